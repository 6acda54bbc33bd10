"""The nine operators of AutoKernel's kernel_fn contract, on libak_b200.so.

Each function keeps the signature, argument meaning, output shape and output
dtype of the reference oracle (reference.py) and of the reference starters'
``kernel_fn`` (kernels/<op>.py), so AutoKernel's bench.py / verify.py and
model code can call them unchanged:

    matmul(A, B)                                   reference.py:10-12
    softmax(x)                                     reference.py:15-17
    layernorm(x, weight, bias, eps=1e-5)           reference.py:20-23
    rmsnorm(x, weight, eps=1e-6)                   reference.py:26-29
    flash_attention(Q, K, V, causal=True, sm_scale=None)   reference.py:32-42
    fused_mlp(x, w_gate, w_up, w_down, activation="silu")  reference.py:45-55
    cross_entropy(logits, targets)                 reference.py:58-60
    rotary_embedding(x, cos, sin)                  reference.py:63-69
    reduce(x, dim=-1)                              reference.py:72-74

Python only validates arguments, allocates outputs/workspaces with torch and
passes raw pointers plus the current CUDA stream to the C ABI.  Inputs must
be CUDA tensors; there is no CPU path.  Non-contiguous inputs are made
contiguous first (a copy), except that matmul accepts a transposed [N, K]
weight view as B, and attention accepts strided [B, H, S, D] views (e.g. the
[B, T, H, D] projection outputs transposed), without copying.
"""
from __future__ import annotations

import ctypes
import math

import torch

from . import _lib
from ._lib import call, dtype_code, require_cuda, stream_ptr

IGNORE_INDEX = -100  # F.cross_entropy default, reference.py:60


def _rows_view(x: torch.Tensor) -> torch.Tensor:
    """2-D [rows, cols] view whose last dim is unit-stride (copying if needed)."""
    if x.dim() == 0:
        x = x.reshape(1, 1)
    if x.stride(-1) != 1 and x.numel() > 0:
        x = x.contiguous()
    if x.dim() == 1:
        return x.reshape(1, -1)
    if x.dim() == 2:
        return x
    try:
        return x.view(-1, x.shape[-1])
    except RuntimeError:
        return x.contiguous().view(-1, x.shape[-1])


def _same_dtype(x: torch.Tensor, *ps: torch.Tensor) -> list[torch.Tensor]:
    return [p if p.dtype == x.dtype else p.to(x.dtype) for p in ps]


# ---------------------------------------------------------------- row ops

def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """y = x / sqrt(mean(x^2, -1) + eps) * weight (reference.py:26-29), each step rounded to
    x's dtype as reference.py rounds it."""
    return _rmsnorm("ak_rmsnorm", x, weight, eps)


def rmsnorm_fp32(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """y = x * rsqrt(mean(x^2, -1) + eps) * weight with fp32 intermediates and one rounding
    (models/llama_7b.py:22-30 RMSNorm without the 16-bit overflow of x^2)."""
    return _rmsnorm("ak_rmsnorm_fp32", x, weight, eps)


def _rmsnorm(entry: str, x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    require_cuda(x, weight)
    (weight,) = _same_dtype(x, weight.contiguous())
    x2 = _rows_view(x)
    y = torch.empty(x2.shape, dtype=x.dtype, device=x.device)
    call(entry, x2.data_ptr(), weight.data_ptr(), y.data_ptr(), x2.shape[0], x2.shape[1],
         x2.stride(0), y.stride(0), float(eps), dtype_code(x.dtype), stream_ptr(x.device))
    return y.view(x.shape)


def layernorm(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor,
              eps: float = 1e-5) -> torch.Tensor:
    """F.layer_norm over the last dim (reference.py:20-23)."""
    require_cuda(x, weight, bias)
    weight, bias = _same_dtype(x, weight.contiguous(), bias.contiguous())
    x2 = _rows_view(x)
    y = torch.empty(x2.shape, dtype=x.dtype, device=x.device)
    call("ak_layernorm", x2.data_ptr(), weight.data_ptr(), bias.data_ptr(), y.data_ptr(),
         x2.shape[0], x2.shape[1], x2.stride(0), y.stride(0), float(eps), dtype_code(x.dtype),
         stream_ptr(x.device))
    return y.view(x.shape)


def softmax(x: torch.Tensor) -> torch.Tensor:
    """softmax over the last dim (reference.py:15-17; bench calls it without dim)."""
    require_cuda(x)
    x2 = _rows_view(x)
    y = torch.empty(x2.shape, dtype=x.dtype, device=x.device)
    call("ak_softmax", x2.data_ptr(), y.data_ptr(), x2.shape[0], x2.shape[1], x2.stride(0),
         y.stride(0), dtype_code(x.dtype), stream_ptr(x.device))
    return y.view(x.shape)


def _rope_broadcast(lead_x: tuple, cs: torch.Tensor):
    """(cs_div, cs_rows) such that flattened x row r uses cos row (r // cs_div) % cs_rows,
    or None when cos's broadcast pattern is not a contiguous block of x's dims."""
    lead_c = tuple(cs.shape[:-1])
    if len(lead_c) > len(lead_x):
        if any(d != 1 for d in lead_c[: len(lead_c) - len(lead_x)]):
            return None
        lead_c = lead_c[len(lead_c) - len(lead_x):]
    lead_c = (1,) * (len(lead_x) - len(lead_c)) + lead_c
    dims = []
    for d, (lx, lc) in enumerate(zip(lead_x, lead_c)):
        if lc == 1:
            continue
        if lc != lx:
            return None
        dims.append(d)
    if not dims:
        return 1, 1
    i, j = dims[0], dims[-1] + 1
    if any(lead_c[d] != lead_x[d] for d in range(i, j)):
        return None
    return math.prod(lead_x[j:]), math.prod(lead_x[i:j])


def rope_apply(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
               out: torch.Tensor | None = None) -> torch.Tensor:
    """Interleaved RoPE returning x's dtype; cos/sin may be x's dtype or fp32."""
    require_cuda(x, cos, sin)
    d = x.shape[-1]
    if d % 2:
        raise ValueError("head_dim must be even for RoPE")
    if cos.shape[-1] != d // 2 or sin.shape[-1] != d // 2:
        raise ValueError(f"cos/sin last dim must be head_dim/2 = {d // 2}")
    if cos.shape != sin.shape:
        raise ValueError("cos and sin must have the same shape")
    if cos.dtype not in (x.dtype, torch.float32):
        cos, sin = cos.to(x.dtype), sin.to(x.dtype)
    elif sin.dtype != cos.dtype:
        sin = sin.to(cos.dtype)
    xc = x.contiguous()
    lead = tuple(x.shape[:-1])
    rows = math.prod(lead)
    bc = _rope_broadcast(lead, cos)
    if bc is None:
        cos = cos.expand(*lead, d // 2).contiguous()
        sin = sin.expand(*lead, d // 2).contiguous()
        bc = (1, rows)
    else:
        cos, sin = cos.contiguous(), sin.contiguous()
    y = torch.empty_like(xc) if out is None else out
    call("ak_rotary_embedding", xc.data_ptr(), cos.data_ptr(), sin.data_ptr(), y.data_ptr(),
         rows, d, bc[0], max(bc[1], 1), dtype_code(x.dtype), dtype_code(cos.dtype),
         stream_ptr(x.device))
    return y


def rotary_embedding(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Interleaved-pair RoPE (reference.py:63-69); output dtype follows torch promotion."""
    out_dtype = torch.promote_types(x.dtype, torch.promote_types(cos.dtype, sin.dtype))
    if out_dtype != x.dtype:
        x = x.to(out_dtype)
    return rope_apply(x, cos.to(out_dtype) if cos.dtype not in (out_dtype, torch.float32) else cos,
                      sin.to(out_dtype) if sin.dtype not in (out_dtype, torch.float32) else sin)


# ---------------------------------------------------------------- reductions

_ws_cache: dict = {}


def _reduce_workspace(device: torch.device) -> torch.Tensor:
    key = (device.index, stream_ptr(device))
    ws = _ws_cache.get(key)
    if ws is None:
        nbytes = _lib.load().ak_reduce_workspace_size()
        ws = torch.empty(nbytes, dtype=torch.uint8, device=device)
        _ws_cache[key] = ws
    return ws


def reduce_partial(x: torch.Tensor) -> torch.Tensor:
    """fp64 sum of every element of x, as a 1-element device tensor (a rank's partial)."""
    require_cuda(x)
    xc = x.contiguous()
    total = torch.empty(1, dtype=torch.float64, device=x.device)
    ws = _reduce_workspace(x.device)
    call("ak_reduce_sum_full", xc.data_ptr(), xc.numel(), dtype_code(x.dtype), total.data_ptr(),
         None, 0, ws.data_ptr(), ws.numel(), stream_ptr(x.device))
    return total


def scalar_from_total(total: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """0-d tensor of `dtype` holding the fp64 device value total[0]."""
    out = torch.empty((), dtype=dtype, device=total.device)
    call("ak_scalar_from_sum", total.data_ptr(), out.data_ptr(), dtype_code(dtype),
         stream_ptr(total.device))
    return out


def reduce(x: torch.Tensor, dim: int = -1) -> torch.Tensor:
    """x.sum(dim) (reference.py:72-74); a 1-D input gives a 0-d result like torch."""
    require_cuda(x)
    if x.dim() == 0:
        return x.clone()
    nd = x.dim()
    if not -nd <= dim < nd:
        raise IndexError(f"dim {dim} out of range for a {nd}-D tensor")
    dim = dim % nd
    out_shape = x.shape[:dim] + x.shape[dim + 1:]
    xc = x.contiguous()
    code = dtype_code(x.dtype)
    if nd == 1:
        total = torch.empty(1, dtype=torch.float64, device=x.device)
        out = torch.empty((), dtype=x.dtype, device=x.device)
        ws = _reduce_workspace(x.device)
        call("ak_reduce_sum_full", xc.data_ptr(), xc.numel(), code, total.data_ptr(),
             out.data_ptr(), code, ws.data_ptr(), ws.numel(), stream_ptr(x.device))
        return out
    outer = math.prod(x.shape[:dim])
    inner = math.prod(x.shape[dim + 1:])
    out = torch.empty(out_shape, dtype=x.dtype, device=x.device)
    call("ak_reduce_sum", xc.data_ptr(), out.data_ptr(), outer, x.shape[dim], inner, code, code,
         stream_ptr(x.device))
    return out


def cross_entropy_rows(logits: torch.Tensor, targets: torch.Tensor, with_stats: bool = False):
    """Per-row losses (fp32) of logits [N, V]; optionally the exact row max and target logit."""
    require_cuda(logits, targets)
    l2 = _rows_view(logits)
    t = targets.reshape(-1)
    if t.dtype != torch.int64:
        t = t.to(torch.int64)
    t = t.contiguous()
    n = l2.shape[0]
    if t.numel() != n:
        raise ValueError(f"targets has {t.numel()} entries for {n} rows")
    loss = torch.empty(n, dtype=torch.float32, device=logits.device)
    mx = torch.empty(n, dtype=torch.float32, device=logits.device) if with_stats else None
    tl = torch.empty(n, dtype=torch.float32, device=logits.device) if with_stats else None
    call("ak_cross_entropy_rows", l2.data_ptr(), t.data_ptr(), n, l2.shape[1], l2.stride(0),
         dtype_code(logits.dtype), IGNORE_INDEX, loss.data_ptr(),
         mx.data_ptr() if mx is not None else None, tl.data_ptr() if tl is not None else None,
         None, stream_ptr(logits.device))
    return (loss, t, mx, tl) if with_stats else (loss, t)


def cross_entropy_partial(logits: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
    """fp64 [sum of row losses, number of counted rows] for this shard (device tensor)."""
    loss, t = cross_entropy_rows(logits, targets)
    sc = torch.empty(2, dtype=torch.float64, device=logits.device)
    call("ak_cross_entropy_finalize", loss.data_ptr(), t.data_ptr(), loss.numel(), IGNORE_INDEX,
         sc.data_ptr(), None, 0, stream_ptr(logits.device))
    return sc


def mean_from_sum_count(sc: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    out = torch.empty((), dtype=dtype, device=sc.device)
    call("ak_mean_from_sum_count", sc.data_ptr(), out.data_ptr(), dtype_code(dtype),
         stream_ptr(sc.device))
    return out


def cross_entropy(logits: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
    """Mean cross entropy over rows (reference.py:58-60); 0-d in logits' dtype."""
    loss, t = cross_entropy_rows(logits, targets)
    out = torch.empty((), dtype=logits.dtype, device=logits.device)
    call("ak_cross_entropy_finalize", loss.data_ptr(), t.data_ptr(), loss.numel(), IGNORE_INDEX,
         None, out.data_ptr(), dtype_code(logits.dtype), stream_ptr(logits.device))
    return out


def linear_cross_entropy_rows(x: torch.Tensor, weight: torch.Tensor, targets: torch.Tensor,
                              with_stats: bool = False):
    """Per-row cross entropy of the logits x @ weight^T (an LM head [vocab, dim]) without
    materialising them: (loss fp32 [N], targets int64 [N]) and, with_stats, the row max and
    target logit, bitwise those of linear() followed by cross_entropy_rows().  16-bit x and
    weight use the fused tensor-core kernel; other dtypes run linear() and
    cross_entropy_rows() (this package's kernels, with the logits stored)."""
    require_cuda(x, weight, targets)
    x2 = _rows_view(x)
    n, dim = x2.shape
    vocab = weight.shape[0]
    if weight.dim() != 2 or weight.shape[1] != dim or weight.dtype != x.dtype:
        raise ValueError("linear_cross_entropy: weight must be [vocab, dim] of x's dtype")
    t = targets.reshape(-1).to(torch.int64).contiguous()
    if t.numel() != n:
        raise ValueError(f"targets has {t.numel()} entries for {n} rows")
    w = weight if weight.stride(1) == 1 else weight.contiguous()
    fused = (x.dtype in (torch.float16, torch.bfloat16) and x2.stride(1) == 1
             and x2.stride(0) % 8 == 0 and w.stride(0) % 8 == 0 and dim % 8 == 0
             and x2.data_ptr() % 16 == 0 and w.data_ptr() % 16 == 0)
    if not fused:
        return cross_entropy_rows(linear(x2, w), t, with_stats)
    loss = torch.empty(n, dtype=torch.float32, device=x.device)
    mx = torch.empty(n, dtype=torch.float32, device=x.device) if with_stats else None
    tl = torch.empty(n, dtype=torch.float32, device=x.device) if with_stats else None
    ws = torch.empty(_lib.load().ak_linear_cross_entropy_workspace_size(n, vocab),
                     dtype=torch.uint8, device=x.device)
    call("ak_linear_cross_entropy_rows", x2.data_ptr(), w.data_ptr(), t.data_ptr(), n, vocab, dim,
         x2.stride(0), w.stride(0), dtype_code(x.dtype), IGNORE_INDEX, ws.data_ptr(), ws.numel(),
         loss.data_ptr(), mx.data_ptr() if mx is not None else None,
         tl.data_ptr() if tl is not None else None, None, stream_ptr(x.device))
    return (loss, t, mx, tl) if with_stats else (loss, t)


def linear_cross_entropy_partial(x: torch.Tensor, weight: torch.Tensor,
                                 targets: torch.Tensor) -> torch.Tensor:
    """fp64 [sum of row losses, counted rows] of the LM head + cross entropy on this shard."""
    loss, t = linear_cross_entropy_rows(x, weight, targets)
    sc = torch.empty(2, dtype=torch.float64, device=x.device)
    call("ak_cross_entropy_finalize", loss.data_ptr(), t.data_ptr(), loss.numel(), IGNORE_INDEX,
         sc.data_ptr(), None, 0, stream_ptr(x.device))
    return sc


def linear_cross_entropy(x: torch.Tensor, weight: torch.Tensor,
                         targets: torch.Tensor) -> torch.Tensor:
    """Mean cross entropy (reference.py:58-60) of the logits x @ weight^T, without storing
    them; 0-d in x's dtype."""
    loss, t = linear_cross_entropy_rows(x, weight, targets)
    out = torch.empty((), dtype=x.dtype, device=x.device)
    call("ak_cross_entropy_finalize", loss.data_ptr(), t.data_ptr(), loss.numel(), IGNORE_INDEX,
         None, out.data_ptr(), dtype_code(x.dtype), stream_ptr(x.device))
    return out


# ---------------------------------------------------------------- contractions

def _b_operand(B: torch.Tensor):
    """(tensor, ld, b_kmajor) for B [K, N]: row-major, or a transposed [N, K] row-major view."""
    if B.stride(1) == 1 and B.stride(0) >= B.shape[1]:
        return B, B.stride(0), 0
    if B.stride(0) == 1 and B.stride(1) >= B.shape[0]:
        return B, B.stride(1), 1
    Bc = B.contiguous()
    return Bc, Bc.stride(0), 0


def matmul(A: torch.Tensor, B: torch.Tensor) -> torch.Tensor:
    """C = A @ B (reference.py:10-12) for A [..., M, K] and 2-D B [K, N]."""
    require_cuda(A, B)
    if B.dim() != 2 or A.dim() < 1:
        raise ValueError("matmul expects A [..., M, K] and a 2-D B [K, N]")
    if A.dtype != B.dtype:
        raise ValueError(f"matmul dtype mismatch {A.dtype} vs {B.dtype}")
    squeeze = A.dim() == 1
    A2 = _rows_view(A)
    M, K = A2.shape
    if B.shape[0] != K:
        raise ValueError(f"matmul shape mismatch: A [..., {K}] @ B {tuple(B.shape)}")
    N = B.shape[1]
    Bt, ldb, kmaj = _b_operand(B)
    C = torch.empty((M, N), dtype=A.dtype, device=A.device)
    call("ak_matmul", A2.data_ptr(), Bt.data_ptr(), C.data_ptr(), M, N, K, A2.stride(0), ldb,
         C.stride(0), kmaj, dtype_code(A.dtype), stream_ptr(A.device))
    if squeeze:
        return C.view(N)
    return C.view(*A.shape[:-1], N)


def linear(x: torch.Tensor, weight: torch.Tensor, residual: torch.Tensor | None = None,
           out: torch.Tensor | None = None) -> torch.Tensor:
    """x @ weight^T for an nn.Linear weight [N, K] (no copy of the weight).  With `residual`
    (same shape as the result) the sum x @ weight^T + residual is formed in the GEMM epilogue;
    `out` may be the residual itself for an in-place update."""
    if residual is None and out is None:
        return matmul(x, weight.t())
    require_cuda(x, weight)
    x2 = _rows_view(x).contiguous()
    M, K = x2.shape
    N = weight.shape[0]
    if weight.shape[1] != K or weight.dtype != x.dtype:
        raise ValueError("linear: weight must be [N, K] of x's dtype")
    w = weight.contiguous()
    shape = (*x.shape[:-1], N)
    o = torch.empty(shape, dtype=x.dtype, device=x.device) if out is None else out
    if tuple(o.shape) != shape or not o.is_contiguous():
        raise ValueError("linear: out must be a contiguous tensor of the result shape")
    r = None
    if residual is not None:
        if tuple(residual.shape) != shape or residual.dtype != x.dtype:
            raise ValueError("linear: residual must match the result shape and dtype")
        r = residual if residual.is_contiguous() else residual.contiguous()
    call("ak_matmul_add", x2.data_ptr(), w.data_ptr(), o.data_ptr(),
         r.data_ptr() if r is not None else None, M, N, K, x2.stride(0), K, N, N, 1,
         dtype_code(x.dtype), stream_ptr(x.device))
    return o


RMS_TILE = 256  # columns per partial sum of squares


def row_sumsq(x: torch.Tensor) -> torch.Tensor:
    """Per-row sums of squares of x [..., cols] over 256-column tiles: fp32
    [ceil(cols / 256), rows], the input of the RMSNorm-folded GEMMs."""
    require_cuda(x)
    x2 = _rows_view(x)
    rows, cols = x2.shape
    ss = torch.empty((cols + RMS_TILE - 1) // RMS_TILE, rows, dtype=torch.float32, device=x.device)
    call("ak_row_sumsq", x2.data_ptr(), rows, cols, x2.stride(0), dtype_code(x.dtype),
         ss.data_ptr(), stream_ptr(x.device))
    return ss


def fold_norm_weight(weight: torch.Tensor, norm_weight: torch.Tensor) -> torch.Tensor:
    """w * diag(norm_weight) for an nn.Linear weight [N, K] read after an RMSNorm over K:
    the weight the RMSNorm-folded GEMMs multiply by (rounded once to the weight's dtype)."""
    return (weight.float() * norm_weight.float()[None, :]).to(weight.dtype).contiguous()


def linear_rms(x: torch.Tensor, weight: torch.Tensor, rs: torch.Tensor | None = None,
               eps: float = 1e-6, residual: torch.Tensor | None = None,
               out: torch.Tensor | None = None, want_ss: bool = False, rope: tuple | None = None):
    """x @ weight^T with the rows scaled by 1 / sqrt(mean(x^2) + eps) from rs (the
    row_sumsq partials of x) -- RMSNorm(x) @ w^T when weight = fold_norm_weight(w, norm
    weight) -- plus an optional residual added in the epilogue (out may alias it).  With
    want_ss also returns the partial sums of squares of the result, for the next norm.  With
    rope = (cos, sin, T, head_dim) -- fp32 tables [T, head_dim / 2] -- interleaved RoPE is applied
    to every output column before rounding, row r at position r % T."""
    require_cuda(x, weight)
    x2 = _rows_view(x)
    M, K = x2.shape
    N = weight.shape[0]
    if weight.shape[1] != K or weight.dtype != x.dtype or not weight.is_contiguous():
        raise ValueError("linear_rms: weight must be a contiguous [N, K] of x's dtype")
    shape = (*x.shape[:-1], N)
    o = torch.empty(shape, dtype=x.dtype, device=x.device) if out is None else out
    ss = (torch.empty((N + RMS_TILE - 1) // RMS_TILE, M, dtype=torch.float32, device=x.device)
          if want_ss else None)
    r = residual
    c = s_ = None
    T = hd = 0
    if rope is not None:
        c, s_, T, hd = rope
        c = c.reshape(T, hd // 2).float().contiguous()
        s_ = s_.reshape(T, hd // 2).float().contiguous()
    call("ak_linear_rms", x2.data_ptr(), weight.data_ptr(), o.data_ptr(),
         r.data_ptr() if r is not None else None, M, N, K, x2.stride(0), N, N,
         rs.data_ptr() if rs is not None else None, rs.shape[0] if rs is not None else 0,
         float(eps), ss.data_ptr() if ss is not None else None,
         c.data_ptr() if c is not None else None, s_.data_ptr() if s_ is not None else None,
         T, hd, N if rope is not None else 0, dtype_code(x.dtype), stream_ptr(x.device))
    return (o, ss) if want_ss else o


def mlp_hidden_rms(x: torch.Tensor, w_gate: torch.Tensor, w_up: torch.Tensor,
                   rs: torch.Tensor, eps: float = 1e-6, activation: str = "silu") -> torch.Tensor:
    """act(g) * u of the row-scaled projections g = RMSNorm(x) @ w_gate^T, u = ... @ w_up^T,
    with the norm weight folded into w_gate and w_up (fold_norm_weight)."""
    require_cuda(x, w_gate, w_up, rs)
    x2 = _rows_view(x)
    M, D = x2.shape
    H = w_gate.shape[0]
    if x2.stride(0) != D:
        raise ValueError("mlp_hidden_rms: x rows must be contiguous")
    hidden = torch.empty((*x.shape[:-1], H), dtype=x.dtype, device=x.device)
    call("ak_mlp_gate_up_rms", x2.data_ptr(), w_gate.data_ptr(), w_up.data_ptr(), hidden.data_ptr(),
         M, D, H, rs.data_ptr(), rs.shape[0], float(eps), _lib.AK_ACT[activation],
         dtype_code(x.dtype), stream_ptr(x.device))
    return hidden


def linear_rope(x: torch.Tensor, weight: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                seq_len: int, head_dim: int, rope_cols: int) -> torch.Tensor:
    """x @ weight^T with interleaved RoPE applied in the GEMM epilogue to the first rope_cols
    output columns (head_dim-wide groups); row r of the flattened x is position r % seq_len.
    cos / sin: fp32 [seq_len, head_dim / 2] (any broadcastable view that is contiguous)."""
    require_cuda(x, weight, cos, sin)
    x2 = _rows_view(x).contiguous()
    M, K = x2.shape
    N = weight.shape[0]
    c = cos.reshape(-1, head_dim // 2).float().contiguous()
    s_ = sin.reshape(-1, head_dim // 2).float().contiguous()
    if c.shape[0] != seq_len:
        raise ValueError("cos/sin must hold seq_len rows")
    out = torch.empty((*x.shape[:-1], N), dtype=x.dtype, device=x.device)
    call("ak_linear_rope", x2.data_ptr(), weight.contiguous().data_ptr(), out.data_ptr(), M, N, K,
         x2.stride(0), N, c.data_ptr(), s_.data_ptr(), seq_len, head_dim, rope_cols,
         dtype_code(x.dtype), stream_ptr(x.device))
    return out


def mlp_hidden(x: torch.Tensor, w_gate: torch.Tensor, w_up: torch.Tensor,
               activation: str = "silu") -> torch.Tensor:
    """act(x @ w_gate^T) * (x @ w_up^T) from one dual-B tensor-core GEMM."""
    require_cuda(x, w_gate, w_up)
    x2 = _rows_view(x).contiguous()
    M, D = x2.shape
    H = w_gate.shape[0]
    hidden = torch.empty((*x.shape[:-1], H), dtype=x.dtype, device=x.device)
    call("ak_mlp_gate_up", x2.data_ptr(), w_gate.contiguous().data_ptr(),
         w_up.contiguous().data_ptr(), hidden.data_ptr(), M, D, H, _lib.AK_ACT[activation],
         dtype_code(x.dtype), stream_ptr(x.device))
    return hidden


def fused_mlp(x: torch.Tensor, w_gate: torch.Tensor, w_up: torch.Tensor, w_down: torch.Tensor,
              activation: str = "silu") -> torch.Tensor:
    """down(act(x @ w_gate^T) * (x @ w_up^T)) (reference.py:45-55)."""
    require_cuda(x, w_gate, w_up, w_down)
    if activation not in _lib.AK_ACT:
        raise ValueError(f"unknown activation {activation!r}")
    w_gate, w_up, w_down = (w.contiguous() for w in _same_dtype(x, w_gate, w_up, w_down))
    x2 = _rows_view(x).contiguous()
    M, D = x2.shape
    H = w_gate.shape[0]
    if w_gate.shape != (H, D) or w_up.shape != (H, D) or w_down.shape != (D, H):
        raise ValueError("fused_mlp expects w_gate/w_up [H, D] and w_down [D, H]")
    hidden = torch.empty((M, H), dtype=x.dtype, device=x.device)
    out = torch.empty((M, D), dtype=x.dtype, device=x.device)
    call("ak_fused_mlp", x2.data_ptr(), w_gate.data_ptr(), w_up.data_ptr(), w_down.data_ptr(),
         hidden.data_ptr(), out.data_ptr(), M, D, H, _lib.AK_ACT[activation],
         dtype_code(x.dtype), stream_ptr(x.device))
    return out.view(*x.shape[:-1], D)


def _attn_strides(t: torch.Tensor) -> list[int] | None:
    """[batch, head, seq] element strides of a 4-D [B, H, S, D] view usable by the strided
    tensor-core entry (unit-stride D, 16-byte aligned rows), else None."""
    if t.stride(3) != 1 or t.data_ptr() % 16:
        return None
    st = [t.stride(0), t.stride(1), t.stride(2)]
    # a size-1 dim may carry any stride; give TMA a valid one
    for i in range(3):
        if t.shape[i] == 1:
            st[i] = t.shape[2] * t.shape[3] if i < 2 else t.shape[3]
    if any(x <= 0 or x % 8 for x in st):
        return None
    return st


def attention_bhsd(Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, causal: bool = True,
                   sm_scale: float | None = None, out: torch.Tensor | None = None):
    """Tensor-core attention on 4-D views Q [B, H, Sq, D], K/V [B, Hkv, Sk, D] of any strides
    (H a multiple of Hkv; query head h reads key/value head h // (H // Hkv)).  Returns O with
    Q's shape, or writes it into `out` (any 4-D strided view).  Returns None if the layout is
    not eligible for the tensor-core path (the caller falls back)."""
    require_cuda(Q, K, V)
    B, H, Sq, D = Q.shape
    Hkv = K.shape[1]
    if (Q.dtype not in (torch.float16, torch.bfloat16) or D not in (64, 128)
            or K.shape != V.shape or K.shape[0] != B or K.shape[3] != D or H % Hkv
            or not (Q.dtype == K.dtype == V.dtype) or _lib.forced_simt()):
        return None
    o = torch.empty(Q.shape, dtype=Q.dtype, device=Q.device) if out is None else out
    st = [_attn_strides(t) for t in (Q, K, V, o)]
    if any(x is None for x in st):
        return None
    if sm_scale is None:
        sm_scale = D ** -0.5
    arr = [(ctypes.c_int64 * 3)(*x) for x in st]
    call("ak_flash_attention_strided", Q.data_ptr(), K.data_ptr(), V.data_ptr(), o.data_ptr(), B,
         H, Hkv, Sq, K.shape[2], D, *[ctypes.addressof(a) for a in arr], 1 if causal else 0,
         float(sm_scale), dtype_code(Q.dtype), stream_ptr(Q.device))
    return o


def flash_attention(Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, causal: bool = True,
                    sm_scale: float | None = None) -> torch.Tensor:
    """softmax(Q K^T * scale [+ causal mask]) V (reference.py:32-42)."""
    require_cuda(Q, K, V)
    if Q.dim() < 2 or K.dim() != Q.dim() or V.dim() != Q.dim():
        raise ValueError("Q, K, V must have the same rank >= 2")
    if not (Q.dtype == K.dtype == V.dtype):
        raise ValueError("Q, K, V dtypes differ")
    D = Q.shape[-1]
    if K.shape[-1] != D or V.shape[-1] != D:
        raise ValueError("head_dim of K / V must match Q")
    if sm_scale is None:
        sm_scale = D ** -0.5
    Sq, Sk = Q.shape[-2], K.shape[-2]
    if V.shape[-2] != Sk:
        raise ValueError("K and V sequence lengths differ")
    if (Q.dim() == 4 and K.shape == V.shape and K.shape[0] == Q.shape[0]
            and K.shape[1] in (1, Q.shape[1])):
        # strided views and a single broadcast key/value head go to the tensor cores as-is
        o = attention_bhsd(Q, K, V, causal, sm_scale)
        if o is not None:
            return o
    lead = torch.broadcast_shapes(Q.shape[:-2], K.shape[:-2], V.shape[:-2])
    Qc = Q.expand(*lead, Sq, D).contiguous()
    Kc = K.expand(*lead, Sk, D).contiguous()
    Vc = V.expand(*lead, Sk, D).contiguous()
    O = torch.empty_like(Qc)
    bh = math.prod(lead)
    call("ak_flash_attention", Qc.data_ptr(), Kc.data_ptr(), Vc.data_ptr(), O.data_ptr(), bh, Sq,
         Sk, D, 1 if causal else 0, float(sm_scale), dtype_code(Q.dtype), stream_ptr(Q.device))
    return O


OPS = {
    "matmul": matmul,
    "softmax": softmax,
    "layernorm": layernorm,
    "rmsnorm": rmsnorm,
    "flash_attention": flash_attention,
    "fused_mlp": fused_mlp,
    "cross_entropy": cross_entropy,
    "rotary_embedding": rotary_embedding,
    "reduce": reduce,
}
