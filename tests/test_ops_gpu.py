"""GPU parity of the nine operators against the float64 oracle and the reference's own
outputs (tests/golden), plus determinism, edge sizes and the tensor-core / SIMT split."""
from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from conftest import load_golden
from oracle import ref_f64
from oracle import ref_torch
from parity import check, check_like_reference, quantum, reference_mlp_hidden, to_np

pytestmark = pytest.mark.gpu

DEV = "cuda"
DTS = {"f16": torch.float16, "bf16": torch.bfloat16, "f32": torch.float32}


def ops():
    from autokernel_b200 import ops as _ops
    return _ops


def _oracle(op, a: dict, kw: dict):
    if op == "rmsnorm":
        return ref_f64.rmsnorm(a["x"], a["weight"], kw.get("eps", 1e-6))
    if op == "layernorm":
        return ref_f64.layernorm(a["x"], a["weight"], a["bias"], kw.get("eps", 1e-5))
    if op == "softmax":
        return ref_f64.softmax(a["x"])
    if op == "rotary_embedding":
        return ref_f64.rotary_embedding(a["x"], a["cos"], a["sin"])
    if op == "reduce":
        return ref_f64.reduce_sum(a["x"], kw.get("dim", -1))
    if op == "cross_entropy":
        return ref_f64.cross_entropy(a["logits"], a["targets"])
    if op == "matmul":
        return ref_f64.matmul(a["A"], a["B"])
    if op == "fused_mlp":
        return ref_f64.fused_mlp(a["x"], a["w_gate"], a["w_up"], a["w_down"], kw.get("activation", "silu"))
    if op == "flash_attention":
        return ref_f64.attention(a["Q"], a["K"], a["V"], kw.get("causal", True), kw.get("sm_scale"))
    raise KeyError(op)


def _run(op, ins: dict, kw: dict):
    f = ops().OPS[op]
    d = {k: v.to(DEV) for k, v in ins.items()}
    if op == "rmsnorm":
        return f(d["x"], d["weight"], **kw)
    if op == "layernorm":
        return f(d["x"], d["weight"], d["bias"], **kw)
    if op == "softmax":
        return f(d["x"])
    if op == "rotary_embedding":
        return f(d["x"], d["cos"], d["sin"])
    if op == "reduce":
        return f(d["x"], **kw)
    if op == "cross_entropy":
        return f(d["logits"], d["targets"])
    if op == "matmul":
        return f(d["A"], d["B"])
    if op == "fused_mlp":
        return f(d["x"], d["w_gate"], d["w_up"], d["w_down"], **kw)
    if op == "flash_attention":
        return f(d["Q"], d["K"], d["V"], **kw)
    raise KeyError(op)


def _np_inputs(ins):
    return {k: to_np(v) for k, v in ins.items()}


def _reduce_n(op, ins, kw):
    if op == "reduce":
        return ins["x"].shape[kw.get("dim", -1)]
    return None


# kernels that round like reference.py in 16-bit dtypes -> output ulps allowed from its output
# (RoPE: bit-identical; RMSNorm: the fp32 sum inside the mean may add in another order)
LIKE_REFERENCE = {"rotary_embedding": 0, "rmsnorm": 1}

OPS = ["rmsnorm", "layernorm", "softmax", "rotary_embedding", "reduce", "cross_entropy",
       "matmul", "fused_mlp", "flash_attention"]


@pytest.mark.parametrize("op", OPS)
def test_golden_cases(op):
    """Every reference-generated case: within tolerance of the f64 oracle, and within the
    reference bench's per-dtype tolerance (+2 output quanta) of the reference's own output."""
    for case in load_golden(op):
        ins, kw = case["inputs"], case["kwargs"]
        y = _run(op, ins, kw)
        torch.cuda.synchronize()
        ref_native = case["out"]
        assert y.shape == ref_native.shape and y.dtype == ref_native.dtype, case["name"]
        if op in LIKE_REFERENCE and y.dtype != torch.float32:
            check_like_reference(y, ref_native, _oracle(op, _np_inputs(ins), kw), op,
                                 case["name"], max_ulps=LIKE_REFERENCE[op])
        else:
            check(y, _oracle(op, _np_inputs(ins), kw), op, case["name"],
                  reduce_n=_reduce_n(op, ins, kw))
        # against the reference's own (native dtype) output, bench.py-style
        bench_tol = {torch.float16: 1e-2, torch.bfloat16: 2e-2, torch.float32: 1e-4}[y.dtype]
        if op in ("softmax", "layernorm", "rotary_embedding"):
            bench_tol = {torch.float16: 1e-3, torch.bfloat16: 2e-3, torch.float32: 1e-5}[y.dtype]
        if op in ("rmsnorm", "reduce") and y.dtype == torch.bfloat16:
            bench_tol = 5e-2
        if op == "cross_entropy" and y.dtype == torch.float32:
            bench_tol = 1e-5
        g = y.float().cpu().double().numpy()
        r = ref_native.double().numpy()
        # the reference's own rounding noise: its native-dtype output vs its fp32 evaluation
        # (bf16 RoPE, for one, rounds each product before subtracting)
        noise = np.abs(r - case["out_f32"].double().numpy())
        fin = np.isfinite(r) & np.isfinite(noise)
        bound = (bench_tol + bench_tol * np.abs(r[fin]) + 2 * quantum(r[fin], y.dtype)
                 + noise[fin])
        if op == "reduce":
            bound = bound * max(1.0, math.sqrt(ins["x"].shape[kw.get("dim", -1)]) / 32)
        assert (np.abs(g[fin] - r[fin]) <= bound).all(), f"{case['name']} vs reference output"


def _gen(seed):
    g = torch.Generator().manual_seed(seed)
    return lambda *s, scale=1.0: torch.randn(*s, generator=g) * scale


@pytest.mark.parametrize("dt", ["bf16", "f16", "f32"])
@pytest.mark.parametrize("M,N,K", [(256, 512, 384), (300, 200, 136), (1024, 1024, 1024),
                                   (128, 11008, 256), (1023, 1023, 1023), (129, 4097, 64)])
def test_matmul_vs_oracle(dt, M, N, K):
    r = _gen(M + N + K)
    A = r(M, K, scale=1 / math.sqrt(K)).to(DTS[dt])
    B = r(K, N).to(DTS[dt])
    y = ops().matmul(A.to(DEV), B.to(DEV))
    check(y, ref_f64.matmul(to_np(A), to_np(B)), "matmul", f"{M}x{N}x{K}_{dt}")


@pytest.mark.parametrize("dt", ["bf16", "f16"])
def test_matmul_transposed_weight_view(dt):
    """B given as W.t() of an nn.Linear weight [N, K] takes the K-major path without a copy."""
    r = _gen(5)
    A = r(200, 512).to(DTS[dt]).to(DEV)
    W = r(320, 512, scale=0.05).to(DTS[dt]).to(DEV)
    y = ops().matmul(A, W.t())
    check(y, ref_f64.matmul(to_np(A), to_np(W).T), "matmul", "linear")


@pytest.mark.parametrize("dt", ["bf16", "f16"])
@pytest.mark.parametrize("act", ["silu", "gelu", "relu2"])
def test_fused_mlp_vs_oracle(dt, act):
    r = _gen(7)
    M, D, H = 300, 256, 704
    x = r(M, D).to(DTS[dt])
    wg, wu, wd = (r(H, D, scale=0.05).to(DTS[dt]), r(H, D, scale=0.05).to(DTS[dt]),
                  r(D, H, scale=0.05).to(DTS[dt]))
    y = ops().fused_mlp(x.to(DEV), wg.to(DEV), wu.to(DEV), wd.to(DEV), act)
    # the hidden is stored with reference.py's roundings (gate, up, act(gate), product), so the
    # output is held to the float64 down projection of that rounded hidden
    hr = reference_mlp_hidden(x, wg, wu, act, DTS[dt])
    check(y, to_np(hr) @ to_np(wd).T, "fused_mlp", act)


@pytest.mark.parametrize("dt", ["bf16", "f16"])
@pytest.mark.parametrize("B,H,S,D,causal", [(1, 4, 256, 128, True), (2, 2, 300, 64, True),
                                            (1, 2, 512, 128, False), (1, 3, 127, 64, True),
                                            (1, 2, 1023, 64, True)])
def test_attention_vs_oracle(dt, B, H, S, D, causal):
    r = _gen(S + D)
    Q, K, V = (r(B, H, S, D).to(DTS[dt]) for _ in range(3))
    y = ops().flash_attention(Q.to(DEV), K.to(DEV), V.to(DEV), causal=causal)
    check(y, ref_f64.attention(to_np(Q), to_np(K), to_np(V), causal), "flash_attention",
          f"{B}x{H}x{S}x{D}")


@pytest.mark.parametrize("op", ["matmul", "flash_attention", "fused_mlp"])
def test_simt_path_agrees(op):
    """The SIMT fallback (forced) meets the same tolerance as the tensor-core path."""
    from autokernel_b200 import _lib
    r = _gen(11)
    if op == "matmul":
        ins = {"A": r(192, 256).to(torch.bfloat16), "B": r(256, 320).to(torch.bfloat16)}
    elif op == "flash_attention":
        ins = {k: r(1, 2, 200, 128).to(torch.bfloat16) for k in ("Q", "K", "V")}
    else:
        ins = {"x": r(64, 128).to(torch.bfloat16), "w_gate": r(256, 128, scale=0.05).to(torch.bfloat16),
               "w_up": r(256, 128, scale=0.05).to(torch.bfloat16), "w_down": r(128, 256, scale=0.05).to(torch.bfloat16)}
    _lib.force_simt(True)
    try:
        y = _run(op, ins, {})
        torch.cuda.synchronize()
    finally:
        _lib.force_simt(False)
    check(y, _oracle(op, _np_inputs(ins), {}), op, "simt")


@pytest.mark.parametrize("dt", ["bf16", "f16", "f32"])
@pytest.mark.parametrize("rows,cols", [(1, 8), (3, 33), (64, 4096), (17, 8192), (4, 32768),
                                       (2, 65536), (5, 70000), (1000, 128), (3001, 2048),
                                       (601, 16384), (2000, 512)])
def test_row_ops_shapes(dt, rows, cols):
    r = _gen(rows * 7 + cols)
    x = r(rows, cols).to(DTS[dt])
    w = (1 + 0.1 * r(cols)).to(DTS[dt])
    b = (0.1 * r(cols)).to(DTS[dt])
    xd = x.to(DEV)
    a = _np_inputs({"x": x, "w": w, "b": b})
    check_like_reference(ops().rmsnorm(xd, w.to(DEV)), ref_torch.rmsnorm(x, w),
                         ref_f64.rmsnorm(a["x"], a["w"]), "rmsnorm", "rms")
    check(ops().layernorm(xd, w.to(DEV), b.to(DEV)), ref_f64.layernorm(a["x"], a["w"], a["b"]), "layernorm", "ln")
    check(ops().softmax(xd * 2), ref_f64.softmax(to_np((x * 2))), "softmax", "sm")


def test_row_ops_strided_rows():
    """A row-strided (non-contiguous) 2-D view is handled without a copy."""
    base = torch.randn(64, 5000, device=DEV, dtype=torch.bfloat16)
    x = base[:, :4096]
    w = torch.ones(4096, device=DEV, dtype=torch.bfloat16)
    check_like_reference(ops().rmsnorm(x, w), ref_torch.rmsnorm(x.cpu(), w.cpu()),
                         ref_f64.rmsnorm(to_np(x), to_np(w)), "rmsnorm", "strided")


@pytest.mark.parametrize("dt", ["bf16", "f16", "f32"])
@pytest.mark.parametrize("shape,cs", [((2, 4, 64, 128), (64, 64)), ((1, 8, 127, 64), (127, 32)),
                                      ((2, 16, 8, 128), (16, 1, 64)), ((3, 5, 6, 10), (6, 5))])
def test_rope_vs_oracle(dt, shape, cs):
    r = _gen(13)
    x = r(*shape).to(DTS[dt])
    c, s = r(*cs).to(DTS[dt]), r(*cs).to(DTS[dt])
    y = ops().rotary_embedding(x.to(DEV), c.to(DEV), s.to(DEV))
    check_like_reference(y, ref_torch.rotary_embedding(x, c, s),
                         ref_f64.rotary_embedding(to_np(x), to_np(c), to_np(s)),
                         "rotary_embedding", str(shape), max_ulps=0)


def test_rope_fp32_table_with_bf16_x():
    """The model path: bf16 activations with an fp32 cos/sin table, bf16 output."""
    r = _gen(14)
    x = r(2, 16, 4, 128).to(torch.bfloat16)
    c, s = ref_f64.cos_sin_table(16, 64)
    ct, st = torch.tensor(c, dtype=torch.float32)[:, None], torch.tensor(s, dtype=torch.float32)[:, None]
    y = ops().rope_apply(x.to(DEV), ct.to(DEV), st.to(DEV))
    assert y.dtype == torch.bfloat16
    check(y, ref_f64.rotary_embedding(to_np(x), to_np(ct), to_np(st)), "rotary_embedding", "fp32 table")


@pytest.mark.parametrize("dt", ["bf16", "f16", "f32"])
@pytest.mark.parametrize("shape,dim", [((4096,), -1), ((1 << 20,) , 0), ((7,), -1), ((33, 1023), -1),
                                       ((8, 300, 5), 1), ((4, 3, 2), 0), ((100, 4097), 1)])
def test_reduce_vs_oracle(dt, shape, dim):
    x = (torch.rand(*shape, generator=torch.Generator().manual_seed(3)) * 2 - 1).to(DTS[dt])
    y = ops().reduce(x.to(DEV), dim)
    check(y, ref_f64.reduce_sum(to_np(x), dim), "reduce", str(shape), reduce_n=shape[dim])


@pytest.mark.parametrize("dt", ["bf16", "f16", "f32"])
@pytest.mark.parametrize("N,V", [(1, 10), (64, 32000), (33, 50257), (1000, 128), (16, 131072),
                                 (1500, 4096), (700, 32000)])
def test_cross_entropy_vs_oracle(dt, N, V):
    g = torch.Generator().manual_seed(N + V)
    logits = (torch.randn(N, V, generator=g) * 2).to(DTS[dt])
    t = torch.randint(0, V, (N,), generator=g)
    if N > 4:
        t[3] = -100
    y = ops().cross_entropy(logits.to(DEV), t.to(DEV))
    check(y, ref_f64.cross_entropy(to_np(logits), t.numpy()), "cross_entropy", f"{N}x{V}")


@pytest.mark.parametrize("dt", ["bf16", "f16", "f32"])
def test_cross_entropy_exact_fields(dt):
    """The row max and the gathered target logit are exact copies of input values."""
    g = torch.Generator().manual_seed(1)
    logits = torch.randn(257, 32000, generator=g).to(DTS[dt]).to(DEV)
    t = torch.randint(0, 32000, (257,), generator=g).to(DEV)
    loss, tt, mx, tl = ops().cross_entropy_rows(logits, t, with_stats=True)
    assert torch.equal(mx, logits.float().max(-1).values)
    assert torch.equal(tl, logits.float().gather(1, t[:, None])[:, 0])


@pytest.mark.parametrize("op", OPS)
def test_bitwise_determinism(op):
    """bench.py stage 4: three runs give bitwise-identical outputs."""
    case = load_golden(op)[-1]
    outs = [_run(op, case["inputs"], case["kwargs"]) for _ in range(3)]
    torch.cuda.synchronize()
    assert all(torch.equal(outs[0], o) for o in outs[1:])


@pytest.mark.parametrize("kind", ["near_zero", "all_zeros", "all_same", "mixed_scale", "near_max"])
@pytest.mark.parametrize("op", ["softmax", "layernorm", "rmsnorm", "cross_entropy"])
def test_stability_inputs(op, kind):
    """bench.py stage 3 transforms (bench.py:808-816) give finite results matching the oracle."""
    r = _gen(21)
    x = r(64, 1024)
    if kind == "near_zero":
        x = x * 1e-6
    elif kind == "all_zeros":
        x = torch.zeros_like(x)
    elif kind == "all_same":
        x = torch.full_like(x, 0.5)
    elif kind == "mixed_scale":
        x[:, ::2] *= 1e3
        x[:, 1::2] *= 1e-3
    else:
        x = x * 100.0
    x = x.to(torch.bfloat16)
    xd = x.to(DEV)
    w = torch.ones(1024, dtype=torch.bfloat16)
    if op == "softmax":
        check(ops().softmax(xd), ref_f64.softmax(to_np(x)), op, kind)
    elif op == "layernorm":
        check(ops().layernorm(xd, w.to(DEV), torch.zeros_like(w).to(DEV)),
              ref_f64.layernorm(to_np(x), to_np(w), np.zeros(1024)), op, kind)
    elif op == "rmsnorm":
        check_like_reference(ops().rmsnorm(xd, w.to(DEV)), ref_torch.rmsnorm(x, w),
                             ref_f64.rmsnorm(to_np(x), to_np(w)), op, kind)
    else:
        t = torch.randint(0, 1024, (64,), generator=torch.Generator().manual_seed(2))
        check(ops().cross_entropy(xd, t.to(DEV)), ref_f64.cross_entropy(to_np(x), t.numpy()), op, kind)


def test_device_status_clean():
    from autokernel_b200 import _lib
    assert _lib.device_status() == 0


@pytest.mark.parametrize("cols", [1024, 32768])
@pytest.mark.parametrize("op", ["softmax", "cross_entropy"])
def test_huge_magnitude_rows(op, cols):
    """bench.py stage 3 scales bf16 inputs by 1e30 (bench.py:808-816); exponents are taken of
    x - max, which stays exact near the max whatever the magnitude."""
    r = _gen(31)
    x = (r(48, cols) * 1e30).to(torch.bfloat16)
    xd = x.to(DEV)
    if op == "softmax":
        check(ops().softmax(xd), ref_f64.softmax(to_np(x)), op, "1e30")
    else:
        t = torch.randint(0, cols, (48,), generator=torch.Generator().manual_seed(3))
        y = ops().cross_entropy(xd, t.to(DEV))
        e = ref_f64.cross_entropy(to_np(x), t.numpy())
        assert abs(float(y.float()) - e) <= 2e-2 * (1 + abs(e)) + 1e28, (float(y), e)


@pytest.mark.parametrize("dt", ["bf16", "f16"])
@pytest.mark.parametrize("B,T,H,Hkv,D,causal", [(2, 300, 4, 4, 128, True), (1, 256, 8, 2, 64, True),
                                                (2, 130, 4, 1, 128, False), (1, 512, 32, 8, 128, True)])
def test_attention_strided_gqa(dt, B, T, H, Hkv, D, causal):
    """[B, T, H, D] projection outputs read in place; key/value head h // (H // Hkv)."""
    r = _gen(T + H)
    q = r(B, T, H, D).to(DTS[dt])
    k = r(B, T, Hkv, D).to(DTS[dt])
    v = r(B, T, Hkv, D).to(DTS[dt])
    qd, kd, vd = q.to(DEV), k.to(DEV), v.to(DEV)
    out = torch.empty(B, T, H, D, dtype=DTS[dt], device=DEV)
    o = ops().attention_bhsd(qd.transpose(1, 2), kd.transpose(1, 2), vd.transpose(1, 2), causal,
                             out=out.transpose(1, 2))
    assert o is not None
    rep = H // Hkv
    Qn = to_np(q).transpose(0, 2, 1, 3)
    Kn = np.repeat(to_np(k).transpose(0, 2, 1, 3), rep, axis=1)
    Vn = np.repeat(to_np(v).transpose(0, 2, 1, 3), rep, axis=1)
    e = ref_f64.attention(Qn, Kn, Vn, causal).transpose(0, 2, 1, 3)
    check(out, e, "flash_attention", f"gqa {B}x{T}x{H}/{Hkv}x{D}")


def test_flash_attention_noncontiguous_inputs():
    """ops.flash_attention on transposed views takes the strided path, same result."""
    r = _gen(3)
    q, k, v = (r(1, 200, 4, 64).to(torch.bfloat16).to(DEV) for _ in range(3))
    o1 = ops().flash_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2))
    o2 = ops().flash_attention(q.transpose(1, 2).contiguous(), k.transpose(1, 2).contiguous(),
                               v.transpose(1, 2).contiguous())
    torch.cuda.synchronize()
    assert torch.equal(o1, o2)


@pytest.mark.parametrize("dt", ["bf16", "f16"])
@pytest.mark.parametrize("case", ["q_is_k", "rising_keys"])
def test_attention_row_max_jumps(dt, case):
    """Rows whose running max grows by a lot in a later key block (self-similar queries and
    keys put the largest score on the diagonal; growing key norms push it to the last block).
    This exercises the rescale of the TMEM accumulator for some rows of a warp and not others."""
    r = _gen(41)
    B, H, S, D = 2, 4, 640, 128
    q = r(B, H, S, D)
    if case == "q_is_k":
        k = q.clone()
    else:
        k = r(B, H, S, D) * torch.linspace(0.2, 3.0, S)[None, None, :, None]
    v = r(B, H, S, D)
    q, k, v = (t.to(DTS[dt]) for t in (q, k, v))
    from autokernel_b200 import _lib
    for causal in (True, False):
        y = ops().flash_attention(q.to(DEV), k.to(DEV), v.to(DEV), causal=causal)
        check(y, ref_f64.attention(to_np(q), to_np(k), to_np(v), causal), "flash_attention",
              f"{case} causal={causal}")
    assert _lib.device_status() == 0


@pytest.mark.parametrize("dt", ["bf16", "f16"])
@pytest.mark.parametrize("B,H,S,causal", [(1, 2, 2048, True), (1, 2, 1536, False),
                                          (2, 2, 700, True), (1, 3, 1100, False)])
def test_attention_d128_long_rows(dt, B, H, S, causal):
    """head_dim 128 over long rows (many mask-free key blocks); ragged S leaves the second
    128-row query tile of a CTA partly or wholly past the end."""
    from autokernel_b200 import _lib
    r = _gen(S + 7 * H)
    Q, K, V = (r(B, H, S, 128).to(DTS[dt]) for _ in range(3))
    y = ops().flash_attention(Q.to(DEV), K.to(DEV), V.to(DEV), causal=causal)
    torch.cuda.synchronize()
    check(y, ref_f64.attention(to_np(Q), to_np(K), to_np(V), causal), "flash_attention",
          f"{B}x{H}x{S}")
    assert _lib.device_status() == 0


@pytest.mark.parametrize("dt", ["bf16", "f16"])
def test_attention_wide_scores(dt):
    """Scores spread over a wide range (scaled keys): exponent arguments far below -125."""
    r = _gen(77)
    B, H, S, D = 1, 2, 1024, 128
    q = r(B, H, S, D)
    k = r(B, H, S, D) * torch.linspace(0.5, 12.0, S)[None, None, :, None]
    v = r(B, H, S, D)
    q, k, v = (t.to(DTS[dt]) for t in (q, k, v))
    y = ops().flash_attention(q.to(DEV), k.to(DEV), v.to(DEV), causal=False)
    check(y, ref_f64.attention(to_np(q), to_np(k), to_np(v), False), "flash_attention", "wide")


@pytest.mark.parametrize("rows,cols", [(64, 4096), (300, 1024), (8, 32768), (8000, 4096)])
def test_layernorm_large_offset(rows, cols):
    """Mean far from zero (1000 + N(0,1)): the merged per-thread variance stays accurate."""
    r = _gen(51)
    x = (1000.0 + r(rows, cols)).float()
    w = torch.ones(cols)
    b = torch.zeros(cols)
    y = ops().layernorm(x.to(DEV), w.to(DEV), b.to(DEV))
    check(y, ref_f64.layernorm(to_np(x), to_np(w), to_np(b)), "layernorm", "offset", scale_tol=100)


@pytest.mark.parametrize("dt", ["bf16", "f16", "f32"])
@pytest.mark.parametrize("M,N,K,inplace", [(300, 256, 512, False), (256, 520, 136, True),
                                           (1023, 1023, 1023, True)])
def test_linear_with_residual(dt, M, N, K, inplace):
    """C = x @ W^T + R formed in the GEMM epilogue; R may be C itself."""
    r = _gen(M + K)
    x = r(M, K, scale=1 / math.sqrt(K)).to(DTS[dt])
    W = r(N, K).to(DTS[dt])
    R = r(M, N).to(DTS[dt])
    Rd = R.to(DEV)
    y = ops().linear(x.to(DEV), W.to(DEV), residual=Rd, out=Rd if inplace else None)
    if inplace:
        assert y.data_ptr() == Rd.data_ptr()
    check(y, ref_f64.matmul(to_np(x), to_np(W).T) + to_np(R), "matmul", "residual")


@pytest.mark.parametrize("dt", ["bf16", "f16"])
@pytest.mark.parametrize("B,T,H,Hkv,hd", [(2, 100, 4, 2, 64), (1, 300, 2, 2, 128)])
def test_linear_rope_epilogue(dt, B, T, H, Hkv, hd):
    """Fused q/k/v projection: RoPE on the q and k columns at position row % T, v untouched."""
    r = _gen(T + hd)
    D = 256
    x = r(B, T, D).to(DTS[dt])
    W = r((H + 2 * Hkv) * hd, D, scale=0.05).to(DTS[dt])
    c, s = ref_f64.cos_sin_table(T, hd // 2)
    ct, st = torch.tensor(c, dtype=torch.float32), torch.tensor(s, dtype=torch.float32)
    y = ops().linear_rope(x.to(DEV), W.to(DEV), ct.to(DEV), st.to(DEV), T, hd, (H + Hkv) * hd)
    proj = (to_np(x) @ to_np(W).T).reshape(B, T, H + 2 * Hkv, hd)
    e = proj.copy()
    e[:, :, :H + Hkv] = ref_f64.rotary_embedding(proj[:, :, :H + Hkv], c[:, None, :], s[:, None, :])
    check(y, e.reshape(B, T, -1), "matmul", "linear_rope")


@pytest.mark.parametrize("op", OPS)
def test_cuda_graph_capture(op):
    """Every operator can be captured in a CUDA graph (no host synchronisation or device
    allocation inside the C ABI) and replays to the eager result."""
    case = load_golden(op)[0]
    ins = {k: v.to(DEV) for k, v in case["inputs"].items()}
    kw = case["kwargs"]
    eager = _run(op, {k: v for k, v in ins.items()}, kw)
    torch.cuda.synchronize()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        _run(op, ins, kw)  # warm-up on the capture stream
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = _run(op, ins, kw)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager)
