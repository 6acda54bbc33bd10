"""AutoKernel's verify.py flow on the drop-ins: swap a model's modules for kernel_fn wrappers and
compare the whole model's output.

verify.py (verify.py:407-605) loads each optimized `kernel_<type>_*.py`, then replaces every
`nn.Linear` with a wrapper that calls `kernel_fn(x_2d, weight.t().contiguous())` and adds the
bias, every `nn.LayerNorm` with `kernel_fn(x_2d, weight, bias, eps)`, and every RMSNorm-like
module (class name in {RMSNorm, LlamaRMSNorm, ...}, or a `weight` + `eps`, no `bias`, name ending
in "norm") with `kernel_fn(x_2d, weight, eps)`; inputs of rank > 2 are flattened to rows and
reshaped back.  The wrappers below do the same calls on the `autokernel_b200.kernels.<op>`
modules, exactly as verify.py would load them from the workspace.

Models: small GPT-2-style (pre-LN, causal, GELU), BERT-style (post-LN, bidirectional) and
LLaMA-style (RMSNorm, SwiGLU, no biases) stacks, random-initialised and seeded (no checkpoints
on the box).  Criterion: the swapped model's error against the same model run in float64 is no
worse than the stock PyTorch model's own error in the same dtype (RMS within 1.5x, max within
3x, plus an ulp of slack), i.e. the swap costs no accuracy.
"""
from __future__ import annotations

import copy
import math

import pytest
import torch
import torch.nn as nn
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

DEV = "cuda"


def kernels():
    from autokernel_b200.kernels import layernorm, matmul, rmsnorm
    return matmul.kernel_fn, layernorm.kernel_fn, rmsnorm.kernel_fn


# ------------------------------------------------------------------ verify.py-style wrappers

def _rows(x):
    return x.reshape(-1, x.shape[-1]) if x.dim() > 2 else x


class LinearSwap(nn.Module):
    def __init__(self, orig: nn.Linear, fn):
        super().__init__()
        self.weight, self.bias, self.fn = orig.weight, orig.bias, fn

    def forward(self, x):
        out = self.fn(_rows(x), self.weight.t().contiguous())
        if self.bias is not None:
            out = out + self.bias
        return out.reshape(*x.shape[:-1], out.shape[-1]) if x.dim() > 2 else out


class LayerNormSwap(nn.Module):
    def __init__(self, orig: nn.LayerNorm, fn):
        super().__init__()
        self.weight, self.bias, self.eps, self.fn = orig.weight, orig.bias, orig.eps, fn

    def forward(self, x):
        return self.fn(_rows(x), self.weight, self.bias, self.eps).reshape(x.shape)


class RMSNormSwap(nn.Module):
    def __init__(self, orig, fn):
        super().__init__()
        self.weight, self.eps, self.fn = orig.weight, orig.eps, fn

    def forward(self, x):
        return self.fn(_rows(x), self.weight, self.eps).reshape(x.shape)


def swap_modules(model: nn.Module) -> dict:
    """Replace modules the way verify.py's OptimizedModelContext does; returns counts per type."""
    mm, ln, rms = kernels()
    counts = {"matmul": 0, "layernorm": 0, "rmsnorm": 0}
    for name, mod in list(model.named_modules()):
        if isinstance(mod, nn.Linear):
            new, kind = LinearSwap(mod, mm), "matmul"
        elif isinstance(mod, nn.LayerNorm):
            new, kind = LayerNormSwap(mod, ln), "layernorm"
        elif (type(mod).__name__ == "RMSNorm" or (hasattr(mod, "weight") and hasattr(mod, "eps")
                                                  and not hasattr(mod, "bias")
                                                  and type(mod).__name__.lower().endswith("norm"))):
            new, kind = RMSNormSwap(mod, rms), "rmsnorm"
        else:
            continue
        parent = model
        *path, last = name.split(".")
        for p in path:
            parent = getattr(parent, p)
        setattr(parent, last, new)
        counts[kind] += 1
    return counts


# ------------------------------------------------------------------ the three model families

class RMSNorm(nn.Module):
    def __init__(self, d, eps=1e-6):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(d))
        self.eps = eps

    def forward(self, x):
        xf = x.float()
        y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps)
        return (y * self.weight.float()).to(x.dtype)


class Attn(nn.Module):
    def __init__(self, d, heads, bias, causal):
        super().__init__()
        self.qkv = nn.Linear(d, 3 * d, bias=bias)
        self.proj = nn.Linear(d, d, bias=bias)
        self.h, self.causal = heads, causal

    def forward(self, x):
        B, T, D = x.shape
        q, k, v = self.qkv(x).view(B, T, 3, self.h, D // self.h).permute(2, 0, 3, 1, 4)
        o = F.scaled_dot_product_attention(q, k, v, is_causal=self.causal)
        return self.proj(o.transpose(1, 2).reshape(B, T, D))


class GPT2Block(nn.Module):
    def __init__(self, d, heads):
        super().__init__()
        self.ln_1, self.ln_2 = nn.LayerNorm(d), nn.LayerNorm(d)
        self.attn = Attn(d, heads, True, True)
        self.fc, self.out = nn.Linear(d, 4 * d), nn.Linear(4 * d, d)

    def forward(self, x):
        x = x + self.attn(self.ln_1(x))
        return x + self.out(F.gelu(self.fc(self.ln_2(x)), approximate="tanh"))


class BertLayer(nn.Module):
    def __init__(self, d, heads):
        super().__init__()
        self.attn = Attn(d, heads, True, False)
        self.ln_attn, self.ln_out = nn.LayerNorm(d, eps=1e-12), nn.LayerNorm(d, eps=1e-12)
        self.inter, self.out = nn.Linear(d, 4 * d), nn.Linear(4 * d, d)

    def forward(self, x):
        x = self.ln_attn(x + self.attn(x))
        return self.ln_out(x + self.out(F.gelu(self.inter(x))))


class LlamaBlock(nn.Module):
    def __init__(self, d, heads, hidden):
        super().__init__()
        self.attention_norm, self.ffn_norm = RMSNorm(d), RMSNorm(d)
        self.attn = Attn(d, heads, False, True)
        self.w1 = nn.Linear(d, hidden, bias=False)
        self.w3 = nn.Linear(d, hidden, bias=False)
        self.w2 = nn.Linear(hidden, d, bias=False)

    def forward(self, x):
        x = x + self.attn(self.attention_norm(x))
        h = self.ffn_norm(x)
        return x + self.w2(F.silu(self.w1(h)) * self.w3(h))


class Stack(nn.Module):
    def __init__(self, family, d=256, heads=4, layers=2, vocab=1024):
        super().__init__()
        self.embed = nn.Embedding(vocab, d)
        if family == "gpt2":
            self.blocks = nn.ModuleList(GPT2Block(d, heads) for _ in range(layers))
            self.norm = nn.LayerNorm(d)
        elif family == "bert":
            self.blocks = nn.ModuleList(BertLayer(d, heads) for _ in range(layers))
            self.norm = nn.Identity()
        else:
            self.blocks = nn.ModuleList(LlamaBlock(d, heads, 688) for _ in range(layers))
            self.norm = RMSNorm(d)
        self.head = nn.Linear(d, vocab, bias=False)

    def forward(self, tokens):
        x = self.embed(tokens)
        for b in self.blocks:
            x = b(x)
        return self.head(self.norm(x))


def _build(family, seed):
    torch.manual_seed(seed)
    m = Stack(family)
    with torch.no_grad():
        for mod in m.modules():  # norm weights and biases away from their 1 / 0 initial values
            if isinstance(mod, (nn.LayerNorm, RMSNorm)):
                mod.weight.add_(0.1 * torch.randn_like(mod.weight))
                if getattr(mod, "bias", None) is not None:
                    mod.bias.add_(0.1 * torch.randn_like(mod.bias))
    return m.eval()


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("family,expect", [("gpt2", {"matmul": 9, "layernorm": 5, "rmsnorm": 0}),
                                           ("bert", {"matmul": 9, "layernorm": 4, "rmsnorm": 0}),
                                           ("llama", {"matmul": 11, "layernorm": 0, "rmsnorm": 5})])
@torch.no_grad()
def test_verify_style_module_swap(family, expect, dtype):
    base = _build(family, 7)
    tokens = torch.randint(0, 1024, (2, 128), generator=torch.Generator().manual_seed(3)).to(DEV)
    exact = copy.deepcopy(base).to(DEV, torch.float64)(tokens)
    stock = copy.deepcopy(base).to(DEV, dtype)
    want = stock(tokens).double()
    swapped = copy.deepcopy(base).to(DEV, dtype)
    assert swap_modules(swapped) == expect
    got = swapped(tokens)
    torch.cuda.synchronize()
    assert got.dtype == dtype and got.shape == want.shape
    assert torch.isfinite(got).all()
    got = got.double()
    ulp = exact.abs().max().item() * (2.0 ** -10 if dtype == torch.float16 else 2.0 ** -7)
    rms = lambda e: e.pow(2).mean().sqrt().item()  # noqa: E731
    err_stock, err_swap = (want - exact).abs(), (got - exact).abs()
    assert rms(err_swap) <= 1.5 * rms(err_stock) + 0.05 * ulp, (family, rms(err_swap), rms(err_stock))
    assert err_swap.max().item() <= 3.0 * err_stock.max().item() + ulp, \
        (family, err_swap.max().item(), err_stock.max().item())
    assert math.isfinite(err_swap.max().item())
