"""LLaMA forward (+ next-token cross entropy) on the nine B200 operators.

The architecture is AutoKernel's models/llama_7b.py (LlamaModel / LlamaModel7B,
models/llama_7b.py:114-209): token embedding, n_layers x [RMSNorm -> q/k/v
projections -> interleaved RoPE -> causal attention (grouped KV heads) -> output
projection -> residual; RMSNorm -> SwiGLU MLP -> residual], final RMSNorm, LM head.
Parameter names are the reference module's state_dict keys, so
`LlamaB200.from_state_dict(ref_model.state_dict(), cfg)` runs a reference model's
weights unchanged.  This is the model-level drop-in that verify.py performs by
module surgery (verify.py:510-641), extended to attention, RoPE, the MLP and the
loss.

Every arithmetic step is one of this package's kernels:
    RMSNorm              folded into the projections that read it (16-bit weights): the
                         o-/down-projection epilogues write per-row sums of squares of the
                         new hidden state, the q/k/v and gate/up GEMMs scale their rows by
                         1 / rms with the norm weight folded into their weights, so the
                         normalised activations are never stored (ops.linear_rms,
                         ops.mlp_hidden_rms); otherwise ops.rmsnorm_fp32 (csrc/rowops.cu)
    q/k/v/o projections  ops.linear            (tcgen05 GEMM, K-major weights, no copies)
    RoPE                 ops.rope_apply        (fp32 cos/sin table, [B, T, H, D] in place)
    attention            ops.attention_bhsd    (reads [B, T, H, D] views, GQA, causal)
    SwiGLU MLP           ops.mlp_hidden + ops.linear (dual GEMM + SiLU*mul epilogue, down GEMM)
    residual adds        in the o-projection / down-projection GEMM epilogues, in place
    LM head + loss       ops.linear_cross_entropy_partial: one tcgen05 GEMM whose epilogue
                         reduces each vocab tile to (max, sum exp) and the target logit
                         (the logits are never stored; ignore_index masks the last position)
Glue left to torch: the embedding gather.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from . import ops, shard


@dataclass
class LlamaConfig:
    vocab_size: int = 32000
    dim: int = 4096
    n_layers: int = 32
    n_heads: int = 32
    n_kv_heads: int = 32
    hidden_dim: int = 11008
    norm_eps: float = 1e-6
    rope_theta: float = 10000.0

    @property
    def head_dim(self) -> int:
        return self.dim // self.n_heads

    def linear_params(self) -> int:
        hd = self.head_dim
        per_layer = (self.dim * self.n_heads * hd + 2 * self.dim * self.n_kv_heads * hd
                     + self.n_heads * hd * self.dim + 3 * self.dim * self.hidden_dim)
        return self.n_layers * per_layer + self.dim * self.vocab_size

    def flops_per_token(self, seq_len: int) -> float:
        """Forward FLOPs per token: 2 x linear params + causal attention (QK^T and PV over the
        (T+1)/2 visible keys on average)."""
        attn = self.n_layers * 2 * 2 * self.n_heads * self.head_dim * (seq_len + 1) / 2
        return 2.0 * self.linear_params() + attn


LLAMA_7B = LlamaConfig()  # BASELINE e2e config: 32 heads of 128, MHA (n_kv_heads = 32)


def rope_tables(seq_len: int, head_dim: int, theta: float, device):
    """fp32 cos/sin [T, 1, head_dim/2] of angle t * theta^(-2i/head_dim), the table
    precompute_freqs_cis builds (models/llama_7b.py:33-37), shaped to broadcast over heads."""
    inv = 1.0 / theta ** (torch.arange(0, head_dim, 2, device=device, dtype=torch.float32) / head_dim)
    ang = torch.outer(torch.arange(seq_len, device=device, dtype=torch.float32), inv)
    return ang.cos()[:, None, :].contiguous(), ang.sin()[:, None, :].contiguous()


class LlamaB200:
    """Inference-mode LLaMA whose forward runs on the autokernel_b200 kernels."""

    def __init__(self, cfg: LlamaConfig, weights: dict[str, torch.Tensor],
                 fuse_norms: bool | None = None):
        self.cfg = cfg
        self.w = weights
        self._rope: dict = {}
        dt = weights["tok_embeddings.weight"].dtype
        # RMSNorm folded into the projections after it (16-bit weights: tensor-core GEMMs)
        self.fuse_norms = dt in (torch.float16, torch.bfloat16) if fuse_norms is None else fuse_norms
        # with folded norms, RoPE of q and k runs in their projection GEMMs' epilogue
        self.fuse_rope = self.fuse_norms
        self._folded: dict[int, tuple] = {}

    @staticmethod
    def random_weights(cfg: LlamaConfig, device, dtype=torch.float16, seed: int = 0,
                       std: float = 0.02) -> dict[str, torch.Tensor]:
        """N(0, std) linear / embedding weights and unit norms (BASELINE: fp16, N(0, 0.02))."""
        g = torch.Generator(device=device).manual_seed(seed)
        hd = cfg.head_dim

        def rnd(*shape):
            return (torch.randn(*shape, device=device, generator=g) * std).to(dtype)

        w = {"tok_embeddings.weight": rnd(cfg.vocab_size, cfg.dim)}
        for i in range(cfg.n_layers):
            p = f"layers.{i}."
            w[p + "attention.wq.weight"] = rnd(cfg.n_heads * hd, cfg.dim)
            w[p + "attention.wk.weight"] = rnd(cfg.n_kv_heads * hd, cfg.dim)
            w[p + "attention.wv.weight"] = rnd(cfg.n_kv_heads * hd, cfg.dim)
            w[p + "attention.wo.weight"] = rnd(cfg.dim, cfg.n_heads * hd)
            w[p + "feed_forward.w1.weight"] = rnd(cfg.hidden_dim, cfg.dim)
            w[p + "feed_forward.w2.weight"] = rnd(cfg.dim, cfg.hidden_dim)
            w[p + "feed_forward.w3.weight"] = rnd(cfg.hidden_dim, cfg.dim)
            w[p + "attention_norm.weight"] = torch.ones(cfg.dim, device=device, dtype=dtype)
            w[p + "ffn_norm.weight"] = torch.ones(cfg.dim, device=device, dtype=dtype)
        w["norm.weight"] = torch.ones(cfg.dim, device=device, dtype=dtype)
        w["output.weight"] = rnd(cfg.vocab_size, cfg.dim)
        return w

    @classmethod
    def from_state_dict(cls, sd: dict, cfg: LlamaConfig, device="cuda", dtype=torch.float16):
        """Weights of a reference LlamaModel / LlamaModel7B (its state_dict keys)."""
        w = {k: v.detach().to(device=device, dtype=dtype).contiguous()
             for k, v in sd.items() if not k.endswith("freqs_cis")}
        return cls(cfg, w)

    def _tables(self, T: int, device):
        key = (T, str(device))
        if key not in self._rope:
            self._rope[key] = rope_tables(T, self.cfg.head_dim, self.cfg.rope_theta, device)
        return self._rope[key]

    def _layer(self, i: int, h: torch.Tensor, cos, sin) -> torch.Tensor:
        c, w = self.cfg, self.w
        p = f"layers.{i}."
        B, T, _ = h.shape
        hd = c.head_dim
        x = ops.rmsnorm_fp32(h, w[p + "attention_norm.weight"], c.norm_eps)
        q = ops.linear(x, w[p + "attention.wq.weight"]).view(B, T, c.n_heads, hd)
        k = ops.linear(x, w[p + "attention.wk.weight"]).view(B, T, c.n_kv_heads, hd)
        v = ops.linear(x, w[p + "attention.wv.weight"]).view(B, T, c.n_kv_heads, hd)
        q = ops.rope_apply(q, cos, sin)
        k = ops.rope_apply(k, cos, sin)
        o = self._attention(q, k, v, B, T)
        # residual adds happen in the GEMM epilogues, in place on h
        ops.linear(o.view(B, T, c.n_heads * hd), w[p + "attention.wo.weight"], residual=h, out=h)
        x = ops.rmsnorm_fp32(h, w[p + "ffn_norm.weight"], c.norm_eps)
        hidden = ops.mlp_hidden(x, w[p + "feed_forward.w1.weight"], w[p + "feed_forward.w3.weight"])
        ops.linear(hidden, w[p + "feed_forward.w2.weight"], residual=h, out=h)
        return h

    def _fold(self, i: int) -> tuple:
        """Projection weights of layer i with the RMSNorm weight that precedes them folded in
        (w * diag(norm.weight), rounded once): q, k, v after attention_norm, w1, w3 after
        ffn_norm.  Built once; the reference weights are kept for the unfused path."""
        if i not in self._folded:
            w, p = self.w, f"layers.{i}."
            an, fn = w[p + "attention_norm.weight"], w[p + "ffn_norm.weight"]
            self._folded[i] = tuple(
                ops.fold_norm_weight(w[p + k], n) for k, n in (
                    ("attention.wq.weight", an), ("attention.wk.weight", an),
                    ("attention.wv.weight", an), ("feed_forward.w1.weight", fn),
                    ("feed_forward.w3.weight", fn)))
        return self._folded[i]

    def _attention(self, q, k, v, B, T):
        c = self.cfg
        hd = c.head_dim
        o = torch.empty(B, T, c.n_heads, hd, dtype=q.dtype, device=q.device)
        r = ops.attention_bhsd(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2),
                               causal=True, out=o.transpose(1, 2))
        if r is None:  # layouts / head sizes the tensor-core path cannot take
            rep = c.n_heads // c.n_kv_heads
            o = ops.flash_attention(q.transpose(1, 2),
                                    k.transpose(1, 2).repeat_interleave(rep, 1),
                                    v.transpose(1, 2).repeat_interleave(rep, 1))
            o = o.transpose(1, 2).contiguous()
        return o

    def _layer_fused(self, i: int, h: torch.Tensor, ss: torch.Tensor, cos, sin):
        """One decoder layer with both RMSNorms folded into the GEMMs that read them: ss holds
        the per-row partial sums of squares of h, and the o-projection and down-projection
        epilogues (which add the residual into h in place) write those of the new h."""
        c, w = self.cfg, self.w
        p = f"layers.{i}."
        B, T, _ = h.shape
        hd, eps = c.head_dim, c.norm_eps
        wq, wk, wv, w1, w3 = self._fold(i)
        rope = (cos, sin, T, hd) if self.fuse_rope else None
        q = ops.linear_rms(h, wq, ss, eps, rope=rope).view(B, T, c.n_heads, hd)
        k = ops.linear_rms(h, wk, ss, eps, rope=rope).view(B, T, c.n_kv_heads, hd)
        v = ops.linear_rms(h, wv, ss, eps).view(B, T, c.n_kv_heads, hd)
        if not self.fuse_rope:
            q = ops.rope_apply(q, cos, sin)
            k = ops.rope_apply(k, cos, sin)
        o = self._attention(q, k, v, B, T)
        _, ss = ops.linear_rms(o.view(B, T, c.n_heads * hd), w[p + "attention.wo.weight"],
                               residual=h, out=h, want_ss=True)
        hidden = ops.mlp_hidden_rms(h, w1, w3, ss, eps)
        _, ss = ops.linear_rms(hidden, w[p + "feed_forward.w2.weight"], residual=h, out=h,
                               want_ss=True)
        return h, ss

    @torch.no_grad()
    def hidden(self, tokens: torch.Tensor) -> torch.Tensor:
        """The final normalised hidden state [B, T, dim], the LM head's input."""
        _, T = tokens.shape
        cos, sin = self._tables(T, tokens.device)
        h = torch.nn.functional.embedding(tokens, self.w["tok_embeddings.weight"])  # new tensor
        if self.fuse_norms:
            ss = ops.row_sumsq(h)
            for i in range(self.cfg.n_layers):
                h, ss = self._layer_fused(i, h, ss, cos, sin)
        else:
            for i in range(self.cfg.n_layers):
                h = self._layer(i, h, cos, sin)
        return ops.rmsnorm_fp32(h, self.w["norm.weight"], self.cfg.norm_eps)

    @torch.no_grad()
    def forward(self, tokens: torch.Tensor) -> torch.Tensor:
        """Logits [B, T, vocab] (models/llama_7b.py:199-209)."""
        return ops.linear(self.hidden(tokens), self.w["output.weight"])

    __call__ = forward

    @staticmethod
    def next_token_targets(tokens: torch.Tensor) -> torch.Tensor:
        """Targets [B, T]: tokens shifted left by one, the last position ignored (-100), so the
        loss over all B*T logit rows equals the mean over the B*(T-1) predicted positions."""
        t = torch.full_like(tokens, ops.IGNORE_INDEX)
        t[:, :-1] = tokens[:, 1:]
        return t

    @torch.no_grad()
    def loss(self, tokens: torch.Tensor, group=None) -> torch.Tensor:
        """Mean next-token cross entropy; with a process group, the mean over all ranks'
        sequences (one fp64 all-reduce of (sum, count)).  The LM head and the loss run as one
        fused kernel (ops.linear_cross_entropy_rows): the [B*T, vocab] logits are never
        stored."""
        h = self.hidden(tokens)
        targets = self.next_token_targets(tokens)
        W = self.w["output.weight"]
        return shard.cross_entropy_sharded(
            h.view(-1, h.shape[-1]), targets.view(-1), group=group,
            partial_fn=lambda x, t: ops.linear_cross_entropy_partial(x, W, t),
            out_dtype=h.dtype)


def model_flops(cfg: LlamaConfig, batch: int, seq_len: int) -> float:
    return cfg.flops_per_token(seq_len) * batch * seq_len


__all__ = ["LlamaConfig", "LLAMA_7B", "LlamaB200", "rope_tables", "model_flops"]
