"""Generate tests/golden/llama_tiny.pt from AutoKernel's own model code (models/llama_7b.py).

    python tests/golden/make_golden_llama.py [REF_DIR]

A tiny LlamaModel (vocab 256, dim 128, 2 layers, 4 heads, 2 kv heads, hidden 256) with seeded
weights (its state_dict is stored), two 48-token sequences, and the reference's fp32 CPU logits.
"""
from __future__ import annotations

import importlib.util
import sys
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
REF_DIR = Path(sys.argv[1] if len(sys.argv) > 1 else "/root/reference")

spec = importlib.util.spec_from_file_location("ak_ref_llama", REF_DIR / "models" / "llama_7b.py")
m = importlib.util.module_from_spec(spec)
spec.loader.exec_module(m)

CFG = dict(vocab_size=256, dim=128, n_layers=2, n_heads=4, n_kv_heads=2, hidden_dim=256, max_seq_len=64)


def main():
    torch.manual_seed(0)
    model = m.LlamaModel(**CFG).float().eval()
    with torch.no_grad():
        for name, p in model.named_parameters():
            if not name.endswith("norm.weight"):
                p.normal_(0.0, 0.05)
            else:
                p.copy_(1 + 0.1 * torch.randn_like(p))
    tokens = torch.randint(0, CFG["vocab_size"], (2, 48), generator=torch.Generator().manual_seed(1))
    with torch.no_grad():
        logits = model(tokens)
    sd = {k: v.clone() for k, v in model.state_dict().items() if not k.endswith("freqs_cis")}
    torch.save({"cfg": CFG, "state_dict": sd, "tokens": tokens, "logits": logits}, HERE / "llama_tiny.pt")
    print((HERE / "llama_tiny.pt").stat().st_size / 1e3, "KB")


if __name__ == "__main__":
    main()
