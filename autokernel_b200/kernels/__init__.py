"""One drop-in module per operator, each exposing KERNEL_TYPE and kernel_fn."""
import importlib

NAMES = ("matmul", "softmax", "layernorm", "rmsnorm", "flash_attention", "fused_mlp",
         "cross_entropy", "rotary_embedding", "reduce")


def get(name: str):
    """Return the drop-in module for an operator name."""
    if name not in NAMES:
        raise KeyError(f"unknown kernel type {name!r}; one of {NAMES}")
    return importlib.import_module(f"{__name__}.{name}")
