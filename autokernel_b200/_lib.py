"""ctypes binding of libak_b200.so (the C ABI declared in include/ak_b200.h).

The library is built ahead of time in-tree (``python -m autokernel_b200.build``)
and loaded from ``autokernel_b200/libak_b200.so``.  There is no fallback: if the
library is missing or the process has no CUDA device, every op raises.
"""
from __future__ import annotations

import ctypes as C
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "libak_b200.so"

AK_F32, AK_F16, AK_BF16 = 0, 1, 2
AK_ACT = {"silu": 0, "gelu": 1, "relu2": 2}

DTYPE_CODE = {torch.float32: AK_F32, torch.float16: AK_F16, torch.bfloat16: AK_BF16}

_vp, _i64, _i32, _f32, _sz = C.c_void_p, C.c_int64, C.c_int, C.c_float, C.c_size_t

# name -> (restype, argtypes); must match include/ak_b200.h
SIGNATURES = {
    "ak_last_error": (C.c_char_p, []),
    "ak_version": (_i32, []),
    "ak_device_status": (_i32, [_i32]),
    "ak_sm_count": (_i32, []),
    "ak_set_force_simt": (None, [_i32]),
    "ak_rmsnorm": (_i32, [_vp, _vp, _vp, _i64, _i64, _i64, _i64, _f32, _i32, _vp]),
    "ak_rmsnorm_fp32": (_i32, [_vp, _vp, _vp, _i64, _i64, _i64, _i64, _f32, _i32, _vp]),
    "ak_layernorm": (_i32, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _f32, _i32, _vp]),
    "ak_softmax": (_i32, [_vp, _vp, _i64, _i64, _i64, _i64, _i32, _vp]),
    "ak_rotary_embedding": (_i32, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i32, _i32, _vp]),
    "ak_reduce_sum": (_i32, [_vp, _vp, _i64, _i64, _i64, _i32, _i32, _vp]),
    "ak_reduce_workspace_size": (_sz, []),
    "ak_reduce_sum_full": (_i32, [_vp, _i64, _i32, _vp, _vp, _i32, _vp, _sz, _vp]),
    "ak_reduce_sum_full_noalloc": (_i32, [_vp, _i64, _i32, _vp, _vp, _i32, _vp]),
    "ak_scalar_from_sum": (_i32, [_vp, _vp, _i32, _vp]),
    "ak_cross_entropy_rows": (_i32, [_vp, _vp, _i64, _i64, _i64, _i32, _i64, _vp, _vp, _vp, _vp, _vp]),
    "ak_cross_entropy_finalize": (_i32, [_vp, _vp, _i64, _i64, _vp, _vp, _i32, _vp]),
    "ak_mean_from_sum_count": (_i32, [_vp, _vp, _i32, _vp]),
    "ak_linear_cross_entropy_workspace_size": (_sz, [_i64, _i64]),
    "ak_linear_cross_entropy_rows": (_i32, [_vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i32, _i64,
                                            _vp, _sz, _vp, _vp, _vp, _vp, _vp]),
    "ak_matmul": (_i32, [_vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _i32, _i32, _vp]),
    "ak_matmul_add": (_i32, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i32, _i32, _vp]),
    "ak_linear_rope": (_i32, [_vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _vp, _vp, _i64, _i64, _i64, _i32, _vp]),
    "ak_row_sumsq": (_i32, [_vp, _i64, _i64, _i64, _i32, _vp, _vp]),
    "ak_linear_rms": (_i32, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _vp, _i32, _f32,
                             _vp, _vp, _vp, _i64, _i64, _i64, _i32, _vp]),
    "ak_mlp_gate_up_rms": (_i32, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _vp, _i32, _f32, _i32, _i32,
                                  _vp]),
    "ak_mlp_gate_up": (_i32, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i32, _i32, _vp]),
    "ak_fused_mlp": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i32, _i32, _vp]),
    "ak_flash_attention": (_i32, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i32, _f32, _i32, _vp]),
    "ak_flash_attention_strided": (_i32, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64,
                                          _vp, _vp, _vp, _vp, _i32, _f32, _i32, _vp]),
}

_lib = None
_lock = threading.Lock()


class AkError(RuntimeError):
    """A libak_b200 entry point returned an error code."""


def load() -> C.CDLL:
    """Load (once) and return the library with argument types set."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise AkError(
                    f"{LIB_PATH} is missing; build it with `python -m autokernel_b200.build` "
                    "(there is no fallback implementation)")
            lib = C.CDLL(str(LIB_PATH))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def call(name: str, *args) -> None:
    """Invoke an entry point and raise AkError (ValueError for argument errors) on failure."""
    rc = getattr(load(), name)(*args)
    if rc != 0:
        msg = load().ak_last_error().decode(errors="replace")
        if rc in (-1, -2, -3, -4):
            raise ValueError(f"{name}: {msg} (code {rc})")
        raise AkError(f"{name}: {msg} (code {rc})")


def dtype_code(t: torch.dtype) -> int:
    try:
        return DTYPE_CODE[t]
    except KeyError:
        raise ValueError(f"unsupported dtype {t}; expected float32, float16 or bfloat16") from None


def stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def require_cuda(*ts: torch.Tensor) -> torch.device:
    """All tensors must live on one CUDA device; makes it current and returns it."""
    dev = ts[0].device
    if dev.type != "cuda":
        raise ValueError("autokernel_b200 ops run on CUDA tensors only (no CPU fallback)")
    for t in ts[1:]:
        if t.device != dev:
            raise ValueError(f"tensors on different devices: {dev} vs {t.device}")
    if torch.cuda.current_device() != dev.index:
        torch.cuda.set_device(dev)
    return dev


_forced_simt = False


def force_simt(on: bool) -> None:
    """Test hook: route contractions through the SIMT kernels."""
    global _forced_simt
    _forced_simt = bool(on)
    load().ak_set_force_simt(1 if on else 0)


def forced_simt() -> bool:
    import os
    return _forced_simt or os.environ.get("AK_FORCE_SIMT") == "1"


def device_status(clear: bool = True) -> int:
    return load().ak_device_status(1 if clear else 0)
