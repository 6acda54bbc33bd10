"""The C-ABI library loads without a GPU, exports every symbol include/ak_b200.h declares,
and rejects bad arguments with error codes and messages before touching the device."""
from __future__ import annotations

import ctypes
import re

import pytest

from conftest import ROOT


def _declared():
    text = (ROOT / "include" / "ak_b200.h").read_text()
    return sorted(set(re.findall(r"^AK_API\s+[\w\s\*]+?\b(ak_\w+)\(", text, flags=re.M)))


def test_library_exports_every_declared_symbol():
    from autokernel_b200 import _lib
    lib = _lib.load()
    names = _declared()
    assert len(names) >= 20
    for n in names:
        assert hasattr(lib, n), n
    # the ctypes signature table covers the whole header
    assert set(names) == set(_lib.SIGNATURES), set(names) ^ set(_lib.SIGNATURES)


def test_version():
    from autokernel_b200 import _lib
    assert _lib.load().ak_version() == 1


@pytest.mark.parametrize("call,code", [
    (lambda L: L.ak_rmsnorm(1, 1, 1, 4, 4, 4, 4, 1e-6, 7, None), -2),        # bad dtype
    (lambda L: L.ak_rmsnorm(1, 1, 1, 4, 8, 4, 8, 1e-6, 2, None), -3),        # ldx < cols
    (lambda L: L.ak_softmax(None, None, 4, 4, 4, 4, 2, None), -1),           # null pointer
    (lambda L: L.ak_rotary_embedding(1, 1, 1, 1, 4, 7, 1, 1, 2, 2, None), -3),  # odd head_dim
    (lambda L: L.ak_rotary_embedding(1, 1, 1, 1, 4, 8, 1, 1, 2, 1, None), -2),  # cos dtype
    (lambda L: L.ak_matmul(1, 1, 1, 4, 4, 4, 2, 4, 4, 0, 2, None), -3),     # lda < K
    (lambda L: L.ak_mlp_gate_up(1, 1, 1, 1, 4, 4, 4, 9, 2, None), -1),      # activation
    (lambda L: L.ak_flash_attention(1, 1, 1, 1, 2, 4, 0, 64, 1, 0.1, 2, None), -3),  # Sk = 0
    (lambda L: L.ak_reduce_sum_full(1, 10, 2, None, None, 2, None, 0, None), -1),   # no workspace
    (lambda L: L.ak_cross_entropy_rows(1, 1, 4, 0, 0, 2, -100, 1, None, None, None, None), -3),
])
def test_argument_errors_are_reported_not_raised(call, code):
    from autokernel_b200 import _lib
    L = _lib.load()
    assert call(L) == code
    assert L.ak_last_error()  # a message is left behind


def test_empty_inputs_are_noops():
    from autokernel_b200 import _lib
    L = _lib.load()
    assert L.ak_rmsnorm(None, None, None, 0, 16, 16, 16, 1e-6, 2, None) == 0
    assert L.ak_matmul(None, None, None, 0, 8, 8, 8, 8, 8, 0, 2, None) == 0
    assert L.ak_flash_attention(None, None, None, None, 0, 4, 4, 64, 1, 0.1, 2, None) == 0
