"""ak_reduce_sum_full_noalloc: the full sum for callers that cannot allocate device memory.

Such callers (code running inside another framework's allocator, or hosts that forbid
cudaMalloc once they are running) cannot hand the library a workspace, so this entry point keeps
its per-CTA partials in scratch built into the library.  This file is named to be collected
last: if it fails, a stop-at-first-failure run has already run every other test.  The test
calls the entry point twice in a row through the C ABI and compares each result with the
workspace-taking ak_reduce_sum_full on the same input.  Both entry points launch the same two
kernels over the same number of partial slots, so the results must agree bit for bit.  The
second call of each pair sums far fewer elements than the first, so most CTAs get no elements:
their slots still hold the first call's partials unless the second call rewrites them.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dt,sizes", [(torch.float32, ((1 << 24) + 3, 7)),
                                      (torch.bfloat16, (1 << 20, 1000)),
                                      (torch.float16, (100003, 33))])
def test_noalloc_matches_workspace_entry_twice(dt, sizes):
    from autokernel_b200 import _lib
    lib = _lib.load()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    s = torch.cuda.current_stream(dev).cuda_stream
    code = _lib.dtype_code(dt)
    ws = torch.empty(lib.ak_reduce_workspace_size(), dtype=torch.uint8, device=dev)
    for call, n in enumerate(sizes):
        g = torch.Generator(device=dev).manual_seed(call)
        x = (torch.rand(n, device=dev, generator=g) * 2 - 1).to(dt)
        tot_ref = torch.empty(1, dtype=torch.float64, device=dev)
        out_ref = torch.empty((), dtype=dt, device=dev)
        rc = lib.ak_reduce_sum_full(x.data_ptr(), n, code, tot_ref.data_ptr(), out_ref.data_ptr(),
                                    code, ws.data_ptr(), ws.numel(), s)
        assert rc == 0, lib.ak_last_error()
        tot = torch.empty(1, dtype=torch.float64, device=dev)
        out = torch.empty((), dtype=dt, device=dev)
        rc = lib.ak_reduce_sum_full_noalloc(x.data_ptr(), n, code, tot.data_ptr(), out.data_ptr(),
                                            code, s)
        assert rc == 0, lib.ak_last_error()
        torch.cuda.synchronize()
        assert torch.equal(tot, tot_ref), (call, float(tot.item()), float(tot_ref.item()))
        assert torch.equal(out, out_ref), (call, float(out.float().item()), float(out_ref.float().item()))
        # and both are within the reduce tolerance of the float64 sum
        e = float(x.double().sum().item())
        assert abs(float(tot.item()) - e) <= 1e-4 * max(1.0, np.sqrt(n) / 32) + 1e-5 * abs(e)
