"""The no-allocation router entry point (pulsar_op_moe_router_topk_noalloc).

Some callers cannot allocate device memory: their host owns every device byte through its
own memory manager, or they call in from another language without a device allocator. For
them the router top-k has a variant whose scratch is an array compiled into the library.
This test calls it through the C ABI and checks its outputs against the regular entry point
(which takes a caller workspace) on two calls in a row with different inputs, so leftover
scratch contents from the first call cannot leak into the second. Tolerances are those of
the router tests: indices exact, weights 2e-3, probs_mean 2e-3, z-loss 1e-6.

The file name sorts last so that a run stopping at the first failure has run every other
test first; it also passes alone in a fresh process.
"""

from __future__ import annotations

import pytest
import torch

from conftest import assert_close

pytestmark = pytest.mark.gpu


def _call(lib, name, logits, bias, K, zw, with_ws):
    N, E = logits.shape
    dev = logits.device
    idx = torch.empty(N, K, dtype=torch.int64, device=dev)
    w = torch.empty(N, K, dtype=torch.bfloat16, device=dev)
    z = torch.zeros((), dtype=torch.float32, device=dev)
    pm = torch.zeros(E, dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    is_bf16 = 1 if logits.dtype == torch.bfloat16 else 0
    if with_ws:
        ws = torch.empty(max(1, N * (E + 1)), dtype=torch.float32, device=dev)
        st = getattr(lib, name)(logits.data_ptr(), is_bf16, bias.data_ptr(), N, E, K, zw, idx.data_ptr(),
                                w.data_ptr(), z.data_ptr(), pm.data_ptr(), ws.data_ptr(), stream)
    else:
        st = getattr(lib, name)(logits.data_ptr(), is_bf16, bias.data_ptr(), N, E, K, zw, idx.data_ptr(),
                                w.data_ptr(), z.data_ptr(), pm.data_ptr(), stream)
    return st, idx, w, z, pm


def test_noalloc_router_matches_workspace_router_twice():
    if not torch.cuda.is_available():
        pytest.skip("CUDA not available")
    from pulsar_b200 import _lib
    lib = _lib.load()
    g = torch.Generator(device="cpu").manual_seed(5)
    cases = [(torch.randn(3000, 16, generator=g).cuda(), 4), (torch.randn(777, 16, generator=g).bfloat16().cuda(), 4)]
    for logits, K in cases:           # two calls in a row, different sizes and dtypes
        bias = (torch.randn(16, generator=g) * 0.1).cuda()
        st_a, idx_a, w_a, z_a, pm_a = _call(lib, "pulsar_op_moe_router_topk", logits, bias, K, 1e-4, True)
        st_b, idx_b, w_b, z_b, pm_b = _call(lib, "pulsar_op_moe_router_topk_noalloc", logits, bias, K, 1e-4, False)
        torch.cuda.synchronize()
        assert st_a == 0 and st_b == 0, _lib.last_error()
        assert torch.equal(idx_a, idx_b)
        assert_close(w_b, w_a, atol=2e-3, msg="weights")
        assert_close(pm_b, pm_a, atol=2e-3, msg="probs_mean")
        assert_close(z_b, z_a, atol=1e-6, rtol=1e-4, msg="z_loss")


def test_noalloc_router_rejects_oversized_input():
    if not torch.cuda.is_available():
        pytest.skip("CUDA not available")
    from pulsar_b200 import _lib
    lib = _lib.load()
    logits = torch.zeros(70000, 16, device="cuda")
    bias = torch.zeros(16, device="cuda")
    st, *_ = _call(lib, "pulsar_op_moe_router_topk_noalloc", logits, bias, 4, 0.0, False)
    assert st == -6
    assert "exceeds the built-in scratch" in _lib.last_error()
