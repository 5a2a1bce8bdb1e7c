"""The allocation-free BitLinear forward against the regular one.

obn_bitlinear_forward_noalloc serves callers that cannot allocate device memory
(their device memory is reserved up front by another allocator, or they run on
latency-critical threads that must not call cudaMalloc/cudaFree): it takes no
workspace and keeps its scratch in one fixed device array inside the library.
This file checks, through the C ABI, that two calls in a row give the same
outputs as obn_bitlinear_forward (within the suite's 1e-5 relative tolerance),
on both matmul paths that use scratch (dp4a for 8 tokens, tcgen05 for 64), and
that sizes beyond the fixed array are refused with a clear error.

The file name sorts last so a run that stops at the first failure has already
run every other test.
"""
import ctypes

import numpy as np
import pytest

from _util import need_cuda, obn, synth

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-5, 1e-6


def _noalloc(torch, layer, x, n):
    y = torch.empty((n, layer.out_dim), dtype=torch.float32, device=x.device)
    rc = obn().lib().obn_bitlinear_forward_noalloc(
        layer.handle, ctypes.c_void_p(x.data_ptr()), n, ctypes.c_void_p(y.data_ptr()),
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0, obn()._lib.last_error()
    return y


@pytest.mark.parametrize("M,K,n", [(2560, 2560, 8), (6912, 2560, 64)])
def test_noalloc_matches_forward_on_two_calls(M, K, n):
    torch = need_cuda()
    L = synth().layer(4242 + n, M, K)
    layer = obn().BitLinear.from_i2s(L.blob(), K, M, norm_weight=L.gamma)
    xs = [torch.from_numpy(synth().activations(4300 + n + i, n, K)).cuda() for i in range(2)]
    want = [layer.forward(x).cpu().numpy() for x in xs]
    got = [_noalloc(torch, layer, x, n).cpu().numpy() for x in xs]  # two calls in a row
    torch.cuda.synchronize()
    for g, w in zip(got, want):
        np.testing.assert_allclose(g, w, rtol=RTOL, atol=ATOL)
    assert not np.array_equal(got[0], got[1])  # the second call did not reuse stale results
    obn().check_device_errors()


def test_noalloc_rejects_sizes_beyond_its_scratch():
    torch = need_cuda()
    K = 6912
    L = synth().layer(5, 256, K)
    layer = obn().BitLinear.from_i2s(L.blob(), K, 256)
    n = (1 << 20) // K + 1  # one token more than the fixed scratch holds
    x = torch.zeros((n, K), device="cuda")
    y = torch.empty((n, 256), device="cuda")
    rc = obn().lib().obn_bitlinear_forward_noalloc(layer.handle, ctypes.c_void_p(x.data_ptr()), n,
                                                   ctypes.c_void_p(y.data_ptr()), None)
    assert rc == obn()._lib.OBN_ERR_UNSUPPORTED
    assert b"fixed scratch" in obn().lib().obn_error_message()
