"""The allocation-free BitLinear forward against the regular one.

obn_bitlinear_forward_noalloc serves callers that cannot allocate device memory
(their device memory is reserved up front by another allocator, or they run on
latency-critical threads that must not call cudaMalloc/cudaFree): it takes no
workspace and keeps its scratch in one fixed device array inside the library.
This file checks, through the C ABI, that two calls in a row give outputs
identical to obn_bitlinear_forward's on every matmul that reads quantized
activations from the scratch: the warp-MMA decode kernel (3 and 8 tokens), the
split-K tensor-core GEMM (64 tokens), and a gated gate|up layer on the warp-MMA
path (3 and 8 tokens: the epilogue forms act(gate) * up). It also checks that
sizes beyond the fixed array are refused with a clear error.

The file name sorts last so a run that stops at the first failure has already
run every other test.
"""
import ctypes

import numpy as np
import pytest

from _util import need_cuda, obn, synth

pytestmark = pytest.mark.gpu


def _noalloc(torch, layer, x, n):
    y = torch.empty((n, layer.out_dim), dtype=torch.float32, device=x.device)
    rc = obn().lib().obn_bitlinear_forward_noalloc(
        layer.handle, ctypes.c_void_p(x.data_ptr()), n, ctypes.c_void_p(y.data_ptr()),
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0, obn()._lib.last_error()
    return y


def _check_two_calls(torch, layer, K, n, seed):
    xs = [torch.from_numpy(synth().activations(seed + i, n, K)).cuda() for i in range(2)]
    want = [layer.forward(x).cpu().numpy() for x in xs]
    got = [_noalloc(torch, layer, x, n).cpu().numpy() for x in xs]  # two calls in a row
    torch.cuda.synchronize()
    for g, w in zip(got, want):
        assert np.array_equal(g, w)  # the same kernels on the same data: bit-identical
    assert not np.array_equal(got[0], got[1])  # the second call did not reuse stale results
    obn().check_device_errors()


@pytest.mark.parametrize("M,K,n", [(2560, 2560, 3), (2560, 2560, 8), (6912, 2560, 64)])
def test_noalloc_matches_forward_on_two_calls(M, K, n):
    torch = need_cuda()
    L = synth().layer(4242 + n, M, K)
    layer = obn().BitLinear.from_i2s(L.blob(), K, M, norm_weight=L.gamma)
    _check_two_calls(torch, layer, K, n, 4300 + n)
    layer.close()


@pytest.mark.parametrize("n", [3, 8])
def test_noalloc_gated_matches_forward_on_two_calls(n):
    torch = need_cuda()
    M, K = 6912, 2560
    g = synth().layer(5100 + n, M, K)
    u = synth().layer(5200 + n, M, K)
    layer = obn().BitLinear.from_i2s_gated(g.blob(), u.blob(), K, M, norm_weight=g.gamma)
    _check_two_calls(torch, layer, K, n, 5300 + n)
    layer.close()


def _refused(torch, layer, n):
    x = torch.zeros((n, layer.in_dim), device="cuda")
    y = torch.empty((n, layer.out_dim), device="cuda")
    rc = obn().lib().obn_bitlinear_forward_noalloc(layer.handle, ctypes.c_void_p(x.data_ptr()), n,
                                                   ctypes.c_void_p(y.data_ptr()), None)
    assert rc == obn()._lib.OBN_ERR_UNSUPPORTED
    assert b"fixed scratch" in obn().lib().obn_error_message()


def test_noalloc_rejects_activations_beyond_its_scratch():
    torch = need_cuda()
    K = 6912
    L = synth().layer(5, 256, K)
    layer = obn().BitLinear.from_i2s(L.blob(), K, 256)
    _refused(torch, layer, (1 << 20) // K + 1)  # one token more than the array holds
    layer.close()
