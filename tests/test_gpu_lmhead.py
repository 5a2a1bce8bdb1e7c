"""GPU parity of the f16 LM head behind the final RMSNorm (obn_lm_head_f16).

Every logit must equal the oracle's restatement of f32_matmul.wgsl bit for bit
(256 lane partials over d-pairs + the shader's halving tree, f32) after the
rmsnorm.wgsl final norm: small ragged tables, several token counts (one, two
and four tokens per pass, and a count that takes two passes), no norm, tiny dim,
and the full BitNet-2B table (128256 x 2560) for the reference's single token.
"""
import numpy as np
import pytest

import oracle as orc
from _util import need_cuda, obn

pytestmark = pytest.mark.gpu


def run(torch, V, D, n, norm, seed):
    rng = np.random.default_rng(seed)
    embed = (rng.standard_normal((V, D)) * 0.05).astype(np.float16)
    x = rng.standard_normal((n, D)).astype(np.float32)
    g = (1 + 0.1 * rng.standard_normal(D)).astype(np.float32) if norm else None
    got = obn().lm_head_f16(torch.from_numpy(embed).cuda(), torch.from_numpy(x).cuda(),
                            None if g is None else torch.from_numpy(g).cuda(), 1e-5)
    want = orc.lm_head_f16(x, embed, g, 1e-5)
    return got.cpu().numpy(), want


@pytest.mark.parametrize("V,D,n,norm", [(1000, 2560, 1, True), (777, 2560, 2, True),
                                        (513, 1024, 3, False), (300, 8, 1, True),
                                        (129, 3072, 4, True), (64, 2048, 6, True),
                                        (1001, 520, 1, False)])
def test_lm_head_bitexact(V, D, n, norm):
    torch = need_cuda()
    got, want = run(torch, V, D, n, norm, V + D + n)
    assert np.array_equal(got, want)


def test_lm_head_full_table_single_token():
    torch = need_cuda()
    got, want = run(torch, 128256, 2560, 1, True, 7)
    assert np.array_equal(got, want)
    obn().check_device_errors()


def test_lm_head_rejects_bad_dims():
    torch = need_cuda()
    E = obn()._lib
    with pytest.raises(E.ObnError) as ei:
        obn().lm_head_f16(torch.zeros((4, 12), dtype=torch.float16, device="cuda"),
                          torch.zeros((1, 12), device="cuda"))
    assert ei.value.code == E.OBN_ERR_UNSUPPORTED


@pytest.mark.parametrize("V,D,n", [(1000, 2560, 8), (1000, 2560, 64), (777, 512, 100),
                                   (1001, 512, 3), (300, 2560, 130), (128256, 2560, 64)])
def test_lm_head_batched_tensor_cores(V, D, n):
    # the tensor-core form: the same logits to f32 rounding (hi/lo f16 split of the
    # normed hidden rows, tensor-core summation order), checked against the exact
    # dot products of the oracle's normed rows
    torch = need_cuda()
    rng = np.random.default_rng(V + D + n)
    embed = (rng.standard_normal((V, D)) * 0.05).astype(np.float16)
    x = rng.standard_normal((n, D)).astype(np.float32)
    g = (1 + 0.1 * rng.standard_normal(D)).astype(np.float32)
    got = obn().lm_head_f16_batched(torch.from_numpy(embed).cuda(), torch.from_numpy(x).cuda(),
                                    torch.from_numpy(g).cuda(), 1e-5).cpu().numpy()
    y = orc.rmsnorm(x, g, 1e-5).astype(np.float64)
    e64 = embed.astype(np.float64)
    exact = y @ e64.T
    l1 = np.abs(y) @ np.abs(e64).T
    assert np.all(np.abs(got - exact) <= 2e-6 * l1 + 1e-7)
    obn().check_device_errors()
