"""GPU checks of the decode attention kernels against the oracle.

RoPE + fp16 KV append against rope.wgsl's formula (q exact to the math
library's last bits; the caches equal the binary16 rounding of the rotated k and
of v), and the split-KV GQA attention against attention.wgsl + softmax.wgsl on
the same fp16 cache contents: decode (one token, up to 2048 keys, several
sequences), chunked prefill with the causal mask, and group sizes 1, 4 and 8.
The tolerance (1e-4 relative, 1e-5 absolute) covers the math library's exp and
the different summation order of the online softmax.
"""
import numpy as np
import pytest

import oracle as orc
from _util import need_cuda

pytestmark = pytest.mark.gpu


def att():
    import importlib
    return importlib.import_module("0xbitnet_b200.attention")


D = 128


@pytest.mark.parametrize("B,n,H,Hkv,pos", [(2, 3, 20, 5, 100), (1, 1, 8, 8, 0), (3, 1, 16, 2, 2000),
                                            # >= one row per SM: one CTA per row, angles shared
                                            (1, 300, 20, 5, 100), (2, 160, 16, 2, 1500)])
def test_rope_kv_append(B, n, H, Hkv, pos):
    torch = need_cuda()
    S_max = pos + n + 5
    rng = np.random.default_rng(B * 100 + n + pos)
    qkv = rng.standard_normal((B * n, (H + 2 * Hkv) * D)).astype(np.float32)
    cache = att().KVCache(B, S_max, Hkv, D)
    cache.seq_len = pos
    q = att().rope_kv_append(torch.from_numpy(qkv).cuda(), cache, H, n, 500000.0)
    q = q.cpu().numpy()
    kc, vc = cache.k.cpu().numpy(), cache.v.cpu().numpy()
    # theta = pos * base^(-2i/D): pow's last bit, scaled by the largest position
    tol = 1e-5 if pos + n < 200 else 1e-3
    for b in range(B):
        rows = qkv[b * n:(b + 1) * n]
        qr = orc.rope(rows[:, :H * D], H, D, pos, 500000.0)
        kr = orc.rope(rows[:, H * D:(H + Hkv) * D], Hkv, D, pos, 500000.0)
        np.testing.assert_allclose(q[b * n:(b + 1) * n], qr, atol=tol, rtol=0)
        got_k = kc[b, pos:pos + n].reshape(n, Hkv * D).astype(np.float32)
        np.testing.assert_allclose(got_k, kr.astype(np.float16).astype(np.float32),
                                   atol=tol, rtol=2e-3)
        got_v = vc[b, pos:pos + n].reshape(n, Hkv * D)
        assert np.array_equal(got_v, rows[:, (H + Hkv) * D:].astype(np.float16))


@pytest.mark.parametrize("B,n,H,Hkv,S", [(1, 1, 20, 5, 1), (1, 1, 20, 5, 2048), (3, 1, 20, 5, 700),
                                         (2, 5, 20, 5, 300), (1, 7, 8, 8, 7), (2, 1, 16, 2, 129),
                                         (1, 130, 4, 1, 260), (1, 1, 20, 5, 5000),
                                         (1, 1, 16, 8, 4096), (2, 1, 4, 4, 33),
                                         # >= 4 work items per SM: the pipelined split pass
                                         # (decode at the bench's batch, a ragged last chunk,
                                         # causal prefill with empty items, G = 8 and G = 1)
                                         (64, 1, 20, 5, 2048), (8, 1, 20, 5, 1900),
                                         (1, 300, 20, 5, 600), (20, 1, 32, 4, 1100),
                                         (3, 40, 8, 8, 2000),
                                         # >= 16 new rows: the 16-row prefill tile pass, G = 1, 2,
                                         # 4, 8, ragged last tiles, an empty cache (S = n)
                                         (2, 33, 16, 8, 100), (1, 64, 32, 4, 64),
                                         (2, 17, 20, 5, 17), (1, 512, 20, 5, 512)])
def test_attention_matches_oracle(B, n, H, Hkv, S):
    torch = need_cuda()
    S_max = S + 3
    rng = np.random.default_rng(B + n + H + S)
    cache = att().KVCache(B, S_max, Hkv, D)
    k = rng.standard_normal((B, S_max, Hkv, D)).astype(np.float16)
    v = rng.standard_normal((B, S_max, Hkv, D)).astype(np.float16)
    cache.k.copy_(torch.from_numpy(k))
    cache.v.copy_(torch.from_numpy(v))
    q = rng.standard_normal((B * n, H * D)).astype(np.float32)
    out = att().attention(torch.from_numpy(q).cuda(), cache, H, n, S).cpu().numpy()
    for b in range(B):
        want = orc.attention(q[b * n:(b + 1) * n], k[b, :S].reshape(S, Hkv * D).astype(np.float32),
                             v[b, :S].reshape(S, Hkv * D).astype(np.float32), H, Hkv, D)
        np.testing.assert_allclose(out[b * n:(b + 1) * n], want, rtol=1e-4, atol=1e-5)


def test_attention_decode_step_end_to_end():
    # qkv of one new token -> rope + append -> attention, against the oracle on the
    # same rounded cache
    torch = need_cuda()
    B, H, Hkv, S_prev = 2, 20, 5, 500
    S_max = 1024
    rng = np.random.default_rng(9)
    cache = att().KVCache(B, S_max, Hkv, D)
    k = rng.standard_normal((B, S_max, Hkv, D)).astype(np.float16)
    v = rng.standard_normal((B, S_max, Hkv, D)).astype(np.float16)
    cache.k.copy_(torch.from_numpy(k))
    cache.v.copy_(torch.from_numpy(v))
    cache.seq_len = S_prev
    qkv = rng.standard_normal((B, (H + 2 * Hkv) * D)).astype(np.float32)
    q = att().rope_kv_append(torch.from_numpy(qkv).cuda(), cache, H, 1)
    out = att().attention(q, cache, H, 1, S_prev + 1).cpu().numpy()
    kc, vc = cache.k.cpu().numpy(), cache.v.cpu().numpy()
    qn = q.cpu().numpy()
    for b in range(B):
        S = S_prev + 1
        want = orc.attention(qn[b:b + 1], kc[b, :S].reshape(S, -1).astype(np.float32),
                             vc[b, :S].reshape(S, -1).astype(np.float32), H, Hkv, D)
        np.testing.assert_allclose(out[b:b + 1], want, rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("B,H,Hkv,S_prev", [(1, 20, 5, 2047), (3, 20, 5, 127), (2, 16, 2, 128),
                                             (1, 8, 8, 0), (2, 32, 4, 300), (1, 20, 5, 1),
                                             (1, 20, 5, 4100), (1, 20, 5, 9000), (8, 20, 5, 300),
                                             # RoPE split pass against the pipelined one
                                             (64, 20, 5, 2047), (8, 20, 5, 1900)])
def test_fused_rope_attention_is_bit_identical(B, H, Hkv, S_prev):
    """obn_attention_decode_rope == obn_rope_kv_append + obn_attention_decode (n = 1):
    same output bits, same cache contents."""
    torch = need_cuda()
    S_max = S_prev + 9
    rng = np.random.default_rng(B * 7 + H + S_prev)
    k = torch.from_numpy(rng.standard_normal((B, S_max, Hkv, D)).astype(np.float16))
    v = torch.from_numpy(rng.standard_normal((B, S_max, Hkv, D)).astype(np.float16))
    qkv = torch.from_numpy(rng.standard_normal((B, (H + 2 * Hkv) * D)).astype(np.float32)).cuda()
    c1, c2 = att().KVCache(B, S_max, Hkv, D), att().KVCache(B, S_max, Hkv, D)
    for c in (c1, c2):
        c.k.copy_(k)
        c.v.copy_(v)
        c.seq_len = S_prev
    q = att().rope_kv_append(qkv, c1, H, 1, pos=S_prev)
    want = att().attention(q, c1, H, 1, S_prev + 1).cpu()
    got = att().attention_rope(qkv, c2, H, S_prev).cpu()
    torch.cuda.synchronize()
    assert torch.equal(got, want)
    assert torch.equal(c1.k.cpu(), c2.k.cpu()) and torch.equal(c1.v.cpu(), c2.v.cpu())


def _rope_at(qkv, cache, H, pos_dev, out, ws):
    import ctypes
    import torch
    from importlib import import_module
    L = import_module("0xbitnet_b200._lib")
    p = lambda t: ctypes.c_void_p(t.data_ptr())
    L.check(L.lib().obn_attention_decode_rope_at(
        p(qkv), p(cache.k), p(cache.v), cache.B, H, cache.Hkv, D, cache.S_max, p(pos_dev),
        ctypes.c_float(500000.0), ctypes.c_float(float(np.float32(1.0) / np.sqrt(np.float32(D)))),
        p(out), p(ws),
        ctypes.c_size_t(ws.numel()), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)))


@pytest.mark.parametrize("B,H,Hkv,S_max,pos", [(1, 20, 5, 4096, 1000), (1, 20, 5, 4096, 2500),
                                               (2, 32, 4, 2048, 2047), (1, 20, 5, 4096, 4096),
                                               (1, 8, 8, 20000, 130),
                                               # many sequences: the RoPE split pass against
                                               # RoPE append + the persistent pass (and a full cache)
                                               (64, 20, 5, 2048, 1500), (32, 20, 5, 2048, 2048)])
def test_rope_attention_device_position(B, H, Hkv, S_max, pos):
    """The _at form (position read on the device, chunks sized for S_max) equals
    RoPE append + attention at the host position, bit for bit; a position at
    S_max appends nothing and attends over the whole cache."""
    torch = need_cuda()
    rng = np.random.default_rng(S_max + pos)
    k = torch.from_numpy(rng.standard_normal((B, S_max, Hkv, D)).astype(np.float16))
    v = torch.from_numpy(rng.standard_normal((B, S_max, Hkv, D)).astype(np.float16))
    qkv = torch.from_numpy(rng.standard_normal((B, (H + 2 * Hkv) * D)).astype(np.float32)).cuda()
    c1, c2 = att().KVCache(B, S_max, Hkv, D), att().KVCache(B, S_max, Hkv, D)
    for c in (c1, c2):
        c.k.copy_(k)
        c.v.copy_(v)
    if pos < S_max:
        q = att().rope_kv_append(qkv, c1, H, 1, 500000.0, pos=pos)
        want = att().attention(q, c1, H, 1, pos + 1).cpu()
    else:  # a full cache: q rotated at pos (scratch cache one row longer) over all S_max keys
        scratch = att().KVCache(B, S_max + 1, Hkv, D)
        q = att().rope_kv_append(qkv, scratch, H, 1, 500000.0, pos=pos)
        want = att().attention(q, c1, H, 1, S_max).cpu()
    from importlib import import_module
    L = import_module("0xbitnet_b200._lib")
    ws = torch.empty(int(L.lib().obn_attention_workspace_bytes(B, 1, H, D, S_max)),
                     dtype=torch.uint8, device="cuda")
    out = torch.empty((B, H * D), dtype=torch.float32, device="cuda")
    pos_dev = torch.tensor([pos], dtype=torch.int32, device="cuda")
    _rope_at(qkv, c2, H, pos_dev, out, ws)
    torch.cuda.synchronize()
    assert torch.equal(out.cpu(), want)
    assert torch.equal(c1.k.cpu(), c2.k.cpu()) and torch.equal(c1.v.cpu(), c2.v.cpu())


@pytest.mark.parametrize("B", [2, 64])
def test_rope_attention_back_to_back_steps(B):
    """Consecutive decode steps on one cache, enqueued with no host sync between
    them (each reads the row the step before appended), equal the same steps run
    one at a time through RoPE append + attention (B = 2: the clustered pass;
    B = 64: the RoPE split pass, against the persistent one)."""
    torch = need_cuda()
    H, Hkv, S_max, pos0, steps = 20, 5, 2048, 1020, 12
    rng = np.random.default_rng(77)
    k = torch.from_numpy(rng.standard_normal((B, S_max, Hkv, D)).astype(np.float16))
    v = torch.from_numpy(rng.standard_normal((B, S_max, Hkv, D)).astype(np.float16))
    qkvs = [torch.from_numpy(rng.standard_normal((B, (H + 2 * Hkv) * D)).astype(np.float32)).cuda()
            for _ in range(steps)]
    c1, c2 = att().KVCache(B, S_max, Hkv, D), att().KVCache(B, S_max, Hkv, D)
    for c in (c1, c2):
        c.k.copy_(k)
        c.v.copy_(v)
    want = []
    for i in range(steps):
        q = att().rope_kv_append(qkvs[i], c1, H, 1, pos=pos0 + i)
        want.append(att().attention(q, c1, H, 1, pos0 + i + 1).cpu())
        torch.cuda.synchronize()
    outs = [torch.empty((B, H * D), dtype=torch.float32, device="cuda") for _ in range(steps)]
    for i in range(steps):
        att().attention_rope(qkvs[i], c2, H, pos0 + i, out=outs[i])
    torch.cuda.synchronize()
    for i in range(steps):
        assert torch.equal(outs[i].cpu(), want[i]), i
    assert torch.equal(c1.k.cpu(), c2.k.cpu()) and torch.equal(c1.v.cpu(), c2.v.cpu())
