"""A small BitNet decoder step on libobn against the oracle composition.

Two layers (hidden 512 = 4 heads x 128, 2 KV heads, FFN 1024, vocab 1000), two
sequences, position 10 of 64 with random fp16 caches: embedding, merged QKV
BitLinear with the block RMSNorm fused, RoPE + KV append, attention, o_proj
with its sub-norm, residual add, gated gate|up with ReLU^2, down with its
sub-norm, residual add, final RMSNorm + tied f16 LM head. The oracle runs the
reference's sequence of shader restatements on the same weights and caches;
the logits must agree within BASELINE's end-to-end 2e-2 (in practice much
closer), and the residual adds and embedding exactly.
"""
import numpy as np
import pytest

import oracle as orc
from _util import need_cuda

pytestmark = pytest.mark.gpu


def dec():
    import importlib
    return importlib.import_module("0xbitnet_b200.decoder")


@pytest.mark.parametrize("B", [2, 6])
def test_decoder_step_matches_oracle(B):
    # B = 2: the shader-order LM head; B = 6: the tensor-core one
    torch = need_cuda()
    D_ = dec()
    cfg = D_.DecoderConfig(layers=2, hidden=512, ffn=1024, heads=4, kv_heads=2, vocab=1000)
    ctx, pos = 64, 10
    ids = [7, 999, 0, 5, 500, 123][:B]
    m = D_.BitNetDecoder(cfg, B, ctx, seed=3)
    m.fill_caches(pos, seed=4)
    m.ids.copy_(torch.tensor(ids, dtype=torch.int32))
    caches = [(c.k.cpu().numpy().astype(np.float32), c.v.cpu().numpy().astype(np.float32))
              for c in m.caches]
    logits = m.step(pos).cpu().numpy()
    torch.cuda.synchronize()

    H, Hkv, d, D, F = cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.hidden, cfg.ffn
    emb = m.embed.cpu().numpy()
    x = emb[ids].astype(np.float32)
    for L, (kc, vc) in zip(m.layers, caches):
        rows = L.qkv.export_i2s().cpu().numpy()
        sw = np.concatenate([np.full(n_, s_, np.float32) for n_, s_ in
                             zip((H * d, Hkv * d, Hkv * d), L.qkv_scales)])
        qkv, _, _ = orc.bitlinear(x, rows, sw, rows.shape[0], D,
                                  norm_w=L.attn_norm.cpu().numpy())
        # every sequence's new token sits at position pos (rows are sequences)
        q = np.concatenate([orc.rope(qkv[b:b + 1, :H * d], H, d, pos, cfg.rope_theta)
                            for b in range(B)])
        k = np.concatenate([orc.rope(qkv[b:b + 1, H * d:(H + Hkv) * d], Hkv, d, pos,
                                     cfg.rope_theta) for b in range(B)])
        v = qkv[:, (H + Hkv) * d:]
        a = np.empty((B, H * d), np.float32)
        for b in range(B):
            K = kc[b, :pos + 1].reshape(pos + 1, Hkv * d).copy()
            V = vc[b, :pos + 1].reshape(pos + 1, Hkv * d).copy()
            K[pos] = k[b].astype(np.float16).astype(np.float32)
            V[pos] = v[b].astype(np.float16).astype(np.float32)
            a[b] = orc.attention(q[b:b + 1], K, V, H, Hkv, d)[0]
        o_rows = L.o.export_i2s().cpu().numpy()
        o, _, _ = orc.bitlinear(a, o_rows, np.full(D, L.o_scale, np.float32), D, H * d,
                                norm_w=L.attn_sub_norm.cpu().numpy())
        x = (x + o).astype(np.float32)
        gu_rows = L.gate_up.export_i2s().cpu().numpy()
        fn = L.ffn_norm.cpu().numpy()
        gt, _, _ = orc.bitlinear(x, gu_rows[0::2], np.full(F, L.gate_scale, np.float32), F, D,
                                 norm_w=fn)
        up, _, _ = orc.bitlinear(x, gu_rows[1::2], np.full(F, L.up_scale, np.float32), F, D,
                                 norm_w=fn)
        act = orc.relu2_mul(gt, up)
        dn_rows = L.down.export_i2s().cpu().numpy()
        dn, _, _ = orc.bitlinear(act, dn_rows, np.full(D, L.down_scale, np.float32), D, F,
                                 norm_w=L.ffn_sub_norm.cpu().numpy())
        x = (x + dn).astype(np.float32)
    want = orc.lm_head_f16(x, emb, m.final_norm.cpu().numpy(), cfg.eps)
    err = np.abs(logits - want).max()
    assert err <= 2e-2, err
    m.close()
