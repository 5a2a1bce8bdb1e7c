"""A BitNet decoder step on libobn against the oracle composition.

Per layer: embedding, merged QKV BitLinear with the block RMSNorm fused, RoPE +
KV append, attention, o_proj with its sub-norm, residual add, gated gate|up with
ReLU^2, down with its sub-norm, residual add; then the final RMSNorm + tied f16
LM head (model.rs:193-266; one block is transformer.rs:51-75). The oracle runs
the reference's sequence of shader restatements on the same weights and caches:
the weights are the seeded I2_S rows the decoder generated, taken before the
device repack (never read back from the device), and the caches are the
device's fp16 caches. Logits must agree within BASELINE's end-to-end 2e-2.

Two sizes:
* a small model (2 layers, hidden 512, FFN 1024, vocab 1000, context 64), eager;
* the config-3 dimensions the decode benchmark runs (hidden 2560, FFN 6912, 20/5
  heads x 128, vocab 128256, context 2048, position 2047), 2 layers, at B = 1 and
  B = 64, through a captured CUDA graph as the benchmark replays it.
"""
import numpy as np
import pytest

import oracle as orc
from _util import need_cuda

pytestmark = pytest.mark.gpu


def dec():
    import importlib
    return importlib.import_module("0xbitnet_b200.decoder")


def oracle_logits(m, ids, caches, pos, stages=None):
    """The reference forward for one new token per sequence at position `pos`.
    `stages` (a dict), when given, receives the arrays of the reference's
    diagnose() stages (model.ts:449-531)."""
    cfg, B = m.cfg, len(ids)
    H, Hkv, d, D, F = cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.hidden, cfg.ffn
    emb = m.embed.cpu().numpy()
    x = emb[ids].astype(np.float32)
    if stages is not None:
        stages["embedding"] = x.copy()
    for li, (L, (kc, vc)) in enumerate(zip(m.layers, caches)):
        src = L.source
        sw = np.concatenate([np.full(n_, s_, np.float32) for n_, s_ in
                             zip((H * d, Hkv * d, Hkv * d), L.qkv_scales)])
        qkv = orc.bitlinear_omp(x, src["qkv"], sw, (H + 2 * Hkv) * d, D,
                                norm_w=L.attn_norm.cpu().numpy(), eps=cfg.eps)
        # every sequence's new token sits at position pos (rows are sequences)
        q = np.concatenate([orc.rope(qkv[b:b + 1, :H * d], H, d, pos, cfg.rope_theta)
                            for b in range(B)])
        k = np.concatenate([orc.rope(qkv[b:b + 1, H * d:(H + Hkv) * d], Hkv, d, pos,
                                     cfg.rope_theta) for b in range(B)])
        v = qkv[:, (H + Hkv) * d:]
        a = np.empty((B, H * d), np.float32)
        for b in range(B):
            K = kc[b, :pos + 1].reshape(pos + 1, Hkv * d).astype(np.float32)
            V = vc[b, :pos + 1].reshape(pos + 1, Hkv * d).astype(np.float32)
            K[pos] = k[b].astype(np.float16).astype(np.float32)
            V[pos] = v[b].astype(np.float16).astype(np.float32)
            a[b] = orc.attention(q[b:b + 1], K, V, H, Hkv, d)[0]
        o = orc.bitlinear_omp(a, src["o"], np.full(D, L.o_scale, np.float32), D, H * d,
                              norm_w=L.attn_sub_norm.cpu().numpy(), eps=cfg.eps)
        x = (x + o).astype(np.float32)
        fn = L.ffn_norm.cpu().numpy()
        gt = orc.bitlinear_omp(x, src["gate"], np.full(F, L.gate_scale, np.float32), F, D,
                               norm_w=fn, eps=cfg.eps)
        up = orc.bitlinear_omp(x, src["up"], np.full(F, L.up_scale, np.float32), F, D,
                               norm_w=fn, eps=cfg.eps)
        act = orc.relu2_mul(gt, up)
        dn = orc.bitlinear_omp(act, src["down"], np.full(D, L.down_scale, np.float32), D, F,
                               norm_w=L.ffn_sub_norm.cpu().numpy(), eps=cfg.eps)
        x = (x + dn).astype(np.float32)
        if stages is not None and li < 2:
            stages[f"layer_{li}"] = x.copy()
    logits = orc.lm_head_f16(x, emb, m.final_norm.cpu().numpy(), cfg.eps)
    if stages is not None:
        normed = orc.rmsnorm(x, m.final_norm.cpu().numpy(), cfg.eps)
        stages.update(last_layer=x.copy(), final_norm=normed, lm_input=normed,
                      logits_first100=logits[0, :100])
    return logits


def host_caches(m, pos):
    # positions < pos as they are before the step (the step writes position pos)
    return [(c.k[:, :pos + 1].cpu().numpy(), c.v[:, :pos + 1].cpu().numpy()) for c in m.caches]


@pytest.mark.parametrize("B", [1, 2, 6])
def test_decoder_step_matches_oracle(B):
    # B = 1: the shader-order LM head; B = 2, 6: the tensor-core one
    torch = need_cuda()
    D_ = dec()
    cfg = D_.DecoderConfig(layers=2, hidden=512, ffn=1024, heads=4, kv_heads=2, vocab=1000)
    ctx, pos = 64, 10
    ids = [7, 999, 0, 5, 500, 123][:B]
    m = D_.BitNetDecoder(cfg, B, ctx, seed=3, keep_source=True)
    m.fill_caches(pos, seed=4)
    m.ids.copy_(torch.tensor(ids, dtype=torch.int32))
    caches = host_caches(m, pos)
    logits = m.step(pos).cpu().numpy()
    torch.cuda.synchronize()
    err = np.abs(logits - oracle_logits(m, ids, caches, pos)).max()
    assert err <= 2e-2, err
    m.close()


@pytest.mark.parametrize("B", [1, 64])
def test_decoder_config3_dims_graph_matches_oracle(B):
    # the benchmarked model's dimensions, 2 of its 30 layers, last cache position
    torch = need_cuda()
    D_ = dec()
    cfg = D_.DecoderConfig(layers=2)  # 2560 / 6912, 20 / 5 heads x 128, vocab 128256
    ctx = 2048
    pos = ctx - 1
    m = D_.BitNetDecoder(cfg, B, ctx, seed=90 + B, keep_source=True)
    m.fill_caches(pos, seed=91 + B)
    ids = [int(i) for i in np.random.default_rng(B).integers(0, cfg.vocab, B)]
    m.ids.copy_(torch.tensor(ids, dtype=torch.int32))
    caches = host_caches(m, pos)
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        m.step(pos)  # eager warm-up (workspaces); rewrites position pos identically
        stream.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            out = m.step(pos)
        out.fill_(float("nan"))
        g.replay()
        stream.synchronize()
    logits = out.cpu().numpy()
    del g
    want = oracle_logits(m, ids, caches, pos)
    assert np.isfinite(logits).all()
    err = np.abs(logits - want).max()
    assert err <= 2e-2, err
    m.close()


def test_decoder_diagnose_stages_match_oracle():
    """BitNetDecoder.diagnose (the reference's diagnose() stages and statistics)
    against the same stages of the oracle composition; a fault planted in one
    oracle stage's statistics is reported at that stage."""
    import importlib
    torch = need_cuda()
    D_ = dec()
    dg = importlib.import_module("0xbitnet_b200.diagnose")
    cfg = D_.DecoderConfig(layers=3, hidden=512, ffn=1024, heads=4, kv_heads=2, vocab=1000)
    ctx, pos, ids = 64, 10, [3, 777]
    m = D_.BitNetDecoder(cfg, len(ids), ctx, seed=5, keep_source=True)
    m.fill_caches(pos, seed=6)
    m.ids.copy_(torch.tensor(ids, dtype=torch.int32))
    caches = host_caches(m, pos)
    got = m.diagnose(pos)
    stages = {}
    oracle_logits(m, ids, caches, pos, stages=stages)
    want = [dg.stage_stats(n, stages[n]) for n in dg.STAGES]
    assert [s["name"] for s in got] == list(dg.STAGES)
    assert all(s["nan_count"] == 0 and s["inf_count"] == 0 for s in got)
    msg = dg.format_stats(got) + "\n-- oracle --\n" + dg.format_stats(want)
    assert dg.first_divergence(got, want, rtol=1e-2, atol=1e-3) is None, msg
    bad = [dict(s) for s in want]
    bad[2]["rms"] *= 1.1  # layer_1
    assert dg.first_divergence(got, bad, rtol=1e-2, atol=1e-3) == "layer_1"
    m.close()
