"""The model-level ABI (include/oxbitnet.h) on a GPU against the oracle model.

Small random BitNet models are written as GGUF files (gguf_writer), loaded
through oxbitnet_load, and run through prefill (the reference's n > 1 pass
over the whole prompt) and one-token decode steps; the logits of every step
must match the oracle composition of the reference's forward (oracle/
model_ref.py RefModel over the shader restatements) within BASELINE's
end-to-end 2e-2. Variants cover the LM head forms (tied, untied f16, untied
ternary), SiLU with and without a gate, missing sub-norms, and prompts longer
than one prefill chunk. The generation loop (greedy), the text APIs, stop
conditions and errors go through the same ABI.
"""
import importlib
import json
import os

import numpy as np
import pytest

from _util import need_cuda
from oracle import model_ref

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
TOL = 2e-2


def ox():
    return importlib.import_module("0xbitnet_b200.oxbitnet")


def gw():
    return importlib.import_module("0xbitnet_b200.gguf_writer")


@pytest.fixture(scope="module")
def vocab():
    with open(os.path.join(HERE, "golden", "tokenizer", "vocab.json")) as f:
        return json.load(f)


def make(tmp_path, vocab, name="m", seed=1, eos=None, **kw):
    W = gw()
    base = dict(vocab=len(vocab["tokens"]), hidden=256, ffn=512, layers=2, heads=2, kv_heads=1)
    base.update(kw)
    shape = W.BitNetShape(**base)
    keep = {}
    p = str(tmp_path / f"{name}.gguf")
    W.write_bitnet_model(p, shape, vocab["tokens"], vocab["merges"], vocab["bos"],
                         vocab["eos"] if eos is None else eos, seed=seed, keep=keep)
    return p, shape, keep


def check_steps(m, ref, prompt, steps):
    got = m.forward(prompt, reset=True)
    want = ref.forward(prompt)
    assert np.abs(got - want).max() <= TOL, np.abs(got - want).max()
    for t in steps:
        got = m.forward([t])
        want = ref.forward([t])
        assert np.abs(got - want).max() <= TOL, np.abs(got - want).max()


def test_prefill_and_decode_match_oracle(tmp_path, vocab):
    need_cuda()
    p, shape, keep = make(tmp_path, vocab)
    m = ox().BitNet.load_sync(p)
    info = m.info()
    assert (info.vocab_size, info.hidden_size, info.num_layers, info.head_dim) == (705, 256, 2, 128)
    ref = model_ref.RefModel(keep, shape)
    check_steps(m, ref, [vocab["bos"], 17, 300, 42, 5, 600, 7, 8, 9], [11, 650, 3])
    assert m.info().position == 12
    # a one-token prompt takes the GEMV order, as the reference's n == 1 forward
    ref.reset()
    check_steps(m, ref, [vocab["bos"]], [100])
    m.dispose()


@pytest.mark.parametrize("n", [513, 600])
def test_prefill_longer_than_one_chunk(tmp_path, vocab, n):
    need_cuda()
    p, shape, keep = make(tmp_path, vocab, layers=1)
    m = ox().BitNet.load_sync(p)
    ref = model_ref.RefModel(keep, shape)
    rng = np.random.default_rng(n)
    prompt = [int(t) for t in rng.integers(0, 700, n)]
    check_steps(m, ref, prompt, [4])
    m.dispose()


@pytest.mark.parametrize("variant", [
    dict(lm_head="f16"),
    dict(lm_head="i2s"),
    dict(arch="bitnet", rope_theta=10000.0),                  # SiLU gate
    dict(arch="bitnet", rope_theta=10000.0, gated=False),     # SiLU, no gate
    dict(gated=False),                                       # ReLU^2, no gate
    dict(sub_norms=False),
    dict(heads=4, kv_heads=1, hidden=512, ffn=1024),          # 4 query heads per KV head
    dict(heads=2, kv_heads=2),                                # MHA
])
def test_variants_match_oracle(tmp_path, vocab, variant):
    need_cuda()
    p, shape, keep = make(tmp_path, vocab, **variant)
    m = ox().BitNet.load_sync(p)
    ref = model_ref.RefModel(keep, shape)
    check_steps(m, ref, [vocab["bos"], 1, 2, 3, 400], [5, 6])
    m.dispose()


def test_greedy_generation_matches_oracle(tmp_path, vocab):
    need_cuda()
    p, shape, keep = make(tmp_path, vocab, seed=5)
    m = ox().BitNet.load_sync(p)
    prompt = [vocab["bos"], 10, 20, 30]
    got = m.generate_ids(prompt, max_tokens=12, temperature=1.0, top_k=1, repeat_penalty=1.0)
    ref = model_ref.RefModel(keep, shape)
    logits = ref.forward(prompt)
    for i, t in enumerate(got):
        top = np.sort(logits)[::-1]
        if top[0] - top[1] < 2 * TOL:  # a near tie: the order after it is not pinned
            break
        assert t == int(np.argmax(logits)), i
        logits = ref.forward([t])
    assert len(got) <= 12
    m.dispose()


def test_text_apis_and_stops(tmp_path, vocab):
    need_cuda()
    p, shape, keep = make(tmp_path, vocab, seed=7)
    m = ox().BitNet.load_sync(p, on_progress=lambda *a: None)
    tok = ox().Tokenizer(p)
    prompt = "Hello, world!"
    ids = tok.encode(prompt)
    greedy = m.generate_ids(ids, max_tokens=6, top_k=1, repeat_penalty=1.0)
    texts = m.generate_tokens_sync(prompt, max_tokens=6, top_k=1, repeat_penalty=1.0)
    assert texts == [tok.token_text(t) for t in greedy]
    assert m.generate_sync(prompt, max_tokens=6, top_k=1, repeat_penalty=1.0) == "".join(texts)
    # the callback stops generation by returning non-zero
    assert len(m.generate_ids(ids, max_tokens=6, top_k=1, stop_after=2)) == 2
    # chat runs the template; max_tokens bounds the output
    n = m.chat([("user", "hi"), ("assistant", "yo"), ("user", "more")], lambda t: None,
               max_tokens=3)
    assert 0 <= n <= 3
    # sampling with a seed is reproducible
    m.set_seed(123)
    a = m.generate_ids(ids, max_tokens=8, temperature=0.8, top_k=20)
    m.set_seed(123)
    b = m.generate_ids(ids, max_tokens=8, temperature=0.8, top_k=20)
    assert a == b
    m.dispose()
    # EOS: a model whose eos id is the first greedy token generates nothing
    p2, _, _ = make(tmp_path, vocab, name="eos", seed=7, eos=greedy[0])
    m2 = ox().BitNet.load_sync(p2)
    assert m2.generate_ids(ids, max_tokens=6, top_k=1, repeat_penalty=1.0) == []
    m2.dispose()


def test_errors(tmp_path, vocab):
    need_cuda()
    p, _, _ = make(tmp_path, vocab, layers=1)
    m = ox().BitNet.load_sync(p)
    with pytest.raises(ox().OxBitNetError, match="exceeds the 4096-position KV cache"):
        m.generate_ids([1] * 4097, max_tokens=1)
    with pytest.raises(ox().OxBitNetError, match="context full"):
        m.forward([1] * 4096, reset=True)
        m.forward([2])
    m.dispose()
    with pytest.raises(ox().OxBitNetError):
        m.forward([1])  # disposed
    # a head_dim the attention kernels are not built for is refused at load
    p3, _, _ = make(tmp_path, vocab, name="hd64", hidden=256, heads=4, kv_heads=4)
    with pytest.raises(ox().OxBitNetError, match="head_dim 64"):
        ox().BitNet.load_sync(p3)


def test_device_sampling_matches_host_sampler(tmp_path, vocab):
    """The generation loop's sampler (penalty, temperature and top-k on the device,
    the draw on the host) picks the same id as the whole-vocabulary host sampler
    (sampling.rs restated in sampler.cpp) on the same logits and draw."""
    need_cuda()
    p, _, _ = make(tmp_path, vocab, layers=1, seed=9)
    m = ox().BitNet.load_sync(p)
    rng = np.random.default_rng(0)
    prompt = [vocab["bos"], 3, 4, 5]
    for trial in range(60):
        T = float(rng.choice([0.0, 0.5, 1.0, 1.7]))
        k = int(rng.choice([1, 5, 50, 200, 704, 705, 0]))
        pen = float(rng.choice([1.0, 1.1, 2.0]))
        recent = [int(t) for t in rng.integers(0, 705, int(rng.integers(0, 70)))]
        u = float(rng.random()) if trial % 10 else 0.0
        logits = m.forward(prompt, reset=True)
        want = ox().sample(logits, T, k, pen, recent, u)
        got = m.sample_next(T, k, pen, recent, u)
        assert got == want, (trial, T, k, pen, u)
    m.dispose()


def test_graph_and_eager_decode_agree(tmp_path, vocab, monkeypatch):
    """Decode steps replayed from the captured graph (position read on the device,
    attention split over the whole cache) give bit-identical logits to eager steps."""
    need_cuda()
    p, _, _ = make(tmp_path, vocab, seed=11)
    g = ox().BitNet.load_sync(p)
    monkeypatch.setenv("OXBITNET_CUDA_GRAPH", "0")
    e = ox().BitNet.load_sync(p)
    prompt = [vocab["bos"], 9, 8, 7]
    assert np.array_equal(g.forward(prompt, reset=True), e.forward(prompt, reset=True))
    for t in [1, 2, 3, 400, 5, 6, 700, 8]:
        assert np.array_equal(g.forward([t]), e.forward([t]))
    # a reset and a new prompt reuse the captured graph at the new positions
    assert np.array_equal(g.forward(prompt[:2], reset=True), e.forward(prompt[:2], reset=True))
    for t in [11, 12]:
        assert np.array_equal(g.forward([t]), e.forward([t]))
    g.dispose()
    e.dispose()


def test_url_source_loads_from_the_cache(tmp_path, vocab):
    """loader.rs:366-384: a URL source is served from <cache_dir>/<sha256(url)> when
    that file exists (nothing is downloaded)."""
    need_cuda()
    import hashlib
    import shutil
    p, shape, keep = make(tmp_path, vocab, layers=1)
    url = "https://example.com/bitnet/ggml-model-i2_s.gguf"
    cache = tmp_path / "cache"
    cache.mkdir()
    shutil.copy(p, cache / hashlib.sha256(url.encode()).hexdigest())
    phases = []
    m = ox().BitNet.load_sync(url, on_progress=lambda *a: phases.append(a[0]),
                              cache_dir=str(cache))
    ref = model_ref.RefModel(keep, shape)
    check_steps(m, ref, [vocab["bos"], 5, 6], [7])
    assert phases[0] == 0 and 1 in phases and phases[-1] == 2
    m.dispose()
