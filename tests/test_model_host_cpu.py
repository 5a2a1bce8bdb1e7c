"""Host side of the model-level ABI (include/oxbitnet.h) on the CPU.

GGUF parsing (the reference's gguf.rs / loader.rs config rules), the byte-level
BPE tokenizer against the golden vectors of the HF `tokenizers` library the
reference links (tests/golden/tokenizer/, made by make_tokenizer_golden.py),
the chat templates and sampler against the restatements in oracle/model_ref.py,
and the FFI conventions of oxbitnet-ffi/src/lib.rs (defaults, NULL handling,
thread-local errors, logger). Nothing here needs a GPU.
"""
import hashlib
import importlib
import json
import os
import random
import struct
import threading

import numpy as np
import pytest

from oracle import model_ref

HERE = os.path.dirname(os.path.abspath(__file__))
GOLD = os.path.join(HERE, "golden", "tokenizer")


def ox():
    return importlib.import_module("0xbitnet_b200.oxbitnet")


def gw():
    return importlib.import_module("0xbitnet_b200.gguf_writer")


@pytest.fixture(scope="module")
def vocab():
    with open(os.path.join(GOLD, "vocab.json")) as f:
        return json.load(f)


@pytest.fixture(scope="module")
def golden():
    with open(os.path.join(GOLD, "golden.json")) as f:
        return json.load(f)


def tiny_shape(**kw):
    W = gw()
    base = dict(vocab=705, hidden=256, ffn=512, layers=1, heads=2, kv_heads=1)
    base.update(kw)
    return W.BitNetShape(**base)


@pytest.fixture(scope="module")
def tiny_gguf(tmp_path_factory, vocab):
    p = str(tmp_path_factory.mktemp("gguf") / "tiny.gguf")
    gw().write_bitnet_model(p, tiny_shape(), vocab["tokens"], vocab["merges"], vocab["bos"],
                            vocab["eos"], seed=1)
    return p


# ---- the oracle is pinned by the library's own outputs -------------------------

def test_oracle_tokenizer_matches_hf_golden(vocab, golden):
    ref = model_ref.RefTokenizer(vocab["tokens"], vocab["merges"], vocab["bos"], vocab["eos"])
    for c in golden["cases"]:
        assert ref.encode(c["text"], add_bos=False) == c["ids"], c["text"]
        assert ref.decode(c["ids"]) == c["decoded"]
    assert [ref.decode_one(i) for i in range(len(vocab["tokens"]))] == golden["decode_one"]


# ---- C++ tokenizer ---------------------------------------------------------------

def test_tokenizer_golden(tiny_gguf, vocab, golden):
    tok = ox().Tokenizer(tiny_gguf)
    for c in golden["cases"]:
        assert tok.encode(c["text"], add_bos=False) == c["ids"], c["text"]
        assert tok.encode(c["text"]) == [vocab["bos"]] + c["ids"]
        assert tok.decode(c["ids"]) == c["decoded"]
    got = [tok.token_text(i) for i in range(len(vocab["tokens"]))]
    assert got == golden["decode_one"]
    assert tok.token_text(10 ** 6) == ""  # unknown ids decode to nothing


def test_tokenizer_fuzz_vs_oracle(tiny_gguf, vocab):
    tok = ox().Tokenizer(tiny_gguf)
    ref = model_ref.RefTokenizer(vocab["tokens"], vocab["merges"], vocab["bos"], vocab["eos"])
    rng = random.Random(5)
    alphabet = list("abcdefghijklmnopqrstuvwxyz ABCDEF.,!?'\n\t0123456789") + \
        ["é", "ü", "日", "本", "😀", "€", " ", "\x01", "\x7f"]
    for _ in range(300):
        s = "".join(rng.choice(alphabet) for _ in range(rng.randint(0, 60)))
        ids = tok.encode(s, add_bos=False)
        assert ids == ref.encode(s, add_bos=False), repr(s)
        assert tok.decode(ids) == s  # byte-level BPE is lossless
    # decoding arbitrary id sequences (split multi-byte characters -> U+FFFD)
    for _ in range(200):
        ids = [rng.randrange(len(vocab["tokens"])) for _ in range(rng.randint(0, 12))]
        assert tok.decode(ids) == ref.decode(ids)


def test_chat_templates(tmp_path, vocab):
    msgs = [("system", "be brief"), ("user", "Hello, world!"), ("assistant", "hi"),
            ("user", "日本語 😀")]
    W = gw()
    variants = {
        "llama3": vocab["tokens"],
        "chatml": vocab["tokens"] + ["<|im_start|>", "<|im_end|>"],
        "plain": [t for t in vocab["tokens"] if t != "<|eot_id|>"] + ["<|x|>"],
    }
    for name, tokens in variants.items():
        p = str(tmp_path / f"{name}.gguf")
        bos = tokens.index("<|begin_of_text|>")
        eos = tokens.index("<|end_of_text|>")
        W.write_bitnet_model(p, tiny_shape(vocab=len(tokens)), tokens, vocab["merges"], bos, eos)
        tok = ox().Tokenizer(p)
        ref = model_ref.RefTokenizer(tokens, vocab["merges"], bos, eos)
        assert tok.chat_template(msgs) == ref.chat(msgs), name
        assert tok.chat_template([]) == ref.chat([]), name


def test_tokenizer_errors(tmp_path, vocab):
    W = gw()
    w = W.GGUFWriter()
    w.add("general.architecture", W.STRING, "bitnet-25")
    p = str(tmp_path / "notok.gguf")
    w.write(p)
    with pytest.raises(ox().OxBitNetError, match="Missing tokenizer.ggml.tokens"):
        ox().Tokenizer(p)
    w = W.GGUFWriter()
    w.add("tokenizer.ggml.tokens", W.ARRAY, (W.STRING, ["a", "b"]))
    w.add("tokenizer.ggml.merges", W.ARRAY, (W.STRING, ["a b"]))  # "ab" is not in the vocab
    p = str(tmp_path / "badmerge.gguf")
    w.write(p)
    with pytest.raises(ox().OxBitNetError, match="Failed to build BPE"):
        ox().Tokenizer(p)


# ---- GGUF parsing ------------------------------------------------------------------

def test_describe_tiny(tiny_gguf):
    d = ox().describe(tiny_gguf)
    assert d["version"] == 3 and d["data_offset"] % 32 == 0
    c = d["config"]
    assert (c["arch"], c["vocab_size"], c["hidden_size"], c["intermediate_size"],
            c["num_layers"], c["num_heads"], c["num_kv_heads"], c["head_dim"]) == \
        ("bitnet-25", 705, 256, 512, 1, 2, 1, 128)
    assert c["tied"] and c["gated"] and c["activation"] == 0
    assert abs(c["rope_theta"] - 500000.0) < 1e-3 and abs(c["rms_norm_eps"] - 1e-5) < 1e-12
    t = {x["name"]: x for x in d["tensors"]}
    q = t["blk.0.attn_q.weight"]
    assert q["type"] == 36 and q["shape"] == [256, 256] and q["bytes"] == 256 * 256 // 4 + 32
    assert q["hf_name"] == "model.layers.0.self_attn.q_proj.weight"
    assert t["token_embd.weight"]["hf_name"] == "model.embed_tokens.weight"
    assert t["output_norm.weight"]["hf_name"] == "model.norm.weight"
    assert t["blk.0.ffn_sub_norm.weight"]["hf_name"] == "model.layers.0.mlp.sub_norm.weight"
    assert "tokenizer.ggml.tokens" in d["metadata_keys"]
    # offsets are aligned and ascending
    offs = [x["offset"] for x in d["tensors"]]
    assert offs == sorted(offs) and all(o % 32 == 0 for o in offs)


def test_config_defaults_and_fallbacks(tmp_path, vocab):
    """loader.rs:246-313: arch-prefixed keys, then llama./bitnet./bitnet-25. prefixes,
    defaults; a non-bitnet-25 arch means SiLU and theta 1e4; output.weight unties."""
    W = gw()
    w = W.GGUFWriter()
    w.add("general.architecture", W.STRING, "bitnet")
    w.add("llama.embedding_length", W.U32, 1536)
    w.add("bitnet.attention.head_count", W.I32, 16)
    w.add("tokenizer.ggml.tokens", W.ARRAY, (W.STRING, ["x"] * 7))
    w.add_tensor("output.weight", (1536, 7), W.TYPE_F16, b"\0" * (1536 * 7 * 2))
    p = str(tmp_path / "cfg.gguf")
    w.write(p)
    c = ox().describe(p)["config"]
    assert c["hidden_size"] == 1536 and c["num_heads"] == 16 and c["num_kv_heads"] == 16
    assert c["vocab_size"] == 7 and c["num_layers"] == 30 and c["intermediate_size"] == 6912
    assert c["activation"] == 1 and abs(c["rope_theta"] - 10000.0) < 1e-3
    assert c["tied"] is False and c["head_dim"] == 96 and c["context_length"] == 4096


def _header(version=3, n_tensors=0, n_kv=0, magic=0x46554747):
    return struct.pack("<IIQQ", magic, version, n_tensors, n_kv)


@pytest.mark.parametrize("blob,msg", [
    (_header(magic=0x12345678), "Invalid GGUF magic: 0x12345678 (expected 0x46554747)"),
    (_header(version=1), "Unsupported GGUF version: 1"),
    (_header(version=4), "Unsupported GGUF version: 4"),
    (b"GGU", "Unexpected EOF"),
    (_header(n_kv=1) + struct.pack("<Q", 3) + b"key" + struct.pack("<I", 13), "Unknown GGUF metadata type: 13"),
    (_header(n_kv=1) + struct.pack("<Q", 3) + b"key" + struct.pack("<I", 8) + struct.pack("<Q", 99),
     "Unexpected EOF"),
    (_header(n_kv=1) + struct.pack("<Q", 2) + b"\xff\xfe" + struct.pack("<IB", 0, 1), "Invalid UTF-8"),
    (_header(n_tensors=5), "Unexpected EOF"),
])
def test_gguf_parse_errors(tmp_path, blob, msg):
    p = str(tmp_path / "bad.gguf")
    with open(p, "wb") as f:
        f.write(blob)
    with pytest.raises(ox().OxBitNetError, match=msg.replace("(", r"\(").replace(")", r"\)")):
        ox().describe(p)


def test_gguf_v2_and_alignment(tmp_path, vocab):
    W = gw()
    w = W.GGUFWriter(version=2, alignment=64)
    w.add("general.alignment", W.U32, 64)
    w.add("tokenizer.ggml.tokens", W.ARRAY, (W.STRING, vocab["tokens"]))
    w.add_tensor("a", (3,), W.TYPE_F32, np.ones(3, np.float32).tobytes())
    w.add_tensor("b", (5,), W.TYPE_F32, np.ones(5, np.float32).tobytes())
    p = str(tmp_path / "v2.gguf")
    w.write(p)
    d = ox().describe(p)
    assert d["version"] == 2 and d["data_offset"] % 64 == 0
    assert [t["offset"] for t in d["tensors"]] == [0, 64]


# ---- sampler -------------------------------------------------------------------------

def test_sampler_known_answers():
    S = ox().sample
    x = np.array([0.5, 2.0, -1.0, 2.0, 1.0], np.float32)
    assert S(x, 1.0, 1, 1.0, [], 0.999) in (1, 3)        # top-1 keeps the tied maxima
    assert S(x, 1.0, 1, 1.0, [], 0.5) == 1
    # u = 0 gives r = 0, which the running sum (0 over masked entries) already reaches
    # at index 0: sampling.rs:69-74 returns the first index then, and so do we
    assert S(x, 1.0, 1, 1.0, [], 0.0) == 0
    assert S(x, 0.0, 50, 1.0, [], 0.5) == 1              # temperature 0: arg-max
    # penalty: positive logits are divided, others multiplied, once per occurrence
    y = np.array([4.0, 3.0, -1.0], np.float32)
    assert S(y, 1.0, 1, 2.0, [0, 0], 0.5) == 1           # 4 / 2 / 2 = 1 < 3
    assert S(y, 1.0, 1, 2.0, [0], 0.5) == 1              # 4 / 2 = 2 < 3
    assert S(np.array([-1.0, -3.0], np.float32), 1.0, 1, 4.0, [0], 0.5) == 1  # -4 < -3
    # ids outside the vocabulary in the window are ignored
    assert S(y, 1.0, 1, 2.0, [7, 100], 0.5) == 0


def test_sampler_vs_oracle():
    rng = np.random.default_rng(3)
    for trial in range(300):
        V = int(rng.integers(2, 400))
        x = (rng.standard_normal(V) * rng.uniform(0.1, 5)).astype(np.float32)
        if trial % 7 == 0:
            x[rng.integers(0, V, 3)] = x.max()  # ties at the top
        T = float(rng.choice([0.0, 0.3, 0.7, 1.0, 1.5]))
        k = int(rng.choice([0, 1, 5, 50, V, V + 3]))
        pen = float(rng.choice([1.0, 1.1, 1.3]))
        recent = [int(t) for t in rng.integers(0, V + 5, int(rng.integers(0, 10)))]
        u = float(rng.random())
        got = ox().sample(x, T, k, pen, recent, u)
        want = model_ref.sample(x, T, k, pen, recent, u)
        assert got == want, (trial, V, T, k, pen, u)


# ---- FFI conventions (oxbitnet-ffi/src/lib.rs) ----------------------------------------

def test_defaults_and_null_handling():
    L = ox().lib()
    g = L.oxbitnet_default_generate_options()
    assert (g.max_tokens, g.top_k, g.repeat_last_n) == (256, 50, 64)
    assert abs(g.temperature - 1.0) < 1e-7 and abs(g.repeat_penalty - 1.1) < 1e-6
    lo = L.oxbitnet_default_load_options()
    assert not lo.on_progress and not lo.progress_userdata and lo.cache_dir is None
    assert L.oxbitnet_load(None, None) is None
    assert ox().error_message() == "source must not be NULL"
    L.oxbitnet_free(None)  # no-op
    cb = ox().TokenFn(lambda *a: 0)
    assert L.oxbitnet_generate(None, b"hi", None, cb, None) == -1
    assert ox().error_message() == "model must not be NULL"
    assert L.oxbitnet_chat(None, None, 0, None, cb, None) == -1
    assert ox().error_message() == "model must not be NULL"
    assert L.oxbitnet_load(b"\xff\xfe", None) is None
    assert ox().error_message().startswith("invalid UTF-8 in source")


def test_error_is_thread_local(tmp_path):
    L = ox().lib()
    assert L.oxbitnet_load(str(tmp_path / "missing.gguf").encode(), None) is None
    assert ox().error_message().startswith("IO error:")
    seen = []
    t = threading.Thread(target=lambda: seen.append(ox().error_message()))
    t.start()
    t.join()
    assert seen == [None]
    # a successful call clears it
    L.oxbitnet_default_generate_options()
    assert ox().lib().oxbitnet_cache_path(b"x", b"/tmp", None, 0) == 0
    assert ox().error_message() is None


def test_url_sources_use_the_cache(tmp_path):
    url = "https://example.com/models/ggml-model-i2_s.gguf"
    want = str(tmp_path / hashlib.sha256(url.encode()).hexdigest())
    assert ox().cache_path(url, str(tmp_path)) == want
    L = ox().lib()
    opts = L.oxbitnet_default_load_options()
    opts.cache_dir = str(tmp_path).encode()
    assert L.oxbitnet_load(url.encode(), opts) is None
    assert ox().error_message().startswith("HTTP error:") and want in ox().error_message()


def test_load_reports_progress_and_logs_before_the_gpu(tiny_gguf):
    """On a CPU box the load reaches the parse and config steps (progress and the
    debug config line) and then fails cleanly at the first CUDA call."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("this checks the no-GPU failure path")
    L = ox().lib()
    phases = []
    opts = L.oxbitnet_default_load_options()
    cb = ox().ProgressFn(lambda p, ud: phases.append((p.contents.phase, p.contents.fraction)))
    opts.on_progress = cb
    assert L.oxbitnet_load(tiny_gguf.encode(), opts) is None
    msg = ox().error_message()
    assert msg.startswith("GPU error") or "CUDA" in msg or "device" in msg, msg
    assert phases[:3] == [(0, 0.0), (0, 1.0), (1, 0.0)]


def test_oxbitnet_header_symbols_are_exported():
    import re
    text = open(os.path.join(HERE, "..", "include", "oxbitnet.h")).read()
    syms = sorted(set(re.findall(r"OXBITNET_API\s+[\w\s\*]+?\b(oxbitnet_\w+)\s*\(", text)))
    assert len(syms) == 22
    for s in ["oxbitnet_set_logger", "oxbitnet_default_generate_options",
              "oxbitnet_default_load_options", "oxbitnet_load", "oxbitnet_free",
              "oxbitnet_generate", "oxbitnet_chat", "oxbitnet_error_message"]:
        assert s in syms  # the reference's eight (oxbitnet-ffi/oxbitnet.h:135-224)
    lib = ox().lib()
    for s in syms:
        assert hasattr(lib, s), s
    assert sorted(ox().SIGNATURES) == syms


def test_logger_receives_messages_from_a_load(tiny_gguf):
    """oxbitnet_set_logger installs the callback once; the load's debug config line
    reaches it at min_level 0 (it is emitted before any device work)."""
    L = ox().lib()
    got = []
    cb = ox().LogFn(lambda lvl, msg, n, ud: got.append((lvl, msg[:n].decode())))
    test_logger_receives_messages_from_a_load.cb = cb  # keep alive for the process
    L.oxbitnet_set_logger(cb, None, 0)
    L.oxbitnet_load(tiny_gguf.encode(), None)
    L.oxbitnet_set_logger(cb, None, 4)  # later calls only change the level
    assert any(lvl == 1 and m.startswith("config: arch=bitnet-25, heads=2, kv_heads=1, "
                                         "head_dim=128, hidden=256") for lvl, m in got), got
