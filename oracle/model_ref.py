"""CPU restatements of the model-level host logic — TEST INFRASTRUCTURE ONLY.

Checkers for the GGUF / tokenizer / sampler / generation code behind the
oxbitnet_* C ABI. Only tests/ import this module. Each function restates the
reference file it names, in plain Python, with an algorithm chosen for
clarity (not the library's): the BPE here merges by rescanning the whole
symbol list each round, the top-k threshold comes from a full sort.

Pinned by tests/golden/tokenizer/ (outputs of the HF `tokenizers` library the
reference links, built the way tokenizer.rs builds it) and by the sampler
known-answer cases in tests/test_model_host_cpu.py.
"""
from __future__ import annotations

import math

import numpy as np


# ---- tokenizer (packages/rust/crates/oxbitnet/src/tokenizer.rs) -------------

def byte_alphabet() -> dict:
    """GPT-2 byte -> character table: printable Latin-1 bytes map to themselves,
    the remaining 68 bytes to U+0100, U+0101, ... in byte order."""
    keep = list(range(33, 127)) + list(range(161, 173)) + list(range(174, 256))
    table, n = {}, 0
    for b in range(256):
        if b in keep:
            table[b] = chr(b)
        else:
            table[b] = chr(256 + n)
            n += 1
    return table


class RefTokenizer:
    """tokenizer.rs:20-217 over a GGUF token list and merge list."""

    def __init__(self, tokens: list, merges: list, bos: int = 1, eos: int = 2):
        self.tokens = list(tokens)
        self.vocab = {t: i for i, t in enumerate(tokens)}  # last id wins for repeats
        self.ranks = {}
        for r, m in enumerate(merges):
            parts = m.split(" ", 1)                       # splitn(2, ' ')
            if len(parts) == 2:
                self.ranks[(parts[0], parts[1])] = r      # last rank wins for repeats
        self.b2c = byte_alphabet()
        self.c2b = {c: b for b, c in self.b2c.items()}
        self.bos, self.eos = bos, eos

    def _bpe(self, word: str) -> list:
        syms = list(word)
        while len(syms) > 1:
            best = None
            for i in range(len(syms) - 1):
                r = self.ranks.get((syms[i], syms[i + 1]))
                if r is not None and (best is None or r < best[0]):
                    best = (r, i)
            if best is None:
                break
            i = best[1]
            syms[i:i + 2] = [syms[i] + syms[i + 1]]
        out = []
        for s in syms:
            if s in self.vocab:
                out.append(self.vocab[s])
            else:  # single characters outside the vocabulary become <unk>
                out.append(self.vocab["<unk>"])
        return out

    def encode(self, text: str, add_bos: bool = True) -> list:
        word = "".join(self.b2c[b] for b in text.encode("utf-8"))
        return ([self.bos] if add_bos else []) + (self._bpe(word) if word else [])

    def token_bytes(self, i: int) -> bytes:
        if not 0 <= i < len(self.tokens):
            return b""
        t = self.tokens[i]
        if all(c in self.c2b for c in t):
            return bytes(self.c2b[c] for c in t)
        return t.encode("utf-8")

    def decode_one(self, i: int) -> str:
        return self.token_bytes(i).decode("utf-8", errors="replace")

    def decode(self, ids) -> str:
        b = b"".join(self.token_bytes(i) for i in ids if i not in (self.bos, self.eos))
        return b.decode("utf-8", errors="replace")

    def chat(self, messages: list) -> list:
        v = self.vocab
        if "<|im_start|>" in v and "<|im_end|>" in v:
            ids = [self.bos]
            for role, content in messages:
                ids += [v["<|im_start|>"]] + self.encode(f"{role}\n{content}", False)
                ids += [v["<|im_end|>"]] + self.encode("\n", False)
            return ids + [v["<|im_start|>"]] + self.encode("assistant\n", False)
        need = ("<|start_header_id|>", "<|end_header_id|>", "<|eot_id|>")
        if not all(k in v for k in need):
            return self.encode("\n".join(c for _, c in messages), True)
        sh, eh, eot = (v[k] for k in need)
        ids = [self.bos]
        for role, content in messages:
            ids += [sh] + self.encode(role, False) + [eh]
            ids += self.encode("\n\n" + content, False) + [eot]
        return ids + [sh] + self.encode("assistant", False) + [eh] + self.encode("\n\n", False)


# ---- sampling (packages/rust/crates/oxbitnet/src/sampling.rs:4-77) ------------

def sample(logits: np.ndarray, temperature: float, top_k: int, repeat_penalty: float,
           recent: list, u: float) -> int:
    """One draw with the uniform value u in [0, 1) supplied; float32 throughout."""
    x = np.array(logits, dtype=np.float32)
    V = x.shape[0]
    if repeat_penalty != 1.0 and recent:
        p = np.float32(repeat_penalty)
        for t in recent:
            if t < V:
                x[t] = x[t] / p if x[t] > 0 else x[t] * p
    if not temperature > 0:
        return int(np.argmax(x))
    if temperature != 1.0:
        x = (x * (np.float32(1.0) / np.float32(temperature))).astype(np.float32)
    if 0 < top_k < V:
        thr = np.sort(x)[::-1][top_k - 1]
        x = np.where(x < thr, np.float32(-np.inf), x).astype(np.float32)
    mx = np.float32(max(x))
    e = [np.float32(math.exp(float(np.float32(v - mx)))) if v != -np.inf else np.float32(0)
         for v in x]
    s = np.float32(0)
    for v in e:
        s = np.float32(s + v)
    r = np.float32(np.float32(u) * s)
    c = np.float32(0)
    for i, v in enumerate(e):
        c = np.float32(c + v)
        if c >= r:
            return i
    return V - 1


# ---- the model forward (nn/model.rs:200-262, transformer.rs:51-72, attention.rs:85-124,
#      ffn.rs:58-92) over the shader restatements of oracle/obn_oracle.c -------------

class RefModel:
    """BitNetModel::forward on the CPU for a model written by gguf_writer with
    keep={...}. The KV cache holds binary16-rounded keys and values (the B200
    cache format; the reference keeps f32), so a comparison isolates the kernels."""

    def __init__(self, keep: dict, shape):
        import oracle as orc
        from importlib import import_module
        self.orc = orc
        self.pack = import_module("0xbitnet_b200.gguf_writer").pack_i2s
        self.k, self.s = keep, shape
        self.d = shape.hidden // shape.heads
        self.reset()

    def reset(self):
        self.K = [np.zeros((0, self.s.kv_heads * self.d), np.float32) for _ in range(self.s.layers)]
        self.V = [np.zeros((0, self.s.kv_heads * self.d), np.float32) for _ in range(self.s.layers)]
        self.pos = 0

    def _lin(self, x, names, norm, eps):
        rows, sw = [], []
        for n in names:
            codes, scale = self.k[n]
            rows.append(self.pack(codes))
            sw.append(np.full(codes.shape[0], scale, np.float32))
        rows, sw = np.concatenate(rows), np.concatenate(sw)
        K = rows.shape[1] * 4
        return self.orc.bitlinear(x, rows, sw, rows.shape[0], K, norm_w=norm, eps=eps)[0]

    def forward(self, ids: list) -> np.ndarray:
        orc, s, d, k = self.orc, self.s, self.d, self.k
        H, Hkv, n = s.heads, s.kv_heads, len(ids)
        x = k["token_embd.weight"][ids].astype(np.float32)
        for i in range(s.layers):
            p = f"blk.{i}."
            qkv = self._lin(x, [p + "attn_q.weight", p + "attn_k.weight", p + "attn_v.weight"],
                            k[p + "attn_norm.weight"], s.eps)
            q = orc.rope(qkv[:, :H * d], H, d, self.pos, s.rope_theta)
            kk = orc.rope(qkv[:, H * d:(H + Hkv) * d], Hkv, d, self.pos, s.rope_theta)
            vv = qkv[:, (H + Hkv) * d:]
            self.K[i] = np.concatenate([self.K[i], kk.astype(np.float16).astype(np.float32)])
            self.V[i] = np.concatenate([self.V[i], vv.astype(np.float16).astype(np.float32)])
            a = orc.attention(q, self.K[i], self.V[i], H, Hkv, d)
            o = self._lin(a, [p + "attn_output.weight"], k.get(p + "attn_sub_norm.weight"), 1e-5)
            x = (x + o).astype(np.float32)
            fn = k[p + "ffn_norm.weight"]
            up = self._lin(x, [p + "ffn_up.weight"], fn, s.eps)
            silu = s.arch != "bitnet-25"
            if s.gated:
                g = self._lin(x, [p + "ffn_gate.weight"], fn, s.eps)
                if silu:
                    act = (g / (np.float32(1) + np.exp(-g))).astype(np.float32) * up
                else:
                    act = orc.relu2_mul(g, up)
            else:
                act = (up / (np.float32(1) + np.exp(-up))).astype(np.float32) if silu else \
                    np.square(np.maximum(up, 0)).astype(np.float32)
            act = act.astype(np.float32)
            dn = self._lin(act, [p + "ffn_down.weight"], k.get(p + "ffn_sub_norm.weight"), 1e-5)
            x = (x + dn).astype(np.float32)
        self.pos += n
        last = x[-1:]
        fnorm = k["output_norm.weight"]
        if "output.weight" in k and isinstance(k["output.weight"], tuple):
            normed = orc.rmsnorm(last, fnorm, s.eps)
            return self._lin(normed, ["output.weight"], fnorm, 1e-5)[0]
        table = k["output.weight"] if "output.weight" in k else k["token_embd.weight"]
        return orc.lm_head_f16(last, table, fnorm, s.eps)[0]
