"""GGUF writer for BitNet b1.58 models (I2_S ternary weights).

Writes the container the reference's parser reads (packages/rust/crates/
oxbitnet/src/model/gguf.rs:140-323; GGUF v3: header, typed metadata, tensor
infos, aligned tensor data) with the tensor names, types and shapes its loader
expects (model/loader.rs:78-171, 214-313). I2_S tensors hold ceil(n/4) packed
bytes (four 2-bit codes per byte in the reference's block interleave,
loader.rs:104-137; codes 0, 1, 2 = -1, 0, +1) followed by a 32-byte trailer
whose first float32 is the per-tensor scale.

`write_bitnet_model` makes a seeded random model of any BitNet shape, so the
full loader -> generate path runs without a checkpoint (none is available
offline). The weights follow the distributions the benchmarks use: ternary
P(-1) = P(+1) = 0.3, scales U(0.5, 2), norm gammas N(1, 0.1), embeddings
N(0, 0.02) in binary16.
"""
from __future__ import annotations

import struct
from dataclasses import dataclass, field

import numpy as np

# metadata value types (gguf.rs:8-20)
U8, I8, U16, I16, U32, I32, F32, BOOL, STRING, ARRAY, U64, I64, F64 = range(13)
# ggml tensor types (gguf.rs:22-36)
TYPE_F32, TYPE_F16, TYPE_I2_S = 0, 1, 36

_SCALAR = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f",
           BOOL: "<?", U64: "<Q", I64: "<q", F64: "<d"}


def _str(s: str | bytes) -> bytes:
    b = s.encode() if isinstance(s, str) else s
    return struct.pack("<Q", len(b)) + b


def _value(vtype: int, v) -> bytes:
    if vtype == STRING:
        return _str(v)
    if vtype == ARRAY:
        etype, items = v
        out = [struct.pack("<IQ", etype, len(items))]
        out += [_value(etype, x) for x in items]
        return b"".join(out)
    return struct.pack(_SCALAR[vtype], v)


@dataclass
class GGUFWriter:
    """Collects metadata and tensors, then writes one GGUF file."""
    version: int = 3
    alignment: int = 32
    metadata: list = field(default_factory=list)   # (key, type, value)
    tensors: list = field(default_factory=list)    # (name, shape ne0-first, ggml type, bytes)

    def add(self, key: str, vtype: int, value) -> None:
        self.metadata.append((key, vtype, value))

    def add_tensor(self, name: str, shape, ggml_type: int, data: bytes) -> None:
        self.tensors.append((name, tuple(int(s) for s in shape), ggml_type, bytes(data)))

    def _header(self) -> bytes:
        head = [struct.pack("<IIQQ", 0x46554747, self.version, len(self.tensors),
                            len(self.metadata))]
        for key, vtype, value in self.metadata:
            head.append(_str(key) + struct.pack("<I", vtype) + _value(vtype, value))
        off = 0
        for name, shape, gtype, data in self.tensors:
            head.append(_str(name) + struct.pack("<I", len(shape))
                        + b"".join(struct.pack("<Q", s) for s in shape)
                        + struct.pack("<IQ", gtype, off))
            off += (len(data) + self.alignment - 1) // self.alignment * self.alignment
        h = b"".join(head)
        return h + b"\0" * ((-len(h)) % self.alignment)

    def write(self, path: str) -> None:
        """Streams the header, then each tensor padded to the alignment."""
        with open(path, "wb") as f:
            f.write(self._header())
            for _, _, _, data in self.tensors:
                f.write(data)
                f.write(b"\0" * ((-len(data)) % self.alignment))


def pack_i2s(codes: np.ndarray) -> np.ndarray:
    """codes [M, K] uint8 in {0,1,2} -> I2_S rows [M, K/4]: within each
    128-column block, byte j (j < 32) of the block holds the codes of columns
    j, 32 + j, 64 + j, 96 + j at bits 7-6, 5-4, 3-2, 1-0."""
    M, K = codes.shape
    c = codes.reshape(M, K // 128, 4, 32).astype(np.uint8)
    return ((c[:, :, 0] << 6) | (c[:, :, 1] << 4) | (c[:, :, 2] << 2) | c[:, :, 3]).reshape(M, K // 4)


def i2s_tensor(rng: np.random.Generator, M: int, K: int, scale: float | None = None) -> tuple:
    """A random ternary [M, K] weight as GGUF I2_S bytes; returns (bytes, codes, scale)."""
    u = rng.random((M, K), dtype=np.float32)
    codes = np.where(u < 0.3, 0, np.where(u < 0.7, 1, 2)).astype(np.uint8)
    if scale is None:
        scale = float(np.float32(0.5 + 1.5 * rng.random()))
    trailer = np.zeros(8, dtype=np.float32)
    trailer[0] = scale
    return pack_i2s(codes).tobytes() + trailer.tobytes(), codes, scale


_FAST_LUT = None


def fast_i2s_tensor(rng: np.random.Generator, M: int, K: int) -> bytes:
    """A random ternary tensor as I2_S bytes without materialising the codes:
    each packed byte comes from 16 random bits, one nibble per 2-bit code
    (nibble < 5 -> -1, < 11 -> 0, else +1: P(-1) = P(+1) = 5/16, P(0) = 6/16).
    For large synthetic models (the 2B shape holds 2.1e9 weights)."""
    global _FAST_LUT
    if _FAST_LUT is None:
        v = np.arange(65536, dtype=np.uint32)
        lut = np.zeros(65536, np.uint8)
        for j in range(4):
            nib = (v >> (4 * j)) & 15
            code = np.where(nib < 5, 0, np.where(nib < 11, 1, 2)).astype(np.uint8)
            lut |= (code << (2 * j)).astype(np.uint8)
        _FAST_LUT = lut
    r = rng.integers(0, 65536, size=M * K // 4, dtype=np.uint16)
    trailer = np.zeros(8, dtype=np.float32)
    trailer[0] = np.float32(0.5 + 1.5 * rng.random())
    return _FAST_LUT[r].tobytes() + trailer.tobytes()


@dataclass
class BitNetShape:
    vocab: int = 128256
    hidden: int = 2560
    ffn: int = 6912
    layers: int = 30
    heads: int = 20
    kv_heads: int = 5
    context_length: int = 4096
    eps: float = 1e-5
    rope_theta: float = 500000.0
    arch: str = "bitnet-25"
    gated: bool = True
    sub_norms: bool = True
    lm_head: str = "tied"   # "tied", "f16" or "i2s"


def write_bitnet_model(path: str, shape: BitNetShape, tokens: list, merges: list,
                       bos: int, eos: int, seed: int = 0, keep: dict | None = None,
                       fast: bool = False) -> None:
    """Writes a seeded random BitNet model with the given tokenizer vocabulary.
    If `keep` is a dict, the host copies of every tensor go into it (name ->
    (codes, scale) for I2_S, float32 array otherwise) for reference checks.
    fast=True draws the ternary weights with fast_i2s_tensor (no `keep`)."""
    s = shape
    rng = np.random.default_rng(seed)
    w = GGUFWriter()
    a = s.arch
    w.add("general.architecture", STRING, a)
    w.add("general.name", STRING, "synthetic bitnet")
    for k, t, v in [("vocab_size", U32, s.vocab), ("embedding_length", U32, s.hidden),
                    ("feed_forward_length", U32, s.ffn), ("block_count", U32, s.layers),
                    ("attention.head_count", U32, s.heads),
                    ("attention.head_count_kv", U32, s.kv_heads),
                    ("context_length", U32, s.context_length),
                    ("attention.layer_norm_rms_epsilon", F32, s.eps),
                    ("rope.freq_base", F32, s.rope_theta)]:
        w.add(f"{a}.{k}", t, v)
    w.add("tokenizer.ggml.model", STRING, "gpt2")
    w.add("tokenizer.ggml.tokens", ARRAY, (STRING, tokens))
    w.add("tokenizer.ggml.merges", ARRAY, (STRING, merges))
    w.add("tokenizer.ggml.bos_token_id", U32, bos)
    w.add("tokenizer.ggml.eos_token_id", U32, eos)

    d = s.hidden // s.heads

    def gamma(name, n):
        g = (1.0 + 0.1 * rng.standard_normal(n)).astype(np.float32)
        w.add_tensor(name, (n,), TYPE_F32, g.tobytes())
        if keep is not None:
            keep[name] = g

    def tern(name, M, K):
        if fast:
            w.add_tensor(name, (K, M), TYPE_I2_S, fast_i2s_tensor(rng, M, K))
            return
        data, codes, scale = i2s_tensor(rng, M, K)
        w.add_tensor(name, (K, M), TYPE_I2_S, data)
        if keep is not None:
            keep[name] = (codes, scale)

    emb = (0.02 * rng.standard_normal((s.vocab, s.hidden), dtype=np.float32)).astype(np.float16)
    w.add_tensor("token_embd.weight", (s.hidden, s.vocab), TYPE_F16, emb.tobytes())
    if keep is not None:
        keep["token_embd.weight"] = emb
    for i in range(s.layers):
        p = f"blk.{i}."
        gamma(p + "attn_norm.weight", s.hidden)
        tern(p + "attn_q.weight", s.heads * d, s.hidden)
        tern(p + "attn_k.weight", s.kv_heads * d, s.hidden)
        tern(p + "attn_v.weight", s.kv_heads * d, s.hidden)
        if s.sub_norms:
            gamma(p + "attn_sub_norm.weight", s.heads * d)
        tern(p + "attn_output.weight", s.hidden, s.heads * d)
        gamma(p + "ffn_norm.weight", s.hidden)
        if s.gated:
            tern(p + "ffn_gate.weight", s.ffn, s.hidden)
        tern(p + "ffn_up.weight", s.ffn, s.hidden)
        if s.sub_norms:
            gamma(p + "ffn_sub_norm.weight", s.ffn)
        tern(p + "ffn_down.weight", s.hidden, s.ffn)
    gamma("output_norm.weight", s.hidden)
    if s.lm_head == "f16":
        out = (0.02 * rng.standard_normal((s.vocab, s.hidden))).astype(np.float16)
        w.add_tensor("output.weight", (s.hidden, s.vocab), TYPE_F16, out.tobytes())
        if keep is not None:
            keep["output.weight"] = out
    elif s.lm_head == "i2s":
        tern("output.weight", s.vocab, s.hidden)
    w.write(path)


def synthetic_vocab(n: int) -> tuple:
    """A vocabulary of n tokens for synthetic models: the 256 byte-alphabet
    characters, filler tokens, and the LLaMA 3 specials last; no merges.
    Returns (tokens, merges, bos, eos)."""
    keep = list(range(33, 127)) + list(range(161, 173)) + list(range(174, 256))
    chars, k = [], 0
    for b in range(256):
        if b in keep:
            chars.append(chr(b))
        else:
            chars.append(chr(256 + k))
            k += 1
    specials = ["<|begin_of_text|>", "<|end_of_text|>", "<|start_header_id|>",
                "<|end_header_id|>", "<|eot_id|>"]
    filler = [f"<tok{i}>" for i in range(n - 256 - len(specials))]
    tokens = chars + filler + specials
    return tokens, [], tokens.index("<|begin_of_text|>"), tokens.index("<|end_of_text|>")
