"""Model-level Python API over the oxbitnet_* C ABI of libobn.so.

Mirrors the reference's Python package (packages/rust/crates/oxbitnet-python/
src/lib.rs): ``BitNet.load_sync(source)``, ``generate(prompt, on_token, ...)``
and ``chat(messages, on_token, ...)`` returning the number of tokens,
``generate_sync`` returning the text, ``generate_tokens_sync`` returning the
token strings, ``dispose()``. Chat messages are (role, content) pairs, as in
the reference. Additions: generation from token ids, raw logits, seeding,
model info, and ``Tokenizer`` (GGUF tokenizer without a GPU).
"""
from __future__ import annotations

import ctypes
from typing import Callable, Iterable, Sequence

import numpy as np

from ._lib import lib as _obn_lib

_P = ctypes.c_void_p
_U = ctypes.c_size_t  # uintptr_t
_I32 = ctypes.c_int32
_U32 = ctypes.c_uint32
_F = ctypes.c_float


class GenerateOptions(ctypes.Structure):
    _fields_ = [("max_tokens", _U), ("temperature", _F), ("top_k", _U),
                ("repeat_penalty", _F), ("repeat_last_n", _U)]


class LoadProgress(ctypes.Structure):
    _fields_ = [("phase", ctypes.c_int), ("loaded", ctypes.c_uint64),
                ("total", ctypes.c_uint64), ("fraction", ctypes.c_double)]


ProgressFn = ctypes.CFUNCTYPE(None, ctypes.POINTER(LoadProgress), _P)
LogFn = ctypes.CFUNCTYPE(None, ctypes.c_int, ctypes.c_char_p, _U, _P)
TokenFn = ctypes.CFUNCTYPE(_I32, ctypes.POINTER(ctypes.c_char), _U, _P)
TokenIdFn = ctypes.CFUNCTYPE(_I32, _U32, ctypes.POINTER(ctypes.c_char), _U, _P)


class LoadOptions(ctypes.Structure):
    _fields_ = [("on_progress", ProgressFn), ("progress_userdata", _P),
                ("cache_dir", ctypes.c_char_p)]


class ChatMessage(ctypes.Structure):
    _fields_ = [("role", ctypes.c_char_p), ("content", ctypes.c_char_p)]


class ModelInfo(ctypes.Structure):
    _fields_ = [(n, _U32) for n in ("vocab_size", "hidden_size", "intermediate_size",
                                    "num_layers", "num_heads", "num_kv_heads", "head_dim",
                                    "max_seq_len", "position")] + \
               [("rms_norm_eps", _F), ("rope_theta", _F)] + \
               [(n, _I32) for n in ("tied_embeddings", "lm_head_f16", "gated_ffn", "activation")]


# Every oxbitnet_* symbol include/oxbitnet.h declares, with (restype, argtypes).
SIGNATURES = {
    "oxbitnet_set_logger": (None, [LogFn, _P, ctypes.c_uint8]),
    "oxbitnet_default_generate_options": (GenerateOptions, []),
    "oxbitnet_default_load_options": (LoadOptions, []),
    "oxbitnet_load": (_P, [ctypes.c_char_p, ctypes.POINTER(LoadOptions)]),
    "oxbitnet_free": (None, [_P]),
    "oxbitnet_generate": (_I32, [_P, ctypes.c_char_p, ctypes.POINTER(GenerateOptions), TokenFn,
                                 _P]),
    "oxbitnet_chat": (_I32, [_P, ctypes.POINTER(ChatMessage), _U,
                             ctypes.POINTER(GenerateOptions), TokenFn, _P]),
    "oxbitnet_error_message": (ctypes.c_char_p, []),
    "oxbitnet_generate_ids": (_I32, [_P, ctypes.POINTER(_U32), _U,
                                     ctypes.POINTER(GenerateOptions), TokenIdFn, _P]),
    "oxbitnet_set_seed": (_I32, [_P, ctypes.c_uint64]),
    "oxbitnet_forward": (_I32, [_P, ctypes.POINTER(_U32), _U, _I32, ctypes.POINTER(_F), _U]),
    "oxbitnet_model_info": (_I32, [_P, ctypes.POINTER(ModelInfo)]),
    "oxbitnet_tokenizer_load": (_P, [ctypes.c_char_p]),
    "oxbitnet_tokenizer_free": (None, [_P]),
    "oxbitnet_tokenize": (_I32, [_P, ctypes.c_char_p, _I32, ctypes.POINTER(_U32), _U,
                                 ctypes.POINTER(_U)]),
    "oxbitnet_chat_template": (_I32, [_P, ctypes.POINTER(ChatMessage), _U,
                                      ctypes.POINTER(_U32), _U, ctypes.POINTER(_U)]),
    "oxbitnet_detokenize": (_I32, [_P, ctypes.POINTER(_U32), _U, ctypes.c_char_p, _U,
                                   ctypes.POINTER(_U)]),
    "oxbitnet_token_text": (_I32, [_P, _U32, ctypes.c_char_p, _U, ctypes.POINTER(_U)]),
    "oxbitnet_sample_next": (_I32, [_P, _F, _U, _F, ctypes.POINTER(_U32), _U, _F,
                                    ctypes.POINTER(_U32)]),
    "oxbitnet_sample": (_U32, [ctypes.POINTER(_F), _U, _F, _U, _F, ctypes.POINTER(_U32), _U, _F]),
    "oxbitnet_gguf_describe": (ctypes.c_char_p, [ctypes.c_char_p]),
    "oxbitnet_cache_path": (_I32, [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_char_p, _U]),
}

_bound = None


def lib() -> ctypes.CDLL:
    global _bound
    if _bound is None:
        L = _obn_lib()
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _bound = L
    return _bound


class OxBitNetError(RuntimeError):
    pass


def error_message() -> str | None:
    m = lib().oxbitnet_error_message()
    return m.decode("utf-8", "replace") if m is not None else None


def _raise(what: str):
    raise OxBitNetError(f"{what}: {error_message()}")


def _ids_array(ids: Sequence[int]):
    arr = (_U32 * max(1, len(ids)))(*ids)
    return arr, len(ids)


def _messages(messages: Iterable) -> tuple:
    msgs = [(r.encode(), c.encode()) for r, c in messages]
    arr = (ChatMessage * max(1, len(msgs)))(*[ChatMessage(r, c) for r, c in msgs])
    return arr, len(msgs), msgs  # keep the byte strings alive


def _options(max_tokens, temperature, top_k, repeat_penalty, repeat_last_n=64):
    return GenerateOptions(max_tokens, temperature, top_k, repeat_penalty, repeat_last_n)


class BitNet:
    """A model on the current CUDA device (oxbitnet-python/src/lib.rs:27-210)."""

    def __init__(self, handle):
        self._h = handle

    @staticmethod
    def load_sync(source: str, on_progress: Callable | None = None,
                  cache_dir: str | None = None) -> "BitNet":
        opts = lib().oxbitnet_default_load_options()
        keep = []
        if on_progress is not None:
            cb = ProgressFn(lambda p, _ud: on_progress(p.contents.phase, p.contents.loaded,
                                                       p.contents.total, p.contents.fraction))
            keep.append(cb)
            opts.on_progress = cb
        if cache_dir is not None:
            opts.cache_dir = cache_dir.encode()
        h = lib().oxbitnet_load(source.encode(), ctypes.byref(opts))
        if not h:
            _raise("load failed")
        return BitNet(h)

    def _handle(self):
        if not self._h:
            raise OxBitNetError("Model disposed")
        return self._h

    def _run(self, fn, *args, on_token=None):
        count = [0]

        def cb(ptr, n, _ud):
            count[0] += 1
            if on_token is not None:
                try:
                    on_token(ctypes.string_at(ptr, n).decode("utf-8", "replace"))
                except Exception:  # the reference ignores callback errors
                    pass
            return 0

        c = TokenFn(cb)
        if fn(self._handle(), *args, c, None) != 0:
            _raise("generation failed")
        return count[0]

    def generate(self, prompt: str, on_token: Callable, max_tokens: int = 256,
                 temperature: float = 1.0, top_k: int = 50, repeat_penalty: float = 1.1) -> int:
        o = _options(max_tokens, temperature, top_k, repeat_penalty)
        return self._run(lib().oxbitnet_generate, prompt.encode(), ctypes.byref(o),
                         on_token=on_token)

    def chat(self, messages, on_token: Callable, max_tokens: int = 256, temperature: float = 1.0,
             top_k: int = 50, repeat_penalty: float = 1.1) -> int:
        arr, n, _keep = _messages(messages)
        o = _options(max_tokens, temperature, top_k, repeat_penalty)
        return self._run(lib().oxbitnet_chat, arr, n, ctypes.byref(o), on_token=on_token)

    def generate_sync(self, prompt: str, max_tokens: int = 256, temperature: float = 1.0,
                      top_k: int = 50, repeat_penalty: float = 1.1) -> str:
        return "".join(self.generate_tokens_sync(prompt, max_tokens, temperature, top_k,
                                                 repeat_penalty))

    def generate_tokens_sync(self, prompt: str, max_tokens: int = 256, temperature: float = 1.0,
                             top_k: int = 50, repeat_penalty: float = 1.1) -> list:
        out = []
        self.generate(prompt, out.append, max_tokens, temperature, top_k, repeat_penalty)
        return out

    # ---- additions ----
    def generate_ids(self, ids: Sequence[int], max_tokens: int = 256, temperature: float = 1.0,
                     top_k: int = 50, repeat_penalty: float = 1.1, repeat_last_n: int = 64,
                     stop_after: int | None = None) -> list:
        """Generated token ids for a prompt given as ids (no BOS added)."""
        got = []

        def cb(i, _ptr, _n, _ud):
            got.append(int(i))
            return 1 if stop_after is not None and len(got) >= stop_after else 0

        c = TokenIdFn(cb)
        arr, n = _ids_array(ids)
        o = _options(max_tokens, temperature, top_k, repeat_penalty, repeat_last_n)
        if lib().oxbitnet_generate_ids(self._handle(), arr, n, ctypes.byref(o), c, None) != 0:
            _raise("generation failed")
        return got

    def forward(self, ids: Sequence[int], reset: bool = False) -> np.ndarray:
        """Logits [vocab] of the last of `ids`, run at the current position."""
        info = self.info()
        out = np.empty(info.vocab_size, np.float32)
        arr, n = _ids_array(ids)
        if lib().oxbitnet_forward(self._handle(), arr, n, int(reset),
                                  out.ctypes.data_as(ctypes.POINTER(_F)), out.size) != 0:
            _raise("forward failed")
        return out

    def sample_next(self, temperature: float, top_k: int, repeat_penalty: float,
                    recent: Sequence[int], u: float) -> int:
        """The next token from the last forward's logits (device top-k path)."""
        arr, n = _ids_array(list(recent))
        out = _U32(0)
        if lib().oxbitnet_sample_next(self._handle(), temperature, top_k, repeat_penalty, arr, n,
                                      u, ctypes.byref(out)) != 0:
            _raise("sample_next failed")
        return int(out.value)

    def set_seed(self, seed: int) -> None:
        if lib().oxbitnet_set_seed(self._handle(), seed) != 0:
            _raise("set_seed failed")

    def info(self) -> ModelInfo:
        mi = ModelInfo()
        if lib().oxbitnet_model_info(self._handle(), ctypes.byref(mi)) != 0:
            _raise("model_info failed")
        return mi

    def dispose(self) -> None:
        if self._h:
            lib().oxbitnet_free(self._h)
        self._h = None

    def __del__(self):
        try:
            self.dispose()
        except Exception:
            pass

    def __repr__(self) -> str:
        return "BitNet(loaded)" if self._h else "BitNet(disposed)"


class Tokenizer:
    """The tokenizer of a GGUF file (works without a GPU)."""

    def __init__(self, path: str):
        self._h = lib().oxbitnet_tokenizer_load(path.encode())
        if not self._h:
            _raise("tokenizer load failed")

    def _ids(self, fn, *args) -> list:
        n = _U(0)
        if fn(self._h, *args, None, 0, ctypes.byref(n)) != 0:
            _raise("tokenizer call failed")
        buf = (_U32 * max(1, n.value))()
        if fn(self._h, *args, buf, n.value, ctypes.byref(n)) != 0:
            _raise("tokenizer call failed")
        return list(buf[:n.value])

    def encode(self, text: str, add_bos: bool = True) -> list:
        return self._ids(lib().oxbitnet_tokenize, text.encode(), int(add_bos))

    def chat_template(self, messages) -> list:
        arr, n, _keep = _messages(messages)
        return self._ids(lib().oxbitnet_chat_template, arr, n)

    def _text(self, fn, *args) -> str:
        n = _U(0)
        if fn(self._h, *args, None, 0, ctypes.byref(n)) != 0:
            _raise("tokenizer call failed")
        buf = ctypes.create_string_buffer(n.value + 1)
        if fn(self._h, *args, buf, n.value + 1, ctypes.byref(n)) != 0:
            _raise("tokenizer call failed")
        return buf.raw[:n.value].decode("utf-8")

    def decode(self, ids: Sequence[int]) -> str:
        arr, n = _ids_array(ids)
        return self._text(lib().oxbitnet_detokenize, arr, n)

    def token_text(self, i: int) -> str:
        return self._text(lib().oxbitnet_token_text, i)

    def close(self) -> None:
        if self._h:
            lib().oxbitnet_tokenizer_free(self._h)
        self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def sample(logits: np.ndarray, temperature: float, top_k: int, repeat_penalty: float,
           recent: Sequence[int], u: float) -> int:
    """One host sampling step with the uniform draw u (logits are copied)."""
    x = np.array(logits, dtype=np.float32)
    arr, n = _ids_array(list(recent))
    return int(lib().oxbitnet_sample(x.ctypes.data_as(ctypes.POINTER(_F)), x.size, temperature,
                                     top_k, repeat_penalty, arr, n, u))


def describe(path: str) -> dict:
    import json
    s = lib().oxbitnet_gguf_describe(path.encode())
    if s is None:
        _raise("describe failed")
    return json.loads(s.decode("utf-8"))


def cache_path(source: str, cache_dir: str | None = None) -> str:
    buf = ctypes.create_string_buffer(4096)
    if lib().oxbitnet_cache_path(source.encode(), cache_dir.encode() if cache_dir else None,
                                 buf, 4096) != 0:
        _raise("cache_path failed")
    return buf.value.decode()
