"""Host tokenizers of the reference (src/gten/tokenizer.{h,cpp}) through the library's C ABI.

``LLamaTokenizer`` and ``Gpt2Tokenizer`` take the reference's constructor arguments
(tokenizer.h:27-31, :51) and vocabulary files, and ``encode`` / ``decode`` return the reference's
ids and bytes for every input (``decode`` returns bytes: a piece may be part of a UTF-8
character). ``for_model`` builds the tokenizer each model uses in the reference's chat program
(nanochat.cpp:188-229). ``greedy_text`` and ``topk_text`` are greedy_sample / topk_sample
(sampler.cpp:11-53, :63-143) with their tokenization and EOS stop, on top of the model's
``generate`` / ``generate_topk``.

The work runs in C++ inside lib/libgten_b200.so (host code, no GPU needed).
"""
from __future__ import annotations

import ctypes as C
import os
from typing import List, Optional, Sequence, Tuple, Union

from . import _check, lib

Text = Union[str, bytes]

_bound = False


def _lib() -> C.CDLL:
    global _bound
    L = lib()
    if not _bound:
        L.gtn_tokenizer_create_llama.argtypes = [C.c_char_p, C.c_int, C.c_int, C.c_char_p, C.c_char_p, C.c_void_p,
                                                 C.c_int, C.c_void_p, C.c_int, C.POINTER(C.c_void_p)]
        L.gtn_tokenizer_create_gpt2.argtypes = [C.c_char_p, C.c_int, C.c_int, C.POINTER(C.c_void_p)]
        L.gtn_tokenizer_free.argtypes = [C.c_void_p]
        L.gtn_tokenizer_free.restype = None
        L.gtn_tokenizer_vocab_size.argtypes = [C.c_void_p]
        L.gtn_tokenizer_eos.argtypes = [C.c_void_p]
        L.gtn_tokenizer_encode.argtypes = [C.c_void_p, C.c_char_p, C.c_size_t, C.c_void_p, C.c_int,
                                           C.POINTER(C.c_int)]
        L.gtn_tokenizer_decode.argtypes = [C.c_void_p, C.c_int, C.c_int, C.POINTER(C.c_void_p),
                                           C.POINTER(C.c_size_t)]
        _bound = True
    return L


def _bytes(s: Text) -> bytes:
    return s.encode("utf-8") if isinstance(s, str) else bytes(s)


def _ids(xs: Sequence[int]):
    arr = (C.c_int32 * max(1, len(xs)))(*xs)
    return arr, len(xs)


class Tokenizer:
    """Tokenizer (abc.h:31-54): encode(prompt) -> ids, decode(prev_token, token) -> bytes."""

    def __init__(self, handle: C.c_void_p):
        self._h = handle
        L = _lib()
        self.vocab_size = L.gtn_tokenizer_vocab_size(self._h)
        self.eos_token = L.gtn_tokenizer_eos(self._h)

    def encode(self, prompt: Text) -> List[int]:
        L = _lib()
        data = _bytes(prompt)
        cap = len(data) + 64  # the reference yields at most one id per byte plus its fixed ids
        while True:
            out = (C.c_int32 * cap)()
            n = C.c_int(0)
            rc = L.gtn_tokenizer_encode(self._h, data, len(data), out, cap, C.byref(n))
            if rc != 0 and n.value > cap:
                cap = n.value
                continue
            _check(rc, "tokenizer_encode")
            return list(out[:n.value])

    def decode(self, prev_token: int, token: int) -> bytes:
        p, n = C.c_void_p(), C.c_size_t()
        _check(_lib().gtn_tokenizer_decode(self._h, prev_token, token, C.byref(p), C.byref(n)), "tokenizer_decode")
        return C.string_at(p, n.value) if n.value else b""

    def decode_all(self, tokens: Sequence[int], first_prev: int = 1) -> bytes:
        """The bytes the reference's sampler prints for `tokens` (each decoded after its predecessor;
        the first after id 1, as sampler.cpp:47 does)."""
        out, prev = [], first_prev
        for t in tokens:
            out.append(self.decode(prev, t))
            prev = t
        return b"".join(out)

    def close(self) -> None:
        if self._h:
            _lib().gtn_tokenizer_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class LLamaTokenizer(Tokenizer):
    """LLamaTokenizer(path, vocab_size, eos, prompt_prefix, prompt_suffix, tokens_prefix, tokens_suffix)."""

    def __init__(self, path: str, vocab_size: int, eos: int, prompt_prefix: Text = "", prompt_suffix: Text = "",
                 tokens_prefix: Sequence[int] = (), tokens_suffix: Sequence[int] = ()):
        tp, ntp = _ids(list(tokens_prefix))
        ts, nts = _ids(list(tokens_suffix))
        h = C.c_void_p()
        _check(_lib().gtn_tokenizer_create_llama(os.fsencode(path), vocab_size, eos, _bytes(prompt_prefix),
                                                 _bytes(prompt_suffix), tp, ntp, ts, nts, C.byref(h)),
               "tokenizer_create_llama")
        super().__init__(h)


class Gpt2Tokenizer(Tokenizer):
    """Gpt2Tokenizer(vocab_path, n_vocab, eos)."""

    def __init__(self, vocab_path: str, n_vocab: int, eos: int):
        h = C.c_void_p()
        _check(_lib().gtn_tokenizer_create_gpt2(os.fsencode(vocab_path), n_vocab, eos, C.byref(h)),
               "tokenizer_create_gpt2")
        super().__init__(h)


# nanochat.cpp:188-229: file, vocabulary size, eos, prompt strings and fixed ids per model
_MODELS = {
    "tinyllama": ("llama", "tinyllama_tokenizer.bin", 32000, 32002, "user\n", "", [1, 32001],
                  [32002, 29871, 13, 32001, 20255, 13]),
    "zephyr": ("gpt2", "zephyr_tokenizer.bin", 100352, 100257),
    "minicpm": ("llama", "minicpm_tokenizer.bin", 122753, 2, "<用户>", "<AI>", [], []),
    "openelm": ("llama", "tinyllama_tokenizer.bin", 32000, 32002, "", "", [1], []),
}


def for_model(name: str, assets_dir: str) -> Tokenizer:
    """The tokenizer of model `name` ("tinyllama", "zephyr", "minicpm", or an "openelm*" size) as the
    reference's chat program builds it, from the directory holding its tokenizer files."""
    key = "openelm" if name.startswith("openelm") else name
    if key not in _MODELS:
        raise ValueError(f"unknown model {name!r}")
    cfg = _MODELS[key]
    path = os.path.join(assets_dir, cfg[1])
    if cfg[0] == "gpt2":
        return Gpt2Tokenizer(path, cfg[2], cfg[3])
    return LLamaTokenizer(path, cfg[2], cfg[3], cfg[4], cfg[5], cfg[6], cfg[7])


def _until_eos(ids: Sequence[int], eos: int) -> List[int]:
    out = []
    for t in ids:
        if int(t) == eos:
            break
        out.append(int(t))
    return out


def greedy_text(model, tokenizer: Tokenizer, prompt: Text, n_predict: Optional[int] = None) -> Tuple[List[int], bytes]:
    """greedy_sample (sampler.cpp:11-53): encode the prompt, greedy ids until the eos id or until
    prompt + ids reach n_predict tokens (the reference's min(inference ctx, train ctx); default: the
    model's max_ctx), and the bytes the reference prints for them. Returns (ids, text)."""
    tokens = tokenizer.encode(prompt)
    n_predict = model.max_ctx if n_predict is None else n_predict
    n_gen = n_predict - len(tokens)
    if n_gen <= 0:
        return [], b""
    ids = _until_eos(model.generate(tokens, n_gen), tokenizer.eos_token)
    return ids, tokenizer.decode_all(ids)


def topk_text(model, tokenizer: Tokenizer, prompt: Text, temp: float, top_k: int, rng,
              n_predict: Optional[int] = None) -> Tuple[List[int], bytes]:
    """topk_sample (sampler.cpp:63-143) with the caller's seeded generator (the reference seeds from
    std::random_device): as greedy_text, with each id drawn as the reference draws it."""
    tokens = tokenizer.encode(prompt)
    n_predict = model.max_ctx if n_predict is None else n_predict
    n_gen = n_predict - len(tokens)
    if n_gen <= 0:
        return [], b""
    ids = _until_eos(model.generate_topk(tokens, n_gen, temp, top_k, rng), tokenizer.eos_token)
    return ids, tokenizer.decode_all(ids)
