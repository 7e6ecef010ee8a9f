"""Test infrastructure only: a plain-Python restatement of the reference's two host tokenizers.

This module is a checker. Only tests/ and tests/golden/ may import it; the product tokenizers
are the C++ ones in the library (gten_b200.tokenizer binds them). Its outputs are pinned against
the reference's own compiled tokenizer (oracle/_ref, built from src/gten/tokenizer.cpp by
build_ref.sh) through tests/golden/tokenizer_cases.json.

LLamaTokenizer (src/gten/tokenizer.cpp:30-245, llama2.c's SentencePiece-BPE encoder):
  * vocabulary file (tokenizer.cpp:46-64): int32 max_token_length, then per token float32 score,
    int32 length, bytes; strings compare as C strings (up to the first NUL);
  * lookups (tokenizer.cpp:95-100, 139-147): qsort of (string, id) by strcmp, then bsearch. Among
    equal strings (MiniCPM's vocabulary holds " " twice) the element the binary search meets
    first is returned; the sort keeps equal strings in id order;
  * encode (tokenizer.cpp:103-132): prompt_prefix + text + prompt_suffix, encoded up to its first
    NUL, between tokens_prefix and tokens_suffix;
  * encode_internal (tokenizer.cpp:134-241): the id of " " first (only for non-empty text), then
    one token per UTF-8 group (a byte and at most 3 following continuation bytes) or, when the
    group is not in the vocabulary, one token per byte (byte + 3); then repeatedly merge the
    adjacent pair whose concatenation has the highest score (strictly above -1e10; the leftmost
    pair among equal scores);
  * decode (tokenizer.cpp:77-93): "" for ids >= vocab_size; after id 1 a leading space is dropped;
    pieces that scan as "<0x%02hhX>" become that single byte; the result is a C string.

Gpt2Tokenizer (tokenizer.cpp:249-334):
  * vocabulary file (tokenizer.cpp:249-268): per token uint32 length, bytes; n_vocab records are
    read; when the file holds fewer, the reference's reads past its end leave the last record's
    string in place, so the remaining ids repeat it (observed on the compiled reference: Zephyr's
    file holds 100,256 records for n_vocab 100,352);
  * string -> id keeps the last id of equal strings; id -> string is "" for unknown ids;
  * encode (tokenizer.cpp:278-331): split with the pattern
    's|'t|'re|'ve|'m|'ll|'d| ?[[:alpha:]]+| ?[[:digit:]]+| ?[^\\s[:alpha:][:digit:]]+|\\s+(?!\\S)|\\s+
    (std::regex, ECMAScript, "C" locale: ASCII classes), then each word greedily by its longest
    prefix in the vocabulary; after every such prefix that does not end the word, the next single
    byte is emitted as its own token (the loop's `j == i` branch also runs after a match), and
    bytes with no entry are skipped (the reference prints a warning);
    fixed prefix ids {27, 91, 882, 91, 29, 397} and suffix ids {100257, 198, 27, 91, 78191, 91, 397}.
"""
from __future__ import annotations

import ctypes
import struct
from typing import Dict, List, Optional, Sequence

_libc = ctypes.CDLL(None)
_libc.sscanf.restype = ctypes.c_int


def _cstr(b: bytes) -> bytes:
    i = b.find(b"\0")
    return b if i < 0 else b[:i]


class LlamaOracle:
    def __init__(self, path: str, vocab_size: int, eos: int, prompt_prefix: bytes = b"",
                 prompt_suffix: bytes = b"", tokens_prefix: Sequence[int] = (), tokens_suffix: Sequence[int] = ()):
        self.path = path
        data = open(path, "rb").read()
        self.max_token_length = struct.unpack_from("<i", data, 0)[0]
        off = 4
        self.vocab: List[bytes] = []
        self.scores: List[float] = []
        for _ in range(vocab_size):
            score, n = struct.unpack_from("<fi", data, off)
            off += 8
            self.vocab.append(data[off:off + n])
            self.scores.append(score)
            off += n
        self.vocab_size, self.eos = vocab_size, eos
        self.prompt_prefix, self.prompt_suffix = prompt_prefix, prompt_suffix
        self.tokens_prefix, self.tokens_suffix = list(tokens_prefix), list(tokens_suffix)
        # qsort by strcmp (equal strings stay in id order), then bsearch
        self.sorted = sorted(((_cstr(s), i) for i, s in enumerate(self.vocab)), key=lambda t: t[0])

    def lookup(self, key: bytes) -> int:
        lo, hi = 0, len(self.sorted)
        while lo < hi:
            mid = (lo + hi) // 2
            k = self.sorted[mid][0]
            if key < k:
                hi = mid
            elif key > k:
                lo = mid + 1
            else:
                return self.sorted[mid][1]
        return -1

    def encode_internal(self, text: bytes) -> List[int]:
        text = _cstr(text)
        out: List[int] = []
        if text:
            out.append(self.lookup(b" "))
        i, n = 0, len(text)
        while i < n:
            j = i + 1
            while j < n and (text[j] & 0xC0) == 0x80 and j - i < 4:
                j += 1
            group = text[i:j]
            tid = self.lookup(group)
            if tid != -1:
                out.append(tid)
            else:
                out.extend(b + 3 for b in group)
            i = j
        while True:
            best, best_id, best_idx = -1e10, -1, -1
            for k in range(len(out) - 1):
                tid = self.lookup(_cstr(self.vocab[out[k]]) + _cstr(self.vocab[out[k + 1]]))
                if tid != -1 and self.scores[tid] > best:
                    best, best_id, best_idx = self.scores[tid], tid, k
            if best_idx == -1:
                break
            out[best_idx] = best_id
            del out[best_idx + 1]
        return out

    def encode(self, text: bytes) -> List[int]:
        return self.tokens_prefix + self.encode_internal(self.prompt_prefix + text + self.prompt_suffix) \
            + self.tokens_suffix

    def decode(self, prev: int, token: int) -> bytes:
        if token >= self.vocab_size:
            return b""
        piece = _cstr(self.vocab[token])
        if prev == 1 and piece[:1] == b" ":
            piece = piece[1:]
        v = ctypes.c_ubyte(0)
        if _libc.sscanf(ctypes.c_char_p(piece), b"<0x%02hhX>", ctypes.byref(v)) == 1:
            return _cstr(bytes([v.value]))
        return piece


# "C" locale classes of the GPT-2 split pattern
_SPACE = frozenset(b" \t\n\v\f\r")
_ALPHA = frozenset(range(ord("A"), ord("Z") + 1)) | frozenset(range(ord("a"), ord("z") + 1))
_DIGIT = frozenset(range(ord("0"), ord("9") + 1))
_CONTRACTIONS = (b"'s", b"'t", b"'re", b"'ve", b"'m", b"'ll", b"'d")


def _cls(c: int) -> int:
    return 0 if c in _SPACE else (1 if c in _ALPHA else (2 if c in _DIGIT else 3))


def gpt2_split(text: bytes) -> List[bytes]:
    """The matches of the split pattern, leftmost-first alternation as ECMAScript evaluates it."""
    words, p, n = [], 0, len(text)
    while p < n:
        m = None
        for c in _CONTRACTIONS:
            if text.startswith(c, p):
                m = p + len(c)
                break
        if m is None:
            for want in (1, 2, 3):  # ' ?[[:alpha:]]+', ' ?[[:digit:]]+', ' ?[^\s[:alpha:][:digit:]]+'
                s = p + 1 if text[p] == 0x20 and p + 1 < n and _cls(text[p + 1]) == want else p
                if s < n and _cls(text[s]) == want:
                    e = s
                    while e < n and _cls(text[e]) == want:
                        e += 1
                    m = e
                    break
        if m is None:  # text[p] is whitespace: '\s+(?!\S)' then '\s+'
            e = p
            while e < n and _cls(text[e]) == 0:
                e += 1
            m = e if (e == n or e - p == 1) else e - 1
        words.append(text[p:m])
        p = m
    return words


class Gpt2Oracle:
    PREFIX = [27, 91, 882, 91, 29, 397]
    SUFFIX = [100257, 198, 27, 91, 78191, 91, 397]

    def __init__(self, path: str, n_vocab: int, eos: int):
        self.path = path
        data = open(path, "rb").read()
        off, last = 0, b""
        self.id_to_token: Dict[int, bytes] = {}
        self.token_to_id: Dict[bytes, int] = {}
        for i in range(n_vocab):
            if off + 4 <= len(data):
                n = struct.unpack_from("<I", data, off)[0]
                last = data[off + 4:off + 4 + n]
                off += 4 + n
            self.token_to_id[last] = i
            self.id_to_token[i] = last
        self.n_vocab, self.eos = n_vocab, eos

    def encode(self, text: bytes) -> List[int]:
        out = list(self.PREFIX)
        for w in gpt2_split(text):
            i, n = 0, len(w)
            while i < n:
                j = n
                while j > i and w[i:j] not in self.token_to_id:
                    j -= 1
                if j > i:
                    out.append(self.token_to_id[w[i:j]])
                    i = j
                    if i == n:
                        break
                # i == j here in both cases (tokenizer.cpp:318-327): the byte at i is looked up
                # alone and emitted, or skipped when the vocabulary lacks it
                tid = self.token_to_id.get(w[i:i + 1])
                if tid is not None:
                    out.append(tid)
                i += 1
        return out + self.SUFFIX

    def decode(self, prev: int, token: int) -> bytes:
        return _cstr(self.id_to_token.get(token, b""))


def for_model(name: str, assets: str) -> Optional[object]:
    """The tokenizer each model uses in the reference's chat program (nanochat.cpp:188-229)."""
    if name == "tinyllama":
        return LlamaOracle(f"{assets}/tinyllama_tokenizer.bin", 32000, 32002, b"user\n", b"", [1, 32001],
                           [32002, 29871, 13, 32001, 20255, 13])
    if name == "zephyr":
        return Gpt2Oracle(f"{assets}/zephyr_tokenizer.bin", 100352, 100257)
    if name == "minicpm":
        return LlamaOracle(f"{assets}/minicpm_tokenizer.bin", 122753, 2, "<用户>".encode(), "<AI>".encode())
    if name == "openelm":
        return LlamaOracle(f"{assets}/tinyllama_tokenizer.bin", 32000, 32002, b"", b"", [1], [])
    return None


class ReferenceTokenizer:
    """The reference's own LLamaTokenizer / Gpt2Tokenizer, compiled into oracle/_ref/libgtenref.so
    (oracle/tok_harness.cpp over src/gten/tokenizer.cpp), driven through ctypes."""

    def __init__(self, lib_path: str, oracle_tok):
        L = ctypes.CDLL(lib_path)
        c = ctypes
        L.tokref_llama.restype = c.c_void_p
        L.tokref_llama.argtypes = [c.c_char_p, c.c_int, c.c_int, c.c_char_p, c.c_char_p, c.c_void_p, c.c_int,
                                   c.c_void_p, c.c_int]
        L.tokref_gpt2.restype = c.c_void_p
        L.tokref_gpt2.argtypes = [c.c_char_p, c.c_int, c.c_int]
        L.tokref_encode.argtypes = [c.c_void_p, c.c_char_p, c.c_int, c.c_void_p, c.c_int]
        L.tokref_decode.argtypes = [c.c_void_p, c.c_int, c.c_int, c.c_char_p, c.c_int]
        L.tokref_free.argtypes = [c.c_void_p, c.c_int]
        self._L = L
        o = oracle_tok
        if isinstance(o, Gpt2Oracle):
            self.kind = 1
            self._h = L.tokref_gpt2(o.path.encode(), o.n_vocab, o.eos)
        else:
            self.kind = 0
            tp = (c.c_int * max(1, len(o.tokens_prefix)))(*o.tokens_prefix)
            ts = (c.c_int * max(1, len(o.tokens_suffix)))(*o.tokens_suffix)
            self._h = L.tokref_llama(o.path.encode(), o.vocab_size, o.eos, o.prompt_prefix, o.prompt_suffix, tp,
                                     len(o.tokens_prefix), ts, len(o.tokens_suffix))

    def encode(self, text: bytes) -> List[int]:
        cap = len(text) + 64
        out = (ctypes.c_int * cap)()
        n = self._L.tokref_encode(self._h, text, len(text), out, cap)
        return list(out[:n])

    def decode(self, prev: int, token: int) -> bytes:
        buf = ctypes.create_string_buffer(4096)
        n = self._L.tokref_decode(self._h, prev, token, buf, 4096)
        return buf.raw[:n]

    def close(self) -> None:
        if self._h:
            self._L.tokref_free(self._h, self.kind)
            self._h = None
