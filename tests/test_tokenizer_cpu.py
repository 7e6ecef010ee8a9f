"""Host tokenizers (src/gten/tokenizer.{h,cpp}; row f4): the library's C++ tokenizers and the
oracle's Python restatement against the reference's own ids and bytes.

* tests/golden/tokenizer_cases.json holds the compiled reference's encode ids and decode bytes
  for the four chat-program configurations (nanochat.cpp:188-229); the oracle and the library
  must reproduce them (these tests read the reference's vocabulary files and skip without the
  reference checkout);
* the live compiled reference (oracle/_ref) on further seeded strings, where it was built;
* synthetic vocabularies written by the tests (no reference needed) that exercise every rule the
  reference has: equal strings (bsearch's pick, the last id in the GPT-2 map), pieces with a NUL,
  byte pieces, BOS-space stripping, tied merge scores, scores at -1e10, missing single bytes,
  records past the end of a GPT-2 file;
* error statuses (missing or short files, a too-small id buffer).
No GPU is used: the tokenizers are host code.
"""
import json
import os
import random
import struct

import pytest

import gten_b200 as G
from gten_b200 import tokenizer as T
from oracle.oracle import reference_dir
from oracle.tokenizer_oracle import Gpt2Oracle, LlamaOracle, ReferenceTokenizer, for_model, gpt2_split

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden", "tokenizer_cases.json")
MODELS = ("tinyllama", "zephyr", "minicpm", "openelm")


def assets_dir():
    ref = reference_dir()
    d = os.path.join(ref, "assets", "tokenizers") if ref else None
    if not d or not os.path.isdir(d):
        pytest.skip("the reference's tokenizer files are not here (reference checkout absent)")
    return d


@pytest.fixture(scope="module")
def golden():
    with open(GOLDEN) as f:
        g = json.load(f)
    g["texts"] = [bytes.fromhex(t) for t in g["texts"]]
    return g


@pytest.mark.parametrize("name", MODELS)
def test_oracle_matches_reference_golden(golden, name):
    o = for_model(name, assets_dir())
    m = golden["models"][name]
    for text, ids in zip(golden["texts"], m["encode"]):
        assert o.encode(text) == ids, text
    for prev, cases in m["decode"].items():
        for i, hexb in cases:
            assert o.decode(int(prev), i) == bytes.fromhex(hexb), (prev, i)


@pytest.mark.parametrize("name", MODELS)
def test_library_matches_reference_golden(golden, name):
    tok = T.for_model(name, assets_dir())
    m = golden["models"][name]
    for text, ids in zip(golden["texts"], m["encode"]):
        assert tok.encode(text) == ids, text
    for prev, cases in m["decode"].items():
        for i, hexb in cases:
            assert tok.decode(int(prev), i) == bytes.fromhex(hexb), (prev, i)
    assert tok.eos_token == for_model(name, assets_dir()).eos


def random_texts(seed, n, alphabet, max_len=64):
    rng = random.Random(seed)
    return [b"".join(rng.choice(alphabet) for _ in range(rng.randint(0, max_len))) for _ in range(n)]


MIXED = ([bytes([c]) for c in b"aeiouxyzAEZ059 '\t\n.,!?-<>"] +
         [s.encode() for s in ("é", "中", "の", "🙂", "'s", "'ve", "  ")] + [b"\x80", b"\xc3", b"\xff"])


@pytest.mark.parametrize("name", MODELS)
def test_library_matches_live_reference(name):
    lib = os.path.join(ROOT, "oracle", "_ref", "libgtenref.so")
    if not os.path.exists(lib):
        pytest.skip("reference harness not built")
    o = for_model(name, assets_dir())
    ref = ReferenceTokenizer(lib, o)
    tok = T.for_model(name, assets_dir())
    try:
        for text in random_texts(99, 150, MIXED) + [b" ".join(random_texts(5, 80, MIXED))]:
            assert tok.encode(text) == ref.encode(text), text
        rng = random.Random(3)
        for i in [rng.randrange(tok.vocab_size) for _ in range(300)]:
            for prev in (0, 1, i):
                assert tok.decode(prev, i) == ref.decode(prev, i), (prev, i)
    finally:
        ref.close()


# ---- synthetic vocabularies (no reference needed)

def write_sp(path, pieces, scores, max_len=None):
    with open(path, "wb") as f:
        f.write(struct.pack("<i", max_len or max(len(p) for p in pieces)))
        for p, s in zip(pieces, scores):
            f.write(struct.pack("<fi", s, len(p)))
            f.write(p)


def sp_vocab(rng):
    pieces = [b"<unk>", b"\n<s>\n", b"\n</s>\n"] + [b"<0x%02X>" % b for b in range(256)]
    letters = [bytes([c]) for c in b"abcde xyz'!"] + ["é".encode(), "中".encode()]
    pieces += letters
    # merges of 2-4 letters, some repeated (equal strings at different ids)
    for _ in range(300):
        pieces.append(b"".join(rng.choice(letters[:9]) for _ in range(rng.randint(2, 4))))
    pieces += [b" ", b"ab", b"x\x00y", b"<0x4G>", b" <0x41>", b"<0x7>", b"<0x+5>", b" a b"]
    # scores: small integers (many ties), a few at or below -1e10
    scores = [float(rng.randint(-6, 0)) for _ in pieces]
    for k in rng.sample(range(259, len(pieces)), 12):
        scores[k] = -1e10 if k % 2 else -3e10
    return pieces, scores


@pytest.mark.parametrize("seed", [1, 2, 3])
def test_sentencepiece_synthetic_matches_oracle(tmp_path, seed):
    rng = random.Random(seed)
    pieces, scores = sp_vocab(rng)
    path = str(tmp_path / "sp.bin")
    write_sp(path, pieces, scores)
    n = len(pieces)
    args = (n, 2, b"pre ", b" post", [1, 7], [9])
    o = LlamaOracle(path, *args)
    tok = T.LLamaTokenizer(path, *args)
    alphabet = [bytes([c]) for c in b"abcdexyz '!q"] + ["é".encode(), "中".encode(), b"\x80", b"\xff", b"\x00"]
    for text in random_texts(seed, 200, alphabet, 40):
        assert tok.encode(text) == o.encode(text), text
    for prev in (0, 1, 5):
        for i in list(range(-2, n + 3)):
            if i < 0:
                assert tok.decode(prev, i) == b""
            else:
                assert tok.decode(prev, i) == o.decode(prev, i), (prev, i, pieces[i] if i < n else None)
    # equal strings resolve as the reference's sorted binary search does
    assert tok.encode(b"") == [1, 7] + o.encode_internal(b"pre  post") + [9]
    check_live_reference(o, tok, random_texts(seed + 10, 100, alphabet, 40), range(n + 2))


def check_live_reference(o, tok, texts, ids):
    """The same vocabulary file through the compiled reference, where it was built."""
    lib = os.path.join(ROOT, "oracle", "_ref", "libgtenref.so")
    if not os.path.exists(lib):
        return
    ref = ReferenceTokenizer(lib, o)
    try:
        for text in texts:
            assert tok.encode(text) == ref.encode(text), text
        for prev in (0, 1):
            for i in ids:
                assert tok.decode(prev, i) == ref.decode(prev, i), (prev, i)
    finally:
        ref.close()


def test_sentencepiece_without_prompt_strings(tmp_path):
    pieces, scores = sp_vocab(random.Random(4))
    path = str(tmp_path / "sp.bin")
    write_sp(path, pieces, scores)
    o = LlamaOracle(path, len(pieces), 2)
    tok = T.LLamaTokenizer(path, len(pieces), 2)
    assert tok.encode(b"") == o.encode(b"") == []
    assert tok.encode(b"\x00abc") == []  # encoded as a C string: empty
    assert tok.encode(b"ab\x00cd") == o.encode(b"ab")


def write_gpt2(path, words, truncate_last=0):
    data = b"".join(struct.pack("<I", len(w)) + w for w in words)
    with open(path, "wb") as f:
        f.write(data[:len(data) - truncate_last])


def gpt2_vocab(rng, drop_bytes=()):
    words = [bytes([b]) for b in range(256) if b not in drop_bytes]
    chunks = [b"a", b"b", b"c", b" ", b"'", b"1", b"2", b"\n", b"!", b"\xc3\xa9", b"  "]
    for _ in range(400):
        words.append(b"".join(rng.choice(chunks) for _ in range(rng.randint(2, 5))))
    words += [b"ab", b"x\x00y", b"ab"]  # an equal string: the later id wins
    return words


@pytest.mark.parametrize("seed,drop", [(1, ()), (2, (ord("!"), ord("\n"), 0xA9))])
def test_gpt2_synthetic_matches_oracle(tmp_path, seed, drop, capfd):
    rng = random.Random(seed)
    words = gpt2_vocab(rng, drop)
    path = str(tmp_path / "g.bin")
    write_gpt2(path, words)
    n_vocab = len(words) + 20  # ids past the file's end repeat its last record
    o = Gpt2Oracle(path, n_vocab, 7)
    tok = T.Gpt2Tokenizer(path, n_vocab, 7)
    alphabet = [bytes([c]) for c in b"abcq12 '\t\n!?"] + [b"'s", b"'ll", "é".encode(), b"\xff", b"\x00"]
    for text in random_texts(seed, 250, alphabet, 48):
        assert tok.encode(text) == o.encode(text), text
    for i in range(-3, n_vocab + 3):
        assert tok.decode(0, i) == o.decode(0, i), i
    assert tok.decode(0, n_vocab - 1) == words[-1]
    check_live_reference(o, tok, random_texts(seed + 10, 100, alphabet, 48), range(n_vocab + 2))
    capfd.readouterr()


def test_gpt2_split_rules():
    """The split pattern's leftmost-first alternation, as std::regex matches it."""
    assert gpt2_split(b"\n    return") == [b"\n   ", b" return"]
    assert gpt2_split(b"a    b") == [b"a", b"   ", b" b"]
    assert gpt2_split(b"  \xff") == [b" ", b" \xff"]
    assert gpt2_split(b"?!'ll'x") == [b"?!'", b"ll", b"'", b"x"]
    assert gpt2_split(b"x  ") == [b"x", b"  "]
    assert gpt2_split(b"\t\tx") == [b"\t", b"\t", b"x"]
    assert gpt2_split(b" \t x") == [b" \t", b" x"]
    assert gpt2_split(b"it's 12ab") == [b"it", b"'s", b" 12", b"ab"]


def test_errors(tmp_path):
    with pytest.raises(G.GtenError, match="status 1"):
        T.LLamaTokenizer(str(tmp_path / "missing.bin"), 10, 2)
    pieces, scores = sp_vocab(random.Random(5))
    path = str(tmp_path / "sp.bin")
    write_sp(path, pieces, scores)
    with pytest.raises(G.GtenError, match="status 4"):
        T.LLamaTokenizer(path, len(pieces) + 1, 2)  # fewer records than vocab_size
    gp = str(tmp_path / "g.bin")
    write_gpt2(gp, gpt2_vocab(random.Random(5)), truncate_last=1)
    with pytest.raises(G.GtenError, match="status 4"):
        T.Gpt2Tokenizer(gp, 1000, 7)  # the file ends inside a record
    # a buffer too small: GTN_ERR_ARG with the needed count; the binding then retries
    tok = T.LLamaTokenizer(path, len(pieces), 2, tokens_prefix=[1] * 100)
    import ctypes as C
    out = (C.c_int32 * 4)()
    n = C.c_int(0)
    rc = T._lib().gtn_tokenizer_encode(tok._h, b"abc", 3, out, 4, C.byref(n))
    assert rc == 1 and n.value > 100
    assert len(tok.encode(b"abc")) == n.value
