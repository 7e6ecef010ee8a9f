"""Generates tests/golden/tokenizer_cases.json from the REFERENCE's own tokenizers.

Run in the build container, where the reference checkout (its src/gten/tokenizer.cpp and
assets/tokenizers/*.bin) exists. oracle/build_ref.sh compiles the unmodified tokenizer.cpp with
oracle/tok_harness.cpp into oracle/_ref/libgtenref.so; this script drives it through
oracle.tokenizer_oracle.ReferenceTokenizer for the four configurations the reference's chat program
builds (nanochat.cpp:188-229: tinyllama, zephyr, minicpm, openelm) and records, per configuration:

* encode: the ids of every case text (hand-written texts covering contractions, digits, runs of
  whitespace, multi-byte UTF-8, invalid UTF-8, an embedded NUL, chat-tag lookalikes; seeded
  random strings over a mixed alphabet; one ~4 KB text joining them);
* decode: the bytes of decode(prev, id) for prev in {0, 1} over the special, byte-piece and
  seeded random ids, and ids at and past the vocabulary's end.

Only ids and decoded bytes are stored, not the vocabularies. Texts are stored as hex.

Usage: python tests/golden/make_tokenizer_golden.py [reference_dir]
"""
import json
import os
import random
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle.oracle import reference_dir  # noqa: E402
from oracle.tokenizer_oracle import ReferenceTokenizer, for_model  # noqa: E402

MODELS = ("tinyllama", "zephyr", "minicpm", "openelm")

HAND = [
    "", " ", "  ", "a", "Hello world", "Hello, world!",
    "I'm sure it's fine, they've said we'll see what'd happen.",
    "Order 66 shipped 2024-05-01 at 13:45; total $1,234.56 (incl. 7% tax).",
    "tabs\tand\nnewlines\r\n  double  spaces   end   ",
    "naïve café résumé — déjà vu",
    "日本語のテキストを分割します。",
    "中文分词测试，句号。",
    "emoji 🙂👍 and symbols ©®™ ∑∞",
    "def f(x):\n    return x ** 2  # square\n",
    "<0x41> <s> </s> <unk> <|endoftext|> <用户><AI>",
    "URL: https://example.com/path?q=1&r=two#frag",
    "MiXeD CaSe WoRdS and ALLCAPS and lowercase",
    "'s 't 're 've 'm 'll 'd ''' \"quoted\" it'S",
    "   leading and trailing   ",
    "\n\n\nblank lines\n\n",
    "a b and a b",
]
HAND_BYTES = [b"\xff\xfe\x80abc", b"\x80\x80\x80\x80\x80x", b"\xe4\xbd", b"abc\x00def", b"\x01\x02\x7f", b"\x00"]

ALPHABET = ([bytes([c]) for c in b"abcdefXYZ0123456789 '\t\n\r.,;:!?-_<>()/\"#"] +
            [s.encode() for s in ("é", "ü", "中", "文", "の", "🙂", "—", "'s", "'ll", "'re", "  ", "   ", " ")] +
            [b"\x80", b"\xbf", b"\xc3", b"\xe4", b"\xf0", b"\xff"])


def cases():
    rng = random.Random(20241202)
    texts = [t.encode("utf-8") for t in HAND] + HAND_BYTES
    rand = [b"".join(rng.choice(ALPHABET) for _ in range(rng.randint(0, 48))) for _ in range(120)]
    texts += rand
    texts.append(b" ".join(rand)[:4096])
    return texts


def decode_ids(name, n, rng):
    ids = list(range(0, 300)) + [n - 2, n - 1, n, n + 7]
    if name == "minicpm":
        ids += list(range(1080, 1350)) + [95320, 116876]
    if name == "zephyr":
        ids += [100255, 100256, 100257, 100300, 100351]
    if name in ("tinyllama", "openelm"):
        ids += [13, 29871, 29889, 31999]
    ids += [rng.randrange(n) for _ in range(200)]
    return ids


def main():
    ref = sys.argv[1] if len(sys.argv) > 1 else reference_dir()
    if not ref:
        sys.exit("reference checkout not found (argument, GTEN_REFERENCE_DIR or BASELINE.json reference_path)")
    lib = os.path.join(ROOT, "oracle", "_ref", "libgtenref.so")
    if not os.path.exists(lib):
        sys.exit("build oracle/_ref first: bash oracle/build_ref.sh")
    assets = os.path.join(ref, "assets", "tokenizers")
    texts = cases()
    out = {"texts": [t.hex() for t in texts], "models": {}}
    rng = random.Random(7)
    for name in MODELS:
        o = for_model(name, assets)
        r = ReferenceTokenizer(lib, o)
        n = o.n_vocab if hasattr(o, "n_vocab") else o.vocab_size
        enc = [r.encode(t) for t in texts]
        ids = decode_ids(name, n, rng)
        dec = {str(prev): [[i, r.decode(prev, i).hex()] for i in ids] for prev in (0, 1)}
        r.close()
        out["models"][name] = {"encode": enc, "decode": dec}
        print(name, len(texts), "texts,", sum(len(e) for e in enc), "ids,", len(ids), "decode ids")
    with open(os.path.join(HERE, "tokenizer_cases.json"), "w") as f:
        json.dump(out, f, separators=(",", ":"))


if __name__ == "__main__":
    main()
