"""Text in, text out on the GPU: greedy_text / topk_text (sampler.cpp:11-53, :63-143 with their
tokenization, EOS stop and printed bytes) through the library's tokenizer and model, against the
oracle's tokenizer restatement and model wiring. The vocabularies are synthetic files written by
the test (the reference's own vocabularies are pinned on the CPU in test_tokenizer_cpu.py)."""
import random
import struct

import numpy as np
import pytest

import gten_b200 as G
from gten_b200 import gtenfile
from gten_b200 import tokenizer as T
from helpers import Q8

pytestmark = pytest.mark.gpu


def cpu_pack(orc):
    def pack(w, dt):
        return orc.pack_q8(w.numpy()) if dt == Q8 else orc.pack_q4(w.numpy())
    return pack


def write_sp(path, n, rng):
    pieces = [b"<unk>", b"\n<s>\n", b"\n</s>\n"] + [b"<0x%02X>" % b for b in range(256)]
    letters = [bytes([c]) for c in b"abcdefghij klmnop"]
    pieces += letters
    seen = set(pieces)
    while len(pieces) < n:
        p = b"".join(rng.choice(letters) for _ in range(rng.randint(2, 5)))
        if p not in seen:
            seen.add(p)
            pieces.append(p)
    with open(path, "wb") as f:
        f.write(struct.pack("<i", max(len(p) for p in pieces)))
        for p in pieces:
            f.write(struct.pack("<fi", float(-rng.randint(0, 50)), len(p)))
            f.write(p)


def write_gpt2(path, n, rng):
    words = [bytes([b]) for b in range(256)]
    chunks = [b"a", b"b", b"c", b"d", b" ", b"e", b"\n", b"'", b"x"]
    seen = set(words)
    while len(words) < n:
        w = b"".join(rng.choice(chunks) for _ in range(rng.randint(2, 7)))
        if w not in seen:
            seen.add(w)
            words.append(w)
    with open(path, "wb") as f:
        for w in words:
            f.write(struct.pack("<I", len(w)) + w)


CASES = {
    # n_vocab, n_embd, n_layers, n_heads, n_kv_heads, n_ffn, family
    "sentencepiece": [1000, 256, 2, 4, 2, 512, 0],
    "gpt2": [100352, 128, 2, 2, 2, 256, 1],  # the GPT-2 tokenizer's fixed ids reach 100257
}


@pytest.mark.parametrize("kind", list(CASES))
def test_greedy_text_matches_oracle(orc, gpu, tmp_path, kind):
    from oracle.oracle import OracleModel
    from oracle.tokenizer_oracle import Gpt2Oracle, LlamaOracle
    dims = CASES[kind]
    n_vocab = dims[0]
    rng = random.Random(11)
    path = str(tmp_path / "vocab.bin")
    prompt = b"abc dab fig hij kalm\nnop 'e"
    if kind == "sentencepiece":
        write_sp(path, n_vocab, rng)
        mk_oracle = lambda eos: LlamaOracle(path, n_vocab, eos, b"user\n", b"", [1], [2])  # noqa: E731
        mk_tok = lambda eos: T.LLamaTokenizer(path, n_vocab, eos, "user\n", "", [1], [2])  # noqa: E731
    else:
        write_gpt2(path, n_vocab, rng)
        mk_oracle = lambda eos: Gpt2Oracle(path, n_vocab, eos)  # noqa: E731
        mk_tok = lambda eos: T.Gpt2Tokenizer(path, n_vocab, eos)  # noqa: E731
    img = gtenfile.synthetic_image(6, Q8, 21, cpu_pack(orc), dims=dims, std=0.05, gain_std=0.1)
    n_predict = 64
    max_ctx = 2 * n_predict
    ptoks = mk_oracle(0).encode(prompt)
    assert 0 < len(ptoks) < n_predict - 8
    full = list(OracleModel(orc, 6, Q8, max_ctx, img, dims=dims).greedy(np.array(ptoks, np.int32),
                                                                        n_predict - len(ptoks)))
    m = G.Model(G.CUSTOM, Q8, max_ctx, dims=dims)
    m.load(img)
    # an eos that never comes: every id up to n_predict; then one that stops the loop early
    for eos in (n_vocab + 1, full[6]):
        o, tok = mk_oracle(eos), mk_tok(eos)
        ids, text = T.greedy_text(m, tok, prompt, n_predict)
        want = full[:full.index(eos)] if eos in full else full
        assert ids == want
        pieces, prev = [], 1
        for t in want:
            pieces.append(o.decode(prev, t))
            prev = t
        assert text == b"".join(pieces)
        tok.close()
    m.close()
