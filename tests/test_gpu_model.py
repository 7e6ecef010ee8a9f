"""Model-level GPU parity: the engine (gtn_model_*) against the oracle's model wiring on small
custom architectures of each family (bit-exact logits and greedy tokens), and against the
reference's own greedy tokens on full-size TinyLlama (committed golden tokens; the live compiled
reference too where it is present)."""
import json
import os

import numpy as np
import pytest
import torch

import gten_b200 as G
from gten_b200 import gtenfile
from helpers import F16, Q4, Q8

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


def cpu_pack(orc):
    def pack(w, dt):
        return orc.pack_q8(w.numpy()) if dt == Q8 else orc.pack_q4(w.numpy())
    return pack


CUSTOM = {
    "llama": [1000, 256, 2, 4, 2, 512, 0],
    "zephyr": [777, 192, 2, 3, 3, 320, 1],
    "minicpm": [900, 128, 3, 2, 2, 288, 2],
    "openelm": [1100, 192, 2, 6, 2, 352, 3],
}


@pytest.mark.parametrize("name", list(CUSTOM))
@pytest.mark.parametrize("wdt", [Q8, Q4, F16])
def test_custom_model_matches_oracle(orc, gpu, name, wdt):
    from oracle.oracle import OracleModel
    dims = CUSTOM[name]
    img = gtenfile.synthetic_image(6, wdt, 99, cpu_pack(orc), dims=dims, std=0.05, gain_std=0.1)
    n_prompt, n_gen = 21, 12
    max_ctx = 2 * (n_prompt + n_gen)  # keeps the reference's qk rows apart (fp16 needs 2x)
    prompt = np.random.default_rng(5).integers(0, dims[0], n_prompt).astype(np.int32)
    om = OracleModel(orc, 6, wdt, max_ctx, img, dims=dims)
    m = G.Model(G.CUSTOM, wdt, max_ctx, dims=dims)
    m.load(img)
    # prefill logits, then one decode step
    assert np.array_equal(m.logits(prompt, 0), om.logits(prompt, 0))
    p2 = np.concatenate([prompt, [7]]).astype(np.int32)
    assert np.array_equal(m.logits(p2, n_prompt), om.logits(p2, n_prompt))
    # greedy decode from scratch
    om2 = OracleModel(orc, 6, wdt, max_ctx, img, dims=dims)
    assert np.array_equal(m.generate(prompt, n_gen), om2.greedy(prompt, n_gen))
    m.close()


def test_long_prefill_in_passes_matches_oracle(orc, gpu):
    """A 520-token prefill: the engine's activation image for the tensor-core GEMM holds 512 rows,
    so each projection runs in two passes (512 rows, then 8); logits and greedy ids must still be
    the oracle's bit for bit."""
    from oracle.oracle import OracleModel
    dims = CUSTOM["llama"]
    img = gtenfile.synthetic_image(6, Q8, 31, cpu_pack(orc), dims=dims, std=0.05, gain_std=0.1)
    n_prompt, n_gen = 520, 4
    max_ctx = 2 * (n_prompt + n_gen)
    prompt = np.random.default_rng(8).integers(0, dims[0], n_prompt).astype(np.int32)
    m = G.Model(G.CUSTOM, Q8, max_ctx, dims=dims)
    m.load(img)
    assert np.array_equal(m.logits(prompt, 0), OracleModel(orc, 6, Q8, max_ctx, img, dims=dims).logits(prompt, 0))
    assert np.array_equal(m.generate(prompt, n_gen), OracleModel(orc, 6, Q8, max_ctx, img, dims=dims).greedy(prompt, n_gen))
    m.close()


@pytest.mark.parametrize("name", list(CUSTOM))
@pytest.mark.parametrize("wdt", [Q8, Q4, F16])
@pytest.mark.parametrize("batch", [3, 11, 20, 40])
def test_batched_generation_matches_single_sequences(orc, gpu, name, wdt, batch):
    """The reference has no batching: each sequence of a batch must produce exactly the ids the
    oracle gives for it alone (batch 11 exercises a second 8-row tile of the fused GEMVs; 20 and
    40 run the decode steps' Q8/Q4 projections on the tensor-core GEMM, 40 with a partial second
    row tile; fp16 weights run the 8-lane CUDA-core kernel in tiles of 8 rows)."""
    from oracle.oracle import OracleModel
    dims = CUSTOM[name]
    img = gtenfile.synthetic_image(6, wdt, 77, cpu_pack(orc), dims=dims, std=0.05, gain_std=0.1)
    n_prompt, n_gen = 13, 9
    max_ctx = 2 * (n_prompt + n_gen)
    prompts = np.random.default_rng(batch).integers(0, dims[0], (batch, n_prompt)).astype(np.int32)
    m = G.Model(G.CUSTOM, wdt, max_ctx, max_batch=batch, dims=dims)
    m.load(img)
    got = m.generate_batch(prompts, n_gen)
    for b in range(batch):
        om = OracleModel(orc, 6, wdt, max_ctx, img, dims=dims)
        assert np.array_equal(got[b], om.greedy(prompts[b], n_gen)), f"sequence {b}"
    m.close()


def test_load_rejects_bad_images(orc, gpu):
    dims = CUSTOM["llama"]
    img = gtenfile.synthetic_image(6, Q8, 1, cpu_pack(orc), dims=dims)
    m = G.Model(G.CUSTOM, Q8, 16, dims=dims)
    bad = img.copy()
    bad[0] ^= 1
    with pytest.raises(G.GtenError, match="status 4"):
        m.load(bad)
    with pytest.raises(G.GtenError, match="status 4"):
        m.load(img[: img.size // 2])
    with pytest.raises(G.GtenError, match="status 1"):
        m.generate(np.array([1, 2, 3], np.int32), 2)  # not loaded yet
    m.load(img)
    with pytest.raises(G.GtenError, match="status 1"):
        m.generate(np.array([dims[0]], np.int32), 1)  # token id out of range
    m.close()


@pytest.mark.parametrize("name", ["llama", "minicpm"])
def test_load_file_matches_load(orc, gpu, name, tmp_path):
    """gtn_model_load_file (mapped .gten file) gives the same model as gtn_model_load from memory,
    including the padded-row records (MiniCPM's down projection rows are not 16-byte multiples);
    a reload replaces the weights."""
    dims = CUSTOM[name]
    img = gtenfile.synthetic_image(6, Q8, 5, cpu_pack(orc), dims=dims, std=0.05, gain_std=0.1)
    other = gtenfile.synthetic_image(6, Q8, 6, cpu_pack(orc), dims=dims, std=0.05, gain_std=0.1)
    path = tmp_path / "m.gten"
    img.tofile(path)
    prompt = np.random.default_rng(8).integers(0, dims[0], 11).astype(np.int32)
    a = G.Model(G.CUSTOM, Q8, 40, dims=dims)
    a.load(img)
    b = G.Model(G.CUSTOM, Q8, 40, dims=dims)
    b.load(other)
    b.load_file(str(path))
    assert np.array_equal(a.generate(prompt, 6), b.generate(prompt, 6))
    with pytest.raises(G.GtenError):
        b.load_file(str(tmp_path / "missing.gten"))
    a.close()
    b.close()


@pytest.mark.parametrize("name", list(CUSTOM))
@pytest.mark.parametrize("wdt", [Q8, Q4, F16])
def test_continuous_batching_matches_single_sequences(orc, gpu, name, wdt):
    """Eleven requests of mixed prompt lengths and lengths of generation through 4 slots: requests
    join the running batch as slots free up; each must get exactly the oracle's single-sequence
    greedy ids."""
    from gten_b200.serve import ContinuousBatcher
    from oracle.oracle import OracleModel
    dims = CUSTOM[name]
    img = gtenfile.synthetic_image(6, wdt, 41, cpu_pack(orc), dims=dims, std=0.05, gain_std=0.1)
    rng = np.random.default_rng(wdt * 7 + len(name))
    m = G.Model(G.CUSTOM, wdt, 48, max_batch=4, dims=dims)
    m.load(img)
    b = ContinuousBatcher(m)
    reqs = {}
    for i in range(11):
        p = rng.integers(0, dims[0], int(rng.integers(2, 28))).astype(np.int32)
        n = int(rng.integers(1, 48 - p.size + 2)) if i % 3 else 1 + i
        reqs[i] = (p, n)
        b.submit(i, p, n)
    res = b.run()
    assert b.steps < sum(n for _, n in reqs.values())  # the steps were shared
    for i, (p, n) in reqs.items():
        om = OracleModel(orc, 6, wdt, 2 * (p.size + n), img, dims=dims)
        assert res[i] == om.greedy(p, n).tolist(), f"request {i}"
    m.close()


def test_slot_api_errors(orc, gpu):
    dims = CUSTOM["llama"]
    img = gtenfile.synthetic_image(6, Q8, 2, cpu_pack(orc), dims=dims)
    m = G.Model(G.CUSTOM, Q8, 16, max_batch=2, dims=dims)
    m.load(img)
    assert (m.slots_step() == -1).all()  # no busy slot: nothing runs
    s0, _ = m.slot_start(np.arange(15, dtype=np.int32))
    s1, _ = m.slot_start(np.array([1, 2], np.int32))
    with pytest.raises(G.GtenError, match="busy"):
        m.slot_start(np.array([3], np.int32))
    with pytest.raises(G.GtenError, match="in use"):
        m.generate(np.array([1, 2, 3], np.int32), 2)  # the slots own the rows
    ids = m.slots_step()  # slot s0 processes position 15
    assert ids[s0] >= 0 and ids[s1] >= 0
    with pytest.raises(G.GtenError, match="max_ctx"):
        m.slots_step()  # slot s0's last token now sits at position 16
    m.slot_finish(s0)
    with pytest.raises(G.GtenError):
        m.slot_finish(s0)
    m.slot_finish(s1)
    assert m.generate(np.array([1, 2, 3], np.int32), 2).size == 2
    m.close()


GOLDEN = os.path.join(HERE, "golden", "greedy_tokens.json")


@pytest.mark.slow
@pytest.mark.parametrize("wdt", [Q8, Q4, F16])
def test_tinyllama_greedy_matches_reference(orc, gpu, wdt):
    """Full-size TinyLlama, seeded N(0, 0.02) weights, 64-token prompt, 64 greedy tokens: the ids
    must equal the reference CPU build's (tests/golden/greedy_tokens.json, made by
    tests/golden/make_golden.py with the compiled reference)."""
    with open(GOLDEN) as f:
        gold = json.load(f)
    case = gold[f"tinyllama_w{wdt}"]
    img = gtenfile.synthetic_image(0, wdt, case["seed"], gtenfile.cuda_packer())
    prompt = np.array(case["prompt"], np.int32)
    m = G.Model(G.TINYLLAMA, wdt, case["n_ctx"])
    m.load(img)
    got = m.generate(prompt, len(case["tokens"]))
    assert got.tolist() == case["tokens"]
    m.close()


MODELS = os.path.join(HERE, "golden", "model_tokens.json")
with open(MODELS) as _f:
    MODEL_CASES = sorted(json.load(_f))


@pytest.mark.slow
@pytest.mark.parametrize("name", MODEL_CASES)
def test_full_size_model_matches_reference(orc, gpu, name):
    """The other BASELINE architectures at full size (StableLM-2-Zephyr-1.6B Q4 with a 512-token
    prompt, MiniCPM-2B Q8 / Q4 with 128 tokens, OpenELM-1.1B fp16 with 1024 tokens), seeded
    N(0, 0.02) weights: the prefill logits must be the compiled reference's bit for bit (SHA-256 of
    the fp32 vector) and the 64 greedy ids of the fused decode path its ids
    (tests/golden/model_tokens.json, made by tests/golden/make_golden.py --models)."""
    import hashlib
    with open(MODELS) as f:
        case = json.load(f)[name]
    img = gtenfile.synthetic_image(case["kind"], case["wdtype"], case["seed"], gtenfile.cuda_packer())
    prompt = np.array(case["prompt"], np.int32)
    m = G.Model(case["kind"], case["wdtype"], case["n_ctx"])
    m.load(img)
    del img
    lg = m.logits(prompt, 0)
    assert hashlib.sha256(lg.tobytes()).hexdigest() == case["logits_sha256"]["0"]
    got = m.generate(prompt, len(case["tokens"]))
    assert got.tolist() == case["tokens"]
    m.close()


@pytest.mark.slow
@pytest.mark.parametrize("wdt", [Q8, Q4, F16])
def test_openelm_sm_matches_oracle(orc, gpu, wdt):
    """OpenELM-270M (openelm_sm_cfg: per-layer query / KV heads and FFN widths, QK-norm) at full
    size against the oracle's OpenELM wiring: prefill logits bit for bit, then greedy ids through
    the fused decode step. The reference runs OpenELM in fp16 only (its RoPE buffer is fp16,
    modules.cpp:247-249), so Q8 / Q4 follow the generic quantized-model semantics of the other
    families (Q8 activations everywhere), as the oracle restates them."""
    from oracle.oracle import OracleModel

    def pack(w, dt):
        return orc.pack_q8(w.numpy()) if dt == Q8 else orc.pack_q4(w.numpy())

    img = gtenfile.synthetic_image(G.OPENELM_SM, wdt, 4321, pack, std=0.05, gain_std=0.1)
    prompt = np.random.default_rng(3).integers(0, 32000, 12).astype(np.int32)
    n_gen, max_ctx = 6, 64
    m = G.Model(G.OPENELM_SM, wdt, max_ctx)
    m.load(img)
    assert np.array_equal(m.logits(prompt, 0), OracleModel(orc, G.OPENELM_SM, wdt, max_ctx, img).logits(prompt, 0))
    assert np.array_equal(m.generate(prompt, n_gen), OracleModel(orc, G.OPENELM_SM, wdt, max_ctx, img).greedy(prompt, n_gen))
    m.close()


def _oracle_topk_loop(om, sampler, prompt, n_gen, temp, top_k):
    """topk_sample's loop (sampler.cpp:80-139) over the oracle model: logits of the whole prompt,
    then of each new token; asserts no tie across the k-th place (a tie makes the pick
    library-specific)."""
    toks, out = [int(t) for t in prompt], []
    k = min(top_k, 1000)
    for i in range(n_gen):
        lg = om.logits(np.array(toks, np.int32), 0 if i == 0 else len(toks) - 1)
        top = np.sort(lg)[::-1]
        assert k == lg.size or top[k - 1] != top[k], f"tie across the k-th place at step {i}"
        t = sampler.step(lg, temp, top_k)
        out.append(t)
        toks.append(t)
    return out


@pytest.mark.parametrize("name", list(CUSTOM))
@pytest.mark.parametrize("wdt", [Q8, Q4, F16])
def test_topk_generation_matches_oracle(orc, gpu, name, wdt):
    """gtn_model_generate_topk draws inside the decode step; the ids must equal the oracle model's
    logits followed by the reference's sampling step with the same seeded std::mt19937."""
    from oracle.oracle import OracleModel, SamplerOracle
    dims = CUSTOM[name]
    img = gtenfile.synthetic_image(6, wdt, 31, cpu_pack(orc), dims=dims, std=0.05, gain_std=0.1)
    n_prompt, n_gen, temp, top_k, seed = 9, 14, 0.8, 40, 2024 + wdt
    max_ctx = 2 * (n_prompt + n_gen)
    prompt = np.random.default_rng(17).integers(0, dims[0], n_prompt).astype(np.int32)
    want = _oracle_topk_loop(OracleModel(orc, 6, wdt, max_ctx, img, dims=dims), SamplerOracle().generator(seed),
                             prompt, n_gen, temp, top_k)
    m = G.Model(G.CUSTOM, wdt, max_ctx, dims=dims)
    m.load(img)
    r = G.Rng(seed)
    assert m.generate_topk(prompt, n_gen, temp, top_k, r).tolist() == want
    # greedy afterwards rebuilds the captured step without the sampler
    assert np.array_equal(m.generate(prompt, 5), OracleModel(orc, 6, wdt, max_ctx, img, dims=dims).greedy(prompt, 5))
    # top_k = 1 is greedy, through the sampler
    assert np.array_equal(m.generate_topk(prompt, 5, 1.0, 1, r), m.generate(prompt, 5))
    with pytest.raises(G.GtenError, match="status 1"):
        m.generate_topk(prompt, 2, 0.0, 5, r)
    with pytest.raises(G.GtenError, match="status 1"):
        m.generate_topk(prompt, 2, 1.0, 0, r)
    r.close()
    m.close()


SAMPLED = os.path.join(HERE, "golden", "sampled_tokens.json")


@pytest.mark.slow
@pytest.mark.parametrize("wdt", [Q8, Q4])
def test_tinyllama_topk_matches_reference(orc, gpu, wdt):
    """Full-size TinyLlama, seeded weights and prompt as the greedy golden case, 48 top-k draws
    (Q8: temp 0.9, top_k 40; Q4: temp 1.7, top_k 200) from one seeded std::mt19937: the ids must equal
    tests/golden/sampled_tokens.json (compiled reference logits + the reference's sampling step)."""
    with open(SAMPLED) as f:
        case = json.load(f)[f"tinyllama_w{wdt}"]
    img = gtenfile.synthetic_image(0, wdt, case["seed"], gtenfile.cuda_packer())
    m = G.Model(G.TINYLLAMA, wdt, case["n_ctx"])
    m.load(img)
    r = G.Rng(case["rng_seed"])
    got = m.generate_topk(np.array(case["prompt"], np.int32), len(case["tokens"]), case["temp"], case["top_k"], r)
    assert got.tolist() == case["tokens"]
    r.close()
    m.close()
