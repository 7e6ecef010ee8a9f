"""CPU tests of the oracle (oracle/gten_oracle.c), the checker every GPU parity test relies on.

Pinning: against the committed golden vectors made from the reference itself
(tests/golden/make_golden.py: the reference converter's Python packer, the compiled reference
ops and its greedy tokens), and, where the reference harness is built, against the live compiled
reference on fresh seeded cases including edge cases (partial blocks, all-zero blocks, start_pos
> 0, GQA groups, decode rows)."""
import json
import os

import numpy as np
import pytest

from helpers import F16, F32, Q4, Q8, act_rows, fp16_vec, q8_rows, weights

HERE = os.path.dirname(os.path.abspath(__file__))
GOLD = os.path.join(HERE, "golden")


def test_pack_matches_reference_packer_golden(orc):
    g = np.load(os.path.join(GOLD, "pack.npz"))
    assert np.array_equal(orc.pack_q8(g["w"]), g["q8"])
    assert np.array_equal(orc.pack_q4(g["w"]), g["q4"])


def test_ops_match_reference_golden(orc):
    g = np.load(os.path.join(GOLD, "ops.npz"))
    for wname, wdt in (("q8", Q8), ("q4", Q4), ("f16", F16)):
        xdt = F16 if wdt == F16 else Q8
        M, K, N = 3, 256, 64
        x, w = g[f"mm_{wname}_x"], g[f"mm_{wname}_w"]
        assert np.array_equal(orc.matmul_2d(x, xdt, M, K, w, wdt, N, xdt), g[f"mm_{wname}_out"])
        assert np.array_equal(orc.matmul_2d(x, xdt, M, K, w, wdt, N, F32), g[f"mm_{wname}_out32"])
    for dname, dt in (("q8", Q8), ("f16", F16)):
        M, D = 4, 256
        x, y, gg, b = g[f"{dname}_x"], g[f"{dname}_y"], g[f"{dname}_g"], g[f"{dname}_b"]
        assert np.array_equal(orc.rms_norm(x, dt, M, D, gg), g[f"{dname}_rms"])
        assert np.array_equal(orc.layer_norm(x, dt, M, D, gg, b), g[f"{dname}_ln"])
        assert np.array_equal(orc.rotary_emb(x, dt, M, D, 64, 1.0), g[f"{dname}_rope"])
        assert np.array_equal(orc.rotary_emb(x, dt, M, D, 64, 0.25), g[f"{dname}_rope25"])
        assert np.array_equal(orc.silu(x, dt, M, D), g[f"{dname}_silu"])
        assert np.array_equal(orc.multiply(x, y, dt, M, D), g[f"{dname}_mul"])
        assert np.array_equal(orc.add(x, y, dt, M, D), g[f"{dname}_add"])
        assert np.array_equal(orc.scale(x, dt, M, D, 12.0), g[f"{dname}_scale"])
        assert np.array_equal(orc.bias_add_inplace(x, dt, M, D, b), g[f"{dname}_bias"])
        n, H, KVH = 37, 4, 2
        q, k, v = g[f"{dname}_q"], g[f"{dname}_k"], g[f"{dname}_v"]
        assert np.array_equal(orc.qkv_attn(q, k, v, dt, n, H, H * 64, KVH * 64, 0), g[f"{dname}_attn"])
        rb = (H * 64 // 32) * 34 if dt == Q8 else H * 64 * 2
        assert np.array_equal(orc.qkv_attn(q, k, v, dt, n, H, H * 64, KVH * 64, n - 1)[(n - 1) * rb:],
                              g[f"{dname}_attn_dec"][(n - 1) * rb:])


def test_fp16_conversions_exhaustive(orc, ref):
    """Every half value decodes like the reference's table; encodes agree on a dense sweep."""
    import ctypes as C
    for h in range(0, 65536, 1):
        a = orc.lib.or_fp16_to_fp32(C.c_uint16(h))
        b = ref.lib.ref_fp16_to_fp32(C.c_uint16(h))
        assert (a == b) or (np.isnan(a) and np.isnan(b)), h
    rng = np.random.default_rng(0)
    xs = np.concatenate([rng.standard_normal(20000) * s for s in (1e-7, 1e-5, 1.0, 1e3, 7e4)]).astype(np.float32)
    for x in xs:
        assert orc.lib.or_fp32_to_fp16(C.c_float(x)) == ref.lib.ref_fp32_to_fp16(C.c_float(x))


def test_reference_python_packer_live(orc):
    """The reference converter's own q8_quantize / q4_quantize on fresh seeded tensors."""
    from oracle.oracle import reference_dir
    ref_dir = reference_dir()
    if ref_dir is None:
        pytest.skip("no reference checkout (GTEN_REFERENCE_DIR or BASELINE.json reference_path)")
    import io

    import torch

    from tests.golden.make_golden import reference_packer
    ns = reference_packer(ref_dir)
    rng = np.random.default_rng(99)
    for scale in (0.02, 1.0, 1e-4):
        w = (rng.standard_normal((16, 512)) * scale).astype(np.float32)
        w[3, 64:96] = 0.0
        for dt, fn in (("q8", orc.pack_q8), ("q4", orc.pack_q4)):
            buf = io.BytesIO()
            ns["write_layer"](buf, "t", torch.from_numpy(w.copy()), dt)
            assert np.array_equal(fn(w), np.frombuffer(buf.getvalue()[14:], np.uint8))


CASES_MM = [(1, 2048, 256), (3, 256, 96), (4, 5632, 64), (2, 5760, 64), (1, 2304, 40)]


@pytest.mark.parametrize("M,K,N", CASES_MM)
@pytest.mark.parametrize("wdt", [Q8, Q4, F16])
def test_matmul_vs_reference(orc, ref, M, K, N, wdt):
    rng = np.random.default_rng(M + K + N + wdt)
    xdt = F16 if wdt == F16 else Q8
    x = act_rows(orc, rng, xdt, M, K)
    w = weights(orc, rng, wdt, N, K)
    for odt in (xdt, F32):
        for sp in {0, M - 1}:
            a = orc.matmul_2d(x, xdt, M, K, w, wdt, N, odt, start_pos=sp)
            b = ref.matmul_2d(x, xdt, M, K, w, wdt, N, odt, start_pos=sp)
            assert np.array_equal(a, b)
    a = orc.matmul_2d(x, xdt, M, K, w, wdt, N, F32, start_pos=M - 1, out_1d=True)
    b = ref.matmul_2d(x, xdt, M, K, w, wdt, N, F32, start_pos=M - 1, out_1d=True)
    assert np.array_equal(a, b)


@pytest.mark.parametrize("dt", [Q8, F16])
def test_rowops_vs_reference(orc, ref, dt):
    rng = np.random.default_rng(5 + dt)
    for D in (2048, 2304, 70):
        M = 5 if (D % 32 == 0 or dt == F16) else 1
        x = act_rows(orc, rng, dt, M, D, 2.0)
        y = act_rows(orc, rng, dt, M, D)
        w = fp16_vec(rng, D)
        b = fp16_vec(rng, D, 0.0, 0.1)
        sp = min(1, M - 1)
        assert np.array_equal(orc.rms_norm(x, dt, M, D, w, sp), ref.rms_norm(x, dt, M, D, w, sp))
        assert np.array_equal(orc.layer_norm(x, dt, M, D, w, b, sp), ref.layer_norm(x, dt, M, D, w, b, sp))
        assert np.array_equal(orc.silu(x, dt, M, D, 0), ref.silu(x, dt, M, D, 0))
        assert np.array_equal(orc.multiply(x, y, dt, M, D), ref.multiply(x, y, dt, M, D))
        assert np.array_equal(orc.add(x, y, dt, M, D), ref.add(x, y, dt, M, D))
        assert np.array_equal(orc.scale(x, dt, M, D, 0.221), ref.scale(x, dt, M, D, 0.221))
        assert np.array_equal(orc.bias_add_inplace(x, dt, M, D, b), ref.bias_add_inplace(x, dt, M, D, b))
        if D % 64 == 0:
            for pct in (1.0, 0.25):
                assert np.array_equal(orc.rotary_emb(x, dt, M, D, 64, pct, 2), ref.rotary_emb(x, dt, M, D, 64, pct, 2))
            w64 = w[:64].copy()
            assert np.array_equal(orc.rms_norm_3d(x, dt, M, D // 64, 64, w64),
                                  ref.rms_norm_3d(x, dt, M, D // 64, 64, w64))
    for wdt in (Q8, Q4, F16):
        if (wdt == F16) != (dt == F16):
            continue
        V, D = 300, 256
        wt = weights(orc, rng, wdt, V, D)
        toks = rng.integers(0, V, 7).astype(np.int32)
        assert np.array_equal(orc.token_embed(wt, wdt, V, D, toks, dt, 2), ref.token_embed(wt, wdt, V, D, toks, dt, 2))


@pytest.mark.parametrize("dt", [Q8, F16])
@pytest.mark.parametrize("n,sp,H,KVH", [(9, 0, 8, 2), (40, 39, 8, 2), (70, 69, 4, 4), (33, 0, 4, 1), (1, 0, 2, 2)])
def test_attention_vs_reference(orc, ref, dt, n, sp, H, KVH):
    rng = np.random.default_rng(n + H + dt)
    q = act_rows(orc, rng, dt, n, H * 64)
    k = act_rows(orc, rng, dt, n, KVH * 64)
    v = act_rows(orc, rng, dt, n, KVH * 64)
    assert np.array_equal(orc.qkv_attn(q, k, v, dt, n, H, H * 64, KVH * 64, sp),
                          ref.qkv_attn(q, k, v, dt, n, H, H * 64, KVH * 64, sp, max_ctx=4 * n))


def test_q8_quantize_partial_blocks_vs_reference(orc, ref):
    rng = np.random.default_rng(3)
    for n in (1, 31, 32, 33, 70, 2048):
        x = (rng.standard_normal(n) * 5).astype(np.float32)
        assert np.array_equal(orc.q8_quantize_row(x), ref.q8_quantize_row(x))
    assert np.array_equal(orc.q8_quantize_row(np.zeros(40, np.float32)), ref.q8_quantize_row(np.zeros(40, np.float32)))


def test_tinyllama_greedy_oracle_matches_reference_golden(orc):
    """Full-size TinyLlama Q8 through the oracle's model wiring: the 64 greedy ids equal the
    reference's (golden)."""
    from oracle.oracle import OracleModel
    import gten_b200 as G
    from gten_b200 import gtenfile
    with open(os.path.join(GOLD, "greedy_tokens.json")) as f:
        case = json.load(f)[f"tinyllama_w{Q8}"]

    def pack(w, dt):
        return orc.pack_q8(w.numpy()) if dt == Q8 else orc.pack_q4(w.numpy())

    img = gtenfile.synthetic_image(G.TINYLLAMA, Q8, case["seed"], pack)
    om = OracleModel(orc, 0, Q8, case["n_ctx"], img)
    got = om.greedy(np.array(case["prompt"], np.int32), len(case["tokens"]))
    assert got.tolist() == case["tokens"]
