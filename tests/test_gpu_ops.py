"""GPU parity of every gten op (C-ABI, sm_100a kernels) against the CPU oracle, bit for bit.

Each case builds seeded inputs in the reference formats, runs the op through
lib/libgten_b200.so and compares the output bytes with the oracle's restatement of the
reference (oracle/gten_oracle.c), which is itself pinned to the compiled reference."""
import numpy as np
import pytest
import torch

import gten_b200 as G
from helpers import F16, F32, I32, Q4, Q8, act_rows, fp16_vec, from_dev, row_bytes, to_dev, weights

pytestmark = pytest.mark.gpu


def dev_out(nbytes, device, fill=None):
    t = torch.zeros(nbytes, dtype=torch.uint8, device=device)
    if fill is not None:
        t.copy_(to_dev(fill, device))
    return t


@pytest.mark.parametrize("wdt", [Q8, Q4, F16])
@pytest.mark.parametrize("M,K,N", [(1, 2048, 256), (1, 2048, 2048), (1, 5632, 2048), (3, 256, 96), (16, 2048, 64),
                                   (9, 5760, 64), (64, 2304, 96), (1, 2048, 32003), (1, 2048, 40),
                                   # tensor-core GEMM (M >= 16): partial row / column tiles, one raw
                                   # chunk, ring wrap-around (K = 5632: 22 chunks); 32-row weight
                                   # tiles for small grids, 64-row tiles from one CTA per SM on
                                   # (9632 rows: 151 tiles, the last one half full)
                                   (16, 256, 64), (33, 2048, 96), (100, 5632, 160), (128, 2304, 256),
                                   (47, 256, 32), (40, 2048, 9632)])
@pytest.mark.parametrize("odt_kind", ["act", "f32"])
def test_matmul_2d(orc, gpu, wdt, M, K, N, odt_kind):
    rng = np.random.default_rng(M * 1000 + K + N + wdt)
    xdt = F16 if wdt == F16 else Q8
    odt = xdt if odt_kind == "act" else F32
    x = act_rows(orc, rng, xdt, M, K)
    w = weights(orc, rng, wdt, N, K)
    for sp in sorted({0, M - 1}):
        want = orc.matmul_2d(x, xdt, M, K, w, wdt, N, odt, start_pos=sp)
        out = dev_out(row_bytes(odt, N) * M, gpu)
        G.matmul_2d(G.GT(to_dev(x, gpu), xdt, (M, K)), G.GT(to_dev(w, gpu), wdt, (N, K)),
                    G.GT(out, odt, (M, N)), start_pos=sp)
        got = from_dev(out)
        rb = row_bytes(odt, N)
        assert np.array_equal(got[sp * rb:], want[sp * rb:]), f"start_pos={sp}"


@pytest.mark.parametrize("wdt", [Q8, Q4])
@pytest.mark.parametrize("K", [2304, 5632, 5760])
@pytest.mark.parametrize("M", [2, 5, 8, 12, 15])
def test_small_batch_gemm(orc, gpu, wdt, K, M):
    """The batched decode steps' GEMM for 2-15 rows (k_gemm4) on the models' row lengths: groups of
    14 or 5 weight rows with a ragged last group (N = 97), two CTAs per SM for K = 2304 and one with
    larger product chunks for the long rows, activation rows staged in one or several passes."""
    import ctypes as C
    rng = np.random.default_rng(M * 100 + K + wdt)
    N = 97
    x = act_rows(orc, rng, Q8, M, K)
    w = weights(orc, rng, wdt, N, K)
    want = orc.matmul_2d(x, Q8, M, K, w, wdt, N, F32, start_pos=0)
    # weight rows padded to a multiple of 8 blocks (16-byte rows, as the model arena lays them out;
    # K = 5760 is 180 blocks): the row stride of the descriptor says so
    nb, bb = K // 32, 34 if wdt == Q8 else 18
    nbp = (nb + 7) // 8 * 8
    wp = np.zeros((N, nbp * bb), np.uint8)
    wp[:, :nb * bb] = np.asarray(w, np.uint8).reshape(N, nb * bb)
    w_dev, x_dev, out = to_dev(wp, gpu), to_dev(x, gpu), dev_out(4 * N * M, gpu)  # alive through the call
    wd = G.GT(w_dev, wdt, (N, K)).desc()
    wd.strides[0] = nbp * 32
    xd = G.GT(x_dev, Q8, (M, K)).desc()
    od = G.GT(out, F32, (M, N)).desc()
    rc = G.lib().gtn_matmul_2d(C.byref(xd), C.byref(wd), C.byref(od), 0, G._stream(None))
    assert rc == 0, G.lib().gtn_last_error()
    assert np.array_equal(from_dev(out), want)


@pytest.mark.parametrize("wdt", [Q8, Q4, F16])
def test_matmul_1d_logits(orc, gpu, wdt):
    """EmbeddingLinear's stride-0 fp32 output (modules.cpp:111-122): last row only."""
    rng = np.random.default_rng(7 + wdt)
    xdt = F16 if wdt == F16 else Q8
    M, K, N = 5, 2048, 1000
    x = act_rows(orc, rng, xdt, M, K)
    w = weights(orc, rng, wdt, N, K)
    want = orc.matmul_2d(x, xdt, M, K, w, wdt, N, F32, start_pos=M - 1, out_1d=True)
    out = dev_out(4 * N, gpu)
    G.matmul_2d(G.GT(to_dev(x, gpu), xdt, (M, K)), G.GT(to_dev(w, gpu), wdt, (N, K)), G.GT(out, F32, (N,)),
                start_pos=M - 1)
    assert np.array_equal(from_dev(out), want)


@pytest.mark.parametrize("dt", [Q8, F16])
@pytest.mark.parametrize("n,sp,H,KVH", [(1, 0, 4, 4), (9, 0, 8, 2), (40, 39, 8, 2), (70, 69, 32, 4), (33, 0, 4, 1),
                                        (300, 299, 32, 4), (257, 250, 36, 36), (1536, 1535, 16, 4)])
def test_qkv_attn(orc, gpu, dt, n, sp, H, KVH):
    rng = np.random.default_rng(n * 7 + H + dt)
    q = act_rows(orc, rng, dt, n, H * 64)
    k = act_rows(orc, rng, dt, n, KVH * 64)
    v = act_rows(orc, rng, dt, n, KVH * 64)
    want = orc.qkv_attn(q, k, v, dt, n, H, H * 64, KVH * 64, sp)
    out = dev_out(row_bytes(dt, H * 64) * n, gpu)
    G.qkv_attn(G.GT(to_dev(q, gpu), dt, (n, H * 64)), G.GT(to_dev(k, gpu), dt, (n, KVH * 64)),
               G.GT(to_dev(v, gpu), dt, (n, KVH * 64)), None, G.GT(out, dt, (n, H * 64)), max_ctx=n, start_pos=sp)
    rb = row_bytes(dt, H * 64)
    assert np.array_equal(from_dev(out)[sp * rb:], want[sp * rb:])


@pytest.mark.parametrize("dt", [Q8, F16])
@pytest.mark.parametrize("D", [2048, 2304, 96])
def test_norms(orc, gpu, dt, D):
    rng = np.random.default_rng(D + dt)
    M = 5
    x = act_rows(orc, rng, dt, M, D)
    w = fp16_vec(rng, D)
    b = fp16_vec(rng, D, 0.0, 0.1)
    rb = row_bytes(dt, D)
    xin = G.GT(to_dev(x, gpu), dt, (M, D))
    out = dev_out(rb * M, gpu)
    G.rms_norm(xin, G.GT(to_dev(w, gpu), F16, (D,)), G.GT(out, dt, (M, D)), start_pos=1)
    assert np.array_equal(from_dev(out)[rb:], orc.rms_norm(x, dt, M, D, w, 1)[rb:])
    out = dev_out(rb * M, gpu)
    G.layer_norm(xin, G.GT(to_dev(w, gpu), F16, (D,)), G.GT(to_dev(b, gpu), F16, (D,)), G.GT(out, dt, (M, D)),
                 start_pos=1)
    assert np.array_equal(from_dev(out)[rb:], orc.layer_norm(x, dt, M, D, w, b, 1)[rb:])


@pytest.mark.parametrize("D", [2048, 2304, 64, 1000])
def test_rms_norm_sequential_sum_adversarial(orc, gpu, D):
    """The RMSNorm sum of squares is computed by an exact parallel emulation of the reference's
    sequential fp32 loop (seqsum.cuh): rows built to stress binade crossings, ties, zeros and
    extreme ranges must still match the serial loop bit for bit."""
    rng = np.random.default_rng(D)
    rows = [
        rng.standard_normal(D),
        np.ones(D),
        np.full(D, 3.0),
        2.0 ** rng.integers(-20, 20, D),
        np.concatenate([np.zeros(D // 2), rng.standard_normal(D - D // 2)]),
        np.zeros(D),
        np.where(rng.random(D) < 0.01, 1e6, 1e-3) * rng.standard_normal(D),
        1.0 + 2.0 ** -12 * rng.integers(0, 8, D),          # short mantissas: rounding ties
        np.sqrt(np.arange(1, D + 1, dtype=np.float64)),   # squares near integers
        rng.standard_normal(D) * 1e-20,                    # subnormal squares
        np.linspace(1e-3, 1e3, D),
        rng.integers(-127, 128, D) * 2.0 ** -7,            # int8 grid: many ties per binade
        # Q8-dequantized values q * fp16(delta) per 32-block, as the residual stream holds them
        rng.integers(-127, 128, D) * np.repeat(
            rng.uniform(1e-3, 1e-1, (D + 31) // 32).astype(np.float16).astype(np.float64), 32)[:D],
        np.concatenate([rng.standard_normal(D - 1) * 1e-30, [1.0]]),  # tiny terms, then a huge one
    ]
    x = np.stack(rows).astype(np.float32)
    M = x.shape[0]
    w = fp16_vec(rng, D)
    out = torch.zeros(M * D * 4, dtype=torch.uint8, device=gpu)
    G.rms_norm(G.GT(to_dev(x, gpu), F32, (M, D)), G.GT(to_dev(w, gpu), F16, (D,)), G.GT(out, F32, (M, D)))
    want = orc.rms_norm(x.view(np.uint8).ravel().copy(), F32, M, D, w, 0)
    got = from_dev(out)
    for r in range(M):
        assert np.array_equal(got[r * D * 4:(r + 1) * D * 4], want[r * D * 4:(r + 1) * D * 4]), f"row {r}"


@pytest.mark.parametrize("D", [2048, 2304])
def test_rms_norm_sequential_sum_many_rows(orc, gpu, D):
    """1,024 seeded rows of mixed distributions (Gaussian with outlier dimensions, Q8-dequantized
    residual blocks, coarse grids with many rounding ties, wide log-uniform ranges): the exact
    parallel sum of squares must equal the serial loop bit for bit on every one."""
    rng = np.random.default_rng(77 + D)
    M = 1024
    x = np.empty((M, D), np.float64)
    for r in range(M):
        kind = r % 6
        if kind == 0:
            v = rng.standard_normal(D) * 10.0 ** rng.uniform(-3, 3)
        elif kind == 1:
            v = rng.standard_normal(D)
            v[rng.integers(0, D, 4)] *= rng.uniform(10, 200)
        elif kind == 2:
            d = rng.uniform(1e-3, 1.0, (D + 31) // 32).astype(np.float16).astype(np.float64)
            v = rng.integers(-127, 128, D) * np.repeat(d, 32)[:D]
        elif kind == 3:
            v = rng.integers(-8, 9, D) * 2.0 ** int(rng.integers(-10, 10))
        elif kind == 4:
            v = np.sign(rng.standard_normal(D)) * 10.0 ** rng.uniform(-6, 4, D)
        else:
            v = rng.standard_normal(D) * np.where(rng.random(D) < 0.5, 0.0, 1.0)
        x[r] = v
    x = x.astype(np.float32)
    w = fp16_vec(rng, D)
    out = torch.zeros(M * D * 4, dtype=torch.uint8, device=gpu)
    G.rms_norm(G.GT(to_dev(x, gpu), F32, (M, D)), G.GT(to_dev(w, gpu), F16, (D,)), G.GT(out, F32, (M, D)))
    want = orc.rms_norm(x.view(np.uint8).ravel().copy(), F32, M, D, w, 0)
    got = from_dev(out)
    bad = [r for r in range(M) if not np.array_equal(got[r * D * 4:(r + 1) * D * 4], want[r * D * 4:(r + 1) * D * 4])]
    assert not bad, f"rows {bad[:10]} of {len(bad)}"


@pytest.mark.parametrize("dt", [Q8, F16])
def test_rms_norm_3d(orc, gpu, dt):
    rng = np.random.default_rng(3 + dt)
    M, Hh, dh = 4, 20, 64
    x = act_rows(orc, rng, dt, M, Hh * dh)
    w = fp16_vec(rng, dh)
    out = dev_out(row_bytes(dt, Hh * dh) * M, gpu)
    G.rms_norm(G.GT(to_dev(x, gpu), dt, (M, Hh, dh)), G.GT(to_dev(w, gpu), F16, (dh,)), G.GT(out, dt, (M, Hh * dh)))
    assert np.array_equal(from_dev(out), orc.rms_norm_3d(x, dt, M, Hh, dh, w, 0))


@pytest.mark.parametrize("dt", [Q8, F16])
@pytest.mark.parametrize("pct", [1.0, 0.25])
@pytest.mark.parametrize("M,sp", [(5, 2), (1, 0), (700, 690)])
def test_rotary_emb(orc, gpu, dt, pct, M, sp):
    rng = np.random.default_rng(M + int(pct * 4) + dt)
    D = 2048
    x = act_rows(orc, rng, dt, M, D)
    want = orc.rotary_emb(x, dt, M, D, 64, pct, sp)
    buf = to_dev(x, gpu)
    G.rotary_emb(G.GT(buf, dt, (M, D)), G.GT(buf, dt, (M, D)), 64, pct, start_pos=sp)
    rb = row_bytes(dt, D)
    assert np.array_equal(from_dev(buf)[sp * rb:], want[sp * rb:])


@pytest.mark.parametrize("dt", [Q8, F16])
@pytest.mark.parametrize("D", [5632, 5760, 2048, 70])
def test_elementwise(orc, gpu, dt, D):
    rng = np.random.default_rng(D + 11 * dt)
    M = 3 if (D % 32 == 0 or dt == F16) else 1
    rb = row_bytes(dt, D)
    x = act_rows(orc, rng, dt, M, D, 3.0)
    y = act_rows(orc, rng, dt, M, D)
    bias = fp16_vec(rng, D, 0.0, 0.5)

    # silu (out of place)
    out = dev_out(rb * M, gpu)
    sp = min(1, M - 1)
    G.silu(G.GT(to_dev(x, gpu), dt, (M, D)), G.GT(out, dt, (M, D)), start_pos=sp)
    assert np.array_equal(from_dev(out)[sp * rb:], orc.silu(x, dt, M, D, sp)[sp * rb:])
    # silu_inplace
    buf = to_dev(x, gpu)
    G.silu_inplace(G.GT(buf, dt, (M, D)))
    assert np.array_equal(from_dev(buf), orc.silu(x, dt, M, D, 0))
    # multiply / add
    out = dev_out(rb * M, gpu)
    G.multiply(G.GT(to_dev(x, gpu), dt, (M, D)), G.GT(to_dev(y, gpu), dt, (M, D)), G.GT(out, dt, (M, D)))
    assert np.array_equal(from_dev(out), orc.multiply(x, y, dt, M, D))
    buf = to_dev(x, gpu)
    G.multiply_inplace(G.GT(buf, dt, (M, D)), G.GT(to_dev(y, gpu), dt, (M, D)))
    assert np.array_equal(from_dev(buf), orc.multiply(x, y, dt, M, D))
    out = dev_out(rb * M, gpu)
    G.add(G.GT(to_dev(x, gpu), dt, (M, D)), G.GT(to_dev(y, gpu), dt, (M, D)), G.GT(out, dt, (M, D)))
    assert np.array_equal(from_dev(out), orc.add(x, y, dt, M, D))
    # scale (minicpm's three constants) and bias
    for s in (12.0, float(np.float32(1.4) / np.sqrt(40.0)), 1.0 / 9):
        buf = to_dev(x, gpu)
        G.scale(G.GT(buf, dt, (M, D)), s, start_pos=M - 1)
        assert np.array_equal(from_dev(buf), orc.scale(x, dt, M, D, s, M - 1))
    buf = to_dev(x, gpu)
    G.bias_add_inplace(G.GT(buf, dt, (M, D)), G.GT(to_dev(bias, gpu), F16, (D,)))
    assert np.array_equal(from_dev(buf), orc.bias_add_inplace(x, dt, M, D, bias))


def test_silu_uses_the_reference_expf(orc, gpu):
    """silu on fp32 rows at inputs where the reference's expf (glibc's, ops.cpp:733-772) and a
    correctly rounded exp differ and the difference reaches silu's result
    (tests/golden/expf_cases.npy, made by make_expf_cases.py from the host's libm): the device must
    give the host library's bits. The oracle calls the host's expf."""
    import os
    x = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "expf_cases.npy"))
    D = 128
    M = (x.size + D - 1) // D
    xs = np.zeros(M * D, np.float32)
    xs[: x.size] = x
    out = dev_out(xs.nbytes, gpu)
    G.silu(G.GT(to_dev(xs, gpu), F32, (M, D)), G.GT(out, F32, (M, D)))
    want = orc.silu(xs.view(np.uint8), F32, M, D, 0)
    got = from_dev(out)
    bad = np.flatnonzero(got.view(np.uint32) != want.view(np.uint32))
    assert bad.size == 0, f"{bad.size} of {xs.size} differ, e.g. x = {xs[bad[:4]]}"


@pytest.mark.parametrize("wdt", [Q8, Q4, F16])
def test_token_embed(orc, gpu, wdt):
    rng = np.random.default_rng(21 + wdt)
    V, D = 300, 2304
    w = weights(orc, rng, wdt, V, D)
    toks = rng.integers(0, V, 9).astype(np.int32)
    odt = F16 if wdt == F16 else Q8
    out = dev_out(row_bytes(odt, D) * toks.size, gpu)
    G.token_embed(G.GT(to_dev(w, gpu), wdt, (V, D)), G.GT(torch.from_numpy(toks).to(gpu), I32, (toks.size,)),
                  G.GT(out, odt, (toks.size, D)), start_pos=2)
    rb = row_bytes(odt, D)
    assert np.array_equal(from_dev(out)[2 * rb:], orc.token_embed(w, wdt, V, D, toks, odt, 2)[2 * rb:])


@pytest.mark.parametrize("rows,cols", [(37, 2048), (1, 32), (256, 5760)])
def test_pack_and_quantize(orc, gpu, rows, cols):
    rng = np.random.default_rng(rows + cols)
    w = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32)
    w[0, :32] = 0.0                      # an all-zero block (delta 0)
    if cols >= 64:
        w[-1, 32:64] = np.float32(0.5) * (np.arange(32) % 3 - 1)  # block with absmax 0.5 and zeros
    wd = torch.from_numpy(w).to(gpu)
    for dt, packer, ref in ((Q8, G.pack_q8, orc.pack_q8), (Q4, G.pack_q4, orc.pack_q4)):
        out = torch.zeros(rows * row_bytes(dt, cols), dtype=torch.uint8, device=gpu)
        packer(wd, out)
        assert np.array_equal(from_dev(out), ref(w))
    # activation quantizer with a partial last block
    x = (rng.standard_normal((rows, cols + 7)) * 3).astype(np.float32)
    out = torch.zeros(rows * row_bytes(Q8, cols + 7), dtype=torch.uint8, device=gpu)
    G.quantize_q8_rows(torch.from_numpy(x).to(gpu), out)
    want = np.concatenate([orc.q8_quantize_row(x[i]) for i in range(rows)])
    got = from_dev(out)
    rb = row_bytes(Q8, cols + 7)
    valid = np.ones(rb, bool)
    valid[rb - 32 + 7:] = False  # bytes past the partial block's 7 values are unspecified
    for i in range(rows):
        assert np.array_equal(got[i * rb:(i + 1) * rb][valid], want[i * rb:(i + 1) * rb][valid])


@pytest.mark.parametrize("n", [1, 32003, 100352, 122753])
def test_argmax(orc, gpu, n):
    rng = np.random.default_rng(n)
    x = rng.standard_normal(n).astype(np.float32)
    if n > 10:
        x[[3, n // 2, n - 1]] = x.max() + 1.0  # ties: the first index wins (sampler.cpp:189-195)
    out = torch.zeros(1, dtype=torch.int32, device=gpu)
    G.argmax(torch.from_numpy(x).to(gpu), out)
    assert int(out.item()) == orc.argmax(x)


def test_errors_are_status_codes(gpu):
    """Shape/dtype violations return GTN_ERR_ARG (the reference asserts and exits)."""
    x = torch.zeros(64, dtype=torch.uint8, device=gpu)
    with pytest.raises(G.GtenError, match="status 1"):
        G.matmul_2d(G.GT(x, Q8, (1, 32)), G.GT(x, Q8, (1, 64)), G.GT(x, F32, (1, 1)))
    with pytest.raises(G.GtenError, match="status 1"):
        G.add(G.GT(x, Q8, (1, 32)), G.GT(x, F16, (1, 32)), G.GT(x, Q8, (1, 32)))
    # multi-row quantized tensors need whole blocks per row (see check_tensor in abi.cu)
    with pytest.raises(G.GtenError, match="overlap"):
        G.silu_inplace(G.GT(x, Q8, (2, 40)))
