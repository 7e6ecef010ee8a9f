"""gtn_matmul_2d_noalloc: the matmul operator for callers that may not allocate device memory.

Some callers cannot call cudaMalloc: they run under a fixed device-memory budget that they hand
out themselves, or inside an allocator / memory-pool callback, or on paths where an allocation's
implicit synchronization is not acceptable. For them the library stages the fp32 dot products of
a quantized or fp16 output in a fixed array of its own instead of allocating scratch.

These tests call the entry point through the C ABI and check that it returns exactly what
gtn_matmul_2d returns and what the CPU oracle returns (the parity bar of every test here is bit
equality), on two calls in a row (the shared staging array keeps the previous call's contents),
including 32-row inputs, where gtn_matmul_2d runs the tensor-core GEMM and this variant (which has
no scratch for its activation image) the CUDA-core GEMM, and a single new row written to a 1-D
output; and that a request larger than the fixed array is refused with a clear error. The file is
collected last on purpose."""
import ctypes as C

import numpy as np
import pytest
import torch

import gten_b200 as G
from helpers import F16, F32, Q4, Q8, act_rows, from_dev, row_bytes, to_dev, weights

pytestmark = pytest.mark.gpu


def call_noalloc(x: G.GT, w: G.GT, out: G.GT, start_pos: int = 0) -> int:
    lib = G.lib()
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    return lib.gtn_matmul_2d_noalloc(C.byref(x.desc()), C.byref(w.desc()), C.byref(out.desc()), start_pos, stream)


@pytest.mark.parametrize("wdt", [Q8, Q4, F16])
def test_noalloc_matches_matmul_2d_twice(orc, gpu, wdt):
    xdt = F16 if wdt == F16 else Q8
    # two calls in a row on the same shape with different data, then a different shape
    cases = [(5, 2048, 2560, 0), (5, 2048, 2560, 0), (3, 5632, 2048, 2), (32, 2048, 2560, 0), (32, 2048, 2560, 0)]
    for call, (M, K, N, sp) in enumerate(cases):
        rng = np.random.default_rng(100 + 10 * call + wdt)
        x = act_rows(orc, rng, xdt, M, K)
        w = weights(orc, rng, wdt, N, K)
        X, W = G.GT(to_dev(x, gpu), xdt, (M, K)), G.GT(to_dev(w, gpu), wdt, (N, K))
        for odt in (xdt, F32):
            want = torch.zeros(row_bytes(odt, N) * M, dtype=torch.uint8, device=gpu)
            got = torch.zeros_like(want)
            G.matmul_2d(X, W, G.GT(want, odt, (M, N)), start_pos=sp)
            rc = call_noalloc(X, W, G.GT(got, odt, (M, N)), start_pos=sp)
            assert rc == 0, G.lib().gtn_last_error().decode()
            torch.cuda.synchronize()
            assert np.array_equal(from_dev(got), from_dev(want)), f"call {call}, out dtype {odt}"
            ref = orc.matmul_2d(x, xdt, M, K, w, wdt, N, odt, start_pos=sp)
            rb = row_bytes(odt, N)
            assert np.array_equal(from_dev(got)[sp * rb:], ref[sp * rb:]), f"call {call}, out dtype {odt} vs oracle"


@pytest.mark.parametrize("wdt", [Q8, Q4, F16])
def test_noalloc_single_row_1d_output(orc, gpu, wdt):
    """One new row (start_pos = n_ctx - 1) into a 1-D output, as EmbeddingLinear's logits
    (modules.cpp:111-122), with n_out not a multiple of 32: Q8 / fp16 (staged) and fp32 outputs,
    twice in a row, equal to gtn_matmul_2d and to the oracle."""
    xdt = F16 if wdt == F16 else Q8
    n_ctx, K, N = 4, 2048, 1000
    for call in range(2):
        rng = np.random.default_rng(7 + call + 3 * wdt)
        x = act_rows(orc, rng, xdt, n_ctx, K)
        w = weights(orc, rng, wdt, N, K)
        X, W = G.GT(to_dev(x, gpu), xdt, (n_ctx, K)), G.GT(to_dev(w, gpu), wdt, (N, K))
        for odt in (xdt, F32):
            want = torch.zeros(row_bytes(odt, N), dtype=torch.uint8, device=gpu)
            got = torch.zeros_like(want)
            G.matmul_2d(X, W, G.GT(want, odt, (N,)), start_pos=n_ctx - 1)
            rc = call_noalloc(X, W, G.GT(got, odt, (N,)), start_pos=n_ctx - 1)
            assert rc == 0, G.lib().gtn_last_error().decode()
            torch.cuda.synchronize()
            assert np.array_equal(from_dev(got), from_dev(want)), f"call {call}, out dtype {odt}"
            ref = orc.matmul_2d(x, xdt, n_ctx, K, w, wdt, N, odt, start_pos=n_ctx - 1, out_1d=True)
            assert np.array_equal(from_dev(got), ref), f"call {call}, out dtype {odt} vs oracle"


def test_noalloc_rejects_requests_beyond_the_fixed_scratch(orc, gpu):
    M, K, N = 65, 32, 32768  # 65 * 32768 = 2,129,920 staging floats > 2,097,152
    x = torch.zeros(row_bytes(Q8, K) * M, dtype=torch.uint8, device=gpu)
    w = torch.zeros(row_bytes(Q8, K) * N, dtype=torch.uint8, device=gpu)
    out = torch.zeros(row_bytes(Q8, N) * M, dtype=torch.uint8, device=gpu)
    rc = call_noalloc(G.GT(x, Q8, (M, K)), G.GT(w, Q8, (N, K)), G.GT(out, Q8, (M, N)))
    assert rc == 1
    assert "fixed scratch" in G.lib().gtn_last_error().decode()
