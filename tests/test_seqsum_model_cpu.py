"""The method behind the exact parallel sum of squares, checked on the CPU.

The reference's RMSNorm adds the squares one at a time in fp32 (ops.cpp:830-836). The library
reproduces that chain in parallel (nanochatllms.cpp_b200/csrc/seqsum.cuh):
  * an exact fixed-point prefix sum predicts the binade of the running sum after every term;
  * inside a binade every add rounds to multiples of one ulp, so each term becomes an integer
    increment, and a tie (half an ulp) rounds by the parity of the running value;
  * one record per binade (head term, exponent field, first-tie parity, increments saturated at
    2^25) is walked in 32-bit integer steps, and every crossing is checked;
  * any failed check takes the plain serial loop.

`exact_sum_model` restates that integer arithmetic in numpy, step for step, so that the method can
be checked against the serial fp32 loop on many more rows than a GPU test holds. The GPU tests
(tests/test_gpu_ops.py) compare the CUDA code itself with the oracle. Pure CPU test infrastructure.
"""
from collections import defaultdict

import numpy as np
import pytest

FRAC_BITS = 25  # the largest term becomes < 2^(24 + 25) in fixed point
TIES_MAX = 128


def serial_sum(p: np.ndarray) -> np.float32:
    """The reference's loop: fl(...fl(fl(0 + p0) + p1)... + p_{n-1}); numpy's accumulate is a
    strictly sequential float32 loop."""
    return np.float32(0.0) if p.size == 0 else np.cumsum(p, dtype=np.float32)[-1]


def bit_length(q: np.ndarray) -> np.ndarray:
    """floor(log2(q)) + 1 for non-negative int64 values, exactly (0 for 0)."""
    bl = np.zeros(q.shape, np.int64)
    for b in range(63):
        bl += (q >> b) > 0
    return bl


def exact_sum_model(p: np.ndarray):
    """(sum, fast): the sum as the parallel method computes it, and whether it took the fast path
    (False: one of its checks failed and the serial loop gave the result)."""
    p = np.ascontiguousarray(p, np.float32)
    n = p.size
    if n == 0:
        return np.float32(0.0), True
    bits = p.view(np.uint32).astype(np.int64)
    maxbits = int(bits.max())
    if maxbits == 0:
        return np.float32(0.0), True
    if maxbits >= 0x7F800000 or n > (1 << 14):  # inf / nan / a negative term; the int64 bound
        return serial_sum(p), False
    emax = (maxbits >> 23) - 127 if maxbits >= 0x800000 else -126
    eoff = 23 + FRAC_BITS - emax  # binade exponent of fixed-point slot sl: e = sl - eoff
    ef = bits >> 23
    m = (bits & 0x7FFFFF) | np.where(ef != 0, 0x800000, 0)
    e_term = np.where(ef != 0, ef - 127, -126)
    # fixed-point terms floor(p * 2^eoff) and their exact prefix: the predicted binade slots
    sh = e_term - emax + FRAC_BITS
    fx = np.where(sh >= 0, m << np.clip(sh, 0, 63), np.where(sh > -32, m >> np.clip(-sh, 0, 63), 0))
    q = np.cumsum(fx)
    slot = bit_length(q) - 1
    if np.any((q == 0) & (p != 0)):  # a non-zero term below the fixed-point resolution
        return serial_sum(p), False
    prev = np.concatenate([[-1], slot[:-1]])
    live = slot >= 0
    head = live & (slot != prev)
    rest = live & ~head
    e = slot - eoff
    sh2 = e - e_term  # p / u = m * 2^-sh2 with u the binade's ulp
    if np.any(rest & ((sh2 < 0) | (e < -126))):
        return serial_sum(p), False
    shc = np.clip(sh2, 1, 31)
    rem = m & ((np.int64(1) << shc) - 1)
    half = np.int64(1) << (shc - 1)
    v = np.where(sh2 == 0, m, (m >> shc) + (rem > half))
    v = np.where((sh2 < 0) | (sh2 >= 32), 0, v)
    inc = np.where(rest, v, 0)
    tie = rest & (sh2 > 0) & (sh2 < 32) & (rem == half)
    cur = np.cumsum(inc)  # inclusive increment prefix (a head's own increment is 0)
    total = int(cur[-1])
    heads = np.nonzero(head)[0]
    hpre = {int(slot[h]): int(cur[h]) for h in heads}
    phead = {int(slot[h]): p[h] for h in heads}
    # ties in index order: the first tie of a binade rounds by the parity of its increments since
    # the head; later ones by the change of that parity since the previous tie
    ties = np.nonzero(tie)[0]
    if ties.size > TIES_MAX:
        return serial_sum(p), False
    tslot = [int(slot[t]) for t in ties]
    tpar = [int(cur[t]) & 1 for t in ties]
    d0, x = {}, defaultdict(int)
    for r, sl in enumerate(tslot):
        if r == 0 or tslot[r - 1] != sl:
            d0[sl] = (tpar[r] ^ (hpre[sl] & 1)) & 1
        else:
            x[sl] += (tpar[r] ^ tpar[r - 1]) & 1
    # the walk over the binade records
    order = [int(slot[h]) for h in heads]
    s = np.float32(0.0)
    ok = True
    for j, sl in enumerate(order):
        nxt = hpre[order[j + 1]] if j + 1 < len(order) else total
        add = min(nxt - hpre[sl] + x[sl], 1 << 25)
        eb = sl - eoff
        y = (eb + 127) << 23 if -126 <= eb <= 127 else -1
        z = d0.get(sl, -1)
        s = np.float32(s + phead[sl])
        b = int(np.array([s], np.float32).view(np.int32)[0])
        sb = (b & 0x7FFFFF) | 0x800000
        up = (sb + z) & (1 if z >= 0 else 0)
        sn = sb + add + up
        ok = ok and (b & 0x7F800000) == y and sn < (1 << 24)
        if not ok:
            break
        s = np.array([y | (sn & 0x7FFFFF)], np.int32).view(np.float32)[0]
    if not ok:
        return serial_sum(p), False
    return np.float32(s), True


def _rows(rng, d, count):
    """Mixed distributions of residual-like rows, as float32."""
    out = []
    for r in range(count):
        kind = r % 8
        if kind == 0:
            v = rng.standard_normal(d) * 10.0 ** rng.uniform(-3, 3)
        elif kind == 1:
            v = rng.standard_normal(d)
            v[rng.integers(0, d, 4)] *= rng.uniform(10, 200)
        elif kind == 2:  # Q8-dequantized blocks: q * fp16(delta)
            dl = rng.uniform(1e-3, 1.0, (d + 31) // 32).astype(np.float16).astype(np.float64)
            v = rng.integers(-127, 128, d) * np.repeat(dl, 32)[:d]
        elif kind == 3:  # a coarse grid: many exact ties
            v = rng.integers(-8, 9, d) * 2.0 ** int(rng.integers(-10, 10))
        elif kind == 4:
            v = np.sign(rng.standard_normal(d)) * 10.0 ** rng.uniform(-6, 4, d)
        elif kind == 5:
            v = rng.standard_normal(d) * (rng.random(d) < 0.5)
        elif kind == 6:  # short mantissas
            v = 1.0 + 2.0 ** -12 * rng.integers(0, 8, d)
        else:  # tiny terms, then large ones (the first terms fall below the fixed-point
            # resolution, so the method takes the serial loop)
            v = np.concatenate([rng.standard_normal(d // 2) * 1e-6, rng.standard_normal(d - d // 2)])
        out.append((kind, (v.astype(np.float32) ** 2).astype(np.float32)))
    return out


@pytest.mark.parametrize("d", [2048, 2304, 1000])
def test_model_matches_serial_loop(d):
    rng = np.random.default_rng(d)
    fast = defaultdict(int)
    rows = _rows(rng, d, 240)
    for kind, p in rows:
        got, used_fast = exact_sum_model(p)
        want = serial_sum(p)
        assert got.tobytes() == want.tobytes(), (kind, got, want)
        fast[kind] += used_fast
    # the residual-like rows take the parallel path almost always
    for kind in (0, 1, 2, 5):
        assert fast[kind] >= 0.9 * (len(rows) // 8), (kind, fast[kind])


def test_model_edge_cases():
    cases = [
        np.zeros(2048, np.float32),
        np.full(2048, 3.0, np.float32),
        np.ones(1, np.float32),
        np.array([0.0, 0.0, 5.0, 0.0], np.float32),
        np.full(2048, np.float32(1e-20) ** 2, np.float32),  # subnormal squares
        np.array([1.0, np.inf, 2.0], np.float32),
        (2.0 ** np.arange(-20, 20, dtype=np.float64)).astype(np.float32),
        np.array([2.0 ** 24] + [1.0] * 100, np.float32),  # every later add is a tie at 2^24
        np.array([2.0 ** 24 + 2] + [1.0] * 100, np.float32),
    ]
    for p in cases:
        got, _ = exact_sum_model(p)
        want = serial_sum(p)
        assert got.tobytes() == want.tobytes(), (p[:4], got, want)
