"""Top-k / temperature sampling (sampler.cpp:63-128) with a seeded generator: the CPU oracle
(oracle/sampler_oracle.cpp, libstdc++'s std::mt19937 and std::discrete_distribution), and a numpy
restatement of the MT19937 steps the device sampler runs, checked against std::mt19937."""
import ctypes as C

import numpy as np
import pytest

from oracle.oracle import SamplerOracle


@pytest.fixture(scope="module")
def so():
    return SamplerOracle()


def mt19937_np(seed: int, n: int) -> np.ndarray:
    """The generator of csrc/sample.cu (seeding of gtn_rng_create, twist and tempering of mt_next)."""
    st = [seed & 0xFFFFFFFF]
    for i in range(1, 624):
        st.append((1812433253 * (st[-1] ^ (st[-1] >> 30)) + i) & 0xFFFFFFFF)
    out, idx = [], 624
    for _ in range(n):
        if idx >= 624:
            for k in range(624):
                y = (st[k] & 0x80000000) | (st[(k + 1) % 624] & 0x7FFFFFFF)
                st[k] = st[(k + 397) % 624] ^ (y >> 1) ^ (0x9908B0DF if y & 1 else 0)
            idx = 0
        y = st[idx]
        idx += 1
        y ^= y >> 11
        y ^= (y << 7) & 0x9D2C5680
        y ^= (y << 15) & 0xEFC60000
        y ^= y >> 18
        out.append(y & 0xFFFFFFFF)
    return np.array(out, np.uint32)


@pytest.mark.parametrize("seed", [0, 1, 5489, 0xDEADBEEF])
def test_mt19937_restatement_matches_std(so, seed):
    n = 1500  # crosses two twists
    want = np.zeros(n, np.uint32)
    so.lib.or_mt19937(C.c_uint32(seed), n, want.ctypes.data_as(C.c_void_p))
    assert np.array_equal(mt19937_np(seed, n), want)


def test_oracle_top1_is_first_argmax(so):
    rng = np.random.default_rng(1)
    x = rng.standard_normal((20, 300)).astype(np.float32)
    got = so.topk_sample(x, 0.8, 1, seed=3)
    assert np.array_equal(got, np.argmax(x, axis=1))


def test_oracle_draws_stay_in_top_k_and_repeat_with_the_seed(so):
    rng = np.random.default_rng(2)
    x = rng.standard_normal((200, 1000)).astype(np.float32) * 3
    a = so.topk_sample(x, 1.0, 7, seed=11)
    b = so.topk_sample(x, 1.0, 7, seed=11)
    assert np.array_equal(a, b)
    top = np.argsort(-x, axis=1)[:, :7]
    assert all(a[i] in top[i] for i in range(len(a)))
    assert len(set(a.tolist())) > 1


def test_oracle_rejects_bad_arguments(so):
    x = np.zeros((1, 10), np.float32)
    with pytest.raises(ValueError):
        so.topk_sample(x, 1.0, 11, seed=0)
    with pytest.raises(ValueError):
        so.topk_sample(x, 0.0, 3, seed=0)
