"""Device top-k / temperature sampling (gtn_sample_topk) against the CPU oracle running the
reference's step with the same std::mt19937 seed: identical token ids draw after draw (the
generator state carries over between draws and across its 624-word twists)."""
import numpy as np
import pytest
import torch

import gten_b200 as G
from oracle.oracle import SamplerOracle

pytestmark = pytest.mark.gpu


def _distinct(x):
    """Rows whose values are all distinct (ties at the top-k boundary are resolved differently)."""
    return all(len(np.unique(r)) == r.size for r in x)


def _logits(rng, draws, n):
    """Rows of n distinct float32 values drawn from a normal distribution of scale 2.5."""
    rows = []
    for _ in range(draws):
        v = np.unique((rng.standard_normal(2 * n) * 2.5).astype(np.float32))
        assert v.size >= n
        rows.append(rng.permutation(v)[:n])
    return np.stack(rows)


@pytest.mark.parametrize("n,temp,top_k,draws,seed", [
    (32003, 1.0, 40, 24, 7),      # TinyLlama vocabulary
    (32003, 0.7, 1000, 8, 8),     # the reference's clamp of top_k
    (4096, 3.5, 5, 40, 9),        # temp clamped to 2.0
    (50, 1.0, 50, 400, 10),       # all tokens; 800 outputs: two twists of the generator
    (100, 0.25, 1, 10, 11),       # greedy through the sampler
    (1000, 1.3, 1700, 6, 12),     # top_k above 1000 clamps
])
def test_sample_topk_matches_reference_step(gpu, n, temp, top_k, draws, seed):
    rng = np.random.default_rng(seed)
    x = _logits(rng, draws, n)
    assert _distinct(x)
    want = SamplerOracle().topk_sample(x, temp, top_k, seed)
    r = G.Rng(seed)
    dev = torch.from_numpy(x).to(gpu)
    out = torch.zeros(draws, dtype=torch.int32, device=gpu)
    for d in range(draws):
        G.sample_topk(dev[d], temp, top_k, r, out[d:d + 1])
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy(), want)
    r.close()


def test_sample_topk_argument_errors(gpu):
    x = torch.zeros(10, dtype=torch.float32, device=gpu)
    out = torch.zeros(1, dtype=torch.int32, device=gpu)
    r = G.Rng(1)
    with pytest.raises(G.GtenError):
        G.sample_topk(x, 1.0, 11, r, out)
    with pytest.raises(G.GtenError):
        G.sample_topk(x, 0.0, 3, r, out)
    r.close()


def _device_steps(gpu, rows, temp, top_k, seed):
    r = G.Rng(seed)
    out = torch.zeros(len(rows), dtype=torch.int32, device=gpu)
    for d, row in enumerate(rows):
        G.sample_topk(torch.from_numpy(np.ascontiguousarray(row, np.float32)).to(gpu), temp, top_k, r, out[d:d + 1])
    torch.cuda.synchronize()
    r.close()
    return out.cpu().numpy().tolist()


def test_sample_topk_duplicates_inside_the_selection(gpu):
    """Values repeated inside the top k (a gap below the k-th largest): the selection is unambiguous."""
    rng = np.random.default_rng(3)
    n, k, rows = 5000, 60, []
    for _ in range(30):
        hi = np.repeat(rng.standard_normal(20).astype(np.float32) + 10, 3)
        lo = np.minimum(rng.standard_normal(n - hi.size).astype(np.float32), hi.min() - 1)
        row = np.concatenate([hi, lo])
        rng.shuffle(row)
        rows.append(row)
    g = SamplerOracle().generator(44)
    assert _device_steps(gpu, rows, 0.9, k, 44) == [g.step(r, 0.9, k) for r in rows]


def test_sample_topk_all_equal_takes_the_first_k(gpu):
    """All logits equal: the reference's heap selection keeps the first k indices, as the device does
    (this takes the refining radix passes and the in-order gather of tied keys)."""
    rows = [np.full(3000, 0.5, np.float32) for _ in range(20)]
    g = SamplerOracle().generator(45)
    want = [g.step(r, 1.0, 50) for r in rows]
    assert max(want) < 50
    assert _device_steps(gpu, rows, 1.0, 50, 45) == want


def test_sample_topk_single_entry_draws_nothing(gpu):
    """n = 1 returns 0 without advancing the generator (std::discrete_distribution with one weight)."""
    rng = np.random.default_rng(4)
    rows = [rng.standard_normal(m).astype(np.float32) for m in (7, 1, 9, 1, 1, 2, 300)]
    g = SamplerOracle().generator(46)
    want = [g.step(r, 1.0, min(5, r.size)) for r in rows]
    r = G.Rng(46)
    out = torch.zeros(len(rows), dtype=torch.int32, device=gpu)
    for d, row in enumerate(rows):
        G.sample_topk(torch.from_numpy(row).to(gpu), 1.0, min(5, row.size), r, out[d:d + 1])
    torch.cuda.synchronize()
    r.close()
    assert out.cpu().numpy().tolist() == want
