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
