"""The continuous-batching scheduler (gten_b200/serve.py) on a fake slot engine (no GPU): every
request gets exactly its single-sequence ids, slots never exceed max_batch and are reused, EOS
stops a request, and requests that cannot fit the context are refused."""
import numpy as np
import pytest

from gten_b200.serve import ContinuousBatcher


def _next(prompt_sum, t):
    return (prompt_sum * 31 + t * 17 + 7) % 1000


class FakeSlots:
    """A deterministic engine: the id after token t of a sequence depends on t and its prompt."""

    def __init__(self, max_batch, max_ctx):
        self.max_batch, self.max_ctx = max_batch, max_ctx
        self.state = {}  # slot -> [prompt_sum, last id, position]
        self.starts = self.max_busy = 0

    def slot_start(self, prompt):
        free = [s for s in range(self.max_batch) if s not in self.state]
        assert free, "slot_start with every slot busy"
        s = free[0]
        ps = sum(prompt)
        first = _next(ps, prompt[-1])
        self.state[s] = [ps, first, len(prompt)]
        self.starts += 1
        self.max_busy = max(self.max_busy, len(self.state))
        return s, first

    def slots_step(self):
        ids = np.full(self.max_batch, -1, np.int32)
        for s, st in self.state.items():
            assert st[2] < self.max_ctx, "a slot stepped past max_ctx"
            st[1] = _next(st[0], st[1])
            st[2] += 1
            ids[s] = st[1]
        return ids

    def slot_finish(self, s):
        del self.state[s]


def _alone(prompt, n_gen, eos=None):
    out, t, ps = [], prompt[-1], sum(prompt)
    for _ in range(n_gen):
        t = _next(ps, t)
        out.append(t)
        if eos is not None and t == eos:
            break
    return out


@pytest.mark.parametrize("max_batch", [1, 3, 8])
def test_every_request_gets_its_single_sequence_ids(max_batch):
    rng = np.random.default_rng(max_batch)
    eng = FakeSlots(max_batch, 64)
    b = ContinuousBatcher(eng)
    reqs = {}
    for i in range(25):
        p = rng.integers(0, 1000, int(rng.integers(1, 30))).tolist()
        n = int(rng.integers(1, 64 - len(p) + 2))
        reqs[i] = (p, n)
        b.submit(i, p, n)
    res = b.run()
    assert set(res) == set(reqs)
    for i, (p, n) in reqs.items():
        assert res[i] == _alone(p, n)
    assert eng.max_busy <= max_batch and not eng.state and eng.starts == 25
    assert b.busy_slot_steps == sum(n - 1 for _, n in reqs.values())


def test_eos_stops_a_request():
    eng = FakeSlots(2, 100)
    b = ContinuousBatcher(eng)
    p = [5, 9, 11]
    full = _alone(p, 40)
    eos = full[6]
    b.submit("a", p, 40, eos=eos)
    b.submit("b", [3], 10)
    res = b.run()
    assert res["a"] == full[:7] and res["b"] == _alone([3], 10)


def test_requests_that_do_not_fit_are_refused():
    b = ContinuousBatcher(FakeSlots(2, 16))
    with pytest.raises(ValueError):
        b.submit(0, list(range(10)), 8)
    with pytest.raises(ValueError):
        b.submit(1, [], 3)
    b.submit(2, list(range(10)), 7)  # 10 + 7 - 1 = 16 fits
    assert b.run()[2] == _alone(list(range(10)), 7)
