"""Continuous batching over a model's slots (gtn_slot_start / gtn_slots_step / gtn_slot_finish).

The reference decodes one sequence per greedy_sample call (src/gten/sampler.cpp:11-53, driven by
the chat loop of src/nanochat.cpp), so a server built on it runs requests one after another. Here
requests of any prompt length and any number of new tokens share the decode steps: a request is
prefilled into a free slot as soon as one opens, every step advances all busy slots, and a slot is
freed the moment its request has its tokens (or produced the EOS id, where the reference's loop
stops, sampler.cpp:44-46). Each request gets exactly the ids it would get alone.

The engine object needs ``slot_start(prompt) -> (slot, first_id)``, ``slots_step() -> ids``
(one entry per slot, -1 for idle ones), ``slot_finish(slot)``, ``max_batch`` and ``max_ctx``:
gten_b200.Model provides them.
"""
from __future__ import annotations

from collections import deque
from dataclasses import dataclass, field


@dataclass
class Request:
    rid: object
    prompt: list
    n_gen: int
    eos: int | None = None
    out: list = field(default_factory=list)


class ContinuousBatcher:
    def __init__(self, engine):
        self.engine = engine
        self.queue: deque[Request] = deque()
        self.slots: dict[int, Request] = {}
        self.steps = 0          # decode steps run
        self.busy_slot_steps = 0  # sum over steps of the busy slots

    def submit(self, rid, prompt, n_gen: int, eos: int | None = None) -> None:
        """Queues a request; prompt + n_gen - 1 must fit the model's context (as gtn_model_generate)."""
        prompt = [int(t) for t in prompt]
        if not prompt or n_gen < 1:
            raise ValueError("a request needs a prompt and at least one new token")
        if len(prompt) + n_gen - 1 > self.engine.max_ctx:
            raise ValueError(f"request {rid!r}: {len(prompt)} + {n_gen} - 1 tokens exceed max_ctx "
                             f"{self.engine.max_ctx}")
        self.queue.append(Request(rid, prompt, n_gen, eos))

    def _done(self, r: Request) -> bool:
        return len(r.out) >= r.n_gen or (r.eos is not None and r.out and r.out[-1] == r.eos)

    def _admit(self, results: dict) -> None:
        while self.queue and len(self.slots) < self.engine.max_batch:
            r = self.queue.popleft()
            slot, first = self.engine.slot_start(r.prompt)
            r.out.append(int(first))
            if self._done(r):
                self.engine.slot_finish(slot)
                results[r.rid] = r.out
            else:
                self.slots[slot] = r

    def run(self) -> dict:
        """Serves every queued request; returns {rid: generated ids}."""
        results: dict = {}
        self._admit(results)
        while self.slots:
            ids = self.engine.slots_step()
            self.steps += 1
            self.busy_slot_steps += len(self.slots)
            for slot in list(self.slots):
                r = self.slots[slot]
                t = int(ids[slot])
                if t < 0:
                    raise RuntimeError(f"slot {slot} of request {r.rid!r} returned no id")
                r.out.append(t)
                if self._done(r):
                    self.engine.slot_finish(slot)
                    del self.slots[slot]
                    results[r.rid] = r.out
            self._admit(results)
        return results
