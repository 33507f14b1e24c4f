"""A minimal continuous-batching scheduler over the engine's sequence slots (eahmmf_engine_set_slots /
prefill_slot / step_slots).

The reference serves one sequence at a time (its Engine holds one KV cache, qwen3moe.cpp:791, :910-913,
and its generate loop feeds one token per forward call, :1294-1310). Here requests queue up; whenever a
slot is free the next request's prompt is prefilled into it, and every step runs one token of every
active sequence as a single forward pass. A sequence leaves when it has its tokens, and its slot takes
the next request at once. Greedy selection; per-sequence tokens equal that sequence decoded alone.
"""
from __future__ import annotations

import dataclasses
from collections import deque


@dataclasses.dataclass
class Request:
    prompt: list
    n_gen: int
    tokens: list = dataclasses.field(default_factory=list)  # generated so far (the first from the prompt)
    slot: int = -1
    pos: int = 0  # position of the next input token


class ContinuousBatcher:
    """Run requests through an engine with `n_slots` sequence slots, at most `max_rows` (<= 64) per step."""

    def __init__(self, engine, n_slots: int, max_rows: int = 64, n_batch: int = 64):
        if engine.set_slots(n_slots):
            raise RuntimeError("eahmmf_engine_set_slots failed")
        self.e, self.n_slots, self.max_rows, self.n_batch = engine, n_slots, min(max_rows, 64), n_batch
        self.queue: deque = deque()
        self.active: dict = {}  # slot -> Request
        self.steps = 0
        self.rows = 0  # sequence-tokens decoded by steps (throughput accounting)

    def submit(self, prompt, n_gen: int) -> Request:
        r = Request(list(map(int, prompt)), int(n_gen))
        self.queue.append(r)
        return r

    def _admit(self):
        free = [s for s in range(self.n_slots) if s not in self.active]
        while free and self.queue and len(self.active) < self.max_rows:
            r = self.queue.popleft()
            r.slot = free.pop(0)
            rc, first = self.e.prefill_slot(r.slot, r.prompt, self.n_batch)
            if rc:
                raise RuntimeError(f"eahmmf_engine_prefill_slot returned {rc}")
            r.tokens.append(first)
            r.pos = len(r.prompt)
            if len(r.tokens) < r.n_gen:
                self.active[r.slot] = r

    def step(self) -> bool:
        """Admit what fits, then one token of every active sequence. False when nothing is left."""
        self._admit()
        if not self.active:
            return False
        rs = list(self.active.values())
        rc, nxt = self.e.step_slots([r.slot for r in rs], [r.pos for r in rs], [r.tokens[-1] for r in rs])
        if rc:
            raise RuntimeError(f"eahmmf_engine_step_slots returned {rc}")
        self.steps += 1
        self.rows += len(rs)
        for r, t in zip(rs, nxt):
            r.tokens.append(int(t))
            r.pos += 1
            if len(r.tokens) >= r.n_gen:
                del self.active[r.slot]
        return True

    def run(self):
        while self.step():
            pass
