"""Commit policies and the decode loop, restated in NumPy / Python (test infrastructure).

Restates from ``python/src/edllm/backends/diffusion_runtime.py``:
  * ``MaskState.masked_positions`` / ``finalize`` (:387-558)
  * ``BlockLayout`` with origin 0 (:1099-1141)
  * ``BD3FixedQuotaCommit.plan`` / ``select`` (:1200-1346)
  * ``_block_frontier_plan`` + ``BlockThresholdCommit`` (:1023-1095), plus an optional per-block
    round budget (``rounds_cap``) that the reference does not have (0 = reference rule)
  * ``EntropyCountCommit`` (:904-941)
  * ``run_decode_loop`` (:1829-1991): plan -> (forward + score) -> select -> commit.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Callable

import numpy as np

from . import selector


@dataclass
class Canvas:
    x: list
    prompt_len: int
    mask_id: int
    eos_id: int

    def masked(self) -> list[int]:
        return [p for p in range(self.prompt_len, len(self.x)) if self.x[p] == self.mask_id]

    def finalize(self) -> dict:
        gen = self.x[self.prompt_len:]
        if self.eos_id in gen:
            answer, hit, reason = gen[: gen.index(self.eos_id)], True, "stop"
        else:
            answer, hit, reason = gen, False, "length"
        remaining = answer.count(self.mask_id)
        visible = answer[: answer.index(self.mask_id)] if remaining else answer
        return {"visible_token_ids": list(visible), "hit_eos": hit, "remaining_mask_count": remaining,
                "finish_reason": "length" if remaining else reason}


@dataclass
class Plan:
    action: str  # "proceed" | "skip" | "stop"
    frontier: list = field(default_factory=list)
    window_end: int | None = None


class BD3FixedQuota:
    """Absolute blocks from origin 0; steps_per_block rounds; quota divmod(initial, rounds)."""

    def __init__(self, *, block_size: int, steps: int, prompt_len: int, gen_len: int, require_alignment: bool = True):
        self.bs, self.steps = int(block_size), int(steps)
        self.start, self.length = int(prompt_len), int(gen_len)
        self.require_alignment = require_alignment
        self._active = None
        self._base = self._rem = self._round = 0

    @property
    def block_count(self) -> int:
        if self.length == 0:
            return 0
        return (self.start + self.length - 1) // self.bs - self.start // self.bs + 1

    @property
    def steps_per_block(self) -> int:
        if self.block_count == 0:
            return 0
        sched = (self.length + self.bs - 1) // self.bs
        return (self.steps + sched - 1) // sched

    @property
    def iteration_limit(self) -> int:
        return self.block_count * self.steps_per_block

    def span(self, index: int) -> tuple[int, int]:
        grid = (self.start // self.bs + index) * self.bs
        return max(self.start, grid), min(self.start + self.length, grid + self.bs)

    def plan(self, c: Canvas, step: int) -> Plan:
        if step >= self.iteration_limit:
            return Plan("stop")
        if self.require_alignment and c.prompt_len % self.bs:
            raise ValueError("BD3LM Candidate prompt length must be a multiple of block_size")
        spb = self.steps_per_block
        if step % spb == 0 and c.eos_id in c.x[c.prompt_len:]:
            return Plan("stop")
        masked = c.masked()
        if not masked:
            return Plan("stop")
        block = step // spb
        lo, hi = self.span(block)
        frontier = [p for p in masked if lo <= p < hi]
        if self._active != block:
            self._active = block
            self._base, self._rem = divmod(len(frontier), spb)
        self._round = step % spb
        if not frontier or self._base + int(self._round < self._rem) == 0:
            return Plan("skip")
        return Plan("proceed", frontier, hi)

    def quota(self) -> int:
        return self._base + int(self._round < self._rem)

    def select(self, scores) -> list[int]:
        return selector.topk_choices(scores, self.quota())


class BlockThreshold:
    """Prompt-relative left-to-right blocks; commit conf >= tau (floor one). ``rounds_cap``>0
    advances past a block after that many rounds with its residual masks left."""

    def __init__(self, *, block_size: int, threshold: float, rounds_cap: int = 0):
        self.bs, self.tau, self.cap = int(block_size), float(threshold), int(rounds_cap)
        self._index = 0
        self._rounds = 0

    def plan(self, c: Canvas, step: int) -> Plan:
        fill = list(range(c.prompt_len, len(c.x)))
        if self.cap > 0 and self._rounds >= self.cap:
            self._index += self.bs
            self._rounds = 0
        while self._index < len(fill):
            block = fill[self._index:self._index + self.bs]
            frontier = [p for p in block if c.x[p] == c.mask_id]
            if frontier:
                return Plan("proceed", frontier, block[-1] + 1)
            self._index += self.bs
            self._rounds = 0
        return Plan("stop")

    def select(self, scores) -> list[int]:
        self._rounds += 1
        return selector.threshold_choices(scores, self.tau)


class EntropyCount:
    """linspace(1, eps, steps + 1, f32) schedule; transfer int(N * (1 - s / t)), all at the end."""

    def __init__(self, *, eps: float, steps: int):
        self.eps, self.steps = float(eps), int(steps)
        self._k = 0

    def plan(self, c: Canvas, step: int) -> Plan:
        ts = np.linspace(1.0, self.eps, self.steps + 1, dtype=np.float32)
        masked = c.masked()
        if not masked:
            return Plan("stop")
        t, s = float(ts[step]), float(ts[step + 1])
        self._k = int(len(masked) * (1.0 - s / t)) if step < self.steps - 1 else len(masked)
        if self._k <= 0:
            return Plan("skip", masked)
        return Plan("proceed", masked, None)

    def select(self, scores) -> list[int]:
        return selector.topk_choices(scores, self._k)


ScoreFn = Callable[[Canvas, list, "int | None", int], tuple]


def run_loop(c: Canvas, policy, score_fn: ScoreFn, iteration_limit: int, trace: list | None = None) -> dict:
    """The generic loop; ``score_fn(canvas, frontier, window_end, step) -> (scores, tokens)``."""
    forwards = committed = 0
    for step in range(int(iteration_limit)):
        plan = policy.plan(c, step)
        if plan.action == "stop":
            break
        if plan.action == "skip":
            continue
        scores, tokens = score_fn(c, list(plan.frontier), plan.window_end, step)
        forwards += 1
        rows = policy.select(scores)
        for r in rows:
            c.x[plan.frontier[r]] = int(tokens[r])
        committed += len(rows)
        if trace is not None:
            trace.append({"step": step, "frontier": list(plan.frontier), "window_end": plan.window_end,
                          "scores": np.asarray(scores, dtype=np.float64).copy(), "tokens": [int(t) for t in tokens],
                          "chosen": sorted(int(r) for r in rows)})
    out = c.finalize()
    out.update(forward_count=forwards, committed_token_count=committed, x=list(c.x))
    return out
