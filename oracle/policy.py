"""Commit policies and the decode loop, restated in NumPy / Python (test infrastructure).

Restates from ``python/src/edllm/backends/diffusion_runtime.py``:
  * ``MaskState.masked_positions`` / ``finalize`` (:387-558)
  * ``BlockLayout`` with origin 0 (:1099-1141)
  * ``BD3FixedQuotaCommit.plan`` / ``select`` (:1200-1346)
  * ``_block_frontier_plan`` + ``BlockThresholdCommit`` (:1023-1095), plus an optional per-block
    round budget (``rounds_cap``) that the reference does not have (0 = reference rule)
  * ``EntropyCountCommit`` (:904-941)
  * ``D2FBlockPipelineCommit`` (:1416-1694), threshold commit rule, no revision window, no
    initial frozen blocks
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


class D2FPipeline:
    """A sliding window of prompt-relative blocks decoded together (D2FBlockPipelineCommit):

    plan, per step: blocks with no mask leave the window oldest-first (frozen); a committed EOS in
    the appended region stops appending; at most one new block joins when the last appended
    block's decoded ratio is >= tau_add (the prompt counts as 1.0); block j is fully activated when
    block j - 1's ratio is >= tau_act (the prompt / a frozen block: 1.0); the frontier is every
    masked position of the unfrozen appended blocks, the window ends at the last appended block.
    select: per unfrozen appended block, the rows whose score is strictly > tau_conf, else, for a
    fully-activated block, its first most-confident row.

    Activation is sticky in the reference; decoded ratios never fall (nothing is remasked), so
    "block j - 1's ratio is >= tau_act now" is the same set."""

    def __init__(self, *, block_size: int, threshold: float, add_threshold: float = 0.1,
                 activate_threshold: float = 0.95):
        self.bs, self.tau = int(block_size), float(threshold)
        self.tau_add, self.tau_act = float(add_threshold), float(activate_threshold)
        self._spans = None
        self._frozen = 0
        self._appended = 0
        self._eos = False
        self._active = []       # (lo, hi, activated) of this step's unfrozen appended blocks
        self._frontier = []

    def _ratio(self, c: Canvas, j: int) -> float:
        lo, hi = self._spans[j]
        masked = sum(1 for p in range(lo, hi) if c.x[p] == c.mask_id)
        return (hi - lo - masked) / (hi - lo)

    def plan(self, c: Canvas, step: int) -> Plan:
        if self._spans is None:
            start, n = c.prompt_len, len(c.x) - c.prompt_len
            self._spans = [(start + j, min(start + j + self.bs, start + n)) for j in range(0, n, self.bs)]
        while self._frozen < self._appended:
            lo, hi = self._spans[self._frozen]
            if any(c.x[p] == c.mask_id for p in range(lo, hi)):
                break
            self._frozen += 1
        if not self._eos and self._appended:
            lo, hi = self._spans[0][0], self._spans[self._appended - 1][1]
            self._eos = any(c.x[p] == c.eos_id for p in range(lo, hi))
        if self._appended < len(self._spans) and not self._eos:
            last = 1.0 if self._appended == 0 else self._ratio(c, self._appended - 1)
            if last >= self.tau_add:
                self._appended += 1
        self._active = []
        for j in range(self._frozen, self._appended):
            prev = 1.0 if j == 0 else self._ratio(c, j - 1)
            self._active.append((*self._spans[j], prev >= self.tau_act))
        if not self._active:
            return Plan("stop")
        self._frontier = [p for lo, hi, _ in self._active for p in range(lo, hi) if c.x[p] == c.mask_id]
        return Plan("proceed", list(self._frontier), self._spans[self._appended - 1][1])

    @property
    def frozen_end(self) -> int:
        """First position of the oldest unfrozen block (the exact K/V prefix ends there)."""
        return self._active[0][0] if self._active else len(self._spans or [])

    def select(self, scores) -> list[int]:
        conf = np.asarray(scores, dtype=np.float64)
        chosen = []
        for lo, hi, activated in self._active:
            rows = [r for r, p in enumerate(self._frontier) if lo <= p < hi]
            if not rows:
                continue
            clear = [r for r in rows if conf[r] > self.tau]
            if clear:
                chosen.extend(clear)
            elif activated:
                chosen.append(rows[int(np.argmax(conf[rows]))])
        return chosen


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
