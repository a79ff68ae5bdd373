"""Executable model of the peer-memory all-reduce protocols, for race detection on the CPU.

The fused all-reduce kernels (csrc/allreduce.cuh, csrc/allreduce_norm.cuh) coordinate W
ranks through flags in each other's memory: CTA b of every rank handles the same units,
publishes a flag per (phase, block, source) with the per-block epoch e, and waits until
the W flags it needs reach e.  Consecutive calls reuse the same slots, so correctness
also depends on no rank overwriting a slot that a slower peer still reads.  This module
replays those protocols step by step (every peer store, flag store and slot read is one
step) under a randomised scheduler that runs the ranks' CTAs in any interleaving,
including ranks that fall a whole call behind, and checks:

* every slot read returns the value written for that call by that source (no stale
  data, no overwrite by a later call, across calls whose grid size and message size
  differ, so that unit ownership and slot strides move between calls);
* the run finishes (no deadlock), also when only ``capacity`` CTAs of a rank are
  resident at a time and the rest are dispatched in block order as CTAs retire.

The memory model is sequentially consistent: the release / acquire pairs of the kernels
(st.release.sys / ld.acquire.sys, with __syncthreads between a CTA's stores and its flag
release) are abstracted as ordered steps.  What is checked is the protocol's logic.

Protocols (``algo`` of a call):
  two_shot        phase 1 scatter -> RS flags -> reduce -> AG scatter -> AG flags -> gather
                  (two_shot_kernel, two_shot16_kernel, two_shot_norm*_kernel)
  one_shot        every rank pushes its whole tensor; slots double-buffered by the parity
                  of the rank's one-shot call count, shared by all blocks of a call
                  (one_shot_kernel)
  gemm_scatter + from_gemm   the GEMM-fed two-shot: the row-parallel GEMM's epilogue
                  scatters into the reduce-scatter slots and publishes a per-rank GEMM
                  epoch; the next kernel waits for every rank's epoch and runs phases 2-3
                  (two calls of the list, always in this order)
  argmax          the cross-rank argmax gather: one CTA, double-buffered by its epoch
  one_shot_block  the same with the parity taken from each block's own epoch.  Unsafe
                  when the grid changes between calls (a unit moves to a block whose epoch
                  has the other parity); the checker finds it, and the kernel uses the
                  call count instead.
  two_shot_staged_offset  two_shot16s_kernel: each CTA's units in two stages, phase 1 of
                  stage 1 issued before the wait for stage 0, stage 1's flags at the fixed
                  block index b + STAGE_OFF of the same phases and epochs (every two-shot
                  grid stays below STAGE_OFF; a grid that does not can collide, which the
                  checker finds)
Candidate schedules, checked before they are built:
  two_shot_staged the same schedule with stage 1's flags in separate flag phases
  two_shot_staged_shared  the same with stage 1's flags at block index b + G of the
                  stage-0 phase (unsafe: a flag word is then written under two different
                  blocks' epochs)
"""
from __future__ import annotations

import random
from dataclasses import dataclass, field
from typing import Callable, Dict, Iterator, List, Optional, Tuple


class ProtocolViolation(AssertionError):
    pass


# Block index of the staged kernel's second flag set (kStageBlockOff in the kernels, where
# every two-shot grid is capped below it); the model's grids stay below this value.
STAGE_OFF = 8


@dataclass
class Call:
    algo: str
    units: int      # two-shot: units per chunk (each rank owns one chunk); one-shot: units in the tensor
    grid: int       # CTAs per rank


@dataclass
class _Rank:
    epochs: Dict[Tuple[str, int], int] = field(default_factory=dict)
    counters: Dict[str, int] = field(default_factory=dict)
    mem: Dict[Tuple, Tuple] = field(default_factory=dict)     # slot address -> tag
    flags: Dict[Tuple, int] = field(default_factory=dict)     # (phase, block, src) -> epoch


Step = Optional[Callable[[], bool]]  # None: a plain step; else a wait condition


class Model:
    def __init__(self, world: int, calls: List[Call], seed: int = 0, capacity: Optional[int] = None,
                 slow_rank_bias: float = 0.5):
        self.W = world
        self.calls = calls
        self.rng = random.Random(seed)
        self.capacity = capacity
        self.ranks = [_Rank() for _ in range(world)]
        # a skewed scheduler: one rank runs less often, so that ranks drift whole calls apart
        self.slow = self.rng.randrange(world)
        self.slow_bias = slow_rank_bias

    # -------------------------------------------------------------- memory helpers
    def _write(self, holder: int, addr: Tuple, tag: Tuple) -> None:
        self.ranks[holder].mem[addr] = tag

    def _read(self, holder: int, addr: Tuple, expect: Tuple, what: str) -> None:
        got = self.ranks[holder].mem.get(addr)
        if got != expect:
            raise ProtocolViolation(f"{what}: rank {holder} read {addr} -> {got}, expected {expect}")

    def _flag(self, holder: int, key: Tuple, e: int) -> None:
        f = self.ranks[holder].flags
        f[key] = max(f.get(key, 0), e)  # flags only move forward (epochs are monotonic)

    def _flag_geq(self, holder: int, key: Tuple, e: int) -> bool:
        return self.ranks[holder].flags.get(key, 0) >= e

    # -------------------------------------------------------------- slot addresses
    # A slot address is (region, source, unit) flattened with the call's slot stride, so
    # that calls with different sizes alias the same words the way byte offsets do.
    @staticmethod
    def _addr(region: str, src: int, unit: int, stride: int) -> Tuple:
        return (region, src * stride + unit)

    # -------------------------------------------------------------- CTA programs
    def _two_shot(self, r: int, k: int, call: Call, b: int, staged: str = "") -> Iterator[Step]:
        W, G, C = self.W, call.grid, call.units
        R = self.ranks[r]
        e = R.epochs.get(("two_shot", b), 0) + 1
        mine = [u for u in range(C) if u % G == b]
        stages = [mine] if not staged else [mine[: (len(mine) + 1) // 2], mine[(len(mine) + 1) // 2:]]

        def key(phase: str, s: int) -> Tuple:
            if not staged or s == 0:
                return (phase, b)
            if staged == "shared":  # stage 1 at block index b + G of the same phase
                return (phase, b + G)
            if staged == "offset":  # stage 1 at the fixed block index b + STAGE_OFF (the kernel's layout)
                return (phase, b + STAGE_OFF)
            return (phase + "1", b)

        for s, us in enumerate(stages):          # phase 1 of every stage
            for u in us:
                for j in range(W):
                    self._write(j, self._addr("rs", r, u, C), (k, r, u))
                    yield None
            for j in range(W):
                self._flag(j, key("rs", s) + (r,), e)
                yield None
        for s, us in enumerate(stages):          # phase 2 of every stage
            for src in range(W):
                yield (lambda src=src, s=s: self._flag_geq(r, key("rs", s) + (src,), e))
            for u in us:
                for src in range(W):
                    self._read(r, self._addr("rs", src, u, C), (k, src, u), f"two_shot{staged} phase 2 call {k}")
                    yield None
                for j in range(W):
                    if j != r:
                        self._write(j, self._addr("ag", r, u, C), (k, r, u))
                        yield None
            for j in range(W):
                if j != r:
                    self._flag(j, key("ag", s) + (r,), e)
                    yield None
        for s, us in enumerate(stages):          # phase 3 of every stage
            for src in range(W):
                if src != r:
                    yield (lambda src=src, s=s: self._flag_geq(r, key("ag", s) + (src,), e))
            for u in us:
                for src in range(W):
                    if src != r:
                        self._read(r, self._addr("ag", src, u, C), (k, src, u), f"two_shot{staged} phase 3 call {k}")
                        yield None
        R.epochs[("two_shot", b)] = e

    def _one_shot(self, r: int, k: int, call: Call, b: int, per_block_parity: bool) -> Iterator[Step]:
        W, G, U = self.W, call.grid, call.units
        R = self.ranks[r]
        e = R.epochs.get(("one_shot", b), 0) + 1
        parity = (e & 1) if per_block_parity else (R.counters.get("one_shot_calls", 0) & 1)
        region = f"os{parity}"
        mine = [u for u in range(U) if u % G == b]
        for u in mine:
            for j in range(W):
                if j != r:
                    self._write(j, self._addr(region, r, u, U), (k, r, u))
                    yield None
        for j in range(W):
            if j != r:
                self._flag(j, ("os", b, r), e)
                yield None
        for src in range(W):
            if src != r:
                yield (lambda src=src: self._flag_geq(r, ("os", b, src), e))
        for u in mine:
            for src in range(W):
                if src != r:
                    self._read(r, self._addr(region, src, u, U), (k, src, u), f"one_shot call {k}")
                    yield None
        R.epochs[("one_shot", b)] = e
        if not per_block_parity:
            # the last CTA of the call to finish advances the rank's call counter
            done = R.counters.get("one_shot_done", 0) + 1
            if done == G:
                R.counters["one_shot_done"] = 0
                R.counters["one_shot_calls"] = R.counters.get("one_shot_calls", 0) + 1
            else:
                R.counters["one_shot_done"] = done
            yield None

    def _gemm_scatter(self, r: int, k: int, call: Call, b: int) -> Iterator[Step]:
        """A row-parallel GEMM whose epilogue stores every tile straight into its owner's
        reduce-scatter slot, without waiting for anything; the last CTA to finish advances
        the rank's GEMM epoch and publishes it to every rank (gemm.cu, EPI_QS*)."""
        W, G, C = self.W, call.grid, call.units
        R = self.ranks[r]
        for j in range(W):                     # tile b covers units b, b + G, ... of every chunk
            for u in range(b, C, G):
                self._write(j, self._addr("rs", r, u, C), (k, r, u))
                yield None
        done = R.counters.get("gemm_done", 0) + 1
        if done < G:
            R.counters["gemm_done"] = done
            return
        R.counters["gemm_done"] = 0
        eg = R.counters.get("gemm_epoch", 0) + 1
        R.counters["gemm_epoch"] = eg
        for j in range(W):
            self._flag(j, ("gemm", 0, r), eg)
            yield None

    def _from_gemm(self, r: int, k: int, call: Call, b: int) -> Iterator[Step]:
        """Phases 2 and 3 after _gemm_scatter (two_shot16_kernel<..., FROM_GEMM>): wait for
        every rank's GEMM epoch, then reduce, all-gather and gather as the two-shot does.
        The data it reads were written by the previous call of the list (the GEMM)."""
        W, G, C = self.W, call.grid, call.units
        R = self.ranks[r]
        e = R.epochs.get(("two_shot", b), 0) + 1
        eg = R.counters.get("gemm_epoch", 0)   # the value this rank's GEMM just published
        kg = k - 1                             # the call index of the GEMM that wrote the slots
        for src in range(W):
            yield (lambda src=src: self._flag_geq(r, ("gemm", 0, src), eg))
        mine = [u for u in range(C) if u % G == b]
        for u in mine:
            for src in range(W):
                self._read(r, self._addr("rs", src, u, C), (kg, src, u), f"from_gemm phase 2 call {k}")
                yield None
            for j in range(W):
                if j != r:
                    self._write(j, self._addr("ag", r, u, C), (k, r, u))
                    yield None
        for j in range(W):
            if j != r:
                self._flag(j, ("ag", b, r), e)
                yield None
        for src in range(W):
            if src != r:
                yield (lambda src=src: self._flag_geq(r, ("ag", b, src), e))
        for u in mine:
            for src in range(W):
                if src != r:
                    self._read(r, self._addr("ag", src, u, C), (k, src, u), f"from_gemm phase 3 call {k}")
                    yield None
        R.epochs[("two_shot", b)] = e

    def _argmax(self, r: int, k: int, call: Call, b: int) -> Iterator[Step]:
        """argmax_gather_kernel: one CTA, (score, index) pairs pushed to every peer, slots
        double-buffered by the parity of its single epoch, fixed slot stride."""
        W, U = self.W, call.units
        R = self.ranks[r]
        e = R.epochs.get(("argmax", 0), 0) + 1
        region = f"am{e & 1}"
        for u in range(U):
            for j in range(W):
                if j != r:
                    self._write(j, self._addr(region, r, u, 512), (k, r, u))
                    yield None
        for j in range(W):
            if j != r:
                self._flag(j, ("argmax", 0, r), e)
                yield None
        for src in range(W):
            if src != r:
                yield (lambda src=src: self._flag_geq(r, ("argmax", 0, src), e))
        for u in range(U):
            for src in range(W):
                if src != r:
                    self._read(r, self._addr(region, src, u, 512), (k, src, u), f"argmax call {k}")
                    yield None
        R.epochs[("argmax", 0)] = e

    def _program(self, r: int, k: int, call: Call, b: int) -> Iterator[Step]:
        a = call.algo
        if a == "gemm_scatter":
            return self._gemm_scatter(r, k, call, b)
        if a == "from_gemm":
            return self._from_gemm(r, k, call, b)
        if a == "argmax":
            return self._argmax(r, k, call, b)
        if a == "two_shot":
            return self._two_shot(r, k, call, b)
        if a == "two_shot_staged":
            return self._two_shot(r, k, call, b, staged="sep")
        if a == "two_shot_staged_offset":
            return self._two_shot(r, k, call, b, staged="offset")
        if a == "two_shot_staged_shared":
            return self._two_shot(r, k, call, b, staged="shared")
        if a == "one_shot":
            return self._one_shot(r, k, call, b, per_block_parity=False)
        if a == "one_shot_block":
            return self._one_shot(r, k, call, b, per_block_parity=True)
        raise ValueError(a)

    # -------------------------------------------------------------- scheduler
    def run(self, max_steps: int = 2_000_000) -> int:
        """Run every rank's calls to completion; returns the number of steps taken."""
        W = self.W
        call_idx = [0] * W
        pending: List[List[int]] = [[] for _ in range(W)]   # blocks not yet dispatched
        live: List[Dict[int, Tuple[Iterator[Step], Step]]] = [dict() for _ in range(W)]

        def start_call(r: int) -> None:
            k = call_idx[r]
            if k < len(self.calls):
                pending[r] = list(range(self.calls[k].grid))

        def dispatch(r: int) -> None:
            cap = self.capacity or 1 << 30
            k = call_idx[r]
            while pending[r] and len(live[r]) < cap:
                b = pending[r].pop(0)
                live[r][b] = (self._program(r, k, self.calls[k], b), None)

        for r in range(W):
            start_call(r)
            dispatch(r)
        steps = 0
        while True:
            runnable = []
            for r in range(W):
                for b, (gen, cond) in live[r].items():
                    if cond is None or cond():
                        runnable.append((r, b))
            if not runnable:
                if any(live[r] or pending[r] or call_idx[r] < len(self.calls) for r in range(W)):
                    raise ProtocolViolation(f"deadlock: calls {call_idx}, live {[sorted(l) for l in live]}")
                return steps
            weights = [self.slow_bias if r == self.slow else 1.0 for r, _ in runnable]
            r, b = self.rng.choices(runnable, weights)[0]
            gen, _ = live[r][b]
            try:
                nxt = next(gen)
                live[r][b] = (gen, nxt)
            except StopIteration:
                del live[r][b]
                dispatch(r)
                if not live[r] and not pending[r]:
                    call_idx[r] += 1         # the call's kernel has ended on this rank
                    start_call(r)
                    dispatch(r)
            steps += 1
            if steps > max_steps:
                raise ProtocolViolation("step limit reached")


def random_calls(rng: random.Random, algo: str, n: int, max_units: int = 24, max_grid: int = 6) -> List[Call]:
    """n calls of one algorithm (or of a random mix with algo == "mixed") with varying
    message and grid sizes.  A GEMM-fed all-reduce is two calls: the GEMM, then phases 2-3."""
    out: List[Call] = []
    while len(out) < n:
        a = rng.choice(["two_shot", "one_shot", "gemm", "argmax"]) if algo == "mixed" else algo
        units = rng.randint(1, max_units)
        grid = rng.randint(1, min(max_grid, units))
        if a == "gemm":
            out.append(Call("gemm_scatter", units, rng.randint(1, min(max_grid, units))))
            out.append(Call("from_gemm", units, grid))
        elif a == "argmax":
            out.append(Call("argmax", min(units, 8), 1))
        else:
            out.append(Call(a, units, grid))
    return out
