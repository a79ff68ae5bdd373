"""Race and deadlock checks of the peer-memory all-reduce protocols (tests/protocol_model.py).

Each case replays W ranks' CTAs through a sequence of calls whose message and grid sizes
change from call to call, under a skewed random scheduler (one rank runs slower, so ranks
drift whole calls apart), and checks that every slot read sees the value its source wrote
for that call and that the run finishes.  The unsafe variants are negative controls: the
checker must find their races.
"""
import random

import pytest

from protocol_model import Call, Model, ProtocolViolation, random_calls

SEEDS = range(60)


def _violations(algo, seeds=SEEDS, capacity_choices=(None,), calls=6):
    bad = 0
    for seed in seeds:
        rng = random.Random(seed)
        W = rng.choice([2, 3, 4, 8])
        try:
            Model(W, random_calls(rng, algo, calls), seed=seed, capacity=rng.choice(capacity_choices)).run()
        except ProtocolViolation:
            bad += 1
    return bad


@pytest.mark.parametrize("algo", ["two_shot", "one_shot", "two_shot_staged", "two_shot_staged_offset"])
def test_protocol_has_no_race_or_deadlock(algo):
    assert _violations(algo) == 0


@pytest.mark.parametrize("algo", ["two_shot", "one_shot"])
def test_progress_with_partial_residency(algo):
    """Only 1-2 CTAs of a rank resident at a time, the rest dispatched in block order."""
    assert _violations(algo, capacity_choices=(1, 2)) == 0


@pytest.mark.parametrize("algo", ["gemm", "argmax"])
def test_gemm_fed_and_argmax_protocols(algo):
    assert _violations(algo, capacity_choices=(None, 2)) == 0


def test_mixed_algorithms_share_the_workspace():
    """Two-shot, one-shot, GEMM-fed two-shot and argmax calls back to back on one
    workspace: the reduce-scatter slots are shared by the two-shot and the GEMM-fed path."""
    assert _violations("mixed", calls=10, capacity_choices=(None, 2)) == 0


@pytest.mark.parametrize("algo", ["one_shot_block", "two_shot_staged_shared"])
def test_checker_finds_the_unsafe_variants(algo):
    assert _violations(algo) > len(SEEDS) // 4


def test_block_parity_is_safe_while_the_grid_is_fixed():
    """The race of per-block parity needs a grid change between calls."""
    for seed in SEEDS:
        rng = random.Random(seed)
        Model(rng.choice([2, 3, 4]), [Call("one_shot_block", rng.randint(4, 24), 4) for _ in range(6)],
              seed=seed).run()


def test_deadlock_is_reported():
    """A rank that skips a call leaves its peers waiting: the model must say so."""
    m = Model(2, [Call("two_shot", 4, 2)], seed=0)
    m.calls = [Call("two_shot", 4, 2)]
    orig = m._program

    def prog(r, k, call, b):
        if r == 1:
            return iter(())  # rank 1's CTAs exit at once without taking part
        return orig(r, k, call, b)
    m._program = prog
    with pytest.raises(ProtocolViolation, match="deadlock"):
        m.run()


class _SkipWaits(Model):
    """A mutant whose waits on one flag family always succeed."""
    skip = ""

    def _flag_geq(self, holder, key, e):
        return True if key[0] == self.skip else super()._flag_geq(holder, key, e)


@pytest.mark.parametrize("algo,skip", [("two_shot", "rs"), ("two_shot", "ag"), ("gemm", "gemm"),
                                       ("one_shot", "os"), ("argmax", "argmax")])
def test_checker_finds_a_missing_wait(algo, skip):
    """Dropping any one wait of a protocol must show up as a stale or missing read."""
    bad = 0
    for seed in SEEDS:
        rng = random.Random(seed)
        m = type("Mutant", (_SkipWaits,), {"skip": skip})(rng.choice([2, 3, 4]), random_calls(rng, algo, 6),
                                                             seed=seed)
        try:
            m.run()
        except ProtocolViolation:
            bad += 1
    assert bad > len(SEEDS) // 4, bad


def test_staged_and_plain_two_shot_share_flags_below_the_offset():
    """Staged and one-stage two-shot calls interleaved on one workspace, every grid below
    the stage offset: safe.  The same with one-stage grids reaching past the offset (its
    CTAs then write the staged kernel's stage-1 flag words under their own epochs): the
    checker must find the collision, which is why the kernels cap their grids."""
    from protocol_model import STAGE_OFF

    def run(max_grid_plain):
        bad = 0
        for seed in SEEDS:
            rng = random.Random(seed)
            calls = []
            for _ in range(8):
                if rng.random() < 0.5:
                    units = rng.randint(1, 24)
                    calls.append(Call("two_shot_staged_offset", units, rng.randint(1, min(6, units))))
                else:
                    units = rng.randint(1, 40)
                    calls.append(Call("two_shot", units, rng.randint(1, min(max_grid_plain, units))))
            try:
                Model(rng.choice([2, 3, 4]), calls, seed=seed).run()
            except ProtocolViolation:
                bad += 1
        return bad
    assert run(STAGE_OFF) == 0
    assert run(4 * STAGE_OFF) > 0
