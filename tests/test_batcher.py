"""The token-budget batcher (libr97host.so r97host_batcher_*, r97training_b200/data.py) against the
reference's own r97::Batcher (src/batcher.cpp, compiled into oracle/_ref): the same plan -- steps,
sub-batches, their sequences and their order -- for every (seed, epoch) over generated datasets and the
shapes the reference's own tests pin (tests/host/batcher.cpp), plus the contract's invariants: the budget
holds per sub-batch, every kept sequence appears once an epoch, skipped ones never, seek clamps and a saved
position resumes identically."""
import ctypes

import numpy as np
import pytest

import oracle
from r97training_b200 import data as D


def _ref():
    if not oracle.ref_available():
        pytest.skip("reference host library not built and reference tree absent")
    ref = oracle.ref_lib()
    f = ref.ref_batcher_plan
    f.restype = ctypes.c_int64
    f.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int, ctypes.c_uint64, ctypes.c_int64,
                  ctypes.c_int, ctypes.c_void_p, ctypes.c_int64]
    ref.ref_last_error.restype = ctypes.c_char_p
    return ref


def ref_plan(lens, budget, devices, seed, epoch0, epochs):
    ref = _ref()
    lens = np.ascontiguousarray(lens, dtype=np.int64)
    args = (lens.ctypes.data if len(lens) else None, len(lens), budget, devices, seed, epoch0, epochs)
    n = ref.ref_batcher_plan(*args, None, 0)
    assert n >= 0, ref.ref_last_error()
    out = np.zeros(n, dtype=np.int64)
    assert ref.ref_batcher_plan(*args, out.ctypes.data, n) == n
    return [int(v) for v in out]


def our_plan(lens, budget, devices, seed, epoch0, epochs):
    b = D.Batcher([D.TokenSeq([0] * int(n), [0] * int(n)) for n in lens], D.BatcherConfig(budget, devices, seed))
    flat = []
    for e in range(epoch0, epoch0 + epochs):
        b.seek(D.Position(e, 0))
        flat.append(b.steps_in_epoch(e))
        while (step := b.next_indices()) is not None:
            flat.append(len(step))
            for sub in step:
                flat.append(len(sub))
                flat.extend(sub)
    sk = b.skipped()
    return flat + [len(sk)] + sk


def _check(lens, budget, devices, seed, epoch0=0, epochs=3):
    want = ref_plan(lens, budget, devices, seed, epoch0, epochs)
    got = our_plan(lens, budget, devices, seed, epoch0, epochs)
    assert got == want, f"plan differs from the reference's (n={len(lens)}, budget={budget}, devices={devices}, seed={seed})"


# the shapes the reference's own batcher tests use (tests/host/batcher.cpp)
PINNED = [
    ([500] * 33 + [12] * 32, 1200, 2),     # a short bucket tail fills the idle device from the next bucket
    ([500] * 5, 1200, 2),                  # an epoch's last odd tail
    ([500] * 3, 1200, 2), ([1] * 3, 2, 2),  # smaller odd residues
    ([1000, 1000, 1000, 10, 10, 10], 1500, 2),  # three longs beside three shorts
    ([500] * 101, 2000, 3),                # fixed lengths: the exact step plan
    ([100] * 100, 1000, 2), ([100] * 1000, 4096, 4), ([128] * 800, 4096, 4),
    ([50] * 20, 500, 2), ([12] * 8, 36, 2), ([7] * 12, 30, 2), ([50] * 20, 500, 1),  # one bucket
    ([400] * 32 + [10] * 32, 4096, 1), ([400] * 33 + [10] * 32, 4096, 1),  # two classes 40x apart
    ([3, 900], 1000, 2), ([2 ** k + 1 for k in range(8)], 1000, 2),  # one sequence a bucket
    ([9000, 300, 200, 100], 1000, 2),      # one over the budget: skipped
    ([0, 0, 5, 6, 0, 7], 16, 2),           # zero-token sequences are a class of their own
    ([], 100, 2),                          # no data
]


@pytest.mark.parametrize("case", range(len(PINNED)))
def test_batcher_matches_reference_on_pinned_shapes(case):
    lens, budget, devices = PINNED[case]
    for seed in (0, 1, 12345, 2**63 + 7):
        _check(lens, budget, devices, seed, 0, 4)


def test_batcher_matches_reference_on_generated_datasets():
    rs = np.random.RandomState(2024)
    for t in range(300):
        n = int(rs.randint(1, 120))
        classes = rs.choice(np.arange(1, 12), size=int(rs.randint(1, 6)), replace=False)
        cls = rs.choice(classes, size=n)
        lens = (2 ** (cls - 1) + rs.randint(0, 2 ** (cls - 1))).astype(np.int64)
        if t % 7 == 0:
            lens[rs.randint(0, n)] = 0
        budget = int(max(lens.max() * rs.uniform(0.7, 4.0), 1))
        devices = int(rs.randint(1, 5))
        _check(lens, budget, devices, int(rs.randint(0, 2**31)), int(rs.randint(0, 5)), 2)


def test_batcher_matches_reference_on_realistic_sizes():
    rs = np.random.RandomState(7)
    lens = rs.randint(17, 4097, size=3000)
    for devices in (1, 2, 4, 8):
        _check(lens, 4096, devices, 99, 0, 2)
    _check(rs.randint(50, 81, size=1000), 4096, 2, 5, 0, 2)


def _epoch(b, e):
    b.seek(D.Position(e, 0))
    steps = []
    while (s := b.next_indices()) is not None:
        steps.append(s)
    return steps


def test_batcher_contract():
    rs = np.random.RandomState(3)
    lens = list(rs.randint(20, 900, size=300)) + [9000]
    seqs = [D.TokenSeq([i] * int(n), [1] * int(n)) for i, n in enumerate(lens)]
    b = D.Batcher(seqs, D.BatcherConfig(token_budget=2000, devices=3, seed=11))
    assert b.skipped() == [300] and b.skipped_tokens() == 9000
    plans = []
    for e in range(3):
        steps = _epoch(b, e)
        assert len(steps) == b.steps_in_epoch(e)
        seen = [i for st in steps for sub in st for i in sub]
        assert sorted(seen) == list(range(300))  # every kept sequence once, the skipped one never
        for st in steps:
            assert 1 <= len(st) <= 3 and all(st)
            for sub in st:
                assert sum(lens[i] for i in sub) <= 2000  # the budget is per sub-batch
        plans.append(steps)
    assert plans[0] != plans[1] != plans[2]
    # next() hands out the sequences themselves
    b.reset()
    first = b.next()
    assert [[s.ids[0] for s in sub] for sub in first] == plans[0][0]
    # a saved position resumes identically
    b.seek(D.Position(1, 2))
    assert b.position() == D.Position(1, 2)
    assert b.next_indices() == plans[1][2]
    # seek clamps: negative epoch / step to the first, past the end to the end (nothing handed out there)
    b.seek(D.Position(-4, -9))
    assert b.position() == D.Position(0, 0)
    b.seek(D.Position(2, 10**6))
    assert b.position() == D.Position(2, b.steps_in_epoch(2))
    assert b.next_indices() is None and b.position() == D.Position(2, b.steps_in_epoch(2))
    b.reset()
    assert b.position() == D.Position(0, 0) and b.next_indices() == plans[0][0]


def test_batcher_rejects_bad_config():
    with pytest.raises(ValueError, match="token_budget"):
        D.Batcher([D.TokenSeq([1], [0])], D.BatcherConfig(0, 1, 0))
    with pytest.raises(ValueError, match="devices"):
        D.Batcher([D.TokenSeq([1], [0])], D.BatcherConfig(10, 0, 0))


def test_step_rows_targets_follow_scores():
    batch = [D.TokenSeq([5, 6, 7, 8], [0, 0, 1, 1]), D.TokenSeq([9, 10], [0, 1])]
    ids, tgt, scored = D.step_rows(batch, rows=3, seq=5)
    assert ids.tolist() == [[5, 6, 7, 8, 0], [9, 10, 0, 0, 0], [0, 0, 0, 0, 0]]
    assert tgt.reshape(3, 5).tolist() == [[-1, 7, 8, -1, -1], [10, -1, -1, -1, -1], [-1] * 5]
    assert scored == 3
    with pytest.raises(ValueError):
        D.step_rows(batch, rows=1, seq=5)
    with pytest.raises(ValueError):
        D.step_rows(batch, rows=2, seq=3)
