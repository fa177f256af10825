"""The IVF-PQ merge closed form used on the device (pq.cu, bsl_resolve_kernel)
equals a direct simulation of BoundedSortedList (BoundedSelection.swift
:158-214): capacity K, equal-score newcomer rejected when full, otherwise
inserted ahead of equal scores, last entry evicted on overflow.  Fuzzed over
score streams with heavy ties (no GPU)."""
import numpy as np
import pytest


def bsl_simulate(scores, cap):
    out = []  # (score, seq)
    for seq, s in enumerate(scores):
        if cap <= 0:
            continue
        if len(out) >= cap and not (s < out[-1][0]):
            continue
        pos = 0
        while pos < len(out) and out[pos][0] < s:
            pos += 1
        out.insert(pos, (s, seq))
        del out[cap:]
    return out


def closed_form(scores, cap):
    """Mirror of bsl_resolve_kernel, fed the 2*cap smallest (score, seq)."""
    cand = sorted((s, i) for i, s in enumerate(scores))[:2 * cap]
    c = len(cand)
    if c <= cap:
        ordered = sorted(cand, key=lambda x: (x[0], -x[1]))
        return ordered
    w = cand[cap - 1][0]
    L = [x for x in cand if x[0] < w]
    E = [x for x in cand if x[0] == w][:cap]
    l = len(L)
    tagged = sorted([(x[1], 0) for x in L] + [(x[1], 1) for x in E])[:cap]
    ins = sum(t for _, t in tagged)
    keep = cap - l
    kept = E[ins - keep:ins]
    return sorted(L, key=lambda x: (x[0], -x[1])) + sorted(kept, key=lambda x: -x[1])


@pytest.mark.parametrize("seed", range(40))
def test_closed_form_matches_simulation(seed):
    rng = np.random.default_rng(seed)
    n = int(rng.integers(1, 400))
    levels = int(rng.integers(1, 12))
    scores = rng.integers(0, levels, n).astype(float).tolist()
    for cap in (1, 2, 3, 5, 10, 32):
        assert closed_form(scores, cap) == bsl_simulate(scores, cap), (seed, cap)


def test_reference_pin_pairs_newest_first():
    # duplicates a_i, b_i inserted a then b (BoundedSelectionTests.swift:281-317)
    scores = []
    for s in (3.0, 9.0, 1.0, 7.0, 2.0, 8.0):
        scores += [s, s]
    got = closed_form(scores, 6)
    assert [seq for _, seq in got] == [5, 4, 9, 8, 1, 0]
    assert got == bsl_simulate(scores, 6)
