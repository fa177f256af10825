"""Pins of the CPU oracle (no GPU): against the reference's own dots.c, the
golden fixtures of the reference tests' brute force, and the tie rules the
reference tests pin."""
import os

import numpy as np
import pytest

import oracle as O

GOLD = os.path.join(os.path.dirname(__file__), "golden", "flat_lcg.npz")
METRICS = {"cosine": O.COSINE, "l2": O.L2, "ip": O.IP}


@pytest.fixture(scope="module")
def gold():
    return np.load(GOLD)


def test_lcg_matches_numpy_restatement(gold):
    # FlatSearchTests.swift:15-22, restated twice (C oracle, numpy script)
    for n in (64, 100, 2048, 2049, 5000):
        v = O.lcg_vectors(n, 128, n)
        np.testing.assert_array_equal(v[:2], gold[f"corpus_head_{n}"])
        np.testing.assert_array_equal(O.lcg_vectors(1, 128, n + 999)[0], gold[f"query_{n}"])


@pytest.mark.parametrize("dim", [1, 3, 4, 15, 16, 17, 31, 32, 33, 127, 128, 383, 384, 768])
def test_sequential_dot_equals_reference_dots_c(dim):
    if O.ref_lib() is None:
        pytest.skip("reference dots.c was not built on this machine")
    c = O.lcg_vectors(257, dim, 11 + dim)
    q = O.lcg_vectors(1, dim, 5 + dim)[0]
    a = O.dot_rows(c, q)
    b = O.ref_dot_rows(c, q)
    np.testing.assert_array_equal(a.view(np.uint32), b.view(np.uint32))


def test_neon_order_restatement_properties():
    # The arm64 order differs from the scalar one only by rounding.
    c = O.lcg_vectors(300, 384, 3)
    q = O.lcg_vectors(1, 384, 4)[0]
    a = O.dot_rows(c, q, "seq")
    b = O.dot_rows(c, q, "neon")
    exact = c.astype(np.float64) @ q.astype(np.float64)
    assert np.max(np.abs(b - exact)) < 1e-4
    assert np.max(np.abs(a - exact)) < 1e-4
    # shapes the NEON branch does not take fall back to the scalar order
    c2 = O.lcg_vectors(10, 13, 1)
    q2 = O.lcg_vectors(1, 13, 2)[0]
    np.testing.assert_array_equal(O.dot_rows(c2, q2, "neon"), O.dot_rows(c2, q2, "seq"))


@pytest.mark.parametrize("n", [64, 100, 2048, 2049, 5000])
@pytest.mark.parametrize("metric", ["cosine", "l2", "ip"])
def test_oracle_matches_reference_test_bruteforce(gold, n, metric):
    """FlatSearchTests.parityAcrossMetricsAndSizes (FlatSearchTests.swift:73-115)."""
    v = O.lcg_vectors(n, 128, n)
    q = O.lcg_vectors(1, 128, n + 999)[0]
    d, i, c = O.flat_search(v, q, 100, METRICS[metric])
    want = gold[f"ids_{n}_{metric}"]
    assert c[0] == min(100, n)
    assert set(i[0, :c[0]].tolist()) == set(want.tolist())
    assert abs(d[0, 0] - gold[f"dist_{n}_{metric}"][0]) < 1e-3
    assert np.all(np.diff(d[0, :c[0]]) >= 0)


def test_oracle_batch_and_k_exceeds(gold):
    v = O.lcg_vectors(4200, 128, 31)
    qs = O.lcg_vectors(16, 128, 77)
    d, i, c = O.flat_search(v, qs, 50, O.COSINE)
    for r in range(16):
        assert set(i[r].tolist()) == set(gold["batch_ids"][r].tolist())
    v = O.lcg_vectors(70, 32, 7)
    q = O.lcg_vectors(1, 32, 5)[0]
    d, i, c = O.flat_search(v, q, 256, O.L2)
    assert c[0] == 70
    assert set(i[0, :70].tolist()) == set(gold["k_exceeds_ids"].tolist())


def test_parallel_flat_scan_equals_exact_set():
    """ParallelFlatScan returns the exact top-k set (its doc comment :4-10)."""
    v = O.lcg_vectors(20000, 64, 9)
    q = O.lcg_vectors(1, 64, 10)[0]
    for metric in (O.COSINE, O.L2, O.IP):
        pd, pi = O.parallel_flat_scan(v, q, 37, metric, cores=8)
        d, i, c = O.flat_search(v, q, 37, metric)
        assert set(pi.tolist()) == set(i[0].tolist())
        np.testing.assert_array_equal(np.sort(pd), d[0])


def _duplicated(pairs, dim, seed):
    base = O.lcg_vectors(pairs, dim, seed)
    return np.repeat(base, 2, axis=0)


def test_tie_orders_under_duplicate_vectors():
    """Structural form of BoundedSelectionTests.swift:228-277 (the pinned id
    lists there come from Swift's Float.random and cannot be regenerated):
    duplicated rows tie exactly; the GPU tier orders each tied pair by
    ascending id, the host tier in heap-extraction order."""
    v = _duplicated(6, 8, 11)
    q = O.lcg_vectors(1, 8, 99)[0]
    for metric in (O.COSINE, O.L2, O.IP):
        d, i, c = O.flat_search(v, q, 12, metric)
        ids = i[0].tolist()
        for a in range(0, 12, 2):
            assert d[0, a] == d[0, a + 1]
            assert ids[a] < ids[a + 1] and ids[a] // 2 == ids[a + 1] // 2
        # the reference GPU tier (boundedTopK) agrees on every tied pair
        dist_row = np.array([O.lib().orc_distance(metric, float(x), O.norm_sq(q), float(nv))
                             for x, nv in zip(O.dot_rows(v, q), O.row_norms(v))], np.float32)
        gd, gi = O.gpu_tier_topk(dist_row, 12)
        assert gi.tolist() == ids
        # host tier returns the same pairs, its tie order is heap dependent
        pd, pi = O.parallel_flat_scan(v, q, 12, metric, cores=1)
        assert sorted(pi.tolist()) == sorted(ids)
        assert [x // 2 for x in pi.tolist()] == [x // 2 for x in ids]


def test_gpu_tier_boundary_tie_keeps_earlier_rows():
    # strict `<` admission: equal distances at the boundary keep the earlier id
    row = np.array([5, 5, 3, 5, 1], np.float32)
    d, i = O.gpu_tier_topk(row, 3)
    assert i.tolist() == [4, 2, 1] or i.tolist() == [4, 2, 0]
    d2, i2, _ = O.flat_search(np.eye(5, dtype=np.float32), np.zeros(5, np.float32), 3, O.IP)
    assert i2[0].tolist() == [0, 1, 2]  # all distances -0: ties by id


def _bsl_reference(items, cap):
    """Array model of BoundedSortedList (BoundedSelectionTests.swift:107-140)."""
    out = []
    for s, a in items:
        if cap <= 0:
            continue
        if len(out) >= cap and not (s < out[-1][0]):
            continue
        pos = 0
        while pos < len(out) and out[pos][0] < s:
            pos += 1
        out.insert(pos, (s, a))
        del out[cap:]
    return out


def test_ivfpq_merge_rule_newest_first():
    """BoundedSelectionTests.ivfpqMergeTieOrderPinned (:281-317), structurally:
    vectors inserted as a_i then b_i (duplicates) come back b_i, a_i."""
    rng = np.random.default_rng(3)
    dim, m, ks = 16, 4, 256
    codebooks = rng.standard_normal((m, ks, dim // m)).astype(np.float32)
    coarse = rng.standard_normal((4, dim)).astype(np.float32)
    distinct = rng.uniform(-1, 1, (10, dim)).astype(np.float32)
    vecs = np.repeat(distinct, 2, axis=0)  # a0, b0, a1, b1, ...
    codes = np.zeros((20, m), np.uint8)
    lists = [[] for _ in range(4)]
    for idx, v in enumerate(vecs):
        c = O.nearest_coarse(v, coarse, O.L2)
        codes[idx] = O.pq_encode_subtracting(v, coarse[c], codebooks)
        lists[c].append(idx)
    offsets = np.cumsum([0] + [len(x) for x in lists]).astype(np.int64)
    flat = np.array(sum(lists, []), np.uint32)
    d, i, c = O.ivfpq_search(coarse, codebooks, codes, offsets, flat, vecs[0], 6, 4, O.L2)
    ids = i[0, :c[0]].tolist()
    for a in range(0, 6, 2):
        assert d[0, a] == d[0, a + 1]
        assert ids[a] == ids[a + 1] + 1  # b (odd id, newer) ahead of a
    # the restated merge equals the array model of BoundedSortedList
    scores = [float(x) for x in d[0, :c[0]]]
    assert sorted(scores) == scores


def test_pq_encode_subtracting_equals_residual_encode():
    """ProductQuantizerTests.swift:91-109: encode(v, subtracting: c) ==
    encode(v - c), exactly."""
    rng = np.random.default_rng(5)
    cb = rng.standard_normal((8, 256, 4)).astype(np.float32)
    for _ in range(20):
        v = rng.standard_normal(32).astype(np.float32)
        c = rng.standard_normal(32).astype(np.float32)
        a = O.pq_encode_subtracting(v, c, cb)
        b = O.pq_encode_subtracting(v - c, np.zeros(32, np.float32), cb)
        np.testing.assert_array_equal(a, b)


def test_ivf_nprobe_all_equals_bruteforce():
    """IVFFlatSearchTests.swift:193-216: probing every list is exact."""
    rng = np.random.default_rng(1)
    v = rng.standard_normal((3000, 32)).astype(np.float32)
    cent = v[rng.choice(3000, 16, replace=False)]
    for metric in (O.COSINE, O.L2, O.IP):
        assign = O.ivf_assign(v, cent, metric)
        off, ids, packed, pn = O.ivf_layout(v, assign, 16)
        q = rng.standard_normal((5, 32)).astype(np.float32)
        d, i, c = O.ivf_search(cent, packed, pn, ids, off, q, 20, 16, metric)
        d2, i2, c2 = O.flat_search(v, q, 20, metric)
        np.testing.assert_array_equal(i, i2)
        np.testing.assert_array_equal(d, d2)


def test_pq_adc_is_sequential_lut_sum():
    rng = np.random.default_rng(2)
    cb = rng.standard_normal((16, 256, 8)).astype(np.float32)
    q = rng.standard_normal(128).astype(np.float32)
    lut = O.pq_lut(q, cb, O.L2)
    codes = rng.integers(0, 256, (100, 16)).astype(np.uint8)
    out = O.pq_adc(lut, codes)
    for r in range(100):
        t = np.float32(0)
        for s in range(16):
            t = np.float32(t + lut[s, codes[r, s]])
        assert out[r] == t


def _int8_fill_numpy(rows):
    """Independent float32 restatement of Int8CodeBuffer.fill
    (Int8CodeCache.swift:64-99) in numpy."""
    rows = np.asarray(rows, np.float32)
    mx = np.abs(rows).max(axis=1)
    scale = np.where(mx > 0, mx / np.float32(127.0), np.float32(1.0)).astype(np.float32)
    inv = (np.float32(1.0) / scale).astype(np.float32)
    scaled = (rows * inv[:, None]).astype(np.float32)
    shifted = np.where(scaled >= 0, scaled + np.float32(0.5), scaled - np.float32(0.5)).astype(np.float32)
    codes = np.clip(np.trunc(shifted), -127, 127).astype(np.int8)
    return codes, scale


def test_int8_fill_matches_numpy_restatement():
    """Codes and scales of the int8 prefilter (BoundedExactScan's Int8CodeBuffer)
    on the reference test generator's data, zero rows and extreme magnitudes."""
    v = O.lcg32_vectors(700, 384, 7)
    v[::50] = 0.0
    v[1::50] *= np.float32(1e5)
    v[2::50] *= np.float32(1e-5)
    v[3, :5] = [0.5, -0.5, 127.0, -127.0, 63.5]  # exact halves after scaling
    codes, scales = O.int8_fill(v)
    want_c, want_s = _int8_fill_numpy(v)
    np.testing.assert_array_equal(scales, want_s)
    np.testing.assert_array_equal(codes, want_c)
    assert codes.min() >= -127 and codes.max() <= 127
    assert (codes[::50] == 0).all() and (scales[::50] == 1.0).all()
