"""Generate the golden fixtures of tests/golden/ (run from the repository root).

The MetalANNS test suite keeps no stored golden files: its exact-search tests
generate data with a portable LCG and compare against a brute force written
inside the test.  This script restates both independently of the C oracle,
in numpy, and freezes their outputs:

* the LCG of Tests/MetalANNSTests/FlatSearchTests.swift:15-22 (pure Python
  integers, numpy float32 divide / multiply / subtract);
* FlatSearchTests.bruteForceTopK + distance (FlatSearchTests.swift:24-71):
  one pass accumulating dot, |q|^2 and |v|^2 sequentially in fp32, cosine =
  1 - dot / (sqrt(|q|^2) * sqrt(|v|^2)), squared L2 over differences, IP =
  -dot; ranking by (distance, id), first k;

for the cases of FlatSearchTests.swift:73-169 (sizes 64/100/2048/2049/5000 at
d=128 with k=100 over three metrics, the 4200-row / 16-query batch at k=50
and the 70-row corpus at k=256) and of ExactSearchIntegrationTests.
"""
from __future__ import annotations

import os

import numpy as np

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "flat_lcg.npz")
M64 = (1 << 64) - 1


def lcg(count: int, dim: int, seed: int) -> np.ndarray:
    state = seed & M64
    raw = np.empty(count * dim, np.float32)
    for i in range(count * dim):
        state = (state * 6364136223846793005 + 1442695040888963407) & M64
        raw[i] = np.float32((state >> 33) & 0xFFFFFF)
    u = raw / np.float32(0xFFFFFF)
    return (u * np.float32(2.0) - np.float32(1.0)).reshape(count, dim)


def test_distances(query: np.ndarray, vectors: np.ndarray, metric: str) -> np.ndarray:
    n, d = vectors.shape
    f = np.float32
    if metric == "cosine":
        dot = np.zeros(n, f)
        nq = f(0)
        nv = np.zeros(n, f)
        for j in range(d):
            dot = dot + query[j] * vectors[:, j]
            nq = f(nq + f(query[j] * query[j]))
            nv = nv + vectors[:, j] * vectors[:, j]
        denom = np.sqrt(nq) * np.sqrt(nv)
        out = np.where(denom < f(1e-10), f(1.0), f(1.0) - dot / np.where(denom == 0, f(1), denom))
        return out.astype(f)
    if metric == "l2":
        s = np.zeros(n, f)
        for j in range(d):
            diff = query[j] - vectors[:, j]
            s = s + diff * diff
        return s
    dot = np.zeros(n, f)
    for j in range(d):
        dot = dot + query[j] * vectors[:, j]
    return -dot


def brute_topk(query, vectors, k, metric):
    dist = test_distances(query, vectors, metric)
    order = np.lexsort((np.arange(len(dist)), dist))[:k]
    return order.astype(np.uint32), dist[order]


def main():
    out = {}
    dim = 128
    for n in (64, 100, 2048, 2049, 5000):
        vectors = lcg(n, dim, n)
        query = lcg(1, dim, n + 999)[0]
        out[f"corpus_head_{n}"] = vectors[:2].copy()
        out[f"query_{n}"] = query
        for metric in ("cosine", "l2", "ip"):
            ids, dist = brute_topk(query, vectors, 100, metric)
            out[f"ids_{n}_{metric}"] = ids
            out[f"dist_{n}_{metric}"] = dist
    vectors = lcg(4200, dim, 31)
    queries = lcg(16, dim, 77)
    out["batch_queries"] = queries
    out["batch_ids"] = np.stack([brute_topk(q, vectors, 50, "cosine")[0] for q in queries])
    vectors = lcg(70, 32, 7)
    query = lcg(1, 32, 5)[0]
    out["k_exceeds_ids"], out["k_exceeds_dist"] = brute_topk(query, vectors, 256, "l2")
    np.savez_compressed(OUT, **out)
    print(OUT, len(out), "arrays")


if __name__ == "__main__":
    main()
