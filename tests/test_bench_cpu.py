"""The bench's synthetic inputs (no GPU): the routing generators behind cfg 3
(Zipf prefill), cfg 4 (Markov decode batch) and cfg 5s (Zipf streaming trace)
have the shapes, ranges and statistics their configs state."""
from __future__ import annotations

import numpy as np

import bench


def _distinct_rows(ids):
    return all(len(set(r.tolist())) == r.size for r in ids.reshape(-1, ids.shape[-1]))


def test_markov_routing_keeps_eighty_percent():
    ids, w = bench.markov_routing(2, 4, 48)
    assert ids.shape == (2, 48, 4, bench.TOP_K) and w.shape == ids.shape
    assert ids.min() >= 0 and ids.max() < bench.EXPERTS and _distinct_rows(ids)
    np.testing.assert_allclose(w.sum(-1), 1.0, rtol=1e-5)
    kept = np.mean([(ids[s, L, t] == ids[s, L, t - 1]).mean() for s in range(2) for L in range(48) for t in (1, 2, 3)])
    assert 0.74 < kept < 0.86, kept
    distinct = np.mean([np.unique(ids[s, L]).size for s in range(2) for L in range(48)])
    assert 14.0 < distinct < 18.0, distinct   # ~15.9 per block at p_keep = 0.8


def test_zipf_routing_is_skewed():
    ids, w = bench.zipf_routing(2, 512)
    assert ids.shape == (2, 512, bench.TOP_K) and _distinct_rows(ids)
    counts = np.sort(np.bincount(ids[0].ravel(), minlength=bench.EXPERTS))[::-1]
    assert counts[0] > 200 and counts.sum() == 512 * bench.TOP_K   # the top expert takes hundreds of rows
    assert 400 < (counts > 0).sum() < 500                         # ~460 experts touched


def test_stream_routing_follows_a_fixed_popularity_per_block():
    ids, w = bench.stream_routing(64, 4)
    assert ids.shape == (64, 4, bench.TOP_K) and _distinct_rows(ids)
    for L in range(4):
        c = np.bincount(ids[:, L].ravel(), minlength=bench.EXPERTS)
        top = np.argsort(-c)[:5]
        perm = np.random.default_rng(50 + L).permutation(bench.EXPERTS)
        assert set(top) & set(perm[:10])   # the most used experts are the block's top-ranked ones


def test_uniform_routing_tokens():
    ids, w = bench.routing_tokens(1, 64, 2)
    assert ids.shape == (1, 2, 64, bench.TOP_K) and _distinct_rows(ids)
    np.testing.assert_allclose(w.sum(-1), 1.0, rtol=1e-5)
