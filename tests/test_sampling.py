"""The oracle's sampling rule (oracle/llama_ref.c orc_sample_*, the definition of
inf_set_sampling) against a second restatement in numpy, and its distribution: top-k 1 is
greedy, the draw frequencies follow the kept weights, top-p keeps the fewest heaviest tokens."""
import numpy as np
import pytest

import oracle as O


def np_select(q, top_p, top_k, seed, counter):
    q = q.astype(np.uint64)
    s = np.sort(q)[::-1]
    tk = int(s[top_k - 1]) if 0 < top_k < q.size else 0
    zk = int(q[q >= tk].sum())
    tp = tk
    if top_p < 1.0 and zk > 0:
        tgt = min(max(np.ceil(np.float64(np.float32(top_p)) * zk), 1.0), float(zk))
        vals, counts = np.unique(s[s >= tk], return_counts=True)
        c = 0
        for v, n in zip(vals[::-1], counts[::-1]):
            c += int(v) * int(n)
            if c >= tgt:
                tp = int(v)
                break
    kept = q >= tp
    total = int(q[kept].sum())
    w = O.philox([counter & 0xFFFFFFFF, counter >> 32, 0, 0], stream_key(seed, 0x3000000))
    r = (int(w[1]) << 32) | int(w[0])
    target = (r * total) >> 64
    csum = np.cumsum(np.where(kept, q, 0).astype(object))
    return int(np.argmax(csum > target))


def splitmix64(x):
    M = (1 << 64) - 1
    z = (x + 0x9E3779B97F4A7C15) & M
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & M
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & M
    return z ^ (z >> 31)


def stream_key(seed, stream):
    k = splitmix64(splitmix64(seed) ^ stream)
    return [k & 0xFFFFFFFF, k >> 32]


def logits_case(rng, V=5000):
    x = rng.standard_normal(V).astype(np.float32) * 3
    x[rng.integers(0, V, 20)] = x.max()  # ties at the top
    return x


@pytest.mark.parametrize("top_p,top_k", [(1.0, 0), (0.9, 0), (0.5, 40), (1.0, 7), (0.3, 0), (0.999, 3)])
def test_oracle_matches_numpy_restatement(top_p, top_k):
    rng = np.random.default_rng(top_k * 100 + int(top_p * 1000))
    for trial in range(8):
        q = O.sample_weights(logits_case(rng), 1.0 / 0.8)
        for counter in (1, 77, (3 << 32) | 9):
            assert O.sample_select(q, top_p, top_k, 5 + trial, counter) == np_select(q, top_p, top_k, 5 + trial, counter)


def test_weights_fixed_point():
    x = np.array([0.0, -1.0, -50.0, -200.0, 0.0], np.float32)
    q = O.sample_weights(x, 1.0)
    assert q[0] == q[4] == 0xFFFFFFFF
    assert abs(int(q[1]) - int(np.exp(np.float64(-1.0)) * 2**32)) <= 2**32 * 2**-22
    assert q[3] == 0


def test_top_k_one_is_greedy():
    rng = np.random.default_rng(3)
    x = rng.standard_normal(1000).astype(np.float32)
    q = O.sample_weights(x, 1.0)
    for c in range(50):
        assert O.sample_select(q, 1.0, 1, 11, c) == int(np.argmax(x))


def test_draw_frequencies_follow_the_weights():
    x = np.log(np.array([0.5, 0.25, 0.125, 0.0625, 0.0625], np.float32))
    q = O.sample_weights(x, 1.0)
    n = 20000
    ids = np.array([O.sample_select(q, 1.0, 0, 7, c) for c in range(n)])
    freq = np.bincount(ids, minlength=5) / n
    np.testing.assert_allclose(freq, [0.5, 0.25, 0.125, 0.0625, 0.0625], atol=0.015)
    # top-p 0.7: {0, 1} carry 0.75 >= 0.7, so only those two, renormalised
    ids = np.array([O.sample_select(q, 0.7, 0, 7, c) for c in range(n)])
    freq = np.bincount(ids, minlength=5) / n
    np.testing.assert_allclose(freq, [2 / 3, 1 / 3, 0, 0, 0], atol=0.015)
