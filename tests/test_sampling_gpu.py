"""Sampling in the decode loop (k_sample, inf_set_sampling) against the oracle's rule.  Each
decode step's fixed-point weights are read back: the oracle's integer selection on them must
give the device's id exactly (thresholds, Philox draw, index-order search), and the oracle's
weights from the same logits must agree with the device's to within the fp32 exponential's
rounding.  Then determinism per seed, top-k 1 equal to greedy, and greedy restored."""
import numpy as np
import pytest

import infb200 as I
import oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def eng(cuda):
    cfg = I.preset(2, n_layers=2, max_seq=512)
    with I.Engine(cfg, seed=0) as e:
        yield e


@pytest.mark.parametrize("temp,top_p,top_k", [(0.9, 0.9, 0), (1.3, 1.0, 40), (0.6, 0.5, 200)])
def test_each_step_matches_the_oracle(eng, temp, top_p, top_k):
    V = eng.V
    prompt = O.gen_ids(1, 16, V)
    eng.reset()
    _, tok = eng.forward(prompt, 0)
    eng.set_sampling(temp, top_p, top_k, seed=5)
    inv_temp = float(np.float32(1.0 / temp))
    pos = prompt.size
    try:
        differs = 0
        for _ in range(24):
            ids, _ = eng.decode(tok, pos, 1)
            q = eng.debug_read("sample_q")
            logits = eng.debug_read("logits")
            want = O.sample_select(q, top_p, top_k, 5, pos + 1)  # counter: the new token's position, slot 0
            assert int(ids[0]) == want
            q_orc = O.sample_weights(logits, inv_temp).astype(np.int64)
            tol = np.maximum(4, (q_orc >> 20))  # a few ulps of the fp32 exponential
            assert np.all(np.abs(q_orc - q.astype(np.int64)) <= tol)
            differs += int(ids[0]) != int(np.argmax(logits))
            tok, pos = int(ids[0]), pos + 1
        assert differs > 0  # the draws are not all the greedy choice
    finally:
        eng.set_sampling(0.0)


def test_seeded_generate_is_deterministic_and_greedy_restores(eng):
    prompt = O.gen_ids(2, 24, eng.V)
    eng.reset()
    greedy, _ = eng.generate(prompt, 16)
    try:
        eng.set_sampling(1.0, 0.95, 0, seed=1)
        eng.reset()
        a, _ = eng.generate(prompt, 16)
        eng.reset()
        b, _ = eng.generate(prompt, 16)
        eng.set_sampling(1.0, 0.95, 0, seed=2)
        eng.reset()
        c, _ = eng.generate(prompt, 16)
        np.testing.assert_array_equal(a, b)
        assert not np.array_equal(a, c)
        eng.set_sampling(1.0, 1.0, 1, seed=3)  # top-k 1: the argmax
        eng.reset()
        k1, _ = eng.generate(prompt, 16)
        np.testing.assert_array_equal(k1, greedy)
    finally:
        eng.set_sampling(0.0)
    eng.reset()
    again, _ = eng.generate(prompt, 16)
    np.testing.assert_array_equal(again, greedy)


def test_sampling_argument_checks(eng):
    for bad in (dict(temperature=-1.0), dict(temperature=float("nan")), dict(temperature=1.0, top_p=0.0),
                dict(temperature=1.0, top_p=1.5)):
        with pytest.raises(I.InfError) as ei:
            eng.set_sampling(**bad)
        assert ei.value.code == 4


def test_ragged_vocabulary(cuda):
    """A vocabulary that is not a multiple of 4 (50257) exercises the sampler's scalar tails."""
    cfg = I.preset(2, n_layers=1, max_seq=128, vocab_size=50257)
    with I.Engine(cfg, seed=0) as e:
        prompt = O.gen_ids(3, 12, e.V)
        _, tok = e.forward(prompt, 0)
        e.set_sampling(1.1, 0.97, 0, seed=9)
        pos = prompt.size
        for _ in range(12):
            ids, _ = e.decode(tok, pos, 1)
            q = e.debug_read("sample_q")
            assert int(ids[0]) == O.sample_select(q, 0.97, 0, 9, pos + 1)
            tok, pos = int(ids[0]), pos + 1
        e.set_sampling(0.7, 1.0, 50257 - 3, seed=9)  # top-k just below the vocabulary
        ids, _ = e.decode(tok, pos, 1)
        assert int(ids[0]) == O.sample_select(e.debug_read("sample_q"), 1.0, 50257 - 3, 9, pos + 1)


def test_batched_step_samples_each_slot_like_the_oracle(cuda):
    """inf_set_slot_sampling: in the batched step each row draws under its own slot's settings.
    The oracle's integer rule on the row's fixed-point weights (read back) gives the device's id
    with the counter (position of the new token, 0); the weights agree with the oracle's from the
    row's logits to within the fp32 exponential's rounding; greedy slots keep their argmax."""
    cfg = I.preset(2, n_layers=2, max_seq=256, max_batch=8)
    B = 8
    settings = {0: (0.9, 0.9, 0, 5), 1: (1.3, 1.0, 40, 6), 2: (0.6, 0.5, 200, 7), 4: (1.0, 0.95, 0, 8),
                5: (0.7, 1.0, 0, 9)}
    with I.Engine(cfg, seed=0) as e:
        cur, lens = [], []
        for i in range(B):
            p = O.gen_ids(40 + i, 10 + 7 * i, cfg.vocab_size)
            _, am = e.forward(p, 0, slot=i)
            cur.append(am)
            lens.append(p.size)
        for sl, (t, tp, tk, seed) in settings.items():
            e.set_slot_sampling(sl, t, tp, tk, seed)
        pos = np.array(lens, np.uint32)
        differs = 0
        for _ in range(6):
            lg, am = e.forward_batch(np.arange(B), np.array(cur, np.uint32), pos, want_logits=True)
            for i in range(B):
                if i in settings:
                    t, tp, tk, seed = settings[i]
                    q = e.debug_read("sample_q_row", pos=i)
                    assert int(am[i]) == O.sample_select(q, tp, tk, seed, int(pos[i]) + 1), f"row {i}"
                    q_orc = O.sample_weights(lg[i], float(np.float32(1.0 / t))).astype(np.int64)
                    assert np.all(np.abs(q_orc - q.astype(np.int64)) <= np.maximum(4, q_orc >> 20))
                    differs += int(am[i]) != int(np.argmax(lg[i]))
                else:
                    assert int(am[i]) == int(np.argmax(lg[i])), f"greedy row {i}"
            cur = [int(x) for x in am]
            pos += 1
        assert differs > 0  # the draws are not all the greedy choice
        for sl in settings:
            e.set_slot_sampling(sl, 0.0)
        lg, am = e.forward_batch(np.arange(B), np.array(cur, np.uint32), pos, want_logits=True)
        np.testing.assert_array_equal(am, np.argmax(lg, axis=1))  # greedy restored
