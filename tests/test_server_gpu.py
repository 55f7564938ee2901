"""Continuous batching on the B200 (inf_server_* over the engine): requests arriving over time
share batched decode steps, slots and pages turn over, and every request's ids equal the ids it
gets when it runs alone.  That holds bit for bit because the server runs even a lone sequence
through the batched tensor-core step and nothing a sequence computes there depends on its batch
neighbours: each row of the projections accumulates on its own (one 128-row tile, the same K
split for 1 and 8 rows), the attention split count is fixed per model, and the LM head's argmax
is per row.  The first id of each request is the batch-1 prefill's."""
import numpy as np
import pytest

import infb200 as I
import oracle as O

pytestmark = pytest.mark.gpu


def drive(server, reqs, arrivals):
    rids = [None] * len(reqs)
    step = 0
    while True:
        for i, (p, m) in enumerate(reqs):
            if arrivals[i] == step:
                rids[i] = server.submit(p, m)
        server.step()
        step += 1
        if step > max(arrivals) and all(server.result(r)[1] for r in rids):
            return [server.result(r) for r in rids]
        assert step < 2000


def test_batched_requests_equal_solo_runs(cuda):
    cfg = I.preset(2, n_layers=2, max_seq=256, max_batch=8)
    rng = np.random.default_rng(4)
    reqs = [(O.gen_ids(10 + i, int(rng.integers(5, 60)), cfg.vocab_size), int(rng.integers(6, 24))) for i in range(16)]
    arrivals = [int(x) for x in rng.integers(0, 12, len(reqs))]
    with I.Engine(cfg, seed=0) as eng:
        with I.Server(eng) as s:
            together = drive(s, reqs, arrivals)
            st = s.stats()
        assert st["batched_steps"] > 0 and st["batched_tokens"] > st["batched_steps"]  # steps were shared
        for (p, m), (out, done, status) in zip(reqs, together):
            assert done and status == 0 and out.size == m
            with I.Server(eng, max_active=1) as alone:
                (solo, _, _), = drive(alone, [(p, m)], [0])
            np.testing.assert_array_equal(out, solo)
        # the first id is the batch-1 prefill's greedy id
        p, m = reqs[0]
        eng.reset(0)
        first, _ = eng.generate(p, 1)
        assert int(first[0]) == int(together[0][0][0])


def test_sampled_requests_equal_solo_runs(cuda):
    """Requests with their own sampling settings (inf_server_submit_sampled) among greedy ones:
    every request's ids equal its run alone (the draws do not depend on the slot or the batch),
    a sampled request's first id is the batch-1 prefill followed by the same rule (the decode of
    slot 0 with its settings), and the sampled requests do not all decode greedily."""
    cfg = I.preset(2, n_layers=2, max_seq=256, max_batch=8)
    rng = np.random.default_rng(9)
    reqs = []
    for i in range(10):
        smp = (0.8 + 0.05 * i, 0.9, 0 if i % 3 else 50, 100 + i) if i % 2 == 0 else None
        reqs.append((O.gen_ids(60 + i, int(rng.integers(5, 50)), cfg.vocab_size), int(rng.integers(6, 20)), smp))

    def run(server, batch):
        rids = [server.submit(p, m, I.NO_EOS, sampling=smp) for p, m, smp in batch]
        for _ in range(2000):
            server.step()
            if all(server.result(r)[1] for r in rids):
                return [server.result(r) for r in rids]
        raise AssertionError("requests did not retire")

    with I.Engine(cfg, seed=0) as eng:
        with I.Server(eng) as s:
            together = run(s, reqs)
        sampled_differs = 0
        for (p, m, smp), (out, done, status) in zip(reqs, together):
            assert done and status == 0 and out.size == m
            with I.Server(eng, max_active=1) as alone:
                (solo, _, _), = run(alone, [(p, m, smp)])
            np.testing.assert_array_equal(out, solo)
            if smp is not None:
                with I.Server(eng, max_active=1) as alone:
                    (greedy, _, _), = run(alone, [(p, m, None)])
                sampled_differs += int(not np.array_equal(out, greedy))
        assert sampled_differs > 0
        # the first id: the batch-1 prefill, then the batch-1 sampler of slot 0 with the same settings
        p, m, (t, tp, tk, seed) = reqs[0]
        eng.reset(0)
        eng.set_sampling(t, tp, tk, seed)
        try:
            first, _ = eng.generate(p, 1)
        finally:
            eng.set_sampling(0.0)
        assert int(first[0]) == int(together[0][0][0])


def test_server_refuses_sampling(cuda):
    """Model-wide sampling (inf_set_sampling) is refused at admission: requests carry their own."""
    cfg = I.preset(2, n_layers=1, max_seq=64, max_batch=2)
    with I.Engine(cfg, seed=0) as eng:
        eng.set_sampling(1.0, 0.9, 0, seed=1)
        with I.Server(eng) as s:
            r = s.submit(O.gen_ids(1, 5, cfg.vocab_size), 4)
            s.step()
            out, done, status = s.result(r)
            assert done and status == 15 and out.size == 0
