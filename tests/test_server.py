"""Continuous batching (inf_server_*) scheduling on the host-only stand-in model
(inf_server_create_synthetic): its next id depends only on the sequence's own previous id and
position, and it rejects a batch that feeds a slot out of order or twice, so the tests check
admission order, the max_active bound, retirement (eos, max_new, end of positions), slot and page
reuse, and that a request's output does not depend on what shares its batch."""
import numpy as np
import pytest

import infb200 as I


def synthetic_next(prev, pos, vocab):
    M = (1 << 64) - 1

    def mix(x):
        x &= M
        x ^= x >> 33
        x = (x * 0xff51afd7ed558ccd) & M
        x ^= x >> 33
        x = (x * 0xc4ceb9fe1a85ec53) & M
        return (x ^ (x >> 33)) & 0xFFFFFFFF
    return mix((prev << 32) ^ pos) % vocab


def run_all(server, reqs, arrivals=None):
    """Submit (prompt, max_new, eos) at their arrival steps, step until all retire."""
    arrivals = arrivals or [0] * len(reqs)
    ids = [None] * len(reqs)
    step = 0
    while True:
        for i, (p, m, e) in enumerate(reqs):
            if arrivals[i] == step:
                ids[i] = server.submit(p, m, e)
        server.step()
        step += 1
        if step > max(arrivals) and all(ids[i] is not None and server.result(ids[i])[1] for i in range(len(reqs))):
            break
        assert step < 10_000
    return [server.result(r) for r in ids], step


def requests(rng, n, vocab, max_seq):
    out = []
    for _ in range(n):
        lp = int(rng.integers(1, max_seq // 2))
        out.append((rng.integers(0, vocab, lp, dtype=np.uint32), int(rng.integers(1, 40)), I.NO_EOS))
    return out


def test_outputs_do_not_depend_on_the_batch():
    rng = np.random.default_rng(1)
    reqs = requests(rng, 30, 1000, 128)
    arrivals = list(rng.integers(0, 40, len(reqs)))
    with I.Server(synthetic=(6, 128, 1000)) as s:
        together, _ = run_all(s, reqs, arrivals)
        st = s.stats()
        assert st["waiting"] == 0 and st["active"] == 0 and st["batched_steps"] > 0
    for (p, m, e), (out, done, rc) in zip(reqs, together):
        with I.Server(synthetic=(1, 128, 1000)) as alone:
            (solo, _, _), = run_all(alone, [(p, m, e)])[0]
        assert done and rc == 0
        np.testing.assert_array_equal(out, solo)
        assert out.size == m
        # each token after the first follows from the one before at its position
        for k in range(1, out.size):
            assert out[k] == synthetic_next(int(out[k - 1]), len(p) + k - 1, 1000)


def test_max_active_and_fifo_admission():
    rng = np.random.default_rng(2)
    reqs = [(rng.integers(0, 50, 5, dtype=np.uint32), 10, I.NO_EOS) for _ in range(7)]
    with I.Server(synthetic=(8, 64, 50), max_active=3) as s:
        rids = [s.submit(*r) for r in reqs]
        s.step()
        st = s.stats()
        assert st["active"] == 3 and st["waiting"] == 4
        started = [s.result(r)[0].size > 0 for r in rids]
        assert started == [True] * 3 + [False] * 4  # first come, first served
        while not all(s.result(r)[1] for r in rids):
            s.step()
            assert s.stats()["active"] <= 3


def test_eos_and_end_of_positions():
    with I.Server(synthetic=(2, 16, 7)) as s:
        # a vocabulary of 7 ids: some id repeats quickly; use the second output as eos
        probe = s.submit(np.array([1, 2, 3], np.uint32), 5)
        while not s.result(probe)[1]:
            s.step()
        out, _, _ = s.result(probe)
        eos = int(out[1])
        r = s.submit(np.array([1, 2, 3], np.uint32), 50, eos)
        while not s.result(r)[1]:
            s.step()
        got = s.result(r)[0]
        assert got[-1] == eos and eos not in got[:-1].tolist()
        # max_seq 16: a 10-token prompt leaves positions 10..15 to feed -> 7 outputs at most
        r = s.submit(np.arange(10, dtype=np.uint32) % 7, 100)
        while not s.result(r)[1]:
            s.step()
        assert s.result(r)[0].size == 7


def test_slots_are_reused_and_requests_released():
    with I.Server(synthetic=(2, 32, 100)) as s:
        rids = [s.submit(np.array([i + 1], np.uint32), 3) for i in range(10)]
        steps = 0
        while not all(s.result(r)[1] for r in rids):
            s.step()
            steps += 1
        assert steps <= 20  # two slots turn over five times
        for r in rids:
            s.release(r)
        with pytest.raises(I.InfError):
            s.result(rids[0])


def test_submit_checks():
    with I.Server(synthetic=(2, 16, 100)) as s:
        for bad in ((np.array([], np.uint32), 3), (np.arange(16, dtype=np.uint32), 3), (np.array([1], np.uint32), 0)):
            with pytest.raises(I.InfError):
                s.submit(*bad)
        r = s.submit(np.array([1], np.uint32), 5)
        with pytest.raises(I.InfError):
            s.release(r)  # still running


def test_overcommitted_page_pool_admits_only_what_fits():
    """8 slots but pages for about two long requests at once: the scheduler admits a request
    only when every position it may write fits beside the running requests' reservations (the
    stand-in fails like the device cache if a step runs out of pages), keeps first-come order,
    and every request still gets its solo output."""
    rng = np.random.default_rng(4)
    reqs = [(rng.integers(0, 500, 90, dtype=np.uint32), 60, I.NO_EOS) for _ in range(7)]  # 149 positions: 10 pages
    with I.Server(synthetic=(8, 256, 500, 21)) as s:
        rids = [s.submit(p, m, e) for p, m, e in reqs]
        max_active = 0
        while s.stats()["waiting"] or s.stats()["active"]:
            s.step()
            max_active = max(max_active, s.stats()["active"])
        assert max_active == 2  # 21 pages hold two 10-page reservations
        outs = [s.result(r) for r in rids]
    for (p, m, e), (out, done, rc) in zip(reqs, outs):
        assert done and rc == 0 and out.size == m
        with I.Server(synthetic=(1, 256, 500)) as alone:
            (solo, _, _), = run_all(alone, [(p, m, e)])[0]
        np.testing.assert_array_equal(out, solo)


def test_request_larger_than_the_pool_is_refused_at_submit():
    with I.Server(synthetic=(4, 256, 500, 5)) as s:
        with pytest.raises(I.InfError) as e:
            s.submit(np.arange(70, dtype=np.uint32), 20)  # 89 positions: 6 pages of 16
        assert e.value.code == 2
        rid = s.submit(np.arange(60, dtype=np.uint32), 20)   # 79 positions: 5 pages
        while s.stats()["waiting"] or s.stats()["active"]:
            s.step()
        out, done, rc = s.result(rid)
        assert done and rc == 0 and out.size == 20


def test_failing_batched_step_retires_its_requests():
    """A batched step that fails (the stand-in fails every batch that holds a sequence whose
    prompt starts with id vocab - 1) returns its error once and retires the requests of that
    batch with it; their slots and pages go back to the pool, the server does not retry the same
    batch, and requests admitted later run to completion."""
    vocab = 500
    with I.Server(synthetic=(4, 128, vocab, 12)) as s:
        good0 = s.submit(np.arange(1, 20, dtype=np.uint32), 8)
        bad = s.submit(np.array([vocab - 1, 3, 4], np.uint32), 8)
        s.step()                            # both admitted (prefill only)
        with pytest.raises(I.InfError) as e:
            s.step()                        # their first batched step fails
        assert e.value.code == 7
        for rid in (good0, bad):
            out, done, rc = s.result(rid)
            assert done and rc == 7 and out.size == 1
        assert s.stats()["active"] == 0
        later = [s.submit(np.arange(5 + i, 40, dtype=np.uint32), 10) for i in range(3)]
        while s.stats()["waiting"] or s.stats()["active"]:
            s.step()
        for rid in later:
            out, done, rc = s.result(rid)
            assert done and rc == 0 and out.size == 10


def run_sampled(server, reqs):
    """Submit (prompt, max_new, sampling or None) at step 0 and step until all retire."""
    rids = [server.submit(p, m, I.NO_EOS, sampling=smp) for p, m, smp in reqs]
    for _ in range(10_000):
        server.step()
        if all(server.result(r)[1] for r in rids):
            return [server.result(r) for r in rids]
    raise AssertionError("requests did not retire")


def test_each_request_keeps_its_own_sampling_settings():
    """Per-request settings (inf_server_submit_sampled) reach the slot the request runs in: the
    stand-in's ids for a sampling request are a hash keyed by its settings.  A request's ids do not
    depend on what shares its batch, two seeds differ, a greedy request between sampling ones
    stays greedy, and a slot that a sampling request used serves a later greedy request greedily."""
    rng = np.random.default_rng(7)
    base = requests(rng, 12, 1000, 128)
    settings = [None, (0.8, 0.9, 0, 1), (1.2, 1.0, 40, 2), None, (0.8, 0.9, 0, 3)]
    reqs = [(p, m, settings[i % len(settings)]) for i, (p, m, _) in enumerate(base)]
    with I.Server(synthetic=(3, 128, 1000)) as s:
        together = run_sampled(s, reqs)
    for (p, m, smp), (out, done, rc) in zip(reqs, together):
        assert done and rc == 0 and out.size == m
        with I.Server(synthetic=(1, 128, 1000)) as alone:
            (solo, _, _), = run_sampled(alone, [(p, m, smp)])
        np.testing.assert_array_equal(out, solo)
        follows_greedy = all(out[k] == synthetic_next(int(out[k - 1]), len(p) + k - 1, 1000) for k in range(1, out.size))
        if smp is None:
            assert follows_greedy
        elif out.size > 3:
            assert not follows_greedy
    # the same request under two seeds
    p, m, _ = reqs[1]
    outs = []
    for seed in (11, 12):
        with I.Server(synthetic=(1, 128, 1000)) as alone:
            (o, _, _), = run_sampled(alone, [(p, 20, (0.8, 0.9, 0, seed))])
            outs.append(o)
    assert not np.array_equal(outs[0], outs[1])


def test_sampling_settings_are_checked_at_submit():
    with I.Server(synthetic=(1, 64, 100)) as s:
        for bad in [(-1.0, 1.0, 0, 0), (1.0, 0.0, 0, 0), (1.0, 1.5, 0, 0), (float("nan"), 1.0, 0, 0)]:
            with pytest.raises(I.InfError) as e:
                s.submit(np.arange(4, dtype=np.uint32), 4, I.NO_EOS, sampling=bad)
            assert e.value.code == 4
        s.submit(np.arange(4, dtype=np.uint32), 4, I.NO_EOS, sampling=(0.0, 0.0, 0, 0))  # temperature 0: greedy, top_p unused
