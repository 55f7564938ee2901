"""Tensor parallelism's decomposition on CPU with two gloo ranks (no GPU): each rank reads its
own shard in the device layout from a checkpoint (inf_safetensors_read with tp_size 2: QKV heads
and gate/up rows column-parallel, O and down columns row-parallel, LM-head vocabulary rows), runs
its half of one decoder layer in float64, and the two partial sums after O and after down are
added with all_reduce -- the exchanges the projection kernels do over NVLink peer memory -- and
the LM head's argmax is taken across the vocabulary shards (ties to the lowest id).  The result
must equal the single-process computation on the canonical tensors.  And a rank that dies
between steps: the survivor's exchange ends with an error within its short process-group
timeout instead of waiting for good."""
import os
import socket

import numpy as np
import pytest

import infb200 as I
import oracle as O
from st_files import TINY, bf16_round, random_tensors, widen, write_checkpoint

WORLD = 2
POS = 9  # position of the token; positions 0..8 come from a synthetic cache


def rmsnorm(x, eps):
    return x / np.sqrt(np.mean(x * x) + eps)


def rope(v, pos, theta):
    """Rotate-half RoPE on [heads, hd] in canonical order."""
    hd = v.shape[-1]
    half = hd // 2
    inv = theta ** (-2.0 * np.arange(half) / hd)
    c, s = np.cos(pos * inv), np.sin(pos * inv)
    a, b = v[..., :half], v[..., half:]
    return np.concatenate([a * c - b * s, b * c + a * s], axis=-1)


def attention(q, kc, vc, G):
    """q [H, hd]; kc, vc [KV, ctx, hd]."""
    H, hd = q.shape
    out = np.empty_like(q)
    for h in range(H):
        s = kc[h // G] @ q[h] / np.sqrt(hd)
        p = np.exp(s - s.max())
        out[h] = (p / p.sum()) @ vc[h // G]
    return out


def synthetic_cache(cfg):
    rng = np.random.default_rng(33)
    KV, hd = cfg["n_kv_heads"], cfg["head_dim"]
    return rng.standard_normal((KV, POS, hd)), rng.standard_normal((KV, POS, hd))


def full_layer(t, cfg, x):
    """One layer and the LM head on the canonical tensors (float64)."""
    eps, theta = cfg["eps"], cfg["rope_theta"]
    H, KV, hd = cfg["n_heads"], cfg["n_kv_heads"], cfg["head_dim"]
    f = {k: widen(v).astype(np.float64) for k, v in t.items()}
    xn = rmsnorm(x, eps) * f[(O.K_ATTN_NORM, 0)]
    q = rope((f[(O.K_WQ, 0)] @ xn).reshape(H, hd), POS, theta)
    k = rope((f[(O.K_WK, 0)] @ xn).reshape(KV, hd), POS, theta)
    v = (f[(O.K_WV, 0)] @ xn).reshape(KV, hd)
    kc, vc = synthetic_cache(cfg)
    kc = np.concatenate([kc, k[:, None]], axis=1)
    vc = np.concatenate([vc, v[:, None]], axis=1)
    r1 = x + f[(O.K_WO, 0)] @ attention(q, kc, vc, H // KV).ravel()
    xn2 = rmsnorm(r1, eps) * f[(O.K_FFN_NORM, 0)]
    g, u = f[(O.K_WGATE, 0)] @ xn2, f[(O.K_WUP, 0)] @ xn2
    r2 = r1 + f[(O.K_WDOWN, 0)] @ (g / (1 + np.exp(-g)) * u)
    logits = f[(O.K_LM_HEAD, -1)] @ (rmsnorm(r2, eps) * f[(O.K_FINAL_NORM, -1)])
    return r2, int(np.argmax(logits))


def from_pairs(rows, hd):
    """Device row order within each head ((i, i + hd/2) pairs) back to canonical order."""
    heads = rows.reshape(-1, hd)
    out = np.empty_like(heads)
    out[:, :hd // 2] = heads[:, 0::2]
    out[:, hd // 2:] = heads[:, 1::2]
    return out


def rank_main(rank, path, port, ref_path):
    import torch
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=WORLD)
    try:
        cfg = dict(TINY, n_layers=1)
        c = I.config_from_dict(cfg)
        c.tp_size, c.tp_rank = WORLD, rank
        rd = lambda kind: widen(I.safetensors_read(path, c, 0, kind)).astype(np.float64)
        eps, theta = cfg["eps"], cfg["rope_theta"]
        Hl, KVl, hd = cfg["n_heads"] // WORLD, cfg["n_kv_heads"] // WORLD, cfg["head_dim"]
        ref = np.load(ref_path)
        x = ref["x"]

        def all_reduce(v):
            t = torch.from_numpy(np.ascontiguousarray(v))
            dist.all_reduce(t)
            return t.numpy()

        xn = rmsnorm(x, eps) * rd(I.W_ATTN_NORM)[0]
        qkv = rd(I.W_QKV) @ xn  # this rank's q heads, then k heads, then v heads
        q = rope(from_pairs(qkv[:Hl * hd], hd), POS, theta)
        k = rope(from_pairs(qkv[Hl * hd:(Hl + KVl) * hd], hd), POS, theta)
        v = from_pairs(qkv[(Hl + KVl) * hd:], hd)
        kc, vc = synthetic_cache(cfg)
        kc = np.concatenate([kc[rank * KVl:(rank + 1) * KVl], k[:, None]], axis=1)
        vc = np.concatenate([vc[rank * KVl:(rank + 1) * KVl], v[:, None]], axis=1)
        att = attention(q, kc, vc, Hl // KVl)
        r1 = x + all_reduce(rd(I.W_O) @ att.ravel())  # row-parallel O: partial sums
        xn2 = rmsnorm(r1, eps) * rd(I.W_FFN_NORM)[0]
        gu = rd(I.W_GATE_UP) @ xn2  # gate_j, up_j interleaved
        g, u = gu[0::2], gu[1::2]
        r2 = r1 + all_reduce(rd(I.W_DOWN) @ (g / (1 + np.exp(-g)) * u))
        lg = rd(I.W_LM_HEAD) @ (rmsnorm(r2, eps) * rd(I.W_FINAL_NORM)[0])
        local = int(np.argmax(lg))
        best = [None] * WORLD
        dist.all_gather_object(best, (float(lg[local]), rank * c.vocab_size // WORLD + local))
        am = min(best, key=lambda b: (-b[0], b[1]))[1]
        np.testing.assert_allclose(r2, ref["r2"], rtol=1e-12, atol=1e-12)
        assert am == int(ref["argmax"])
    finally:
        dist.destroy_process_group()


def free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_tp2_layer_matches_single_process(tmp_path):
    import torch.multiprocessing as mp
    cfg = dict(TINY, n_layers=1)
    t = {k: bf16_round(v) for k, v in random_tensors(cfg, np.random.default_rng(12)).items()}
    path = str(tmp_path / "tp.safetensors")
    write_checkpoint(path, cfg, t)
    x = np.random.default_rng(13).standard_normal(cfg["dim"])
    r2, am = full_layer(t, cfg, x)
    ref_path = str(tmp_path / "ref.npz")
    np.savez(ref_path, x=x, r2=r2, argmax=am)
    mp.spawn(rank_main, args=(path, free_port(), ref_path), nprocs=WORLD, join=True)


def failing_rank_main(rank, port, q):
    """Rank 1 dies before the exchange; rank 0's all-reduce must end with an error, not hang."""
    import datetime
    import time

    import torch
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=WORLD,
                            timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        os._exit(3)  # a rank that stops between steps
    t0 = time.time()
    try:
        dist.all_reduce(torch.ones(4))
        q.put(("no error", time.time() - t0))
    except Exception as e:  # noqa: BLE001 -- any error is the detection
        q.put(("error", time.time() - t0, type(e).__name__))


def test_rank_failure_is_detected_not_hung():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=failing_rank_main, args=(r, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    try:
        res = q.get(timeout=120)
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    assert res[0] == "error" and res[1] < 60, res
    assert procs[1].exitcode == 3
