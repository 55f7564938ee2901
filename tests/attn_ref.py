"""Plain fp32 PyTorch attention over a paged KV cache, the reference the attention kernels are
tested against (a helper module for the GPU tests, not a test file)."""


def gather_pages(torch, pool, pages, n, KV, hd):
    """[KV, n, hd] fp32 rows 0..n-1 of one sequence from a [pages][KV][blk][hd] pool."""
    return pool[pages].float().permute(1, 0, 2, 3).reshape(KV, -1, hd)[:, :n]


def decode_attention(torch, q, kp, vp_, bt, slots, pos, H, KV, hd, blk):
    """softmax(q.K^T / sqrt(hd)).V of each token over positions 0..pos[i] of its slot."""
    G = H // KV
    outs = []
    for i in range(q.shape[0]):
        n = int(pos[i]) + 1
        pages = bt[int(slots[i]), : (n + blk - 1) // blk].long()
        K = gather_pages(torch, kp, pages, n, KV, hd)
        V = gather_pages(torch, vp_, pages, n, KV, hd)
        qi = q[i].float().view(KV, G, hd)
        s = torch.einsum("kgd,knd->kgn", qi, K) / hd ** 0.5
        p = torch.softmax(s, dim=-1)
        outs.append(torch.einsum("kgn,knd->kgd", p, V).reshape(H * hd))
    return torch.stack(outs)


def prefill_attention(torch, q, kp, vp_, bt_row, pos0, T, H, KV, hd, blk, rows=512):
    """Causal attention of T consecutive tokens at positions pos0.. of one sequence whose block
    table row is bt_row: token t attends positions 0..pos0+t.  q: [T][H*hd]; returns [T][H*hd]."""
    G = H // KV
    n = pos0 + T
    pages = bt_row[: (n + blk - 1) // blk].long()
    K = gather_pages(torch, kp, pages, n, KV, hd)           # [KV, n, hd]
    V = gather_pages(torch, vp_, pages, n, KV, hd)
    qf = q.float().view(T, KV, G, hd)
    out = torch.empty(T, KV, G, hd, device=q.device, dtype=torch.float32)
    keys = torch.arange(n, device=q.device)
    for t0 in range(0, T, rows):
        t1 = min(T, t0 + rows)
        qb = qf[t0:t1].permute(1, 2, 0, 3)                  # [KV, G, r, hd]
        s = torch.einsum("kgrd,knd->kgrn", qb, K) / hd ** 0.5
        qpos = torch.arange(pos0 + t0, pos0 + t1, device=q.device)
        s = s.masked_fill(keys[None, :] > qpos[:, None], float("-inf"))
        p = torch.softmax(s, dim=-1)
        out[t0:t1] = torch.einsum("kgrn,knd->kgrd", p, V).permute(2, 0, 1, 3)
    return out.reshape(T, H * hd)
