"""The attention kernels at the plans the workloads actually run, against plain fp32 PyTorch
attention over the same paged cache (random page permutations unless stated):

* batch-1 decode of the Llama-3-8B shape with the model's default max_seq 3072: 192 pages per
  sequence, so the decode step runs the tensor-core cluster kernel as 16 CTAs x 12 pages per KV
  head (the SIMT cluster kernel, which serves fp32 models and other head sizes, alongside);
* the 64-sequence batched step (contexts 512-4096 from the seed-2 lengths, max_seq 4352): the
  tensor-core streaming kernel;
* batch-1 decode after the 32k-token prefill (max_seq 32896): beyond one cluster, the split-K
  kernel;
* the tensor-core causal prefill attention on one 4096-token chunk (the default prefill chunk)
  and on the second chunk of an 8192-token prompt, with consecutive and with scattered pages.
"""
import numpy as np
import pytest

import infb200 as I
from attn_ref import decode_attention, prefill_attention

pytestmark = pytest.mark.gpu

RTOL, ATOL = 2 ** -7, 2e-3  # bf16 output (8-bit mantissa); P rounded to bf16 in the tensor-core kernels


def _within_one_ulp(torch, a, b):
    """Two bf16 results of fp32-accurate computations: equal, or one bf16 rounding step apart
    (a value in [2^e, 2^(e+1)) has a step of 2^(e-7) <= 2^-7 |value|), with an absolute floor of
    1e-5 for outputs near zero, where the weighted sum cancels and the two fp32 summation orders
    (~1e-6 of the terms' magnitude) exceed a step of the tiny result.  Returns (ok, fraction
    identical, worst element as (a, b))."""
    a, b = a.float().flatten(), b.float().flatten()
    excess = (a - b).abs() - (torch.maximum(a.abs(), b.abs()) * 2 ** -7 + 1e-5)
    i = int(excess.argmax())
    return bool(excess[i] <= 0), float((a == b).float().mean()), (float(a[i]), float(b[i]))


def _pools(torch, n_pages, KV, blk, hd, seed, q_rows, H, q_scale=1.5):
    g = torch.Generator(device="cuda").manual_seed(seed)
    kp = torch.randn(n_pages, KV, blk, hd, device="cuda", generator=g).to(torch.bfloat16)
    vp_ = torch.randn(n_pages, KV, blk, hd, device="cuda", generator=g).to(torch.bfloat16)
    q = (torch.randn(q_rows, H * hd, device="cuda", generator=g) * q_scale / hd ** 0.25).to(torch.bfloat16)
    return g, kp, vp_, q


def _decode(torch, kernel, q, kp, vp_, bt, slots, pos, pps, n_pages, H, KV, hd, blk):
    n = q.shape[0]
    out = torch.empty_like(q)
    nb = I.attn_decode_scratch_bytes(n, H, KV, hd, blk, pps, I.BF16)
    scratch = torch.full((nb,), 0x7F, dtype=torch.uint8, device="cuda")
    I.attn_decode_with(kernel, q.data_ptr(), kp.data_ptr(), vp_.data_ptr(), bt.data_ptr(), pps, n_pages,
                       slots.data_ptr(), pos.data_ptr(), n, H, KV, hd, blk, I.BF16, out.data_ptr(), scratch.data_ptr(),
                       nb)
    return out


def test_cluster_kernel_at_the_headline_plan(cuda):
    """Llama-3-8B heads (32 q / 8 kv, head_dim 128), max_seq 3072 -> 192 pages per sequence, the
    positions the headline decodes (2048 and on) plus both ends of the plan's range; one token per
    call, as the batch-1 decode step runs it.  The tensor-core cluster kernel keeps each softmax
    weight as three bf16 parts (~24 bits), so its output is the SIMT cluster kernel's (fp32
    weights) or one bf16 rounding step away, and mostly identical."""
    torch = cuda
    H, KV, hd, blk, pps = 32, 8, 128, 16, 3072 // 16
    positions = [0, 15, 191, 2047, 2048, 2049, 2560, 3071]
    n_pages = pps + 5
    g, kp, vp_, q = _pools(torch, n_pages, KV, blk, hd, 11, len(positions), H)
    bt = torch.randperm(n_pages, device="cuda", generator=g).int()[:pps].view(1, pps).contiguous()
    slot = torch.zeros(1, dtype=torch.int32, device="cuda")
    for i, p in enumerate(positions):
        pos = torch.tensor([p], dtype=torch.int32, device="cuda")
        qi = q[i:i + 1].contiguous()
        ref = decode_attention(torch, qi, kp, vp_, bt, slot, pos, H, KV, hd, blk)
        cl = _decode(torch, I.ATTN_CLUSTER, qi, kp, vp_, bt, slot, pos, pps, n_pages, H, KV, hd, blk)
        torch.testing.assert_close(cl.float(), ref, rtol=RTOL, atol=ATOL, msg=f"position {p}")
        ct = _decode(torch, I.ATTN_CLUSTER_TC, qi, kp, vp_, bt, slot, pos, pps, n_pages, H, KV, hd, blk)
        torch.testing.assert_close(ct.float(), ref, rtol=RTOL, atol=ATOL, msg=f"tensor-core cluster at position {p}")
        ok, same, worst = _within_one_ulp(torch, ct, cl)
        assert ok and same >= 0.9, f"position {p}: {same:.3f} identical to the SIMT cluster kernel, worst {worst}"
        auto = _decode(torch, I.ATTN_AUTO, qi, kp, vp_, bt, slot, pos, pps, n_pages, H, KV, hd, blk)
        assert torch.equal(auto, ct), f"position {p}: the automatic choice is not the tensor-core cluster kernel"
        sk = _decode(torch, I.ATTN_SPLITK, qi, kp, vp_, bt, slot, pos, pps, n_pages, H, KV, hd, blk)
        torch.testing.assert_close(sk.float(), ref, rtol=RTOL, atol=ATOL, msg=f"split-K at position {p}")


@pytest.mark.parametrize("H,KV,hd,max_seq", [(32, 8, 128, 3072), (32, 4, 64, 1024), (32, 8, 128, 3328)])
def test_cluster_kernel_every_plan_size(cuda, H, KV, hd, max_seq):
    """TinyLlama heads at its max_seq, and the largest context one 16-CTA cluster holds for the
    Llama-3-8B heads (3328 positions: 13 pages per CTA fill the 112 KB shared-memory budget);
    several tokens in one launch (one cluster per token and KV head)."""
    torch = cuda
    blk = 16
    pps = max_seq // blk
    positions = [max_seq - 1, max_seq // 2, 17, max_seq - 16]
    n = len(positions)
    n_pages = n * pps
    g, kp, vp_, q = _pools(torch, n_pages, KV, blk, hd, H * hd + max_seq, n, H)
    bt = torch.randperm(n_pages, device="cuda", generator=g).int().view(n, pps).contiguous()
    slots = torch.arange(n, dtype=torch.int32, device="cuda")
    pos = torch.tensor(positions, dtype=torch.int32, device="cuda")
    ref = decode_attention(torch, q, kp, vp_, bt, slots, pos, H, KV, hd, blk)
    out = _decode(torch, I.ATTN_CLUSTER, q, kp, vp_, bt, slots, pos, pps, n_pages, H, KV, hd, blk)
    torch.testing.assert_close(out.float(), ref, rtol=RTOL, atol=ATOL)
    ct = _decode(torch, I.ATTN_CLUSTER_TC, q, kp, vp_, bt, slots, pos, pps, n_pages, H, KV, hd, blk)
    torch.testing.assert_close(ct.float(), ref, rtol=RTOL, atol=ATOL)
    ok, same, worst = _within_one_ulp(torch, ct, out)
    assert ok and same >= 0.9, f"{same:.3f} identical to the SIMT cluster kernel, worst {worst}"
    if max_seq == 3328:  # one more page per sequence no longer fits one cluster (refused on the host)
        bt2 = torch.zeros(n, pps + 1, dtype=torch.int32, device="cuda")
        for kernel in (I.ATTN_CLUSTER, I.ATTN_CLUSTER_TC):
            with pytest.raises(I.InfError) as e:
                _decode(torch, kernel, q, kp, vp_, bt2, slots, pos, pps + 1, n_pages, H, KV, hd, blk)
            assert e.value.code == 15


def test_mma_kernel_at_the_batched_workload(cuda):
    """64 sequences, contexts uniform in [512, 4096] (seed 2, the batched workload's lengths),
    max_seq 4352 -> 272 pages per sequence; the automatic choice for several tokens is this kernel."""
    torch = cuda
    H, KV, hd, blk = 32, 8, 128, 16
    B, pps = 64, 4352 // 16
    lens = I.synth_uniform(2, I.STREAM_CTX_LEN, B, 512, 4096)
    n_pages = B * pps
    g, kp, vp_, q = _pools(torch, n_pages, KV, blk, hd, 5, B, H)
    bt = torch.randperm(n_pages, device="cuda", generator=g).int().view(B, pps).contiguous()
    slots = torch.arange(B, dtype=torch.int32, device="cuda")
    pos = torch.from_numpy(lens.astype(np.int32)).cuda()  # the token at position len attends len + 1 keys
    ref = decode_attention(torch, q, kp, vp_, bt, slots, pos, H, KV, hd, blk)
    out = _decode(torch, I.ATTN_MMA, q, kp, vp_, bt, slots, pos, pps, n_pages, H, KV, hd, blk)
    torch.testing.assert_close(out.float(), ref, rtol=RTOL, atol=ATOL)
    auto = _decode(torch, I.ATTN_AUTO, q, kp, vp_, bt, slots, pos, pps, n_pages, H, KV, hd, blk)
    assert torch.equal(auto, out)


def test_split_k_kernel_at_32k_context(cuda):
    """Batch-1 decode after the 32768-token prefill: max_seq 32896 (2056 pages) is beyond one
    cluster, so the decode step runs the split-K kernel."""
    torch = cuda
    H, KV, hd, blk, pps = 32, 8, 128, 16, 32896 // 16
    n_pages = pps
    g, kp, vp_, q = _pools(torch, n_pages, KV, blk, hd, 9, 3, H)
    bt = torch.randperm(n_pages, device="cuda", generator=g).int().view(1, pps).contiguous()
    slot = torch.zeros(1, dtype=torch.int32, device="cuda")
    with pytest.raises(I.InfError) as e:  # the cluster kernel cannot hold 2056 pages
        pos = torch.tensor([100], dtype=torch.int32, device="cuda")
        _decode(torch, I.ATTN_CLUSTER, q[:1].contiguous(), kp, vp_, bt, slot, pos, pps, n_pages, H, KV, hd, blk)
    assert e.value.code == 15
    for i, p in enumerate([32767, 32800, 32895]):
        pos = torch.tensor([p], dtype=torch.int32, device="cuda")
        qi = q[i:i + 1].contiguous()
        ref = decode_attention(torch, qi, kp, vp_, bt, slot, pos, H, KV, hd, blk)
        out = _decode(torch, I.ATTN_AUTO, qi, kp, vp_, bt, slot, pos, pps, n_pages, H, KV, hd, blk)
        torch.testing.assert_close(out.float(), ref, rtol=RTOL, atol=ATOL, msg=f"position {p}")


@pytest.mark.parametrize("pos0,T,scatter", [(0, 4096, False), (0, 4096, True), (4096, 4096, False),
                                             (4096, 4096, True), (0, 300, True)])
def test_tensor_core_prefill_attention(cuda, pos0, T, scatter):
    """Causal attention of one prefill pass of the Llama-3-8B heads: the first 4096-token chunk of
    a prompt, and the second chunk of an 8192-token prompt (its queries attend the first chunk's
    keys too), with the sequence's pages consecutive in the pool (one 8-page TMA box per key tile)
    or scattered (one box per page); a short ragged prompt; the SIMT kernel alongside.

    The tensor-core kernel rounds each softmax weight to bf16 before P.V (relative error <= 2^-8
    per weight, the row sum taken over the rounded weights), so its output is an exact average of
    the values under weights perturbed by at most 2^-8: |out - ref| <= 2^-8 * max|v_i - out| <=
    2^-7 * max|V|.  That bound is reached only by the first tokens, which average a handful of
    values; with hundreds of keys the perturbations average out, so rows with at least 256 keys
    are held to the SIMT kernel's tolerance, and the mean error of every pass must stay small."""
    torch = cuda
    H, KV, hd, blk = 32, 8, 128, 16
    n = pos0 + T
    pps = (n + blk - 1) // blk
    n_pages = pps + 8
    g, kp, vp_, q = _pools(torch, n_pages, KV, blk, hd, n + int(scatter), T, H)
    pages = torch.randperm(n_pages, device="cuda", generator=g).int()[:pps] if scatter else \
        torch.arange(3, 3 + pps, dtype=torch.int32, device="cuda")
    bt = pages.view(1, pps).contiguous()
    tok_pos = torch.arange(pos0, n, dtype=torch.int32, device="cuda")
    tok_slot = torch.zeros(T, dtype=torch.int32, device="cuda")
    ref = prefill_attention(torch, q, kp, vp_, bt[0], pos0, T, H, KV, hd, blk)
    p_bound = 2 ** -7 * float(vp_.float().abs().max())
    long_rows = (tok_pos + 1 >= 256).nonzero().flatten()
    for kernel in (I.PREFILL_AUTO, I.PREFILL_SIMT):
        out = torch.empty_like(q)
        I.attn_prefill(kernel, q.data_ptr(), kp.data_ptr(), vp_.data_ptr(), bt.data_ptr(), pps, n_pages,
                       tok_slot.data_ptr(), tok_pos.data_ptr(), T, H, KV, hd, blk, out.data_ptr())
        err = (out.float() - ref).abs()
        assert float(err.mean()) <= 3e-4, f"kernel {kernel}: mean error {float(err.mean())}"
        if kernel == I.PREFILL_AUTO:
            torch.testing.assert_close(out.float(), ref, rtol=RTOL, atol=p_bound)
        else:
            torch.testing.assert_close(out.float(), ref, rtol=RTOL, atol=ATOL)
        if long_rows.numel():
            torch.testing.assert_close(out[long_rows].float(), ref[long_rows], rtol=RTOL, atol=ATOL)
