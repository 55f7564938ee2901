"""The no-allocation decode attention entry point (inf_attn_decode_noalloc).

It exists for callers that cannot call cudaMalloc: a serving loop that must not stall the
device mid-step, or a runtime whose device memory is all committed to a pre-sized arena.
Instead of caller-provided scratch it uses an array built into libinf.so, shared by every
call.  These tests call it through the C ABI twice in a row (the second call finds the first
call's leftovers in the shared array) and compare each result with the scratch-taking entry
point inf_attn_decode: both run the same kernel with the same split plan, so the outputs must
be bit-identical, whatever the shared array held before.  The file runs last so
that a failure here leaves every other test already run; it also passes on its own in a
fresh process (the first call sets up the array's device address).
"""
import pytest

import infb200 as I

pytestmark = pytest.mark.gpu


def _case(torch, H, KV, hd, positions, seed):
    blk = 16
    pps = (max(positions) + blk) // blk
    n = len(positions)
    n_pages = n * pps + 1
    g = torch.Generator(device="cuda").manual_seed(seed)
    kp = torch.randn(n_pages, KV, blk, hd, device="cuda", generator=g).to(torch.bfloat16)
    vp_ = torch.randn(n_pages, KV, blk, hd, device="cuda", generator=g).to(torch.bfloat16)
    q = (torch.randn(n, H * hd, device="cuda", generator=g) * 0.5).to(torch.bfloat16)
    bt = torch.randperm(n_pages, device="cuda", generator=g).int()[: n * pps].view(n, pps).contiguous()
    slots = torch.arange(n, dtype=torch.int32, device="cuda")
    pos = torch.tensor(positions, dtype=torch.int32, device="cuda")
    return dict(q=q, kp=kp, vp=vp_, bt=bt, slots=slots, pos=pos, pps=pps, n_pages=n_pages, n=n, H=H, KV=KV, hd=hd,
                blk=blk)


def _with_scratch(torch, c):
    out = torch.empty_like(c["q"])
    nb = I.attn_decode_scratch_bytes(c["n"], c["H"], c["KV"], c["hd"], c["blk"], c["pps"], I.BF16)
    scratch = torch.empty(nb, dtype=torch.uint8, device="cuda")
    I.attn_decode(c["q"].data_ptr(), c["kp"].data_ptr(), c["vp"].data_ptr(), c["bt"].data_ptr(), c["pps"],
                  c["n_pages"], c["slots"].data_ptr(), c["pos"].data_ptr(), c["n"], c["H"], c["KV"], c["hd"],
                  c["blk"], I.BF16, out.data_ptr(), scratch.data_ptr(), nb)
    return out


def _no_alloc(torch, c):
    out = torch.empty_like(c["q"])
    I.attn_decode_noalloc(c["q"].data_ptr(), c["kp"].data_ptr(), c["vp"].data_ptr(), c["bt"].data_ptr(), c["pps"],
                          c["n_pages"], c["slots"].data_ptr(), c["pos"].data_ptr(), c["n"], c["H"], c["KV"], c["hd"],
                          c["blk"], I.BF16, out.data_ptr())
    return out


def test_no_alloc_attention_matches_scratch_entry_point_twice(cuda):
    torch = cuda
    first = _case(torch, 32, 8, 128, [0, 17, 2047, 3071], seed=1)   # Llama-3-8B heads, batch 4
    second = _case(torch, 32, 4, 64, [5, 1023], seed=2)             # TinyLlama heads, other sizes
    for c in (first, second):
        want = _with_scratch(torch, c)
        got = _no_alloc(torch, c)
        torch.cuda.synchronize()
        assert torch.equal(got, want)


def test_no_alloc_attention_rejects_shapes_beyond_its_scratch(cuda):
    torch = cuda
    c = _case(torch, 32, 8, 128, [4095] * 64, seed=3)  # 64 sequences at 4k positions: ~23 MB of scratch
    with pytest.raises(I.InfError) as e:
        _no_alloc(torch, c)
    assert e.value.code == 4 and "above the built-in" in str(e.value)


def test_no_alloc_attention_reports_unsupported_shapes_like_the_scratch_entry_point(cuda):
    torch = cuda
    c = _case(torch, 24, 8, 128, [100], seed=4)  # GQA group 3: no kernel serves it
    with pytest.raises(I.InfError) as a:
        _no_alloc(torch, c)
    scratch = torch.empty(256, dtype=torch.uint8, device="cuda")  # the shape's scratch size is 0: unsupported
    out = torch.empty_like(c["q"])
    with pytest.raises(I.InfError) as b:
        I.attn_decode(c["q"].data_ptr(), c["kp"].data_ptr(), c["vp"].data_ptr(), c["bt"].data_ptr(), c["pps"],
                      c["n_pages"], c["slots"].data_ptr(), c["pos"].data_ptr(), c["n"], 24, 8, 128, 16, I.BF16,
                      out.data_ptr(), scratch.data_ptr(), 256)
    assert a.value.code == b.value.code == 15
    assert I.attn_decode_scratch_bytes(1, 24, 8, 128, 16, c["pps"], I.BF16) == 0
