"""Kernel-level GPU parity: the stand-alone gather and RMSNorm of the C ABI against the
oracle and against the reference's own kernels (oracle/_ref, built from
src/cuda/kernels/input_embeddings.cu and rmsnorm.cu)."""
import ctypes as C
import os

import numpy as np
import pytest

import infb200 as I
import oracle as O

pytestmark = pytest.mark.gpu


def _ref_lib():
    if not os.path.exists(O.REF_LIB_PATH):
        pytest.skip("reference kernels not built (oracle/_ref)")
    L = C.CDLL(O.REF_LIB_PATH)
    L.ref_fetch_input_embeddings.restype = C.c_int
    L.ref_fetch_input_embeddings.argtypes = [C.c_void_p, C.c_ulonglong, C.c_uint, C.c_void_p, C.c_void_p, C.c_void_p]
    L.ref_rmsnorm_row0.restype = C.c_int
    L.ref_rmsnorm_row0.argtypes = [C.c_void_p, C.c_uint, C.c_void_p, C.c_void_p]
    return L


def _bf16_table(torch, vocab, dim, seed):
    t = O.fill_tensor(seed, O.tensor_stream(-1, O.K_EMBED), vocab * dim, 0.02, bf16=True)
    return t.reshape(vocab, dim), torch.from_numpy(t.view(np.int16).reshape(vocab, dim)).cuda()


@pytest.mark.parametrize("vocab,dim,n", [(32000, 288, 16), (32000, 2048, 512), (128256, 4096, 64), (1000, 72, 3),
                                         (50, 8, 1)])
def test_gather_bit_exact_vs_oracle(cuda, vocab, dim, n):
    torch = cuda
    h_tab, d_tab = _bf16_table(torch, vocab, dim, 0)
    ids = O.gen_ids(1, n, vocab)
    ids[0] = vocab - 1
    d_ids = torch.from_numpy(ids.view(np.int32)).cuda()
    out = torch.empty((n, dim), dtype=torch.int16, device="cuda")
    I.fetch_input_embeddings(d_ids.data_ptr(), n, dim, vocab, d_tab.data_ptr(), out.data_ptr(), I.BF16)
    got = out.cpu().numpy().view(np.uint16)
    want = O.embed_gather(ids, h_tab, dim)  # fp32 values of the bf16 rows
    np.testing.assert_array_equal(O.bf16_to_f32(got), want)


def test_gather_fp32_bit_exact(cuda):
    torch = cuda
    tab = O.fill_tensor(0, 0, 32000 * 288, 0.02, bf16=False).reshape(32000, 288)
    ids = O.gen_ids(1, 16, 32000)
    out = torch.empty((16, 288), dtype=torch.float32, device="cuda")
    d_tab = torch.from_numpy(tab).cuda()
    d_ids = torch.from_numpy(ids.view(np.int32)).cuda()
    I.fetch_input_embeddings(d_ids.data_ptr(), 16, 288, 32000, d_tab.data_ptr(), out.data_ptr(), I.F32)
    np.testing.assert_array_equal(out.cpu().numpy(), tab[ids])


def test_gather_rejects_out_of_range_id(cuda):
    torch = cuda
    _, d_tab = _bf16_table(torch, 100, 16, 0)
    d_ids = torch.tensor([3, 100, 5], dtype=torch.int32, device="cuda")
    out = torch.empty((3, 16), dtype=torch.int16, device="cuda")
    with pytest.raises(I.InfError) as e:
        I.fetch_input_embeddings(d_ids.data_ptr(), 3, 16, 100, d_tab.data_ptr(), out.data_ptr(), I.BF16)
    assert e.value.code == 10
    assert (out[1] == 0).all()  # the bad row is zeroed, never read out of bounds


@pytest.mark.parametrize("dim,n", [(288, 16), (2048, 64), (4096, 64)])
def test_gather_matches_reference_kernel(cuda, dim, n):
    """The reference's own gather (launched as src/main.cu:396-404) pins the oracle and ours."""
    torch = cuda
    L = _ref_lib()
    vocab = 4096
    h_tab, d_tab = _bf16_table(torch, vocab, dim, 3)
    ids = O.gen_ids(9, n, vocab)
    d_ids = torch.from_numpy(ids.view(np.int32)).cuda()
    ref = torch.empty((n, dim), dtype=torch.int16, device="cuda")
    ours = torch.empty_like(ref)
    assert L.ref_fetch_input_embeddings(d_ids.data_ptr(), n, dim, d_tab.data_ptr(), ref.data_ptr(), None) == 0
    torch.cuda.synchronize()
    I.fetch_input_embeddings(d_ids.data_ptr(), n, dim, vocab, d_tab.data_ptr(), ours.data_ptr(), I.BF16)
    assert torch.equal(ref, ours)
    np.testing.assert_array_equal(O.bf16_to_f32(ref.cpu().numpy().view(np.uint16)), O.embed_gather(ids, h_tab, dim))


@pytest.mark.parametrize("rows,dim", [(1, 288), (16, 4096), (7, 2048), (3, 5632), (2, 72)])
def test_rmsnorm_vs_oracle(cuda, rows, dim):
    torch = cuda
    rng = np.random.default_rng(dim)
    x = rng.standard_normal((rows, dim)).astype(np.float32) * 0.3
    xb = np.vectorize(O.lib().orc_f32_to_bf16, otypes=[np.uint16])(x)
    g = np.full(dim, 0x3F80, np.uint16)
    g[::3] = 0x3FC0  # 1.5
    d_x = torch.from_numpy(xb.view(np.int16)).cuda()
    d_g = torch.from_numpy(g.view(np.int16)).cuda()
    d_y = torch.empty_like(d_x)
    I.rmsnorm(d_x.data_ptr(), d_y.data_ptr(), rows, dim, d_g.data_ptr(), 1e-5, I.BF16)
    got = O.bf16_to_f32(d_y.cpu().numpy().view(np.uint16))
    want = O.rmsnorm(O.bf16_to_f32(xb), g, 1e-5)
    # identical rounding point; fp32 reduction order may move a value by one bf16 ulp
    np.testing.assert_allclose(got, want, rtol=2 ** -7, atol=1e-6)
    assert np.mean(got == want) > 0.99


@pytest.mark.parametrize("dim", [128, 512, 2048])
def test_rmsnorm_matches_reference_kernel_on_its_valid_domain(cuda, dim):
    """k_rmsnorm (src/cuda/kernels/rmsnorm.cu:11-59) has no eps and is only well defined for
    one row with a power-of-two warp count; there it must agree with ours at eps = 0."""
    torch = cuda
    L = _ref_lib()
    rng = np.random.default_rng(dim)
    x = (rng.standard_normal(dim) * 0.5).astype(np.float32)
    xb = np.vectorize(O.lib().orc_f32_to_bf16, otypes=[np.uint16])(x)
    g = np.vectorize(O.lib().orc_f32_to_bf16, otypes=[np.uint16])(1 + 0.1 * rng.standard_normal(dim).astype(np.float32))
    d_ref = torch.from_numpy(xb.view(np.int16)).cuda()
    d_g = torch.from_numpy(g.view(np.int16)).cuda()
    d_ours = torch.empty_like(d_ref)
    I.rmsnorm(d_ref.data_ptr(), d_ours.data_ptr(), 1, dim, d_g.data_ptr(), 0.0, I.BF16)
    assert L.ref_rmsnorm_row0(d_ref.data_ptr(), dim, d_g.data_ptr(), None) == 0  # in place
    torch.cuda.synchronize()
    ref = O.bf16_to_f32(d_ref.cpu().numpy().view(np.uint16))
    ours = O.bf16_to_f32(d_ours.cpu().numpy().view(np.uint16))
    orc = O.rmsnorm(O.bf16_to_f32(xb)[None], g, 0.0)[0]
    np.testing.assert_allclose(ref, ours, rtol=2 ** -7, atol=1e-6)
    np.testing.assert_allclose(orc, ours, rtol=2 ** -7, atol=1e-6)


def _attn_reference(torch, q, kp, vp_, bt, slots, pos, H, KV, hd, blk):
    """Plain fp32 attention of each token over positions 0..pos of its slot."""
    G = H // KV
    outs = []
    for i in range(q.shape[0]):
        n = int(pos[i]) + 1
        pages = bt[int(slots[i]), : (n + blk - 1) // blk].long()
        K = kp[pages].float().permute(1, 0, 2, 3).reshape(KV, -1, hd)[:, :n]   # [KV, n, hd]
        V = vp_[pages].float().permute(1, 0, 2, 3).reshape(KV, -1, hd)[:, :n]
        qi = q[i].float().view(KV, G, hd)
        s = torch.einsum("kgd,knd->kgn", qi, K) / hd ** 0.5
        p = torch.softmax(s, dim=-1)
        outs.append(torch.einsum("kgn,knd->kgd", p, V).reshape(H * hd))
    return torch.stack(outs)


@pytest.mark.parametrize("H,KV,hd,dtype,positions", [
    (32, 8, 128, "bf16", [0, 15, 16, 1000, 2047, 2560]),
    (32, 4, 64, "bf16", [5, 511, 512, 1023]),
    (6, 6, 48, "fp32", [0, 17, 255]),
    (4, 2, 16, "bf16", [3, 63]),
])
def test_attn_decode_kernel_vs_torch_fp32(cuda, H, KV, hd, dtype, positions):
    torch = cuda
    blk = 16
    max_seq = max(positions) + 1
    pps = (max_seq + blk - 1) // blk
    n = len(positions)
    n_pages = n * pps + 3
    g = torch.Generator(device="cuda").manual_seed(H * hd + n)
    tdt = torch.bfloat16 if dtype == "bf16" else torch.float32
    kp = torch.randn(n_pages, KV, blk, hd, device="cuda", generator=g).to(tdt)
    vp_ = torch.randn(n_pages, KV, blk, hd, device="cuda", generator=g).to(tdt)
    q = (torch.randn(n, H * hd, device="cuda", generator=g) * 0.5).to(tdt)
    perm = torch.randperm(n_pages, device="cuda", generator=g).int()
    bt = perm[: n * pps].view(n, pps).contiguous()
    slots = torch.arange(n, dtype=torch.int32, device="cuda")
    pos = torch.tensor(positions, dtype=torch.int32, device="cuda")
    out = torch.empty_like(q)
    code = I.BF16 if dtype == "bf16" else I.F32
    nb = I.attn_decode_scratch_bytes(n, H, KV, hd, blk, pps, code)
    scratch = torch.full((nb,), 0x7F, dtype=torch.uint8, device="cuda")  # contents on entry do not matter
    for _ in range(2):
        I.attn_decode(q.data_ptr(), kp.data_ptr(), vp_.data_ptr(), bt.data_ptr(), pps, n_pages, slots.data_ptr(),
                      pos.data_ptr(), n, H, KV, hd, blk, code, out.data_ptr(), scratch.data_ptr(), nb)
    ref = _attn_reference(torch, q, kp, vp_, bt, slots, pos, H, KV, hd, blk)
    if dtype == "bf16":
        torch.testing.assert_close(out.float(), ref, rtol=2 ** -7, atol=2e-3)
    else:
        torch.testing.assert_close(out, ref, rtol=1e-4, atol=1e-5)


def test_attn_decode_rejects_bad_page(cuda):
    torch = cuda
    H, KV, hd, blk, pps = 8, 2, 64, 16, 4
    kp = torch.zeros(4, KV, blk, hd, dtype=torch.bfloat16, device="cuda")
    q = torch.zeros(1, H * hd, dtype=torch.bfloat16, device="cuda")
    bt = torch.tensor([[0, 1, 99, 2]], dtype=torch.int32, device="cuda")  # page 99 is outside the pool
    slot = torch.zeros(1, dtype=torch.int32, device="cuda")
    pos = torch.tensor([40], dtype=torch.int32, device="cuda")
    out = torch.empty_like(q)
    nb = I.attn_decode_scratch_bytes(1, H, KV, hd, blk, pps, I.BF16)
    scratch = torch.empty(nb, dtype=torch.uint8, device="cuda")
    with pytest.raises(I.InfError) as e:
        I.attn_decode(q.data_ptr(), kp.data_ptr(), kp.data_ptr(), bt.data_ptr(), pps, 4, slot.data_ptr(),
                      pos.data_ptr(), 1, H, KV, hd, blk, I.BF16, out.data_ptr(), scratch.data_ptr(), nb)
    assert e.value.code == 11
