"""The Gemma-style decoder (InfConfig.arch = InfArchGemma) on the B200 against the oracle's
restatement of it (oracle/llama_ref.c, pinned to the independent numpy restatement of
tests/golden/gen_golden.py): embedding scale, (1 + w) RMSNorms, per-head q/k norms, post-attention
and pre/post-FFN norms, GELU-tanh MLP, per-layer-embedding block, tied LM head, logit soft-cap,
and head_dim 512 attention."""
import os

import numpy as np
import pytest

import infb200 as I
import oracle as O
from attn_ref import decode_attention
from test_stages_gpu import assert_bf16_close

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")

TINY_GEMMA = dict(vocab=512, dim=64, n_layers=2, n_heads=4, n_kv_heads=2, head_dim=32, ffn=128, max_seq=64,
                  eps=1e-6, rope_theta=10000.0, arch=1, ple_dim=16, final_softcap=30.0, dtype="bf16")


def cosine(a, b):
    a, b = a.astype(np.float64), b.astype(np.float64)
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b) + 1e-30))


def test_tiny_gemma_against_golden_and_oracle(cuda):
    g = np.load(os.path.join(GOLD, "tiny_gemma_bf16.npz"))
    cfg = I.config_from_dict(TINY_GEMMA)
    with I.Engine(cfg, seed=0) as eng:
        lg, am = eng.forward(g["prompt"], 0)
        ids, logits = [am], [lg]
        for s in range(1, 12):
            lg, am = eng.forward([ids[-1]], len(g["prompt"]) + s - 1)
            ids.append(am)
            logits.append(lg)
    np.testing.assert_array_equal(np.array(ids, np.uint32), g["ids"])
    orc = O.OracleModel(I.oracle_dict(cfg), seed=0)
    o_ids, o_logits = orc.generate(g["prompt"], 12, want_logits=True)
    np.testing.assert_array_equal(o_ids, g["ids"])
    for s in range(12):
        assert float(np.abs(logits[s] - o_logits[s]).max()) <= 2e-2, f"step {s}"
        assert cosine(logits[s], o_logits[s]) >= 0.999, f"step {s}"


def test_gemma_generate_and_sampling_run(cuda):
    cfg = I.config_from_dict(TINY_GEMMA)
    prompt = O.gen_ids(3, 9, cfg.vocab_size)
    with I.Engine(cfg, seed=0) as eng:
        gen, st = eng.generate(prompt, 20)
        eng.reset(0)
        _, am = eng.forward(prompt, 0)
        loop = [am]
        for s in range(1, 20):
            _, am = eng.forward([loop[-1]], 9 + s - 1)
            loop.append(am)
        np.testing.assert_array_equal(gen, np.array(loop, np.uint32))
        eng.set_sampling(0.8, 0.95, 20, seed=3)
        eng.reset(0)
        sampled, _ = eng.generate(prompt, 20)
        assert sampled.max() < cfg.vocab_size


def test_gemma_e2b_shape_one_layer_stages(cuda):
    """The Gemma-4-E2B shape (dim 1536, 8 heads of 512 with 2 KV heads, FFN 6144, per-layer
    inputs of 256), one layer, vocabulary 4096: 12 tokens through the decode step, then q, each
    position's K and V, the attention output (head_dim 512, the split-K kernel), the GELU-tanh
    product and the logits against the oracle."""
    cfg = I.preset(6, n_layers=1, vocab_size=4096, max_seq=256)
    n = 12
    prompt = I.synth_ids(7, n, cfg.vocab_size)
    with I.Engine(cfg) as eng:
        for t in range(n):
            lg, am = eng.forward(prompt[t:t + 1], t)
        got = {k: eng.debug_read(k) for k in ("q", "attn", "h", "resid", "logits")}
        kv = [(eng.debug_read("k", 0, 0, t), eng.debug_read("v", 0, 0, t)) for t in range(n)]
    orc = O.OracleModel(I.oracle_dict(cfg), seed=0)
    o_lg, o_am = orc.forward(prompt, 0)
    q, _, _, att = orc.layer0()
    h, resid = orc.layer0_mlp()
    assert_bf16_close(got["q"], q, "q")
    for t in range(n):
        k, v = orc.kv(0, t)
        assert_bf16_close(kv[t][0], k, f"k[{t}]")
        assert_bf16_close(kv[t][1], v, f"v[{t}]")
    assert_bf16_close(got["attn"], att, "attention", min_exact=0.95)
    assert_bf16_close(got["h"], h, "gelu product", min_exact=0.9)
    scale = float(np.abs(resid).max())
    assert float(np.abs(got["resid"] - resid).max()) <= 2e-2 * scale
    assert float(np.abs(got["logits"] - o_lg).max()) <= 2e-2
    assert cosine(got["logits"], o_lg) >= 0.999
    assert am == o_am or np.sort(o_lg)[-1] - np.sort(o_lg)[-2] < 2e-2


@pytest.mark.parametrize("positions", [[0, 15, 511], [1000, 4095]])
def test_attention_head_dim_512(cuda, positions):
    """head_dim 512 (Gemma's global_head_dim, src/model.cuh:11), GQA group 4: the split-K kernel
    (16 head-dim values a lane) against fp32 attention."""
    torch = cuda
    H, KV, hd, blk = 8, 2, 512, 16
    pps = 4096 // blk
    n = len(positions)
    n_pages = n * pps
    g = torch.Generator(device="cuda").manual_seed(hd + n)
    kp = torch.randn(n_pages, KV, blk, hd, device="cuda", generator=g).to(torch.bfloat16)
    vp_ = torch.randn(n_pages, KV, blk, hd, device="cuda", generator=g).to(torch.bfloat16)
    q = (torch.randn(n, H * hd, device="cuda", generator=g) * 0.3).to(torch.bfloat16)
    bt = torch.randperm(n_pages, device="cuda", generator=g).int().view(n, pps).contiguous()
    slots = torch.arange(n, dtype=torch.int32, device="cuda")
    pos = torch.tensor(positions, dtype=torch.int32, device="cuda")
    out = torch.empty_like(q)
    nb = I.attn_decode_scratch_bytes(n, H, KV, hd, blk, pps, I.BF16)
    scratch = torch.empty(nb, dtype=torch.uint8, device="cuda")
    I.attn_decode(q.data_ptr(), kp.data_ptr(), vp_.data_ptr(), bt.data_ptr(), pps, n_pages, slots.data_ptr(),
                  pos.data_ptr(), n, H, KV, hd, blk, I.BF16, out.data_ptr(), scratch.data_ptr(), nb)
    ref = decode_attention(torch, q, kp, vp_, bt, slots, pos, H, KV, hd, blk)
    torch.testing.assert_close(out.float(), ref, rtol=2 ** -7, atol=2e-3)
