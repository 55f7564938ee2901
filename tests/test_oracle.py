"""CPU tests of the oracle: pinned against published Philox known answers and against the
golden fixtures of the independent numpy restatement (tests/golden/gen_golden.py)."""
import os

import numpy as np
import pytest

import oracle as O

GOLD = os.path.join(os.path.dirname(__file__), "golden")
TINY = dict(vocab=512, dim=64, n_layers=2, n_heads=4, n_kv_heads=2, head_dim=16, ffn=160, max_seq=64,
            eps=1e-5, rope_theta=10000.0)


# Known-answer vectors published with Random123 (Salmon et al., SC'11) for Philox4x32-10.
PHILOX_KAT = [
    ((0, 0, 0, 0), (0, 0), (0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8)),
    ((0xFFFFFFFF,) * 4, (0xFFFFFFFF,) * 2, (0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD)),
    ((0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344), (0xA4093822, 0x299F31D0),
     (0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1)),
]


@pytest.mark.parametrize("ctr,key,want", PHILOX_KAT)
def test_philox_known_answers(ctr, key, want):
    assert tuple(int(x) for x in O.philox(ctr, key)) == want


def test_splitmix64_known_answer():
    # SplitMix64 from state 0: first output of the reference generator (Vigna)
    assert O.lib().orc_splitmix64(0) == 0xE220A8397B1DCDAF


def test_streams_match_numpy_restatement():
    s = np.load(os.path.join(GOLD, "streams.npz"))
    np.testing.assert_array_equal(O.gen_ids(1, 16, 32000), s["prompt_cfg1"])
    np.testing.assert_array_equal(O.gen_ids(1, 64, 128256), s["prompt_cfg3_head"])
    lens = np.array([O.uniform_u32(2, O.STREAM_CTX_LEN, i, 512, 4096) for i in range(64)], np.uint32)
    np.testing.assert_array_equal(lens, s["ctx_lens_cfg4"])
    assert lens.min() >= 512 and lens.max() <= 4096
    v = O.fill_tensor(0, O.tensor_stream(-1, O.K_EMBED), 64, 0.02, bf16=False)
    np.testing.assert_array_equal(v, s["normal_head"])


def test_synthetic_weight_statistics():
    v = O.fill_tensor(0, O.tensor_stream(3, O.K_WQ), 1 << 20, 0.02, bf16=False)
    assert abs(float(v.mean())) < 1e-4
    assert abs(float(v.std()) - 0.02) < 2e-4
    assert float(np.abs(v).max()) <= 0.02 * np.sqrt(3) * 2 + 1e-6  # Irwin-Hall(4) support


@pytest.mark.parametrize("x,want", [
    (1.0, 0x3F80), (-2.0, 0xC000), (0.0, 0x0000), (-0.0, 0x8000),
    (1.00390625, 0x3F80),          # exactly half an ulp above 1.0: ties to even (down)
    (1.01171875, 0x3F82),          # 1.5 ulp: ties to even (up)
    (float("inf"), 0x7F80), (3.4e38, 0x7F80),  # rounds to inf
])
def test_bf16_round_to_nearest_even(x, want):
    assert O.lib().orc_f32_to_bf16(x) == want


def test_bf16_nan_is_quiet():
    assert O.lib().orc_f32_to_bf16(float("nan")) == 0x7FC0


@pytest.mark.parametrize("dtype", ["fp32", "bf16"])
def test_oracle_matches_golden(dtype):
    g = np.load(os.path.join(GOLD, f"tiny_{dtype}.npz"))
    m = O.OracleModel(dict(TINY, dtype=dtype), seed=0)
    emb = m.weight(-1, O.K_EMBED, (512, 64))[:4]
    emb = O.bf16_to_f32(emb) if dtype == "bf16" else emb
    np.testing.assert_array_equal(emb, g["embed_head"])
    wq = m.weight(0, O.K_WQ, (64, 64))[:2]
    np.testing.assert_array_equal(O.bf16_to_f32(wq) if dtype == "bf16" else wq, g["wq0_head"])
    wd = m.weight(1, O.K_WDOWN, (64, 160))[-2:]
    np.testing.assert_array_equal(O.bf16_to_f32(wd) if dtype == "bf16" else wd, g["wd1_tail"])
    ids, logits = m.generate(g["prompt"], 12, want_logits=True)
    np.testing.assert_array_equal(ids, g["ids"])
    np.testing.assert_allclose(logits, g["logits"], atol=2e-5, rtol=0)


@pytest.mark.parametrize("dtype", ["fp32", "bf16"])
def test_oracle_layer0_stages_match_golden(dtype):
    g = np.load(os.path.join(GOLD, f"tiny_{dtype}.npz"))
    m = O.OracleModel(dict(TINY, dtype=dtype), seed=0)
    m.generate(g["prompt"], 12)
    q, k, v, a = m.layer0()
    tol = 1e-2 if dtype == "bf16" else 1e-5  # one bf16 ulp at |x| <= 2
    np.testing.assert_allclose(q, g["layer0_q"], atol=tol)
    np.testing.assert_allclose(k, g["layer0_k"], atol=tol)
    np.testing.assert_allclose(v, g["layer0_v"], atol=tol)
    np.testing.assert_allclose(a, g["layer0_att"], atol=tol)


TINY_GEMMA = dict(vocab=512, dim=64, n_layers=2, n_heads=4, n_kv_heads=2, head_dim=32, ffn=128, max_seq=64,
                  eps=1e-6, rope_theta=10000.0, arch=1, ple_dim=16, final_softcap=30.0)


@pytest.mark.parametrize("dtype", ["fp32", "bf16"])
def test_gemma_oracle_matches_numpy_restatement(dtype):
    """The Gemma-style decoder of the C oracle against the independent numpy restatement
    (tests/golden/gen_golden.py, NpGemma): ids identical, logits and layer-0 stages close."""
    g = np.load(os.path.join(GOLD, f"tiny_gemma_{dtype}.npz"))
    m = O.OracleModel(dict(TINY_GEMMA, dtype=dtype), seed=0)
    ids, logits = m.generate(g["prompt"], 12, want_logits=True)
    np.testing.assert_array_equal(ids, g["ids"])
    np.testing.assert_allclose(logits, g["logits"], atol=2e-5, rtol=0)
    q, k, v, a = m.layer0()
    h, _ = m.layer0_mlp()
    tol = 1e-2 if dtype == "bf16" else 1e-5
    for got, name in ((q, "q"), (k, "k"), (v, "v"), (a, "att"), (h, "h")):
        np.testing.assert_allclose(got, g[f"layer0_{name}"], atol=tol, err_msg=name)
    # the LM head is the embedding (tied), and norm gains are drawn, not ones
    assert m.weight(-1, O.K_LM_HEAD, (4,)).tolist() == m.weight(-1, O.K_EMBED, (4,)).tolist()
    assert len(set(m.weight(0, O.K_ATTN_NORM, (64,)).tolist())) > 10


def test_gemma_prefill_equals_tokenwise():
    cfg = dict(TINY_GEMMA, dtype="bf16")
    m = O.OracleModel(cfg, seed=0)
    ids = O.gen_ids(5, 40, 512)
    la, _ = m.forward(ids, 0, all_logits=True)
    m2 = O.OracleModel(cfg, seed=0)
    for t in range(40):
        lt, _ = m2.forward(ids[t:t + 1], t)
        np.testing.assert_array_equal(lt, la[t])


def test_rope_table_matches_golden():
    g = np.load(os.path.join(GOLD, "tiny_fp32.npz"))
    cs, sn = O.rope_table(64, 16, 10000.0)
    np.testing.assert_array_equal(cs, g["rope_cos"])
    np.testing.assert_array_equal(sn, g["rope_sin"])


def test_gather_and_rmsnorm_stage_oracles():
    rng = np.random.default_rng(0)
    table = rng.standard_normal((100, 24)).astype(np.float32)
    ids = np.array([3, 99, 0, 3], np.uint32)
    np.testing.assert_array_equal(O.embed_gather(ids, table, 24), table[ids])
    x = rng.standard_normal((5, 24)).astype(np.float32)
    g = np.ones(24, np.float32)
    y = O.rmsnorm(x, g, 1e-5)
    want = x / np.sqrt((x.astype(np.float64) ** 2).mean(1, keepdims=True) + 1e-5)
    np.testing.assert_allclose(y, want, rtol=1e-6, atol=1e-6)


def test_oracle_rejects_bad_inputs():
    m = O.OracleModel(dict(TINY, dtype="fp32"), seed=0)
    with pytest.raises(ValueError):
        m.forward([600], 0)           # id >= vocab
    with pytest.raises(ValueError):
        m.forward([1, 2], 63)         # beyond max_seq


@pytest.mark.parametrize("dtype,n", [("bf16", 10), ("bf16", 150), ("fp32", 70)])
def test_prefill_equals_tokenwise(dtype, n):
    """A multi-token forward runs the prompt in blocks of 64 tokens, one layer at a time for the
    block; every logit and every K/V entry equals feeding the tokens one at a time."""
    cfg = dict(TINY, dtype=dtype, max_seq=160)
    m = O.OracleModel(cfg, seed=0)
    ids = O.gen_ids(5, n, 512)
    la, _ = m.forward(ids, 0, all_logits=True)
    m2 = O.OracleModel(cfg, seed=0)
    for t in range(n):
        lt, _ = m2.forward(ids[t:t + 1], t)
        np.testing.assert_array_equal(lt, la[t])
    for layer in range(cfg["n_layers"]):
        for t in range(0, n, 7):
            for a, b in zip(m.kv(layer, t), m2.kv(layer, t)):
                np.testing.assert_array_equal(a, b)
