"""Per-stage GPU parity: one-layer models of every workload shape, compared stage by stage
with the oracle (q, K/V cache, attention output, SwiGLU product, logits) on identical
weights and ids.  One layer keeps fp32 accumulation-order noise from cascading, so each
stored bf16 value must equal the oracle's or sit one bf16 ulp away (a rounding-boundary
flip), and the fraction of exact matches is high.  The SwiGLU product is checked on the
device's own attention output (a single upstream flip moves every residual element)."""
import numpy as np
import pytest

import infb200 as I
import oracle as O

pytestmark = pytest.mark.gpu


def ulp_bf16(x):
    x = np.maximum(np.abs(x), 1e-30)
    return np.exp2(np.floor(np.log2(x)) - 7)


def assert_bf16_close(got, want, name, min_exact=0.97, max_ulps=1.0, abs_frac=1e-5):
    """Each value within max_ulps bf16 ulps, plus an absolute allowance of abs_frac times the
    vector's scale: a dot product's fp32 error is absolute (it scales with the sum of |terms|),
    so a value that cancels to near zero can move several of its own tiny ulps."""
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    allow = max_ulps * ulp_bf16(np.maximum(np.abs(got), np.abs(want))) + abs_frac * float(np.abs(want).max())
    excess = np.abs(got - want) - allow
    exact = float(np.mean(got == want))
    worst = int(np.argmax(excess))
    assert float(excess.max()) <= 1e-12, f"{name}[{worst}]: {got[worst]} vs {want[worst]} (exact {exact:.4f})"
    assert exact >= min_exact, f"{name}: only {exact:.4f} exactly equal"


def _bf16_round(x):
    """fp32 -> nearest-even bf16, returned as fp32."""
    a = np.asarray(x, np.float32).view(np.uint32).astype(np.uint64)
    r = ((a + 0x7FFF + ((a >> 16) & 1)) >> 16) << 16
    return r.astype(np.uint32).view(np.float32)


def mlp_stage(orc, cfg, token, attn):
    """The first layer's SwiGLU product for `token`, computed from a given attention output with
    the oracle's weights and the oracle's rounding points (oracle/llama_ref.c: fp32 O-projection
    output from a double dot product, fp32 residual add, RMSNorm with the double sum of squares
    and fp32 scale, bf16 x-hat, fp32 gate/up from double dot products, silu(gate)*up in double
    stored as bf16).  Lets the MLP stage be checked on the device's own attention output: one
    rounding-boundary flip in the attention moves the whole residual through a W_o column."""
    d, F, H, hd = cfg.dim, cfg.ffn_dim, cfg.n_heads, cfg.head_dim

    def mv(kind, rows, cols, x):
        W = orc.weight(0, kind, (rows, cols))
        x64 = np.asarray(x, np.float64)
        y = np.empty(rows, np.float32)
        for r0 in range(0, rows, 2048):
            y[r0:r0 + 2048] = (O.bf16_to_f32(W[r0:r0 + 2048]).astype(np.float64) @ x64).astype(np.float32)
        return y

    emb = O.bf16_to_f32(orc.weight(-1, 0, (cfg.vocab_size, d))[token]).astype(np.float32)
    r1 = (emb + mv(11, d, H * hd, np.asarray(attn, np.float32))).astype(np.float32)
    ss = float(np.sum(r1.astype(np.float64) ** 2))
    inv = np.float32(1.0) / np.sqrt(np.float32(np.float32(ss) / np.float32(d) + np.float32(cfg.norm_eps)))
    g = O.bf16_to_f32(orc.weight(0, 16, (d,))).astype(np.float32)
    xh = _bf16_round((r1 * inv).astype(np.float32) * g)
    gate = mv(12, F, d, xh).astype(np.float64)
    up = mv(13, F, d, xh).astype(np.float64)
    return _bf16_round((gate / (1.0 + np.exp(-gate)) * up).astype(np.float32)).astype(np.float64)


def cosine(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b) + 1e-30))


def assert_f32_close(got, want, name, rtol=1e-4):
    scale = float(np.abs(want).max()) + 1e-12
    err = float(np.abs(np.asarray(got) - np.asarray(want)).max())
    assert err <= rtol * scale, f"{name}: max-abs {err} vs scale {scale}"


@pytest.mark.parametrize("preset", [1, 2, 3])
def test_decode_path_stages(cuda, preset):
    cfg = I.preset(preset, n_layers=1, max_seq=64)
    n = 12
    prompt = I.synth_ids(7, n, cfg.vocab_size)
    with I.Engine(cfg) as eng:
        for t in range(n):                          # every token through the decode kernels
            lg, am = eng.forward(prompt[t:t + 1], t)
        got = {k: eng.debug_read(k) for k in ("q", "attn", "h", "resid", "logits")}
        kv = [(eng.debug_read("k", 0, 0, t), eng.debug_read("v", 0, 0, t)) for t in range(n)]
    orc = O.OracleModel(I.oracle_dict(cfg), seed=0)
    o_lg, o_am = orc.forward(prompt, 0)
    q, _, _, att = orc.layer0()
    h, resid = orc.layer0_mlp()
    if cfg.dtype == I.BF16:
        assert_bf16_close(got["q"], q, "q")
        for t in range(n):
            k, v = orc.kv(0, t)
            assert_bf16_close(kv[t][0], k, f"k[{t}]")
            assert_bf16_close(kv[t][1], v, f"v[{t}]")
        assert_bf16_close(got["attn"], att, "attention", min_exact=0.95)
        # the MLP on its own input (the device's attention output), and end to end by cosine
        assert_bf16_close(got["h"], mlp_stage(orc, cfg, int(prompt[-1]), got["attn"]), "swiglu", min_exact=0.97)
        assert cosine(got["h"], h) >= 0.99999
        assert_f32_close(got["resid"], resid, "residual", rtol=2e-2)
        assert float(np.abs(got["logits"] - o_lg).max()) <= 2e-2
    else:
        assert_f32_close(got["q"], q, "q")
        assert_f32_close(got["attn"], att, "attention")
        assert_f32_close(got["h"], h, "swiglu")
        assert_f32_close(got["resid"], resid, "residual")
        assert_f32_close(got["logits"], o_lg, "logits")
    np.testing.assert_array_equal(lg, got["logits"])
    assert am == o_am or np.sort(o_lg)[-1] - np.sort(o_lg)[-2] < 2e-2


@pytest.mark.parametrize("preset,n,drift", [(2, 200, 0.0144), (3, 300, 0.0161)])
def test_tensor_core_prefill_stages(cuda, preset, n, drift):
    """One multi-token pass (tcgen05 GEMMs, prefill attention): every position's K and V in
    the paged cache, and the last token's logits within twice the measured drift between
    fp32 and double accumulation of the same one-layer model and prompt (`drift`, from
    oracle/llama_ref.c with orc_set_accum_f32; it grows with the prompt length)."""
    cfg = I.preset(preset, n_layers=1, max_seq=512)
    prompt = I.synth_ids(8, n, cfg.vocab_size)
    with I.Engine(cfg) as eng:
        lg, _ = eng.forward(prompt, 0)
        kv = [(eng.debug_read("k", 0, 0, t), eng.debug_read("v", 0, 0, t)) for t in range(n)]
    orc = O.OracleModel(I.oracle_dict(cfg), seed=0)
    o_lg, _ = orc.forward(prompt, 0)
    for t in range(n):
        k, v = orc.kv(0, t)
        assert_bf16_close(kv[t][0], k, f"k[{t}]")
        assert_bf16_close(kv[t][1], v, f"v[{t}]")
    assert float(np.abs(lg - o_lg).max()) <= 2 * drift


def test_rope_positions_far_into_the_cache(cuda):
    """Positions near max_seq use the far end of the RoPE table and the last KV pages."""
    cfg = I.preset(2, n_layers=1, max_seq=1024)
    start = 1000
    ids = I.synth_ids(9, 24, cfg.vocab_size)
    with I.Engine(cfg) as eng:
        eng.forward(I.synth_ids(10, start, cfg.vocab_size), 0)  # fill the cache with one multi-token pass
        eng.forward(ids, start)
        got = [eng.debug_read("k", 0, 0, start + t) for t in range(24)]
    orc = O.OracleModel(I.oracle_dict(cfg), seed=0)
    orc.forward(I.synth_ids(10, start, cfg.vocab_size), 0)
    orc.forward(ids, start)
    for t in range(24):
        assert_bf16_close(got[t], orc.kv(0, start + t)[0], f"k[{start + t}]")


# The same one-layer model, prompt and ids run by the oracle with fp32 instead of double
# accumulation (orc_set_accum_f32): its logits at positions 2048..2063 differ from the double run's
# by up to 0.0173 max-abs, the spread of two correct implementations after a 2048-token prompt.
DRIFT_HEADLINE_1L = 0.0173


def test_headline_decode_plan_stages(cuda):
    """The batch-1 decode step as the headline runs it: the Llama-3-8B shape at its default
    max_seq 3072 (192 pages per sequence, so the decode graph's attention is the 16-CTA cluster
    kernel with 12 pages per CTA), one layer, vocabulary 8192 to keep the oracle cheap.  A
    2048-token prompt goes through the tensor-core prefill, then 16 tokens through the decode
    graph at positions 2048..2063.  At every step:
    * the attention output is the correctly rounded value (within one bf16 ulp, measured 0.5) of
      attention computed in float64 from the step's q over the engine's own cache (every K/V row
      read back): the kernel, its split plan and the current row it patches in after the
      dependency wait are exact;
    * q, the new K/V row, the attention output, the SwiGLU product and the logits match the
      oracle, which ran the same ids from its own prefill.  The prompt's K/V rows came from the
      tensor-core prefill's fp32 sums, a rounding-boundary flip away from the oracle's double sums
      at a few percent of entries, so the attention output and what follows it carry an absolute
      allowance of 0.4% of the vector's largest value, and the logits twice the measured drift."""
    torch = cuda
    cfg = I.preset(3, n_layers=1, vocab_size=8192)
    assert cfg.max_seq == 3072
    n, steps = 2048, 16
    prompt = I.synth_ids(21, n, cfg.vocab_size)
    ids = I.synth_ids(22, steps, cfg.vocab_size)
    H, KV, hd = cfg.n_heads, cfg.n_kv_heads, cfg.head_dim
    got = []
    with I.Engine(cfg) as eng:
        eng.forward(prompt, 0, want_logits=False)
        for s in range(steps):
            lg, am = eng.forward(ids[s:s + 1], n + s)
            got.append({k: eng.debug_read(k) for k in ("q", "attn", "h")} | {"logits": lg, "am": am})
        K = np.stack([eng.debug_read("k", 0, 0, t) for t in range(n + steps)]).reshape(-1, KV, hd)
        V = np.stack([eng.debug_read("v", 0, 0, t) for t in range(n + steps)]).reshape(-1, KV, hd)
    Kt = torch.from_numpy(K).double().permute(1, 0, 2)  # [KV, pos, hd], the bf16 values widened
    Vt = torch.from_numpy(V).double().permute(1, 0, 2)
    for s in range(steps):
        p = n + s
        q = torch.from_numpy(got[s]["q"]).double().view(KV, H // KV, hd)
        sc = torch.einsum("kgd,knd->kgn", q, Kt[:, :p + 1]) / hd ** 0.5
        ref = torch.einsum("kgn,knd->kgd", torch.softmax(sc, -1), Vt[:, :p + 1]).reshape(-1).numpy()
        assert_bf16_close(got[s]["attn"], ref, f"attention at {p} over the engine's cache", min_exact=0.0,
                          abs_frac=1e-6)
    orc = O.OracleModel(I.oracle_dict(cfg), seed=0)
    orc.forward(prompt, 0)
    for s in range(steps):
        p = n + s
        o_lg, o_am = orc.forward(ids[s:s + 1], p)
        q, k, v, att = orc.layer0()
        h, _ = orc.layer0_mlp()
        g = got[s]
        assert_bf16_close(g["q"], q, f"q at {p}")
        assert_bf16_close(K[p].reshape(-1), k, f"k at {p}")
        assert_bf16_close(V[p].reshape(-1), v, f"v at {p}")
        assert_bf16_close(g["attn"], att, f"attention at {p}", min_exact=0.85, abs_frac=4e-3)
        # the SwiGLU product sits behind the attention output, the O projection and a norm, so the
        # prompt's cache difference flips many of its bf16 roundings: closeness only
        assert_bf16_close(g["h"], h, f"swiglu at {p}", min_exact=0.0, abs_frac=4e-3)
        assert float(np.abs(g["logits"] - o_lg).max()) <= 2 * DRIFT_HEADLINE_1L, f"logits at {p}"
        assert g["am"] == o_am or np.sort(o_lg)[-1] - np.sort(o_lg)[-2] < 2 * DRIFT_HEADLINE_1L
