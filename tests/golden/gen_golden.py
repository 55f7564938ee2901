"""Generate the golden fixtures under tests/golden/ from an independent numpy restatement.

The reference (gosutek/inference-project) ships no tests, fixtures or golden vectors and
has no forward pass beyond the embedding gather (src/cuda/kernels/input_embeddings.cu:23-34)
and a single RMSNorm (src/cuda/kernels/rmsnorm.cu:11-59).  These fixtures therefore come
from a second, independent restatement of the decoder written here in numpy (it shares no
code with the C oracle in oracle/llama_ref.c).  The C oracle is tested against them, so two
independent restatements must agree before either is trusted.

Run:  python tests/golden/gen_golden.py      (writes tests/golden/*.npz)
"""
from __future__ import annotations

import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
M64 = (1 << 64) - 1


# ---------------------------------------------------------------- synthetic data
def splitmix64(x: int) -> int:
    z = (x + 0x9E3779B97F4A7C15) & M64
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & M64
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & M64
    return z ^ (z >> 31)


def stream_key(seed: int, stream: int):
    k = splitmix64(splitmix64(seed) ^ stream)
    return k & 0xFFFFFFFF, k >> 32


def philox_vec(idx: np.ndarray, key):
    """Philox4x32-10 over counters (idx_lo, idx_hi, 0, 0), vectorised."""
    idx = idx.astype(np.uint64)
    c0 = (idx & np.uint64(0xFFFFFFFF)).astype(np.uint64)
    c1 = (idx >> np.uint64(32)).astype(np.uint64)
    c2 = np.zeros_like(c0)
    c3 = np.zeros_like(c0)
    k0, k1 = np.uint64(key[0]), np.uint64(key[1])
    mask = np.uint64(0xFFFFFFFF)
    for _ in range(10):
        p0 = np.uint64(0xD2511F53) * c0
        p1 = np.uint64(0xCD9E8D57) * c2
        hi0, lo0 = p0 >> np.uint64(32), p0 & mask
        hi1, lo1 = p1 >> np.uint64(32), p1 & mask
        c0, c1, c2, c3 = hi1 ^ c1 ^ k0, lo1, hi0 ^ c3 ^ k1, lo0
        k0 = (k0 + np.uint64(0x9E3779B9)) & mask
        k1 = (k1 + np.uint64(0xBB67AE85)) & mask
    return [c.astype(np.uint32) for c in (c0, c1, c2, c3)]


def init_scale(std: float) -> np.float32:
    return np.float32(float(std) * 1.7320508075688772 / 4194304.0)


def normal_tensor(seed: int, stream: int, n: int, std: float) -> np.ndarray:
    w = philox_vec(np.arange(n, dtype=np.uint64), stream_key(seed, stream))
    s = sum((x >> np.uint32(10)).astype(np.int64) for x in w) - (1 << 23)
    return s.astype(np.float32) * init_scale(std)


def bf16_round(x: np.ndarray) -> np.ndarray:
    u = np.asarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = (u + np.uint64(0x7FFF) + ((u >> np.uint64(16)) & np.uint64(1))) >> np.uint64(16)
    return (u.astype(np.uint32) << np.uint32(16)).view(np.float32)


def tensor_stream(layer: int, kind: int) -> int:
    return ((layer + 1) << 8) | kind


def uniform_ids(seed: int, stream: int, n: int, lo: int, hi: int) -> np.ndarray:
    w = philox_vec(np.arange(n, dtype=np.uint64), stream_key(seed, stream))
    rng = np.uint64(hi - lo + 1)
    return (np.uint64(lo) + ((w[0].astype(np.uint64) * rng) >> np.uint64(32))).astype(np.uint32)


# ---------------------------------------------------------------- model
class NpLlama:
    def __init__(self, cfg: dict, seed: int):
        self.cfg = cfg
        bf = cfg["dtype"] == "bf16"
        self.R = bf16_round if bf else (lambda a: np.asarray(a, dtype=np.float32))
        V, d, L = cfg["vocab"], cfg["dim"], cfg["n_layers"]
        H, KV, hd, F = cfg["n_heads"], cfg["n_kv_heads"], cfg["head_dim"], cfg["ffn"]
        std = cfg.get("init_std", 0.02)

        def gen(layer, kind, shape):
            t = normal_tensor(seed, tensor_stream(layer, kind), int(np.prod(shape)), std)
            return self.R(t).reshape(shape)

        self.embed = gen(-1, 0, (V, d))
        self.lm_head = gen(-1, 1, (V, d))
        self.layers = []
        for l in range(L):
            self.layers.append(dict(
                wq=gen(l, 8, (H * hd, d)), wk=gen(l, 9, (KV * hd, d)), wv=gen(l, 10, (KV * hd, d)),
                wo=gen(l, 11, (d, H * hd)), wg=gen(l, 12, (F, d)), wu=gen(l, 13, (F, d)), wd=gen(l, 14, (d, F))))
        half = hd // 2
        p = np.arange(cfg["max_seq"], dtype=np.float64)[:, None]
        inv = np.power(float(np.float32(cfg["rope_theta"])), -2.0 * np.arange(half, dtype=np.float64) / hd)
        self.cos = np.cos(p * inv).astype(np.float32)
        self.sin = np.sin(p * inv).astype(np.float32)
        self.K = np.zeros((L, cfg["max_seq"], KV, hd), np.float32)
        self.V = np.zeros_like(self.K)
        self.dbg = None

    def rmsnorm(self, x):
        ss = np.float32(np.dot(x.astype(np.float64), x.astype(np.float64)))
        inv = np.float32(1.0) / np.sqrt(ss / np.float32(x.size) + np.float32(self.cfg["eps"]), dtype=np.float32)
        return self.R(x * inv)

    def rope(self, x, pos):
        hd = self.cfg["head_dim"]
        half = hd // 2
        x = x.reshape(-1, hd).copy()
        a, b = x[:, :half].copy(), x[:, half:].copy()
        c, s = self.cos[pos], self.sin[pos]
        x[:, :half] = a * c - b * s
        x[:, half:] = b * c + a * s
        return x.reshape(-1)

    def token(self, tid, pos, want_logits):
        cfg = self.cfg
        H, KV, hd = cfg["n_heads"], cfg["n_kv_heads"], cfg["head_dim"]
        grp = H // KV
        r = self.embed[tid].astype(np.float32).copy()
        for l, W in enumerate(self.layers):
            xh = self.rmsnorm(r)
            q = self.R(self.rope(W["wq"] @ xh, pos))
            k = self.R(self.rope(W["wk"] @ xh, pos))
            v = self.R(W["wv"] @ xh)
            self.K[l, pos] = k.reshape(KV, hd)
            self.V[l, pos] = v.reshape(KV, hd)
            att = np.zeros(H * hd, np.float32)
            scale = np.float32(1.0 / np.sqrt(hd))
            for h in range(H):
                g = h // grp
                ks = self.K[l, : pos + 1, g]
                vs = self.V[l, : pos + 1, g]
                s = (ks @ q[h * hd:(h + 1) * hd]) * scale
                p = np.exp(s - s.max())
                att[h * hd:(h + 1) * hd] = (p @ vs) / p.sum()
            att = self.R(att)
            if l == 0:
                self.dbg = (q.copy(), k.copy(), v.copy(), att.copy())
            r = r + W["wo"] @ att
            xh = self.rmsnorm(r)
            gt = W["wg"] @ xh
            up = W["wu"] @ xh
            h_ = self.R((gt / (np.float32(1) + np.exp(-gt))) * up)
            r = r + W["wd"] @ h_
        if not want_logits:
            return None
        return (self.lm_head @ self.rmsnorm(r)).astype(np.float32)

    def generate(self, prompt, n_new):
        for t, tid in enumerate(prompt):
            lg = self.token(int(tid), t, t == len(prompt) - 1)
        ids, logits = [], []
        for s in range(n_new):
            nxt = int(np.argmax(lg))
            ids.append(nxt)
            logits.append(lg)
            if s + 1 < n_new:
                lg = self.token(nxt, len(prompt) + s, True)
        return np.array(ids, np.uint32), np.stack(logits)


def gelu_tanh64(x):
    x = np.asarray(x, np.float64)
    return 0.5 * x * (1.0 + np.tanh(0.7978845608028654 * (x + 0.044715 * x ** 3)))


class NpGemma:
    """The Gemma-style decoder (arch 1 of the oracle) restated in numpy: embedding times
    bf16(sqrt(dim)), every RMSNorm scaled by (1 + w), per-head RMSNorm of q and k before RoPE,
    RMSNorm of the attention and MLP outputs before their residual adds, gelu_tanh(gate) * up,
    the per-layer-embedding block after the MLP, the embedding as LM head, final soft-cap.
    Projections accumulate in float64 and round to float32."""

    def __init__(self, cfg: dict, seed: int):
        self.cfg = cfg
        bf = cfg["dtype"] == "bf16"
        self.R = bf16_round if bf else (lambda a: np.asarray(a, dtype=np.float32))
        V, d, L = cfg["vocab"], cfg["dim"], cfg["n_layers"]
        H, KV, hd, F, P = cfg["n_heads"], cfg["n_kv_heads"], cfg["head_dim"], cfg["ffn"], cfg["ple_dim"]
        std = cfg.get("init_std", 0.02)

        def gen(layer, kind, shape):
            t = normal_tensor(seed, tensor_stream(layer, kind), int(np.prod(shape)), std)
            return self.R(t).reshape(shape)

        self.embed = gen(-1, 0, (V, d))
        self.final_norm = gen(-1, 2, (d,))
        if P:
            self.embed_ple = gen(-1, 3, (V, L * P))
            self.ple_model_proj = gen(-1, 4, (L * P, d))
            self.ple_proj_norm = gen(-1, 5, (P,))
        self.layers = []
        for l in range(L):
            W = dict(wq=gen(l, 8, (H * hd, d)), wk=gen(l, 9, (KV * hd, d)), wv=gen(l, 10, (KV * hd, d)),
                     wo=gen(l, 11, (d, H * hd)), wg=gen(l, 12, (F, d)), wu=gen(l, 13, (F, d)), wd=gen(l, 14, (d, F)),
                     attn_norm=gen(l, 15, (d,)), ffn_norm=gen(l, 16, (d,)), q_norm=gen(l, 17, (hd,)),
                     k_norm=gen(l, 18, (hd,)), post_attn=gen(l, 19, (d,)), post_ffn=gen(l, 20, (d,)))
            if P:
                W.update(ple_gate=gen(l, 21, (P, d)), ple_proj=gen(l, 22, (d, P)), ple_post=gen(l, 23, (d,)))
            self.layers.append(W)
        half = hd // 2
        p = np.arange(cfg["max_seq"], dtype=np.float64)[:, None]
        inv = np.power(float(np.float32(cfg["rope_theta"])), -2.0 * np.arange(half, dtype=np.float64) / hd)
        self.cos = np.cos(p * inv).astype(np.float32)
        self.sin = np.sin(p * inv).astype(np.float32)
        self.K = np.zeros((L, cfg["max_seq"], KV, hd), np.float32)
        self.V = np.zeros_like(self.K)
        self.dbg = None

    @staticmethod
    def mv(W, x):
        return (W.astype(np.float64) @ np.asarray(x, np.float64)).astype(np.float32)

    def rms1p(self, x, w):
        x = np.asarray(x, np.float32)
        ss = np.float32(np.dot(x.astype(np.float64), x.astype(np.float64)))
        inv = np.float32(1.0) / np.sqrt(ss / np.float32(x.size) + np.float32(self.cfg["eps"]), dtype=np.float32)
        return (x * inv) * (np.float32(1.0) + w.astype(np.float32))

    def rope(self, x, pos):
        hd = self.cfg["head_dim"]
        half = hd // 2
        x = x.reshape(-1, hd).copy()
        a, b = x[:, :half].copy(), x[:, half:].copy()
        c, s = self.cos[pos], self.sin[pos]
        x[:, :half] = a * c - b * s
        x[:, half:] = b * c + a * s
        return x.reshape(-1)

    def token(self, tid, pos, want_logits):
        cfg = self.cfg
        d, L = cfg["dim"], cfg["n_layers"]
        H, KV, hd, P = cfg["n_heads"], cfg["n_kv_heads"], cfg["head_dim"], cfg["ple_dim"]
        R = self.R
        c32 = lambda v: bf16_round(np.float32(v))  # a constant in the model dtype
        grp = H // KV
        r = self.embed[tid].astype(np.float32) * c32(np.sqrt(d))
        if P:
            pm = (self.mv(self.ple_model_proj, R(r)) * c32(1.0 / np.sqrt(d))).reshape(L, P)
            a = self.embed_ple[tid].reshape(L, P) * c32(np.sqrt(P))
            ple = np.stack([R((a[l] + self.rms1p(pm[l], self.ple_proj_norm)) * c32(1.0 / np.sqrt(2.0)))
                            for l in range(L)])
        for l, W in enumerate(self.layers):
            xh = R(self.rms1p(r, W["attn_norm"]))
            q = self.mv(W["wq"], xh).reshape(H, hd)
            k = self.mv(W["wk"], xh).reshape(KV, hd)
            v = R(self.mv(W["wv"], xh))
            q = R(self.rope(np.concatenate([self.rms1p(q[h], W["q_norm"]) for h in range(H)]), pos))
            k = R(self.rope(np.concatenate([self.rms1p(k[h], W["k_norm"]) for h in range(KV)]), pos))
            self.K[l, pos] = k.reshape(KV, hd)
            self.V[l, pos] = v.reshape(KV, hd)
            att = np.zeros(H * hd, np.float32)
            scale = np.float32(1.0 / np.sqrt(hd))
            for h in range(H):
                g = h // grp
                s = (self.K[l, : pos + 1, g].astype(np.float64) @ q[h * hd:(h + 1) * hd].astype(np.float64)).astype(
                    np.float32) * scale
                e = np.exp(s.astype(np.float64) - float(s.max()))
                att[h * hd:(h + 1) * hd] = (e @ self.V[l, : pos + 1, g].astype(np.float64)) / e.sum()
            att = R(att)
            r = r + self.rms1p(self.mv(W["wo"], att), W["post_attn"])
            xh = R(self.rms1p(r, W["ffn_norm"]))
            h_ = R((gelu_tanh64(self.mv(W["wg"], xh)) * self.mv(W["wu"], xh).astype(np.float64)).astype(np.float32))
            if l == 0:
                self.dbg = (q.copy(), k.copy(), v.copy(), att.copy(), h_.copy())
            r = r + self.rms1p(self.mv(W["wd"], h_), W["post_ffn"])
            if P:
                z = self.mv(W["ple_gate"], R(r))
                y = R((gelu_tanh64(z) * ple[l].astype(np.float64)).astype(np.float32))
                r = r + self.rms1p(self.mv(W["ple_proj"], y), W["ple_post"])
        if not want_logits:
            return None
        lg = self.mv(self.embed, R(self.rms1p(r, self.final_norm)))
        cap = cfg.get("final_softcap", 0.0)
        if cap > 0:
            lg = (cap * np.tanh(lg.astype(np.float64) / cap)).astype(np.float32)
        return lg

    generate = NpLlama.generate


TINY = dict(vocab=512, dim=64, n_layers=2, n_heads=4, n_kv_heads=2, head_dim=16, ffn=160, max_seq=64,
            eps=1e-5, rope_theta=10000.0)
TINY_GEMMA = dict(vocab=512, dim=64, n_layers=2, n_heads=4, n_kv_heads=2, head_dim=32, ffn=128, max_seq=64,
                  eps=1e-6, rope_theta=10000.0, arch=1, ple_dim=16, final_softcap=30.0)


def main():
    for dtype in ("fp32", "bf16"):
        cfg = dict(TINY, dtype=dtype)
        m = NpLlama(cfg, seed=0)
        prompt = uniform_ids(1, 0x1000000, 8, 0, cfg["vocab"] - 1)
        ids, logits = m.generate(prompt, 12)
        q, k, v, att = m.dbg
        np.savez_compressed(
            os.path.join(HERE, f"tiny_{dtype}.npz"),
            prompt=prompt, ids=ids, logits=logits, layer0_q=q, layer0_k=k, layer0_v=v, layer0_att=att,
            embed_head=m.embed[:4].copy(), wq0_head=m.layers[0]["wq"][:2].copy(),
            wd1_tail=m.layers[1]["wd"][-2:].copy(), lm_head_sum=np.float64(m.lm_head.astype(np.float64).sum()),
            rope_cos=m.cos, rope_sin=m.sin)
        print(dtype, "ids", ids)
    for dtype in ("fp32", "bf16"):
        cfg = dict(TINY_GEMMA, dtype=dtype)
        m = NpGemma(cfg, seed=0)
        prompt = uniform_ids(1, 0x1000000, 8, 0, cfg["vocab"] - 1)
        ids, logits = m.generate(prompt, 12)
        q, k, v, att, h = m.dbg
        np.savez_compressed(os.path.join(HERE, f"tiny_gemma_{dtype}.npz"), prompt=prompt, ids=ids, logits=logits,
                            layer0_q=q, layer0_k=k, layer0_v=v, layer0_att=att, layer0_h=h)
        print("gemma", dtype, "ids", ids)
    # synthetic-stream vectors: raw Philox words, ids and context lengths of the workloads
    words = philox_vec(np.arange(4, dtype=np.uint64), stream_key(0, tensor_stream(0, 8)))
    np.savez_compressed(
        os.path.join(HERE, "streams.npz"),
        philox_words=np.stack(words, axis=1),
        prompt_cfg1=uniform_ids(1, 0x1000000, 16, 0, 31999),
        prompt_cfg3_head=uniform_ids(1, 0x1000000, 64, 0, 128255),
        ctx_lens_cfg4=uniform_ids(2, 0x2000000, 64, 512, 4096),
        normal_head=normal_tensor(0, tensor_stream(-1, 0), 64, 0.02),
    )


if __name__ == "__main__":
    main()
