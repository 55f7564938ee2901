"""ctypes binding of the CPU oracle (oracle/llama_ref.c) -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU legs import this module; the
product library never does.  The oracle restates the decoder the B200 library runs
(see llama_ref.h for the reference anchors: src/cuda/kernels/input_embeddings.cu:23-34,
src/cuda/kernels/rmsnorm.cu:11-59, src/model.cuh:44-50).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libllama_ref.so")
REF_LIB_PATH = os.path.join(HERE, "_ref", "libref_kernels.so")

# tensor kinds (orc_tensor_stream)
K_EMBED, K_LM_HEAD, K_FINAL_NORM = 0, 1, 2
K_EMBED_PLE, K_PLE_MODEL_PROJ, K_PLE_PROJ_NORM = 3, 4, 5  # Gemma-style models
K_WQ, K_WK, K_WV, K_WO, K_WGATE, K_WUP, K_WDOWN, K_ATTN_NORM, K_FFN_NORM = range(8, 17)
K_Q_NORM, K_K_NORM, K_POST_ATTN_NORM, K_POST_FFN_NORM, K_PLE_GATE, K_PLE_PROJ, K_PLE_POST_NORM = range(17, 24)

STREAM_PROMPT = 0x1000000
STREAM_CTX_LEN = 0x2000000


class OrcConfig(C.Structure):
    _fields_ = [
        ("vocab", C.c_uint32), ("dim", C.c_uint32), ("n_layers", C.c_uint32), ("n_heads", C.c_uint32),
        ("n_kv_heads", C.c_uint32), ("head_dim", C.c_uint32), ("ffn", C.c_uint32), ("max_seq", C.c_uint32),
        ("n_slots", C.c_uint32), ("bf16", C.c_uint32), ("eps", C.c_float), ("rope_theta", C.c_float),
        ("init_std", C.c_float), ("arch", C.c_uint32), ("ple_dim", C.c_uint32), ("final_softcap", C.c_float),
    ]


_lib = None


def build() -> None:
    subprocess.run(["make", "-s", "-C", HERE, "libllama_ref.so"], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = C.CDLL(LIB_PATH)
        u32, u64, f32, vp = C.c_uint32, C.c_uint64, C.c_float, C.c_void_p
        L.orc_splitmix64.restype = u64
        L.orc_splitmix64.argtypes = [u64]
        L.orc_philox4x32_10.argtypes = [vp, vp, vp]
        L.orc_init_scale.restype = f32
        L.orc_init_scale.argtypes = [f32]
        L.orc_normal_value.restype = f32
        L.orc_normal_value.argtypes = [u64, u64, u64, f32]
        L.orc_f32_to_bf16.restype = C.c_uint16
        L.orc_f32_to_bf16.argtypes = [f32]
        L.orc_fill_tensor.argtypes = [u64, u64, u64, f32, C.c_int, vp]
        L.orc_uniform_u32.restype = u32
        L.orc_uniform_u32.argtypes = [u64, u64, u64, u32, u32]
        L.orc_gen_ids.argtypes = [u64, u64, u64, u32, vp]
        L.orc_tensor_stream.restype = u64
        L.orc_tensor_stream.argtypes = [C.c_int32, u32]
        L.orc_rope_table.argtypes = [u32, u32, f32, vp, vp]
        L.orc_embed_gather.argtypes = [vp, u64, u32, vp, C.c_int, vp]
        L.orc_rmsnorm.argtypes = [vp, u64, u32, vp, C.c_int, f32, vp]
        L.orc_matvec.argtypes = [vp, C.c_int, u64, u64, vp, vp]
        L.orc_model_create.restype = vp
        L.orc_model_create.argtypes = [C.POINTER(OrcConfig), u64, C.c_int]
        L.orc_model_destroy.argtypes = [vp]
        L.orc_model_weight.restype = vp
        L.orc_model_weight.argtypes = [vp, C.c_int32, u32]
        L.orc_forward.restype = C.c_int
        L.orc_forward.argtypes = [vp, u32, vp, u32, u32, vp, vp, vp]
        L.orc_generate.restype = C.c_int
        L.orc_generate.argtypes = [vp, u32, vp, u32, u32, vp, vp]
        L.orc_fill_kv_synthetic.restype = C.c_int
        L.orc_fill_kv_synthetic.argtypes = [vp, u32, u32, u64]
        L.orc_last_layer0.restype = C.c_int
        L.orc_last_layer0.argtypes = [vp, vp, vp, vp, vp]
        L.orc_last_layer0_mlp.restype = C.c_int
        L.orc_last_layer0_mlp.argtypes = [vp, vp, vp]
        L.orc_kv_read.restype = C.c_int
        L.orc_kv_read.argtypes = [vp, u32, u32, u32, vp, vp]
        L.orc_set_accum_f32.argtypes = [C.c_int]
        L.orc_argmax.restype = u32
        L.orc_argmax.argtypes = [vp, u64]
        L.orc_sample_weights.argtypes = [vp, u64, f32, vp]
        L.orc_sample_weights.restype = None
        L.orc_sample_select.argtypes = [vp, u64, f32, u32, u64, u64]
        L.orc_sample_select.restype = u32
        _lib = L
    return _lib


def _p(a: np.ndarray):
    return a.ctypes.data_as(C.c_void_p)


def philox(ctr, key):
    c = np.asarray(ctr, dtype=np.uint32)
    k = np.asarray(key, dtype=np.uint32)
    out = np.zeros(4, dtype=np.uint32)
    lib().orc_philox4x32_10(_p(c), _p(k), _p(out))
    return out


def fill_tensor(seed: int, stream: int, n: int, std: float, bf16: bool) -> np.ndarray:
    out = np.empty(n, dtype=np.uint16 if bf16 else np.float32)
    lib().orc_fill_tensor(seed, stream, n, std, int(bf16), _p(out))
    return out


def gen_ids(seed: int, n: int, vocab: int, stream: int = STREAM_PROMPT) -> np.ndarray:
    out = np.empty(n, dtype=np.uint32)
    lib().orc_gen_ids(seed, stream, n, vocab, _p(out))
    return out


def uniform_u32(seed: int, stream: int, idx: int, lo: int, hi: int) -> int:
    return int(lib().orc_uniform_u32(seed, stream, idx, lo, hi))


def sample_weights(logits: np.ndarray, inv_temp: float) -> np.ndarray:
    x = np.ascontiguousarray(logits, dtype=np.float32)
    q = np.empty(x.size, dtype=np.uint32)
    lib().orc_sample_weights(_p(x), x.size, inv_temp, _p(q))
    return q


def sample_select(q: np.ndarray, top_p: float, top_k: int, seed: int, counter: int) -> int:
    q = np.ascontiguousarray(q, dtype=np.uint32)
    return int(lib().orc_sample_select(_p(q), q.size, top_p, top_k, seed, counter))


def tensor_stream(layer: int, kind: int) -> int:
    return int(lib().orc_tensor_stream(layer, kind))


def rope_table(max_seq: int, head_dim: int, theta: float):
    cs = np.empty((max_seq, head_dim // 2), dtype=np.float32)
    sn = np.empty_like(cs)
    lib().orc_rope_table(max_seq, head_dim, theta, _p(cs), _p(sn))
    return cs, sn


def bf16_to_f32(h: np.ndarray) -> np.ndarray:
    return (h.astype(np.uint32) << 16).view(np.float32)


def embed_gather(ids: np.ndarray, table: np.ndarray, dim: int) -> np.ndarray:
    ids = np.ascontiguousarray(ids, dtype=np.uint32)
    out = np.empty((ids.size, dim), dtype=np.float32)
    lib().orc_embed_gather(_p(ids), ids.size, dim, _p(table), int(table.dtype == np.uint16), _p(out))
    return out


def rmsnorm(x: np.ndarray, g: np.ndarray, eps: float) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, dim = x.shape
    y = np.empty_like(x)
    lib().orc_rmsnorm(_p(x), rows, dim, _p(g), int(g.dtype == np.uint16), eps, _p(y))
    return y


def matvec(W: np.ndarray, x: np.ndarray) -> np.ndarray:
    rows, cols = W.shape
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty(rows, dtype=np.float32)
    lib().orc_matvec(_p(np.ascontiguousarray(W)), int(W.dtype == np.uint16), rows, cols, _p(x), _p(y))
    return y


class OracleModel:
    """Synthetic-weight Llama decoder on the host cores."""

    def __init__(self, cfg: dict, seed: int = 0, n_slots: int = 1, n_threads: int = 0):
        self.cfg = dict(cfg)
        c = OrcConfig(
            vocab=cfg["vocab"], dim=cfg["dim"], n_layers=cfg["n_layers"], n_heads=cfg["n_heads"],
            n_kv_heads=cfg["n_kv_heads"], head_dim=cfg["head_dim"], ffn=cfg["ffn"], max_seq=cfg["max_seq"],
            n_slots=n_slots, bf16=int(cfg["dtype"] == "bf16"), eps=cfg["eps"], rope_theta=cfg["rope_theta"],
            init_std=cfg.get("init_std", 0.02), arch=int(cfg.get("arch", 0)), ple_dim=int(cfg.get("ple_dim", 0)),
            final_softcap=float(cfg.get("final_softcap", 0.0)),
        )
        self.c = c
        self.h = lib().orc_model_create(C.byref(c), seed, n_threads)
        if not self.h:
            raise MemoryError("orc_model_create failed")

    def close(self):
        if self.h:
            lib().orc_model_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def weight(self, layer: int, kind: int, shape) -> np.ndarray:
        ptr = lib().orc_model_weight(self.h, layer, kind)
        n = int(np.prod(shape))
        ct = C.c_uint16 if self.c.bf16 else C.c_float
        arr = np.ctypeslib.as_array(C.cast(ptr, C.POINTER(ct)), shape=(n,))
        return arr.reshape(shape).copy()

    def forward(self, ids, start_pos: int, slot: int = 0, all_logits: bool = False):
        ids = np.ascontiguousarray(ids, dtype=np.uint32)
        V = self.c.vocab
        la = np.empty((ids.size, V), dtype=np.float32) if all_logits else None
        ll = np.empty(V, dtype=np.float32)
        am = C.c_uint32(0)
        rc = lib().orc_forward(self.h, slot, _p(ids), ids.size, start_pos,
                               _p(la) if la is not None else None, _p(ll), C.byref(am))
        if rc:
            raise ValueError(f"orc_forward failed: {rc}")
        return (la if all_logits else ll), int(am.value)

    def generate(self, prompt, n_new: int, slot: int = 0, want_logits: bool = False):
        prompt = np.ascontiguousarray(prompt, dtype=np.uint32)
        out = np.empty(n_new, dtype=np.uint32)
        lg = np.empty((n_new, self.c.vocab), dtype=np.float32) if want_logits else None
        rc = lib().orc_generate(self.h, slot, _p(prompt), prompt.size, n_new, _p(out),
                                _p(lg) if lg is not None else None)
        if rc:
            raise ValueError(f"orc_generate failed: {rc}")
        return (out, lg) if want_logits else out

    def fill_kv_synthetic(self, ctx: int, seed: int = 7, slot: int = 0):
        rc = lib().orc_fill_kv_synthetic(self.h, slot, ctx, seed)
        if rc:
            raise ValueError("orc_fill_kv_synthetic failed")

    def layer0_mlp(self):
        h = np.empty(self.c.ffn, np.float32)
        r = np.empty(self.c.dim, np.float32)
        lib().orc_last_layer0_mlp(self.h, _p(h), _p(r))
        return h, r

    def kv(self, layer: int, pos: int, slot: int = 0):
        n = self.c.n_kv_heads * self.c.head_dim
        k = np.empty(n, np.float32)
        v = np.empty(n, np.float32)
        if lib().orc_kv_read(self.h, slot, layer, pos, _p(k), _p(v)):
            raise ValueError("orc_kv_read")
        return k, v

    def layer0(self):
        c = self.c
        q = np.empty(c.n_heads * c.head_dim, np.float32)
        k = np.empty(c.n_kv_heads * c.head_dim, np.float32)
        v = np.empty_like(k)
        a = np.empty_like(q)
        lib().orc_last_layer0(self.h, _p(q), _p(k), _p(v), _p(a))
        return q, k, v, a
