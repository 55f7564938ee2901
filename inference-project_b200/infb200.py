"""ctypes binding of libinf.so (include/inf.h) -- the host-side mirror of the reference's
entry points for Python callers (tests, bench.py).

It mirrors gosutek/inference-project's model-load / forward / generate surface
(src/main.cu:200 model_build, src/main.cu:354 model_destroy, the embed -> RMSNorm forward of
src/main.cu:396-412) on top of the C ABI.  There is no fallback: if libinf.so is missing or
fails to load, every call raises.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libinf.so")

u8, u16, u32, u64, i32, f32, f64 = C.c_uint8, C.c_uint16, C.c_uint32, C.c_uint64, C.c_int32, C.c_float, C.c_double
vp = C.c_void_p

ERRORS = {
    0: "Success", 1: "ErrorMemoryAllocation", 2: "ErrorArenaOutOfMemory", 3: "ErrorAlreadyInitialized",
    4: "ErrorInvalidValue", 5: "ErrorInvalidHostPtr", 6: "ErrorInvalidDevPtr", 7: "ErrorGeneric", 8: "ErrorCuda",
    9: "ErrorBadConfig", 10: "ErrorTokenOutOfRange", 11: "ErrorKvOutOfRange", 12: "ErrorNccl", 13: "ErrorTimeout",
    14: "ErrorIo", 15: "ErrorUnsupported",
}
F32, BF16 = 0, 1
ARCH_LLAMA, ARCH_GEMMA = 0, 1  # InfArch
PREFILL_ATTN_AUTO, PREFILL_ATTN_SIMT = 0, 1  # InfPrefillAttention
KERNEL_KINDS = ["embed", "qkv", "attn", "o_proj", "gate_up", "down", "lm_head"]
# InfWeightKind: the weights in their device layout
W_EMBED, W_LM_HEAD, W_FINAL_NORM = 0, 1, 2
W_QKV, W_O, W_GATE_UP, W_DOWN, W_ATTN_NORM, W_FFN_NORM = 8, 11, 12, 14, 15, 16


class InfError(RuntimeError):
    def __init__(self, code: int, where: str, detail: str):
        self.code = code
        self.name = ERRORS.get(code, str(code))
        super().__init__(f"{where}: {self.name} ({detail})")


class InfConfig(C.Structure):
    _fields_ = [
        ("vocab_size", u32), ("dim", u32), ("n_layers", u32), ("n_heads", u32), ("n_kv_heads", u32),
        ("head_dim", u32), ("ffn_dim", u32), ("max_seq", u32), ("max_batch", u32), ("kv_block", u32),
        ("kv_pages", u32), ("prefill_chunk", u32), ("dtype", u32), ("norm_eps", f32), ("rope_theta", f32),
        ("init_std", f32), ("tp_rank", u32), ("tp_size", u32), ("prefill_attention", u32), ("arch", u32),
        ("ple_dim", u32), ("final_softcap", f32),
    ]

    def as_dict(self) -> dict:
        d = {k: getattr(self, k) for k, _ in self._fields_}
        return d


class InfSampling(C.Structure):
    _fields_ = [("temperature", f32), ("top_p", f32), ("top_k", u32), ("reserved", u32), ("seed", u64)]


class HostArena(C.Structure):
    _fields_ = [("reserve_size", u64), ("commit_size", u64), ("commit_pos", u64), ("pos", u64)]


class DevArena(C.Structure):
    _fields_ = [("_d_ptr", vp), ("size", u64), ("pos", u64)]


class ExecCtx(C.Structure):
    _fields_ = [("host_arena", HostArena), ("dev_arena", DevArena)]


class Model(C.Structure):
    _fields_ = [("config", InfConfig), ("data", vp), ("model_bsize", u64), ("engine", vp)]


class InfStats(C.Structure):
    _fields_ = [("prefill_ms", f64), ("decode_ms", f64), ("n_prompt", u32), ("n_new", u32),
                ("kernel_launches", u64)]


EXPORTS = [
    "exec_ctx_create", "exec_ctx_destroy", "arena_host_create", "arena_host_destroy", "arena_host_push",
    "arena_host_pop", "arena_host_pop_at", "mem_arena_host_pos_get", "arena_dev_create", "arena_dev_destroy",
    "arena_dev_push", "arena_dev_pop", "arena_dev_pop_at", "arena_dev_pos_get", "cu_malloc", "cu_free",
    "cu_memcpy_htd", "cu_memcpy_htd_async", "cu_memcpy_dth", "cu_host_register_read_only", "cu_memset",
    "inf_fetch_input_embeddings", "inf_rmsnorm", "inf_gemm_bf16", "inf_attn_decode_scratch_bytes", "inf_attn_decode",
    "inf_attn_decode_with", "inf_attn_prefill",
    "inf_config_preset", "inf_model_build", "inf_model_destroy", "inf_forward", "inf_forward_batch",
    "inf_generate", "inf_decode", "inf_seq_reset", "inf_error_string", "inf_last_error_detail", "inf_model_stream",
    "inf_kernel_launches", "inf_batch_h2d_bytes", "inf_decode_bytes", "inf_profile_decode_step", "inf_synth_ids", "inf_debug_read",
    "inf_tp_export", "inf_tp_connect", "inf_attn_decode_noalloc", "inf_config_from_json", "inf_safetensors_check",
    "inf_safetensors_read", "inf_tokenizer_build", "inf_tokenizer_destroy", "inf_tokenizer_vocab_size",
    "inf_tokenizer_encode", "inf_tokenizer_encode_special", "inf_tokenizer_decode", "inf_set_sampling", "inf_set_slot_sampling", "inf_server_submit_sampled", "inf_server_create",
    "inf_server_create_synthetic", "inf_server_destroy", "inf_server_submit", "inf_server_step", "inf_server_result",
    "inf_server_release", "inf_server_stats",
]

_lib = None


def build() -> None:
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def lib():
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise OSError(f"{LIB_PATH} is not built (run `make -C {HERE}`); there is no fallback path")
    L = C.CDLL(LIB_PATH)
    E = C.c_int
    sig = {
        "exec_ctx_create": (E, [C.POINTER(C.POINTER(ExecCtx))]),
        "exec_ctx_destroy": (E, [C.POINTER(C.POINTER(ExecCtx))]),
        "arena_host_create": (E, [C.POINTER(C.POINTER(HostArena)), u64, u64]),
        "arena_host_destroy": (E, [C.POINTER(HostArena)]),
        "arena_host_push": (E, [C.POINTER(HostArena), u64, C.POINTER(vp)]),
        "arena_host_pop": (None, [C.POINTER(HostArena), u64]),
        "arena_host_pop_at": (None, [C.POINTER(HostArena), u64]),
        "mem_arena_host_pos_get": (u64, [C.POINTER(HostArena)]),
        "arena_dev_create": (E, [C.POINTER(DevArena), u64]),
        "arena_dev_destroy": (E, [C.POINTER(DevArena)]),
        "arena_dev_push": (E, [C.POINTER(DevArena), u64, C.POINTER(vp)]),
        "arena_dev_pop": (None, [C.POINTER(DevArena), u64]),
        "arena_dev_pop_at": (None, [C.POINTER(DevArena), u64]),
        "arena_dev_pos_get": (u64, [C.POINTER(DevArena)]),
        "cu_malloc": (i32, [C.POINTER(vp), u64]),
        "cu_free": (i32, [vp]),
        "cu_memcpy_htd": (E, [vp, vp, u64]),
        "cu_memcpy_htd_async": (i32, [vp, vp, u64, vp]),
        "cu_memcpy_dth": (E, [vp, vp, u64]),
        "cu_host_register_read_only": (i32, [vp, u64]),
        "cu_memset": (i32, [vp, i32, u64]),
        "inf_fetch_input_embeddings": (E, [vp, u64, u32, u32, vp, vp, u32, vp]),
        "inf_rmsnorm": (E, [vp, vp, u32, u32, vp, f32, u32, vp]),
        "inf_gemm_bf16": (E, [vp, vp, vp, u32, u32, u32, u32, vp]),
        "inf_attn_decode_scratch_bytes": (u64, [u32, u32, u32, u32, u32, u32, u32]),
        "inf_attn_decode": (E, [vp, vp, vp, vp, u32, u32, vp, vp, u32, u32, u32, u32, u32, u32, vp, vp, u64, vp]),
        "inf_attn_decode_with": (E, [u32, vp, vp, vp, vp, u32, u32, vp, vp, u32, u32, u32, u32, u32, u32, vp, vp, u64,
                                     vp]),
        "inf_attn_prefill": (E, [u32, vp, vp, vp, vp, u32, u32, vp, vp, u32, u32, u32, u32, u32, vp, vp]),
        "inf_config_preset": (E, [u32, C.POINTER(InfConfig)]),
        "inf_model_build": (E, [C.POINTER(C.POINTER(ExecCtx)), C.POINTER(Model), C.POINTER(InfConfig), C.c_char_p, u64]),
        "inf_model_destroy": (E, [C.POINTER(C.POINTER(ExecCtx)), C.POINTER(Model)]),
        "inf_forward": (E, [C.POINTER(Model), vp, u32, u32, u32, vp, vp]),
        "inf_forward_batch": (E, [C.POINTER(Model), u32, vp, vp, vp, vp, vp]),
        "inf_generate": (E, [C.POINTER(Model), vp, u32, u32, vp, C.POINTER(InfStats)]),
        "inf_decode": (E, [C.POINTER(Model), u32, u32, u32, u32, vp, C.POINTER(InfStats)]),
        "inf_seq_reset": (E, [C.POINTER(Model), u32]),
        "inf_error_string": (C.c_char_p, [E]),
        "inf_last_error_detail": (C.c_char_p, []),
        "inf_model_stream": (vp, [C.POINTER(Model)]),
        "inf_kernel_launches": (u64, [C.POINTER(Model)]),
        "inf_batch_h2d_bytes": (u64, [C.POINTER(Model)]),
        "inf_decode_bytes": (u64, [C.POINTER(InfConfig), u32]),
        "inf_profile_decode_step": (u32, [C.POINTER(Model), u32, u32, u32, C.POINTER(f32), u32]),
        "inf_synth_ids": (E, [u64, u64, u64, u32, u32, vp]),
        "inf_debug_read": (E, [C.POINTER(Model), u32, u32, u32, u32, vp, u64]),
        "inf_tp_export": (E, [C.POINTER(Model), vp, u64]),
        "inf_attn_decode_noalloc": (E, [vp, vp, vp, vp, u32, u32, vp, vp, u32, u32, u32, u32, u32, u32, vp, vp]),
        "inf_tp_connect": (E, [C.POINTER(Model), vp, u32]),
        "inf_config_from_json": (E, [C.c_char_p, C.POINTER(InfConfig)]),
        "inf_safetensors_check": (E, [C.c_char_p, C.POINTER(InfConfig)]),
        "inf_safetensors_read": (E, [C.c_char_p, C.POINTER(InfConfig), u32, u32, vp, u64]),
        "inf_tokenizer_build": (E, [C.c_char_p, C.POINTER(vp)]),
        "inf_tokenizer_destroy": (E, [C.POINTER(vp)]),
        "inf_tokenizer_vocab_size": (u32, [vp]),
        "inf_tokenizer_encode": (E, [vp, C.c_char_p, vp, u64, C.POINTER(u64)]),
        "inf_tokenizer_encode_special": (E, [vp, C.c_char_p, vp, u64, C.POINTER(u64)]),
        "inf_tokenizer_decode": (E, [vp, vp, u64, C.c_char_p, u64, C.POINTER(u64)]),
        "inf_set_sampling": (E, [C.POINTER(Model), C.POINTER(InfSampling)]),
        "inf_set_slot_sampling": (E, [C.POINTER(Model), u32, C.POINTER(InfSampling)]),
        "inf_server_submit_sampled": (E, [vp, vp, u32, u32, u32, C.POINTER(InfSampling), C.POINTER(u64)]),
        "inf_server_create": (E, [C.POINTER(Model), u32, C.POINTER(vp)]),
        "inf_server_create_synthetic": (E, [u32, u32, u32, u32, u32, C.POINTER(vp)]),
        "inf_server_destroy": (E, [C.POINTER(vp)]),
        "inf_server_submit": (E, [vp, vp, u32, u32, u32, C.POINTER(u64)]),
        "inf_server_step": (E, [vp, C.POINTER(u32)]),
        "inf_server_result": (E, [vp, u64, vp, u32, C.POINTER(u32), C.POINTER(u32), C.POINTER(C.c_int)]),
        "inf_server_release": (E, [vp, u64]),
        "inf_server_stats": (E, [vp, C.POINTER(u32), C.POINTER(u32), C.POINTER(u64), C.POINTER(u64)]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def check(rc: int, where: str) -> None:
    if rc != 0:
        raise InfError(rc, where, lib().inf_last_error_detail().decode(errors="replace"))  # details quote file bytes


def preset(n: int, **overrides) -> InfConfig:
    c = InfConfig()
    check(lib().inf_config_preset(n, C.byref(c)), "inf_config_preset")
    for k, v in overrides.items():
        setattr(c, k, v)
    return c


def config_from_dict(d: dict) -> InfConfig:
    c = InfConfig()
    c.kv_block, c.max_batch, c.norm_eps, c.init_std, c.tp_size = 16, 1, 1e-5, 0.02, 1
    names = {"vocab": "vocab_size", "ffn": "ffn_dim", "eps": "norm_eps"}
    for k, v in d.items():
        if k == "dtype":
            c.dtype = BF16 if v == "bf16" else F32
        elif hasattr(c, names.get(k, k)):
            setattr(c, names.get(k, k), v)
    return c


def config_from_json(path: str, base: InfConfig | None = None) -> InfConfig:
    """inf_config_from_json: a Hugging Face config.json over `base` (fields the file lacks keep
    base's values: max_seq, max_batch, KV paging, tensor parallelism)."""
    c = InfConfig()
    if base is not None:
        C.memmove(C.byref(c), C.byref(base), C.sizeof(InfConfig))
    check(lib().inf_config_from_json(os.fsencode(path), C.byref(c)), "inf_config_from_json")
    return c


def safetensors_check(path: str, cfg: InfConfig) -> None:
    check(lib().inf_safetensors_check(os.fsencode(path), C.byref(cfg)), "inf_safetensors_check")


def weight_shape(cfg: InfConfig, kind: int) -> tuple:
    """Rows and columns of one weight in the device layout of rank cfg.tp_rank."""
    tp = max(1, cfg.tp_size)
    d, hd = cfg.dim, cfg.head_dim
    L, P = cfg.n_layers, cfg.ple_dim
    return {W_EMBED: (cfg.vocab_size, d), W_LM_HEAD: (cfg.vocab_size // tp, d), W_FINAL_NORM: (1, d),
            W_QKV: ((cfg.n_heads + 2 * cfg.n_kv_heads) // tp * hd, d), W_O: (d, cfg.n_heads // tp * hd),
            W_GATE_UP: (2 * cfg.ffn_dim // tp, d), W_DOWN: (d, cfg.ffn_dim // tp), W_ATTN_NORM: (1, d),
            W_FFN_NORM: (1, d),
            # Gemma-style models
            3: (cfg.vocab_size, L * P), 4: (L * P, d), 5: (1, P), 17: (1, hd), 18: (1, hd), 19: (1, d), 20: (1, d),
            21: (P, d), 22: (d, P), 23: (1, d)}[kind]


def safetensors_read(path: str, cfg: InfConfig, layer: int, kind: int) -> np.ndarray:
    """inf_safetensors_read: one weight as the device holds it (uint16 bf16 bits or float32)."""
    out = np.empty(weight_shape(cfg, kind), dtype=np.uint16 if cfg.dtype == BF16 else np.float32)
    check(lib().inf_safetensors_read(os.fsencode(path), C.byref(cfg), layer, kind, _ptr(out), out.nbytes),
          "inf_safetensors_read")
    return out


class Tokenizer:
    """inf_tokenizer_*: BPE encode / decode of a Hugging Face tokenizer.json."""

    def __init__(self, path: str):
        self.h = vp()
        check(lib().inf_tokenizer_build(os.fsencode(path), C.byref(self.h)), "inf_tokenizer_build")

    @property
    def vocab_size(self) -> int:
        return int(lib().inf_tokenizer_vocab_size(self.h))

    def encode(self, text, special: bool = False) -> np.ndarray:
        """The reference's encoding; special=True first cuts out added special tokens."""
        fn = lib().inf_tokenizer_encode_special if special else lib().inf_tokenizer_encode
        raw = text.encode() if isinstance(text, str) else bytes(text)
        n = u64()
        out = np.empty(len(raw) + 8, dtype=np.uint32)  # enough unless byte fallback splits "▁"
        rc = fn(self.h, raw, _ptr(out), out.size, C.byref(n))
        if rc == 4 and n.value > out.size:
            out = np.empty(n.value, dtype=np.uint32)
            rc = fn(self.h, raw, _ptr(out), out.size, C.byref(n))
        check(rc, "inf_tokenizer_encode")
        return out[:n.value]

    def decode_bytes(self, ids) -> bytes:
        ids = np.ascontiguousarray(ids, dtype=np.uint32)
        n = u64()
        check(lib().inf_tokenizer_decode(self.h, _ptr(ids), ids.size, None, 0, C.byref(n)), "inf_tokenizer_decode")
        buf = C.create_string_buffer(n.value + 1)
        check(lib().inf_tokenizer_decode(self.h, _ptr(ids), ids.size, buf, n.value + 1, C.byref(n)),
              "inf_tokenizer_decode")
        return buf.raw[:n.value]

    def decode(self, ids) -> str:
        return self.decode_bytes(ids).decode("utf-8", errors="replace")

    def close(self):
        if self.h:
            check(lib().inf_tokenizer_destroy(C.byref(self.h)), "inf_tokenizer_destroy")

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


NO_EOS = 0xFFFFFFFF


class Server:
    """inf_server_*: continuous batching over a model's sequence slots (or, with engine None,
    over the host-only stand-in model of inf_server_create_synthetic)."""

    def __init__(self, engine=None, max_active: int = 0, synthetic: tuple | None = None):
        self.h = vp()
        if engine is not None:
            check(lib().inf_server_create(C.byref(engine.model), max_active, C.byref(self.h)), "inf_server_create")
        else:
            n_slots, max_seq, vocab = synthetic[:3]
            kv_pages = synthetic[3] if len(synthetic) > 3 else 0
            check(lib().inf_server_create_synthetic(n_slots, max_seq, vocab, kv_pages, max_active, C.byref(self.h)),
                  "inf_server_create_synthetic")

    def submit(self, prompt, max_new: int, eos: int = NO_EOS, sampling: tuple | None = None) -> int:
        """sampling: (temperature, top_p, top_k, seed) for this request (inf_server_submit_sampled)."""
        p = np.ascontiguousarray(prompt, dtype=np.uint32)
        rid = u64()
        if sampling is None:
            check(lib().inf_server_submit(self.h, _ptr(p), p.size, max_new, eos, C.byref(rid)), "inf_server_submit")
        else:
            t, tp, tk, seed = sampling
            smp = InfSampling(temperature=t, top_p=tp, top_k=tk, reserved=0, seed=seed)
            check(lib().inf_server_submit_sampled(self.h, _ptr(p), p.size, max_new, eos, C.byref(smp), C.byref(rid)),
                  "inf_server_submit_sampled")
        return rid.value

    def step(self) -> int:
        n = u32()
        check(lib().inf_server_step(self.h, C.byref(n)), "inf_server_step")
        return n.value

    def result(self, rid: int):
        """(ids so far, done, error code that retired it or 0)."""
        n, done, status = u32(), u32(), C.c_int()
        check(lib().inf_server_result(self.h, rid, None, 0, C.byref(n), None, None), "inf_server_result")
        out = np.empty(n.value, dtype=np.uint32)
        check(lib().inf_server_result(self.h, rid, _ptr(out), out.size, C.byref(n), C.byref(done), C.byref(status)),
              "inf_server_result")
        return out, bool(done.value), status.value

    def release(self, rid: int):
        check(lib().inf_server_release(self.h, rid), "inf_server_release")

    def stats(self) -> dict:
        w, a, bs, bt = u32(), u32(), u64(), u64()
        check(lib().inf_server_stats(self.h, C.byref(w), C.byref(a), C.byref(bs), C.byref(bt)), "inf_server_stats")
        return dict(waiting=w.value, active=a.value, batched_steps=bs.value, batched_tokens=bt.value)

    def close(self):
        if self.h:
            check(lib().inf_server_destroy(C.byref(self.h)), "inf_server_destroy")

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def oracle_dict(c: InfConfig) -> dict:
    """The same model as a dict for oracle/oracle.py (tests only)."""
    d = dict(vocab=c.vocab_size, dim=c.dim, n_layers=c.n_layers, n_heads=c.n_heads, n_kv_heads=c.n_kv_heads,
             head_dim=c.head_dim, ffn=c.ffn_dim, max_seq=c.max_seq, eps=c.norm_eps, rope_theta=c.rope_theta,
             dtype="bf16" if c.dtype == BF16 else "fp32", init_std=c.init_std)
    if c.arch:
        d.update(arch=c.arch, ple_dim=c.ple_dim, final_softcap=c.final_softcap)
    return d


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(vp)


class Engine:
    """One model on the current CUDA device (one context per GPU)."""

    def __init__(self, cfg: InfConfig, seed: int = 0, weights_path: str | None = None):
        """Synthetic weights from `seed`, or a safetensors checkpoint (file, index or directory)."""
        self.cfg = cfg
        self.ctx = C.POINTER(ExecCtx)()
        self.model = Model()
        path = os.fsencode(weights_path) if weights_path is not None else None
        check(lib().inf_model_build(C.byref(self.ctx), C.byref(self.model), C.byref(cfg), path, seed),
              "inf_model_build")
        self.V = cfg.vocab_size // max(1, cfg.tp_size)

    def close(self):
        if self.model.engine:
            check(lib().inf_model_destroy(C.byref(self.ctx), C.byref(self.model)), "inf_model_destroy")

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def stream(self) -> int:
        return lib().inf_model_stream(C.byref(self.model)) or 0

    @property
    def launches(self) -> int:
        return int(lib().inf_kernel_launches(C.byref(self.model)))

    @property
    def batch_h2d_bytes(self) -> int:
        """Bytes the batched steps have copied host -> device so far."""
        return int(lib().inf_batch_h2d_bytes(C.byref(self.model)))

    @property
    def weight_bytes(self) -> int:
        return int(self.model.model_bsize)

    def forward(self, ids, start_pos: int, slot: int = 0, want_logits: bool = True):
        ids = np.ascontiguousarray(ids, dtype=np.uint32)
        lg = np.empty(self.V, dtype=np.float32) if want_logits else None
        am = np.zeros(1, dtype=np.uint32)
        check(lib().inf_forward(C.byref(self.model), _ptr(ids), ids.size, start_pos, slot,
                                _ptr(lg) if lg is not None else None, _ptr(am)), "inf_forward")
        return lg, int(am[0])

    def forward_ptr(self, ids_ptr: int, n: int, start_pos: int, slot: int, logits_ptr, argmax_ptr):
        """Device- or host-pointer variant (torch tensors' data_ptr())."""
        check(lib().inf_forward(C.byref(self.model), vp(ids_ptr), n, start_pos, slot,
                                vp(logits_ptr) if logits_ptr else None, vp(argmax_ptr) if argmax_ptr else None),
              "inf_forward")

    def forward_batch(self, slots, ids, positions, want_logits: bool = False):
        slots = np.ascontiguousarray(slots, dtype=np.uint32)
        ids = np.ascontiguousarray(ids, dtype=np.uint32)
        positions = np.ascontiguousarray(positions, dtype=np.uint32)
        n = ids.size
        lg = np.empty((n, self.V), dtype=np.float32) if want_logits else None
        am = np.zeros(n, dtype=np.uint32)
        check(lib().inf_forward_batch(C.byref(self.model), n, _ptr(slots), _ptr(ids), _ptr(positions),
                                      _ptr(lg) if lg is not None else None, _ptr(am)), "inf_forward_batch")
        return lg, am

    def generate(self, prompt, n_new: int):
        prompt = np.ascontiguousarray(prompt, dtype=np.uint32)
        out = np.zeros(n_new, dtype=np.uint32)
        st = InfStats()
        check(lib().inf_generate(C.byref(self.model), _ptr(prompt), prompt.size, n_new, _ptr(out), C.byref(st)),
              "inf_generate")
        return out, st

    def decode(self, first_id: int, start_pos: int, n_steps: int, slot: int = 0, want_ids: bool = True):
        out = np.zeros(n_steps, dtype=np.uint32) if want_ids else None
        st = InfStats()
        check(lib().inf_decode(C.byref(self.model), slot, start_pos, first_id, n_steps,
                               _ptr(out) if out is not None else None, C.byref(st)), "inf_decode")
        return out, st

    def tp_export(self) -> bytes:
        buf = (C.c_uint8 * 64)()
        check(lib().inf_tp_export(C.byref(self.model), buf, 64), "inf_tp_export")
        return bytes(buf)

    def tp_connect(self, handles) -> None:
        """handles: the tp_size exported handles in rank order."""
        blob = b"".join(handles)
        buf = (C.c_uint8 * len(blob)).from_buffer_copy(blob)
        check(lib().inf_tp_connect(C.byref(self.model), buf, len(handles)), "inf_tp_connect")

    BUFFERS = {"resid": 0, "q": 1, "attn": 2, "h": 3, "logits": 4, "k": 5, "v": 6, "sample_q": 7, "sample_q_row": 8}

    def debug_read(self, name: str, layer: int = 0, slot: int = 0, pos: int = 0) -> np.ndarray:
        n = max(self.cfg.dim, self.cfg.ffn_dim, self.V, self.cfg.n_heads * self.cfg.head_dim)
        out = np.empty(n, dtype=np.float32)
        check(lib().inf_debug_read(C.byref(self.model), self.BUFFERS[name], layer, slot, pos, _ptr(out), n),
              "inf_debug_read")
        tp = max(1, self.cfg.tp_size)
        sizes = {"resid": self.cfg.dim, "q": self.cfg.n_heads // tp * self.cfg.head_dim,
                 "attn": self.cfg.n_heads // tp * self.cfg.head_dim, "h": self.cfg.ffn_dim // tp, "logits": self.V,
                 "k": self.cfg.n_kv_heads // tp * self.cfg.head_dim, "v": self.cfg.n_kv_heads // tp * self.cfg.head_dim,
                 "sample_q": self.V, "sample_q_row": self.V}
        r = out[:sizes[name]].copy()
        return r.view(np.uint32) if name in ("sample_q", "sample_q_row") else r

    def set_sampling(self, temperature: float, top_p: float = 1.0, top_k: int = 0, seed: int = 0):
        """inf_set_sampling; temperature 0 restores greedy decoding."""
        s = InfSampling(temperature=temperature, top_p=top_p, top_k=top_k, reserved=0, seed=seed)
        check(lib().inf_set_sampling(C.byref(self.model), C.byref(s)), "inf_set_sampling")

    def set_slot_sampling(self, slot: int, temperature: float, top_p: float = 1.0, top_k: int = 0, seed: int = 0):
        """inf_set_slot_sampling: the slot's settings for the batched step; temperature 0 is greedy."""
        s = InfSampling(temperature=temperature, top_p=top_p, top_k=top_k, reserved=0, seed=seed)
        check(lib().inf_set_slot_sampling(C.byref(self.model), slot, C.byref(s)), "inf_set_slot_sampling")

    def reset(self, slot: int = 0):
        check(lib().inf_seq_reset(C.byref(self.model), slot), "inf_seq_reset")

    def profile_step(self, pos: int, token: int, slot: int = 0) -> dict:
        ms = (f32 * 8)()
        n = lib().inf_profile_decode_step(C.byref(self.model), slot, pos, token, ms, 8)
        if n == 0:
            raise InfError(7, "inf_profile_decode_step", lib().inf_last_error_detail().decode())
        return {KERNEL_KINDS[k]: float(ms[k]) for k in range(n)}


STREAM_PROMPT = 0x1000000
STREAM_CTX_LEN = 0x2000000


def synth_ids(seed: int, n: int, vocab: int, stream: int = STREAM_PROMPT) -> np.ndarray:
    """Seeded uniform ids in [0, vocab) (the workloads' prompts)."""
    out = np.empty(n, dtype=np.uint32)
    check(lib().inf_synth_ids(seed, stream, n, 0, vocab - 1, _ptr(out)), "inf_synth_ids")
    return out


def synth_uniform(seed: int, stream: int, n: int, lo: int, hi: int) -> np.ndarray:
    out = np.empty(n, dtype=np.uint32)
    check(lib().inf_synth_ids(seed, stream, n, lo, hi, _ptr(out)), "inf_synth_ids")
    return out


def decode_bytes(cfg: InfConfig, ctx: int) -> int:
    return int(lib().inf_decode_bytes(C.byref(cfg), ctx))


def fetch_input_embeddings(d_ids: int, n: int, dim: int, vocab: int, d_table: int, d_out: int, dtype: int,
                           stream: int = 0) -> None:
    check(lib().inf_fetch_input_embeddings(vp(d_ids), n, dim, vocab, vp(d_table), vp(d_out), dtype,
                                           vp(stream) if stream else None), "inf_fetch_input_embeddings")


def gemm_bf16(d_x: int, d_w: int, d_y: int, T: int, N: int, K: int, out_f32: bool, stream: int = 0) -> None:
    check(lib().inf_gemm_bf16(vp(d_x), vp(d_w), vp(d_y), T, N, K, int(out_f32), vp(stream) if stream else None),
          "inf_gemm_bf16")


def attn_decode_scratch_bytes(n_tokens, n_heads, n_kv_heads, head_dim, kv_block, pages_per_seq, dtype) -> int:
    return int(lib().inf_attn_decode_scratch_bytes(n_tokens, n_heads, n_kv_heads, head_dim, kv_block, pages_per_seq,
                                                   dtype))


def attn_decode(d_q, d_k, d_v, d_bt, pages_per_seq, n_pages, d_slot, d_pos, n_tokens, n_heads, n_kv_heads, head_dim,
                kv_block, dtype, d_out, d_scratch, scratch_bytes, stream=0) -> None:
    check(lib().inf_attn_decode(vp(d_q), vp(d_k), vp(d_v), vp(d_bt), pages_per_seq, n_pages, vp(d_slot), vp(d_pos),
                                n_tokens, n_heads, n_kv_heads, head_dim, kv_block, dtype, vp(d_out), vp(d_scratch),
                                scratch_bytes, vp(stream) if stream else None), "inf_attn_decode")


ATTN_AUTO, ATTN_SPLITK, ATTN_CLUSTER, ATTN_MMA, ATTN_CLUSTER_TC = 0, 1, 2, 3, 4  # InfAttnKernel


def attn_decode_with(kernel, d_q, d_k, d_v, d_bt, pages_per_seq, n_pages, d_slot, d_pos, n_tokens, n_heads,
                     n_kv_heads, head_dim, kv_block, dtype, d_out, d_scratch, scratch_bytes, stream=0) -> None:
    """inf_attn_decode with one kernel of InfAttnKernel forced."""
    check(lib().inf_attn_decode_with(kernel, vp(d_q), vp(d_k), vp(d_v), vp(d_bt), pages_per_seq, n_pages, vp(d_slot),
                                     vp(d_pos), n_tokens, n_heads, n_kv_heads, head_dim, kv_block, dtype, vp(d_out),
                                     vp(d_scratch), scratch_bytes, vp(stream) if stream else None),
          "inf_attn_decode_with")


PREFILL_AUTO, PREFILL_SIMT = 0, 1  # InfPrefillAttention


def attn_prefill(kernel, d_q, d_k, d_v, d_bt, pages_per_seq, n_pages, d_slot, d_pos, n_tokens, n_heads, n_kv_heads,
                 head_dim, kv_block, d_out, stream=0) -> None:
    """Causal attention of one prefill pass over the paged cache (bf16)."""
    check(lib().inf_attn_prefill(kernel, vp(d_q), vp(d_k), vp(d_v), vp(d_bt), pages_per_seq, n_pages, vp(d_slot),
                                 vp(d_pos), n_tokens, n_heads, n_kv_heads, head_dim, kv_block, vp(d_out),
                                 vp(stream) if stream else None), "inf_attn_prefill")


def attn_decode_noalloc(d_q, d_k, d_v, d_bt, pages_per_seq, n_pages, d_slot, d_pos, n_tokens, n_heads, n_kv_heads,
                        head_dim, kv_block, dtype, d_out, stream=0) -> None:
    """inf_attn_decode without a scratch argument: for callers that cannot allocate."""
    check(lib().inf_attn_decode_noalloc(vp(d_q), vp(d_k), vp(d_v), vp(d_bt), pages_per_seq, n_pages, vp(d_slot),
                                        vp(d_pos), n_tokens, n_heads, n_kv_heads, head_dim, kv_block, dtype,
                                        vp(d_out), vp(stream) if stream else None), "inf_attn_decode_noalloc")


def rmsnorm(d_x: int, d_y: int, rows: int, dim: int, d_gain: int, eps: float, dtype: int, stream: int = 0) -> None:
    check(lib().inf_rmsnorm(vp(d_x), vp(d_y), rows, dim, vp(d_gain), eps, dtype, vp(stream) if stream else None),
          "inf_rmsnorm")
