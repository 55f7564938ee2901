"""Safetensors files for the loader tests: a writer of the format (8-byte little-endian header
length, JSON header, byte buffer) and the canonical Hugging Face Llama tensors of a config,
either from a numpy generator or the synthetic weights of the engine (Philox streams of the
oracle, so a checkpoint written here holds exactly the weights inf_model_build generates from
the same seed)."""
from __future__ import annotations

import json
import struct

import numpy as np

import oracle as O

DTYPES = {"BF16": np.uint16, "F32": np.float32, "F16": np.float16, "I32": np.int32, "U8": np.uint8}

TINY = dict(vocab=512, dim=64, n_layers=2, n_heads=4, n_kv_heads=2, head_dim=16, ffn=160, max_seq=64, eps=1e-5,
            rope_theta=10000.0, dtype="bf16")


def header_bytes(header: dict, pad_to: int = 8) -> bytes:
    h = json.dumps(header, separators=(",", ":")).encode()
    return h + b" " * ((-len(h)) % pad_to)


def write_safetensors(path, tensors, metadata: dict | None = None) -> None:
    """tensors: list of (name, dtype string, array); buffer in list order, no gaps."""
    header, blobs, at = {}, [], 0
    if metadata is not None:
        header["__metadata__"] = metadata
    for name, dt, arr in tensors:
        raw = np.ascontiguousarray(arr, dtype=DTYPES[dt]).tobytes()
        header[name] = {"dtype": dt, "shape": list(np.shape(arr)), "data_offsets": [at, at + len(raw)]}
        blobs.append(raw)
        at += len(raw)
    write_raw(path, header_bytes(header), b"".join(blobs))


def write_raw(path, header: bytes, buf: bytes, hlen: int | None = None) -> None:
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(header) if hlen is None else hlen))
        f.write(header)
        f.write(buf)


def bf16_round(x: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bits, round to nearest even (finite inputs)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def widen(h: np.ndarray) -> np.ndarray:
    return (h.astype(np.uint32) << 16).view(np.float32)


def hf_names(n_layers: int, prefix: str = "model.", tie: bool = False):
    """(name, canonical kind, layer) of every tensor of the decoder, Hugging Face Llama names."""
    out = [(prefix + "embed_tokens.weight", O.K_EMBED, -1)]
    for l in range(n_layers):
        p = f"{prefix}layers.{l}."
        out += [(p + "input_layernorm.weight", O.K_ATTN_NORM, l), (p + "self_attn.q_proj.weight", O.K_WQ, l),
                (p + "self_attn.k_proj.weight", O.K_WK, l), (p + "self_attn.v_proj.weight", O.K_WV, l),
                (p + "self_attn.o_proj.weight", O.K_WO, l), (p + "post_attention_layernorm.weight", O.K_FFN_NORM, l),
                (p + "mlp.gate_proj.weight", O.K_WGATE, l), (p + "mlp.up_proj.weight", O.K_WUP, l),
                (p + "mlp.down_proj.weight", O.K_WDOWN, l)]
    out.append((prefix + "norm.weight", O.K_FINAL_NORM, -1))
    if not tie:
        out.append(("lm_head.weight", O.K_LM_HEAD, -1))
    return out


def gemma_names(n_layers: int, ple: bool, prefix: str = "model.language_model."):
    """(name, canonical kind, layer) of every tensor of the Gemma-style decoder: Gemma names, the
    embedding as LM head (no lm_head.weight), per-layer embeddings when `ple`."""
    out = [(prefix + "embed_tokens.weight", O.K_EMBED, -1)]
    if ple:
        out += [(prefix + "embed_tokens_per_layer.weight", O.K_EMBED_PLE, -1),
                (prefix + "per_layer_model_projection.weight", O.K_PLE_MODEL_PROJ, -1),
                (prefix + "per_layer_projection_norm.weight", O.K_PLE_PROJ_NORM, -1)]
    for l in range(n_layers):
        p = f"{prefix}layers.{l}."
        out += [(p + "input_layernorm.weight", O.K_ATTN_NORM, l), (p + "self_attn.q_proj.weight", O.K_WQ, l),
                (p + "self_attn.k_proj.weight", O.K_WK, l), (p + "self_attn.v_proj.weight", O.K_WV, l),
                (p + "self_attn.q_norm.weight", O.K_Q_NORM, l), (p + "self_attn.k_norm.weight", O.K_K_NORM, l),
                (p + "self_attn.o_proj.weight", O.K_WO, l), (p + "post_attention_layernorm.weight", O.K_POST_ATTN_NORM, l),
                (p + "pre_feedforward_layernorm.weight", O.K_FFN_NORM, l), (p + "mlp.gate_proj.weight", O.K_WGATE, l),
                (p + "mlp.up_proj.weight", O.K_WUP, l), (p + "mlp.down_proj.weight", O.K_WDOWN, l),
                (p + "post_feedforward_layernorm.weight", O.K_POST_FFN_NORM, l)]
        if ple:
            out += [(p + "per_layer_input_gate.weight", O.K_PLE_GATE, l), (p + "per_layer_projection.weight", O.K_PLE_PROJ, l),
                    (p + "post_per_layer_input_norm.weight", O.K_PLE_POST_NORM, l)]
    out.append((prefix + "norm.weight", O.K_FINAL_NORM, -1))
    return out


def canon_shape(shape: dict, kind: int):
    d, hd, V, F = shape["dim"], shape["head_dim"], shape["vocab"], shape["ffn"]
    H, KV, L, P = shape["n_heads"], shape["n_kv_heads"], shape["n_layers"], shape.get("ple_dim", 0)
    return {O.K_EMBED: (V, d), O.K_LM_HEAD: (V, d), O.K_FINAL_NORM: (d,), O.K_ATTN_NORM: (d,), O.K_FFN_NORM: (d,),
            O.K_WQ: (H * hd, d), O.K_WK: (KV * hd, d), O.K_WV: (KV * hd, d), O.K_WO: (d, H * hd),
            O.K_WGATE: (F, d), O.K_WUP: (F, d), O.K_WDOWN: (d, F),
            O.K_EMBED_PLE: (V, L * P), O.K_PLE_MODEL_PROJ: (L * P, d), O.K_PLE_PROJ_NORM: (P,),
            O.K_Q_NORM: (hd,), O.K_K_NORM: (hd,), O.K_POST_ATTN_NORM: (d,), O.K_POST_FFN_NORM: (d,),
            O.K_PLE_GATE: (P, d), O.K_PLE_PROJ: (d, P), O.K_PLE_POST_NORM: (d,)}[kind]


def random_tensors(shape: dict, rng: np.random.Generator):
    """{(kind, layer): float32 array} of random canonical tensors."""
    out = {}
    for _, kind, layer in hf_names(shape["n_layers"]):
        out[(kind, layer)] = rng.standard_normal(canon_shape(shape, kind)).astype(np.float32)
    return out


def synthetic_tensors(shape: dict, seed: int, init_std: float = 0.02, bf16: bool = True):
    """{(kind, layer): array} of the engine's synthetic weights (bf16 bits or float32); Gemma-style
    shapes (arch 1) draw their norm gains like the weights."""
    out = {}
    gemma = shape.get("arch", 0) == 1
    names = gemma_names(shape["n_layers"], shape.get("ple_dim", 0) > 0) if gemma else hf_names(shape["n_layers"])
    for _, kind, layer in names:
        sh = canon_shape(shape, kind)
        n = int(np.prod(sh))
        if kind in (O.K_FINAL_NORM, O.K_ATTN_NORM, O.K_FFN_NORM) and not gemma:
            a = np.full(n, 0x3F80, np.uint16) if bf16 else np.ones(n, np.float32)
        else:
            a = O.fill_tensor(seed, O.tensor_stream(layer, kind), n, init_std, bf16)
        out[(kind, layer)] = a.reshape(sh)
    return out


def write_checkpoint(path, shape: dict, tensors: dict, dtype: str = "BF16", prefix: str = "model.", tie: bool = False,
                     metadata: dict | None = None) -> list:
    """One file; tensors hold bf16 bits (uint16) or float32 and are converted to `dtype`."""
    items = []
    gemma = shape.get("arch", 0) == 1
    names = gemma_names(shape["n_layers"], shape.get("ple_dim", 0) > 0, prefix) if gemma else \
        hf_names(shape["n_layers"], prefix, tie)
    for name, kind, layer in names:
        a = tensors[(kind, layer)]
        if dtype == "F32" and a.dtype == np.uint16:
            a = widen(a)
        elif dtype == "BF16" and a.dtype == np.float32:
            a = bf16_round(a)
        items.append((name, dtype, a))
    write_safetensors(path, items, metadata)
    return items
