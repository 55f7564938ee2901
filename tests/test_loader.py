"""Checkpoint loading on the host (no GPU): safetensors parsing and validation, the device
layout of every weight for every tensor-parallel rank, dtype conversion, sharded checkpoints and
config.json, through the C ABI (inf_safetensors_check, inf_safetensors_read,
inf_config_from_json).  The expected layouts are restated here in numpy from the layout rules:
QKV rows of each head in (i, i + head_dim/2) pairs, gate/up rows interleaved, the rank's rows
(QKV, gate/up, LM head) or columns (O, down).  Error cases follow the reference's model_build
(src/main.cu:177-352) and its defects D7 (offsets from the file start) and D8 (one contiguous
bf16 span assumed)."""
import json
import os

import numpy as np
import pytest

import infb200 as I
import oracle as O
from st_files import (TINY, bf16_round, canon_shape, header_bytes, hf_names, random_tensors, widen,
                      write_checkpoint, write_raw, write_safetensors)

E_IO, E_INVALID, E_CONFIG, E_UNSUPPORTED = 14, 4, 9, 15


def cfg_of(shape=TINY, **kw):
    c = I.config_from_dict(shape)
    for k, v in kw.items():
        setattr(c, k, v)
    return c


def expected(t: dict, c, layer: int, kind: int) -> np.ndarray:
    """Device layout of one weight for rank c.tp_rank, from canonical tensors (bf16 bits or f32)."""
    tp, rk = max(1, c.tp_size), c.tp_rank
    hd, Hl, KVl, Fl, Vl = c.head_dim, c.n_heads // tp, c.n_kv_heads // tp, c.ffn_dim // tp, c.vocab_size // tp
    if kind == I.W_EMBED:
        return t[(O.K_EMBED, -1)]
    if kind == I.W_LM_HEAD:
        return t[(O.K_LM_HEAD, -1)][rk * Vl:(rk + 1) * Vl]
    if kind == I.W_FINAL_NORM:
        return t[(O.K_FINAL_NORM, -1)].reshape(1, -1)
    if kind in (I.W_ATTN_NORM, I.W_FFN_NORM):
        return t[(O.K_ATTN_NORM if kind == I.W_ATTN_NORM else O.K_FFN_NORM, layer)].reshape(1, -1)
    if kind == I.W_QKV:
        pair = np.stack([np.arange(hd // 2), np.arange(hd // 2) + hd // 2], axis=1).ravel()
        rows = []
        for k, h0, n in ((O.K_WQ, rk * Hl, Hl), (O.K_WK, rk * KVl, KVl), (O.K_WV, rk * KVl, KVl)):
            w = t[(k, layer)]
            for h in range(h0, h0 + n):
                rows.append(w[h * hd + pair])
        return np.concatenate(rows)
    if kind == I.W_O:
        return t[(O.K_WO, layer)][:, rk * Hl * hd:(rk + 1) * Hl * hd]
    if kind == I.W_GATE_UP:
        g = t[(O.K_WGATE, layer)][rk * Fl:(rk + 1) * Fl]
        u = t[(O.K_WUP, layer)][rk * Fl:(rk + 1) * Fl]
        return np.stack([g, u], axis=1).reshape(2 * Fl, -1)
    if kind == I.W_DOWN:
        return t[(O.K_WDOWN, layer)][:, rk * Fl:(rk + 1) * Fl]
    raise ValueError(kind)


ALL = [(I.W_EMBED, 0), (I.W_LM_HEAD, 0), (I.W_FINAL_NORM, 0)] + [
    (k, l) for l in range(TINY["n_layers"]) for k in (I.W_QKV, I.W_O, I.W_GATE_UP, I.W_DOWN, I.W_ATTN_NORM, I.W_FFN_NORM)]


def bf16_tensors(seed=0):
    rng = np.random.default_rng(seed)
    return {k: bf16_round(v) for k, v in random_tensors(TINY, rng).items()}


def check_code(code, fn, *args, match=None):
    with pytest.raises(I.InfError) as ei:
        fn(*args)
    assert ei.value.code == code, str(ei.value)
    if match:
        assert match in str(ei.value), str(ei.value)
    return ei.value


# ------------------------------------------------------------------ layout and dtypes
@pytest.mark.parametrize("tp,rank", [(1, 0), (2, 0), (2, 1)])
def test_read_gives_device_layout(tmp_path, tp, rank):
    t = bf16_tensors()
    path = str(tmp_path / "model.safetensors")
    write_checkpoint(path, TINY, t)
    c = cfg_of(tp_size=tp, tp_rank=rank)
    I.safetensors_check(path, c)
    for kind, layer in ALL:
        got = I.safetensors_read(path, c, layer, kind)
        np.testing.assert_array_equal(got, expected(t, c, layer, kind), err_msg=f"kind {kind} layer {layer}")


def test_language_model_prefix_and_tied_lm_head(tmp_path):
    """The reference's checkpoints name tensors model.language_model.*; without lm_head.weight
    the embedding is the LM head."""
    t = bf16_tensors(1)
    path = str(tmp_path / "lm.safetensors")
    write_checkpoint(path, TINY, t, prefix="model.language_model.", tie=True)
    c = cfg_of()
    I.safetensors_check(path, c)
    np.testing.assert_array_equal(I.safetensors_read(path, c, 0, I.W_LM_HEAD), t[(O.K_EMBED, -1)])
    np.testing.assert_array_equal(I.safetensors_read(path, c, 1, I.W_QKV), expected(t, c, 1, I.W_QKV))


def rne_reference(x: np.ndarray) -> np.ndarray:
    """bf16 bits of finite float32 x by round-to-nearest-even, from the two neighbours' distances."""
    u = x.view(np.uint32)
    lo = (u >> 16).astype(np.uint32)
    with np.errstate(invalid="ignore"):  # infinities: lo is exact, the comparisons below are False
        lo_f = (lo << 16).view(np.float32).astype(np.float64)
        hi_f = ((lo + 1) << 16).view(np.float32).astype(np.float64)
        xd = x.astype(np.float64)
        dlo, dhi = np.abs(xd - lo_f), np.abs(hi_f - xd)
        pick_hi = (dhi < dlo) | ((dhi == dlo) & (lo & 1 == 1))
    return np.where(pick_hi, lo + 1, lo).astype(np.uint16)


def test_f32_checkpoint_into_bf16_model(tmp_path):
    """F32 tensors are rounded to bf16 (nearest, ties to even) on the way in."""
    rng = np.random.default_rng(2)
    t = random_tensors(TINY, rng)
    emb = t[(O.K_EMBED, -1)].ravel()
    # exact halfway points (ties both ways), signed zeros, subnormals, infinities
    base = rng.integers(0, 0x7F00, size=256, dtype=np.uint32) << 16
    emb[:256] = (base | 0x8000).view(np.float32)
    emb[256:512] = ((base | 0x18000) & 0x7FFFFFFF).view(np.float32) * -1
    emb[512:520] = np.array([0.0, -0.0, 1e-40, -1e-40, np.inf, -np.inf, 3.0e38, -3.0e38], np.float32)
    path = str(tmp_path / "f32.safetensors")
    write_checkpoint(path, TINY, t, dtype="F32")
    c = cfg_of()
    got = I.safetensors_read(path, c, 0, I.W_EMBED).ravel()
    want = rne_reference(t[(O.K_EMBED, -1)].ravel())
    np.testing.assert_array_equal(got, want)
    np.testing.assert_array_equal(got, bf16_round(t[(O.K_EMBED, -1)]).ravel())
    qkv = I.safetensors_read(path, c, 0, I.W_QKV)
    np.testing.assert_array_equal(qkv, expected({k: bf16_round(v) for k, v in t.items()}, c, 0, I.W_QKV))


def test_f32_nan_stays_nan(tmp_path):
    t = random_tensors(TINY, np.random.default_rng(3))
    t[(O.K_EMBED, -1)][0, :3] = np.array([np.nan, -np.nan, np.float32(np.nan)], np.float32)
    t[(O.K_EMBED, -1)].view(np.uint32)[0, 3] = 0x7F800001  # signalling NaN whose low bits would round away
    path = str(tmp_path / "nan.safetensors")
    write_checkpoint(path, TINY, t, dtype="F32")
    got = I.safetensors_read(path, cfg_of(), 0, I.W_EMBED)[0, :4]
    assert np.all((got & 0x7F80) == 0x7F80) and np.all((got & 0x007F) != 0)


def test_bf16_checkpoint_into_f32_model(tmp_path):
    t = bf16_tensors(4)
    path = str(tmp_path / "b.safetensors")
    write_checkpoint(path, TINY, t)
    c = cfg_of(dict(TINY, dtype="fp32"))
    for kind, layer in ALL:
        got = I.safetensors_read(path, c, layer, kind)
        assert got.dtype == np.float32
        np.testing.assert_array_equal(got, widen(expected(t, c, layer, kind)))


def test_offsets_are_relative_to_the_buffer(tmp_path):
    """Defect D7: offsets count from the end of the header.  A header padded with spaces moves
    the buffer; the tensors must still be found where the offsets say."""
    t = bf16_tensors(5)
    items = []
    for name, kind, layer in hf_names(TINY["n_layers"]):
        items.append((name, "BF16", t[(kind, layer)]))
    header, blobs, at = {}, [], 0
    for name, dt, a in items:
        raw = np.ascontiguousarray(a).tobytes()
        header[name] = {"dtype": dt, "shape": list(a.shape), "data_offsets": [at, at + len(raw)]}
        blobs.append(raw)
        at += len(raw)
    h = header_bytes(header) + b" " * 4096
    path = str(tmp_path / "padded.safetensors")
    write_raw(path, h, b"".join(blobs))
    np.testing.assert_array_equal(I.safetensors_read(path, cfg_of(), 0, I.W_EMBED), t[(O.K_EMBED, -1)])


def test_any_tensor_order(tmp_path):
    """Defect D8: tensors in any order (here reversed) and unrelated tensors of other dtypes."""
    t = bf16_tensors(6)
    items = [(n, "BF16", t[(k, l)]) for n, k, l in hf_names(TINY["n_layers"])][::-1]
    items.insert(3, ("vision_tower.patch.weight", "I32", np.arange(12, dtype=np.int32).reshape(3, 4)))
    path = str(tmp_path / "rev.safetensors")
    write_safetensors(path, items, metadata={"format": "pt"})
    c = cfg_of()
    I.safetensors_check(path, c)
    np.testing.assert_array_equal(I.safetensors_read(path, c, 1, I.W_DOWN), expected(t, c, 1, I.W_DOWN))


@pytest.mark.parametrize("extra,ok", [
    ("model.layers.0.self_attn.rotary_emb.inv_freq", True),   # a buffer, no weights
    ("model.layers.0.self_attn.q_norm.weight", False),         # q/k norms (Gemma 3, Qwen 3)
    ("model.layers.1.pre_feedforward_layernorm.weight", False),
    ("model.layers.0.self_attn.q_proj.bias", False),           # biases (Qwen 2)
    ("model.embed_tokens_per_layer.weight", False),            # per-layer embeddings (Gemma 3n / 4)
])
def test_tensors_of_other_families_are_refused(tmp_path, extra, ok):
    t = bf16_tensors(10)
    items = [(n, "BF16", t[(k, l)]) for n, k, l in hf_names(TINY["n_layers"])]
    items.append((extra, "F32", np.ones(8, np.float32)))
    path = str(tmp_path / "x.safetensors")
    write_safetensors(path, items)
    if ok:
        I.safetensors_check(path, cfg_of())
    else:
        check_code(E_UNSUPPORTED, I.safetensors_check, path, cfg_of(), match=extra)


def test_sharded_index_and_directory(tmp_path):
    t = bf16_tensors(7)
    names = hf_names(TINY["n_layers"])
    half = len(names) // 2
    shards = {"model-00001-of-00002.safetensors": names[:half], "model-00002-of-00002.safetensors": names[half:]}
    wmap = {}
    for fn, part in shards.items():
        write_safetensors(str(tmp_path / fn), [(n, "BF16", t[(k, l)]) for n, k, l in part])
        wmap.update({n: fn for n, _, _ in part})
    with open(tmp_path / "model.safetensors.index.json", "w") as f:
        json.dump({"metadata": {"total_size": 0}, "weight_map": wmap}, f)
    c = cfg_of(tp_size=2, tp_rank=1)
    for path in (str(tmp_path / "model.safetensors.index.json"), str(tmp_path)):
        I.safetensors_check(path, c)
        for kind, layer in ALL:
            np.testing.assert_array_equal(I.safetensors_read(path, c, layer, kind), expected(t, c, layer, kind))
    # an index that puts a tensor in the wrong shard
    name0 = names[0][0]
    wmap[name0] = "model-00002-of-00002.safetensors"
    with open(tmp_path / "bad.index.json", "w") as f:
        json.dump({"weight_map": wmap}, f)
    check_code(E_INVALID, I.safetensors_check, str(tmp_path / "bad.index.json"), c, match=name0)


def test_directory_with_single_file(tmp_path):
    t = bf16_tensors(8)
    write_checkpoint(str(tmp_path / "model.safetensors"), TINY, t)
    I.safetensors_check(str(tmp_path), cfg_of())


# ------------------------------------------------------------------ malformed files
def good_file(tmp_path, name="g.safetensors"):
    t = bf16_tensors(9)
    path = str(tmp_path / name)
    items = write_checkpoint(path, TINY, t)
    return path, items


def header_and_buf(items):
    header, blobs, at = {}, [], 0
    for name, dt, a in items:
        raw = np.ascontiguousarray(a).tobytes()
        header[name] = {"dtype": dt, "shape": list(np.shape(a)), "data_offsets": [at, at + len(raw)]}
        blobs.append(raw)
        at += len(raw)
    return header, b"".join(blobs)


def test_missing_file(tmp_path):
    check_code(E_IO, I.safetensors_check, str(tmp_path / "nope.safetensors"), cfg_of())
    check_code(E_IO, I.safetensors_check, str(tmp_path), cfg_of())  # directory without a checkpoint


def test_short_and_truncated_files(tmp_path):
    path, items = good_file(tmp_path)
    raw = open(path, "rb").read()
    p = str(tmp_path / "x.safetensors")
    open(p, "wb").write(raw[:5])
    check_code(E_INVALID, I.safetensors_check, p, cfg_of(), match="8-byte")
    open(p, "wb").write(raw[:200])  # inside the header
    check_code(E_INVALID, I.safetensors_check, p, cfg_of(), match="truncated")
    open(p, "wb").write(raw[:-100])  # inside the buffer
    check_code(E_INVALID, I.safetensors_check, p, cfg_of())


def test_header_length_limits(tmp_path):
    header, buf = header_and_buf(good_file(tmp_path)[1])
    p = str(tmp_path / "h.safetensors")
    write_raw(p, header_bytes(header), buf, hlen=100_000_001)
    check_code(E_INVALID, I.safetensors_check, p, cfg_of())
    write_raw(p, header_bytes(header), buf, hlen=0)
    check_code(E_INVALID, I.safetensors_check, p, cfg_of())


@pytest.mark.parametrize("text", [b'{"a": ', b'[1, 2]', b'{"x": {"dtype": "BF16"}}', b'{"a" 1}', b'\x00{}'])
def test_malformed_header(tmp_path, text):
    p = str(tmp_path / "m.safetensors")
    write_raw(p, text, b"")
    check_code(E_INVALID, I.safetensors_check, p, cfg_of())


def mutate(tmp_path, fn, name="mut.safetensors"):
    header, buf = header_and_buf(good_file(tmp_path)[1])
    buf = fn(header, buf)
    p = str(tmp_path / name)
    write_raw(p, header_bytes(header) if isinstance(header, dict) else header, buf)
    return p


def test_missing_tensor(tmp_path):
    victim = "model.layers.1.self_attn.k_proj.weight"

    def drop(h, buf):
        b, e = h[victim]["data_offsets"]
        del h[victim]
        for v in h.values():  # close the gap so only the name is missing
            if v["data_offsets"][0] >= e:
                v["data_offsets"] = [v["data_offsets"][0] - (e - b), v["data_offsets"][1] - (e - b)]
        return buf[:b] + buf[e:]
    check_code(E_INVALID, I.safetensors_check, mutate(tmp_path, drop), cfg_of(), match=victim)


def test_shape_mismatch(tmp_path):
    def reshape(h, buf):
        v = h["model.layers.0.mlp.down_proj.weight"]
        v["shape"] = [v["shape"][1], v["shape"][0]]  # same bytes, transposed
        return buf
    check_code(E_CONFIG, I.safetensors_check, mutate(tmp_path, reshape), cfg_of(), match="down_proj")


def test_unsupported_dtype(tmp_path):
    def f16(h, buf):
        h["model.norm.weight"]["dtype"] = "F16"
        return buf
    check_code(E_UNSUPPORTED, I.safetensors_check, mutate(tmp_path, f16), cfg_of(), match="F16")


def test_size_disagrees_with_shape(tmp_path):
    def grow(h, buf):
        h["model.norm.weight"]["shape"] = [TINY["dim"] + 1]
        return buf
    check_code(E_INVALID, I.safetensors_check, mutate(tmp_path, grow), cfg_of(), match="bytes for")


def test_hole_and_overlap(tmp_path):
    def hole(h, buf):
        for v in h.values():
            v["data_offsets"] = [v["data_offsets"][0] + 2, v["data_offsets"][1] + 2]
        return b"\0\0" + buf
    check_code(E_INVALID, I.safetensors_check, mutate(tmp_path, hole, "hole.safetensors"), cfg_of(), match="hole")

    def overlap(h, buf):
        a = h["model.norm.weight"]
        b = h["model.layers.0.input_layernorm.weight"]
        b["data_offsets"] = list(a["data_offsets"])  # two tensors on the same bytes
        return buf
    check_code(E_INVALID, I.safetensors_check, mutate(tmp_path, overlap, "ov.safetensors"), cfg_of())

    def trailing(h, buf):
        return buf + b"\0" * 16
    check_code(E_INVALID, I.safetensors_check, mutate(tmp_path, trailing, "tr.safetensors"), cfg_of())


def test_offsets_past_the_buffer(tmp_path):
    def past(h, buf):
        v = h["lm_head.weight"]
        v["data_offsets"] = [v["data_offsets"][0] + 64, v["data_offsets"][1] + 64]
        return buf
    check_code(E_INVALID, I.safetensors_check, mutate(tmp_path, past), cfg_of())


def test_duplicate_key_and_bad_metadata(tmp_path):
    header, buf = header_and_buf(good_file(tmp_path)[1])
    text = header_bytes(header).rstrip()
    name = "model.norm.weight"
    dup = text[:-1] + b',"' + name.encode() + b'":' + json.dumps(header[name]).encode() + b"}"
    p = str(tmp_path / "dup.safetensors")
    write_raw(p, dup, buf)
    check_code(E_INVALID, I.safetensors_check, p, cfg_of(), match="duplicate")
    header["__metadata__"] = {"format": 1}
    write_raw(p, header_bytes(header), buf)
    check_code(E_INVALID, I.safetensors_check, p, cfg_of(), match="__metadata__")


def test_config_mismatch(tmp_path):
    path, _ = good_file(tmp_path)
    check_code(E_CONFIG, I.safetensors_check, path, cfg_of(dict(TINY, ffn=168)))
    check_code(E_INVALID, I.safetensors_check, path, cfg_of(dict(TINY, n_layers=3)), match="layers.2")


def test_read_argument_checks(tmp_path):
    path, _ = good_file(tmp_path)
    c = cfg_of()
    small = np.empty(4, np.uint16)
    with pytest.raises(I.InfError) as ei:
        I.check(I.lib().inf_safetensors_read(path.encode(), I.C.byref(c), 0, I.W_EMBED, small.ctypes.data_as(I.vp), small.nbytes),
                "read")
    assert ei.value.code == E_INVALID
    check_code(E_INVALID, I.safetensors_read, path, c, TINY["n_layers"], I.W_QKV)
    big = np.empty(1 << 20, np.uint16)
    with pytest.raises(I.InfError) as ei:
        I.check(I.lib().inf_safetensors_read(path.encode(), I.C.byref(c), 0, 99, big.ctypes.data_as(I.vp), big.nbytes),
                "read")
    assert ei.value.code == E_INVALID


def test_model_build_checks_before_the_device(tmp_path):
    """inf_model_build opens and checks the checkpoint before any device work, so a bad file
    fails the same way with or without a GPU."""
    path, _ = good_file(tmp_path)
    p = str(tmp_path / "t.safetensors")
    open(p, "wb").write(open(path, "rb").read()[:300])
    with pytest.raises(I.InfError) as ei:
        I.Engine(cfg_of(), weights_path=p)
    assert ei.value.code == E_INVALID
    with pytest.raises(I.InfError) as ei:
        I.Engine(cfg_of(), weights_path=str(tmp_path / "absent"))
    assert ei.value.code == E_IO


# ------------------------------------------------------------------ config.json
LLAMA3_8B = {"architectures": ["LlamaForCausalLM"], "hidden_act": "silu", "hidden_size": 4096,
             "intermediate_size": 14336, "max_position_embeddings": 8192, "model_type": "llama",
             "num_attention_heads": 32, "num_hidden_layers": 32, "num_key_value_heads": 8, "rms_norm_eps": 1e-05,
             "rope_scaling": None, "rope_theta": 500000.0, "tie_word_embeddings": False, "torch_dtype": "bfloat16",
             "vocab_size": 128256, "attention_bias": False, "mlp_bias": False}


def write_json(tmp_path, obj, name="config.json"):
    p = str(tmp_path / name)
    with open(p, "w") as f:
        f.write(obj if isinstance(obj, str) else json.dumps(obj))
    return p


def test_config_llama3_8b(tmp_path):
    base = I.preset(3)
    c = I.config_from_json(write_json(tmp_path, LLAMA3_8B), I.preset(1))
    for k in ("vocab_size", "dim", "n_layers", "n_heads", "n_kv_heads", "head_dim", "ffn_dim", "dtype"):
        assert getattr(c, k) == getattr(base, k), k
    assert c.rope_theta == 500000.0 and abs(c.norm_eps - 1e-5) < 1e-12
    assert c.max_seq == I.preset(1).max_seq  # never from the file


def test_config_text_config_and_defaults(tmp_path):
    """The reference reads the "text_config" object (src/main.cu:146-157); num_key_value_heads
    defaults to num_attention_heads, head_dim to hidden_size / num_attention_heads."""
    doc = {"vision_config": {"hidden_size": 1}, "text_config": {"hidden_size": 2048, "intermediate_size": 5632,
           "num_attention_heads": 32, "num_hidden_layers": 22, "vocab_size": 32000, "rope_theta": 1e4}}
    c = I.config_from_json(write_json(tmp_path, doc), I.preset(2))
    assert (c.dim, c.n_heads, c.n_kv_heads, c.head_dim, c.n_layers) == (2048, 32, 32, 64, 22)
    doc["text_config"]["head_dim"] = 128
    doc["text_config"]["num_key_value_heads"] = 4
    c = I.config_from_json(write_json(tmp_path, doc), I.preset(2))
    assert (c.head_dim, c.n_kv_heads) == (128, 4)


@pytest.mark.parametrize("doc,code", [
    ("{\"hidden_size\": 4096,", E_INVALID),
    ({"hidden_size": "4096"}, E_INVALID),
    ({"hidden_size": -1}, E_INVALID),
    ({"hidden_size": 4096.5}, E_INVALID),
    ({"num_hidden_layers": 1 << 33}, E_INVALID),
    ({"torch_dtype": "float16"}, E_UNSUPPORTED),
    ({"hidden_act": "gelu"}, E_UNSUPPORTED),
    ({"attention_bias": True}, E_UNSUPPORTED),
    ({"rope_scaling": {"rope_type": "llama3", "factor": 8.0}}, E_UNSUPPORTED),
    ({"model_type": "gemma3_text", "sliding_window": 512}, E_UNSUPPORTED),
    ({"model_type": "gemma3n_text", "altup_num_inputs": 4}, E_UNSUPPORTED),
    ({"model_type": "gemma4_text", "hidden_activation": "silu"}, E_UNSUPPORTED),
    ({"model_type": "gemma4_text", "head_dim": 256, "query_pre_attn_scalar": 224}, E_UNSUPPORTED),
    ({"model_type": "mistral"}, E_UNSUPPORTED),
    ({"hidden_activation": "gelu_pytorch_tanh"}, E_UNSUPPORTED),
    ({"hidden_size": 100, "num_attention_heads": 3}, E_INVALID),
    ("[" * 70 + "]" * 70, E_INVALID),
])
def test_config_errors(tmp_path, doc, code):
    check_code(code, I.config_from_json, write_json(tmp_path, doc), I.preset(1))


def test_config_gemma_e2b_shape(tmp_path):
    """A Gemma-4-E2B-shaped config.json (its text_config, as the reference reads it,
    src/main.cu:139-157) gives the Gemma-style decoder of preset 6: global_head_dim is the head
    dim, hidden_size_per_layer_input the per-layer embedding width."""
    doc = {"model_type": "gemma4", "text_config": {
        "model_type": "gemma4_text", "hidden_size": 1536, "intermediate_size": 6144, "global_head_dim": 512,
        "num_attention_heads": 8, "num_key_value_heads": 2, "vocab_size": 262144, "num_hidden_layers": 35,
        "hidden_size_per_layer_input": 256, "final_logit_softcapping": 30.0, "rms_norm_eps": 1e-6,
        "rope_theta": 1000000.0, "hidden_activation": "gelu_pytorch_tanh", "torch_dtype": "bfloat16"}}
    c = I.config_from_json(write_json(tmp_path, doc), I.preset(3))
    want = I.preset(6)
    for f in ("arch", "dim", "ffn_dim", "head_dim", "n_heads", "n_kv_heads", "vocab_size", "n_layers", "ple_dim",
              "dtype"):
        assert getattr(c, f) == getattr(want, f), f
    assert c.final_softcap == 30.0 and abs(c.norm_eps - 1e-6) < 1e-12 and c.rope_theta == 1e6


def test_config_missing_file(tmp_path):
    check_code(E_IO, I.config_from_json, str(tmp_path / "none.json"), I.preset(1))


def test_json_strings_and_numbers(tmp_path):
    """Escapes (\\u with surrogate pairs) in keys that are ignored, exponents in numbers."""
    text = ('{"_name_or_path": "m\\u00e9ta/\\ud83e\\udd99 \\"llama\\"\\n", "rms_norm_eps": 1E-6, '
            '"rope_theta": 5e5, "hidden_size": 4096, "num_attention_heads": 32}')
    c = I.config_from_json(write_json(tmp_path, text), I.preset(3))
    assert c.rope_theta == 500000.0 and abs(c.norm_eps - 1e-6) < 1e-13 and c.head_dim == 128
    check_code(E_INVALID, I.config_from_json, write_json(tmp_path, '{"a": "\\ud83e"}', "s.json"), I.preset(3))
    check_code(E_INVALID, I.config_from_json, write_json(tmp_path, '{"a": 01}', "n.json"), I.preset(3))


def _gemma_ckpt(tmp_path, drop=None, extra=None):
    from st_files import canon_shape, gemma_names
    cfg = I.preset(6, n_layers=2, vocab_size=256, max_seq=64)
    shape = dict(vocab=256, dim=cfg.dim, n_layers=2, n_heads=cfg.n_heads, n_kv_heads=cfg.n_kv_heads,
                 head_dim=cfg.head_dim, ffn=cfg.ffn_dim, arch=1, ple_dim=cfg.ple_dim)
    rng = np.random.default_rng(0)
    items = [(n, "BF16", bf16_round(rng.standard_normal(canon_shape(shape, k)).astype(np.float32)))
             for n, k, l in gemma_names(2, True) if n != drop]
    items += extra or []
    path = str(tmp_path / "g.safetensors")
    write_safetensors(path, items)
    return cfg, path, {n: a for n, _, a in items}


def test_gemma_checkpoint_names_and_layout(tmp_path):
    """Gemma names map to the device weights: pre_feedforward_layernorm is the MLP's input norm,
    post_attention_layernorm the attention output's; q/k norms are [head_dim]; the per-layer
    embedding tables keep their shapes."""
    cfg, path, t = _gemma_ckpt(tmp_path)
    I.safetensors_check(path, cfg)
    p = "model.language_model.layers.1."
    np.testing.assert_array_equal(I.safetensors_read(path, cfg, 1, 16).view(np.uint16).ravel(),
                                  t[p + "pre_feedforward_layernorm.weight"])
    np.testing.assert_array_equal(I.safetensors_read(path, cfg, 1, 19).view(np.uint16).ravel(),
                                  t[p + "post_attention_layernorm.weight"])
    np.testing.assert_array_equal(I.safetensors_read(path, cfg, 0, 17).view(np.uint16).ravel(),
                                  t["model.language_model.layers.0.self_attn.q_norm.weight"])
    np.testing.assert_array_equal(I.safetensors_read(path, cfg, 0, 3).view(np.uint16).reshape(256, -1),
                                  t["model.language_model.embed_tokens_per_layer.weight"])


@pytest.mark.parametrize("case", ["no_q_norm", "lm_head", "llama_config"])
def test_gemma_checkpoint_errors(tmp_path, case):
    if case == "no_q_norm":
        cfg, path, _ = _gemma_ckpt(tmp_path, drop="model.language_model.layers.1.self_attn.k_norm.weight")
        check_code(E_INVALID, I.safetensors_check, path, cfg)
    elif case == "lm_head":
        cfg, path, _ = _gemma_ckpt(tmp_path, extra=[("lm_head.weight", "BF16", np.zeros((256, 1536), np.uint16))])
        check_code(E_UNSUPPORTED, I.safetensors_check, path, cfg)
    else:  # a Llama config meets Gemma tensors: the extra norms are refused, not ignored
        cfg, path, _ = _gemma_ckpt(tmp_path)
        llama = I.preset(3, n_layers=2, vocab_size=256, dim=cfg.dim, n_heads=8, n_kv_heads=2, head_dim=512,
                         ffn_dim=cfg.ffn_dim)
        import ctypes
        assert I.lib().inf_safetensors_check(path.encode(), ctypes.byref(llama)) in (E_UNSUPPORTED, E_INVALID)
