"""A model loaded from a safetensors checkpoint is the model built from synthetic weights when
the checkpoint holds those weights: the checkpoint is written here from the oracle's Philox
streams (the canonical Hugging Face tensors, before the device layout), loaded through
inf_model_build, and its logits and greedy ids must equal the synthetic model's bit for bit.
A BF16 checkpoint, an F32 one (rounded to bf16 on the way in) and a sharded one with the
reference's "model.language_model." names all give the same model."""
import json
import time

import numpy as np
import pytest

import infb200 as I
import oracle as O
from st_files import hf_names, synthetic_tensors, write_checkpoint, write_safetensors

pytestmark = pytest.mark.gpu

SEED = 11


def shape_of(c) -> dict:
    return dict(vocab=c.vocab_size, dim=c.dim, n_layers=c.n_layers, n_heads=c.n_heads, n_kv_heads=c.n_kv_heads,
                head_dim=c.head_dim, ffn=c.ffn_dim, arch=c.arch, ple_dim=c.ple_dim)


def run(cfg, prompt, weights_path=None):
    with I.Engine(cfg, seed=SEED, weights_path=weights_path) as eng:
        lg, am = eng.forward(prompt, 0)
        ids, _ = eng.generate(prompt, 8)
    return lg, am, ids


@pytest.mark.parametrize("preset,layers,vocab", [(2, 2, 8192), (3, 1, 8192)])
def test_checkpoint_equals_synthetic_bf16(cuda, tmp_path, preset, layers, vocab):
    cfg = I.preset(preset, n_layers=layers, vocab_size=vocab, max_seq=256)
    shape = shape_of(cfg)
    t = synthetic_tensors(shape, SEED, cfg.init_std, bf16=True)
    prompt = O.gen_ids(3, 37, vocab)
    want = run(cfg, prompt)
    for dtype in ("BF16", "F32"):
        path = str(tmp_path / f"m_{dtype}.safetensors")
        write_checkpoint(path, shape, t, dtype=dtype)
        t0 = time.perf_counter()
        got = run(cfg, prompt, path)
        dt = time.perf_counter() - t0
        np.testing.assert_array_equal(got[0], want[0], err_msg=dtype)
        assert got[1] == want[1]
        np.testing.assert_array_equal(got[2], want[2])
        print(f"preset {preset} {dtype}: load + forward + 8 tokens {dt:.2f} s")


def test_checkpoint_sharded_language_model_names(cuda, tmp_path):
    cfg = I.preset(2, n_layers=2, vocab_size=4096, max_seq=128)
    shape = shape_of(cfg)
    t = synthetic_tensors(shape, SEED, cfg.init_std, bf16=True)
    names = hf_names(shape["n_layers"], prefix="model.language_model.")
    wmap = {}
    for i, part in enumerate((names[:7], names[7:])):
        fn = f"model-{i + 1:05d}-of-00002.safetensors"
        write_safetensors(str(tmp_path / fn), [(n, "BF16", t[(k, l)]) for n, k, l in part])
        wmap.update({n: fn for n, _, _ in part})
    with open(tmp_path / "model.safetensors.index.json", "w") as f:
        json.dump({"metadata": {}, "weight_map": wmap}, f)
    prompt = O.gen_ids(4, 21, shape["vocab"])
    want = run(cfg, prompt)
    got = run(cfg, prompt, str(tmp_path))
    np.testing.assert_array_equal(got[0], want[0])
    np.testing.assert_array_equal(got[2], want[2])


def test_checkpoint_fp32_model(cuda, tmp_path):
    cfg = I.preset(1, max_seq=64)
    shape = shape_of(cfg)
    t = synthetic_tensors(shape, SEED, cfg.init_std, bf16=False)
    path = str(tmp_path / "f32.safetensors")
    write_checkpoint(path, shape, t, dtype="F32")
    prompt = O.gen_ids(5, 9, shape["vocab"])
    want = run(cfg, prompt)
    got = run(cfg, prompt, path)
    np.testing.assert_array_equal(got[0], want[0])
    np.testing.assert_array_equal(got[2], want[2])


def test_gemma_checkpoint_equals_synthetic(cuda, tmp_path):
    """The Gemma-style decoder from a checkpoint with Gemma names (q/k norms, the four norms of a
    layer, per-layer embeddings, tied LM head) equals the synthetic model of the same seed."""
    cfg = I.preset(6, n_layers=2, vocab_size=2048, max_seq=128)
    shape = shape_of(cfg)
    t = synthetic_tensors(shape, SEED, cfg.init_std, bf16=True)
    path = str(tmp_path / "gemma.safetensors")
    write_checkpoint(path, shape, t, dtype="BF16", prefix="model.language_model.")
    I.safetensors_check(path, cfg)
    prompt = O.gen_ids(6, 11, shape["vocab"])
    want = run(cfg, prompt)
    got = run(cfg, prompt, path)
    np.testing.assert_array_equal(got[0], want[0])
    assert got[1] == want[1]
    np.testing.assert_array_equal(got[2], want[2])
