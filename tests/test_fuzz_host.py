"""Seeded fuzzing of the host-side parsers in libinf.so: corrupted safetensors headers and
buffers, corrupted config.json and tokenizer.json files, and random byte strings (invalid UTF-8
included) through the tokenizer.  Every case must end in a result or an Error_t -- a crash here
would take the process down."""
import json
import os
import struct

import numpy as np
import pytest

import infb200 as I
from st_files import TINY, bf16_round, random_tensors, write_checkpoint

HERE = os.path.dirname(os.path.abspath(__file__))
TOK = os.path.join(HERE, "golden", "tokenizer_synth.json")


def mutate(raw: bytes, rng, n_edits: int) -> bytes:
    b = bytearray(raw)
    for _ in range(n_edits):
        op = rng.integers(0, 4)
        i = int(rng.integers(0, max(1, len(b))))
        if op == 0 and b:
            b[i % len(b)] = int(rng.integers(0, 256))
        elif op == 1:
            b.insert(i, int(rng.integers(0, 256)))
        elif op == 2 and b:
            del b[i % len(b)]
        else:
            b[i:i] = bytes(rng.choice([b'"', b"{", b"}", b"[", b"]", b",", b":", b"\\", b"-1", b"1e99", b"\\u00"]))
    return bytes(b)


def test_safetensors_header_fuzz(tmp_path):
    cfg = I.config_from_dict(TINY)
    path = str(tmp_path / "good.safetensors")
    t = {k: bf16_round(v) for k, v in random_tensors(TINY, np.random.default_rng(0)).items()}
    write_checkpoint(path, TINY, t)
    raw = open(path, "rb").read()
    hlen = struct.unpack("<Q", raw[:8])[0]
    header, buf = raw[8:8 + hlen], raw[8 + hlen:]
    rng = np.random.default_rng(1)
    p = str(tmp_path / "f.safetensors")
    outcomes = set()
    for trial in range(300):
        h = mutate(header, rng, int(rng.integers(1, 6)))
        body = buf if trial % 3 else mutate(buf[:4096], rng, 3) + buf[4096:]
        with open(p, "wb") as f:
            f.write(struct.pack("<Q", len(h) if trial % 7 else int(rng.integers(0, 1 << 40))))
            f.write(h)
            f.write(body)
        try:
            I.safetensors_check(p, cfg)
            outcomes.add(0)
        except I.InfError as e:
            outcomes.add(e.code)
    assert outcomes - {0}  # the corruptions are caught


def test_json_files_fuzz(tmp_path):
    rng = np.random.default_rng(2)
    cfg_doc = json.dumps({"text_config": {"hidden_size": 64, "num_attention_heads": 4, "num_key_value_heads": 2,
                                          "intermediate_size": 160, "vocab_size": 512, "num_hidden_layers": 2,
                                          "rms_norm_eps": 1e-5, "rope_theta": 1e4, "torch_dtype": "bfloat16"}}).encode()
    tok_doc = open(TOK, "rb").read()[:20000]  # a prefix: malformed by construction, then mutated
    p = str(tmp_path / "c.json")
    for trial in range(300):
        with open(p, "wb") as f:
            f.write(mutate(cfg_doc, rng, int(rng.integers(1, 8))))
        try:
            I.config_from_json(p, I.preset(1))
        except I.InfError as e:
            assert e.code in (4, 14, 15)
        with open(p, "wb") as f:
            f.write(mutate(tok_doc, rng, int(rng.integers(1, 8))))
        try:
            I.Tokenizer(p).close()
        except I.InfError as e:
            assert e.code in (4, 14, 15)


def test_tokenizer_random_bytes():
    rng = np.random.default_rng(3)
    with I.Tokenizer(TOK) as tok:
        for _ in range(500):
            n = int(rng.integers(1, 200))
            raw = bytes(int(x) for x in rng.integers(1, 256, n))  # no NUL: the C string ends there
            ids = tok.encode(raw)  # byte fallback covers every byte
            assert all(0 <= int(i) < tok.vocab_size for i in ids)
            back = tok.decode_bytes(ids)
            # a final space ends the text; a space after another one is an empty word's "▁"
            assert back == (raw[:-1] if raw.endswith(b" ") else raw)
