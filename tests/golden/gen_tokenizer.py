"""Generate the tokenizer fixtures under tests/golden/ with the reference's own tokenizer.

1. tokenizer_synth.json: a synthetic Hugging Face BPE tokenizer.json (no real tokenizer can be
   downloaded here): merges learned by plain BPE training (most frequent adjacent pair, ties to
   the smallest pair) on a seeded corpus of pseudo-words over an alphabet with 1-, 2-, 3- and
   4-byte UTF-8 characters, with the reference's pre-tokenization (words split at ' ', "▁"
   before every word but the first).  The vocabulary holds four special tokens, the 256
   <0xXX> byte tokens, every character, every merge result and a 20 x "▁" token (its length
   also sizes the reference's pair buffer, which is as long as the longest vocabulary token,
   src/tokenizer.c:95-101 and 216, above any pair the texts here form).
2. tokenizer_golden.json: texts and the ids the reference's tokenizer_encode
   (src/tokenizer.c:39-183, compiled from its sources into oracle/_ref/libref_tokenizer.so by
   `make -C oracle ref`) gives for them.  Only texts the reference handles without undefined
   behaviour: no leading space (its piece loop runs to UINT32_MAX, src/tokenizer.c:104) and
   every character in the vocabulary (it drops unknown pieces, defect D13).

Run:  make -C oracle ref && python tests/golden/gen_tokenizer.py
"""
from __future__ import annotations

import ctypes as C
import json
import os
import sys
from collections import Counter

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
SP = "▁"

ALPHABET = (list("etaoinshrdlucmfwypvbgkqjxz") + list("ETAOINS") + list("0123456789") + list(".,;:!?'-()\"")
            + ["é", "ß", "ñ", "ü", "中", "文", "字", "🦙", "🚀"])


def make_lexicon(rng: np.random.Generator, n: int = 2500) -> list[str]:
    w = np.array([1.0 / (i + 1) ** 0.8 for i in range(len(ALPHABET))])
    w /= w.sum()
    lex = set()
    while len(lex) < n:
        k = int(rng.integers(1, 11))
        lex.add("".join(rng.choice(ALPHABET, size=k, p=w)))
    return sorted(lex)


def zipf_words(rng: np.random.Generator, lex: list[str], n: int) -> list[str]:
    p = np.array([1.0 / (i + 1) for i in range(len(lex))])
    p /= p.sum()
    return [lex[i] for i in rng.choice(len(lex), size=n, p=p)]


def train_bpe(words: list[str], n_merges: int):
    seqs = Counter()
    for i, w in enumerate(words):
        seqs[tuple(w if i % 50 == 0 else SP + w)] += 1  # characters; one word in 50 starts a text (no "▁")
    merges = []
    for _ in range(n_merges):
        pairs = Counter()
        for s, c in seqs.items():
            for a, b in zip(s, s[1:]):
                pairs[(a, b)] += c
        if not pairs:
            break
        best = min(pairs.items(), key=lambda kv: (-kv[1], kv[0]))[0]  # most frequent, then smallest
        merges.append(best)
        new = {}
        for s, c in seqs.items():
            out, i = [], 0
            while i < len(s):
                if i + 1 < len(s) and s[i] == best[0] and s[i + 1] == best[1]:
                    out.append(s[i] + s[i + 1])
                    i += 2
                else:
                    out.append(s[i])
                    i += 1
            t = tuple(out)
            new[t] = new.get(t, 0) + c
        seqs = new
    return merges


def build_tokenizer(rng) -> tuple[dict, list[str]]:
    lex = make_lexicon(rng)
    merges = train_bpe(zipf_words(rng, lex, 40000), 700)
    vocab = {"<pad>": 0, "<eos>": 1, "<bos>": 2, "<unk>": 3}
    for b in range(256):
        vocab[f"<0x{b:02X}>"] = len(vocab)
    for ch in [SP] + ALPHABET:
        vocab.setdefault(ch, len(vocab))
    for a, b in merges:
        vocab.setdefault(a + b, len(vocab))
    vocab.setdefault(SP * 20, len(vocab))
    tok = {
        "version": "1.0",
        "added_tokens": [{"id": i, "content": s, "special": True} for s, i in list(vocab.items())[:4]]
        + [{"id": len(vocab), "content": "<start_of_turn>", "special": True}],
        "model": {"type": "BPE", "dropout": None, "unk_token": "<unk>", "byte_fallback": True,
                  "vocab": vocab, "merges": [[a, b] for a, b in merges]},
    }
    return tok, lex


def texts(rng, lex: list[str]) -> list[str]:
    out = ["", "a", "e", "é", "🦙🦙🦙", "the end", "a  b", "trailing ", "x   y  z"]
    for _ in range(120):  # sentences
        n = int(rng.integers(1, 40))
        out.append(" ".join(zipf_words(rng, lex, n)))
    for _ in range(30):  # long unspaced runs
        n = int(rng.integers(20, 200))
        out.append("".join(zipf_words(rng, lex, n)))
    for _ in range(30):  # random characters, random spacing (never a leading space)
        n = int(rng.integers(1, 300))
        s = "".join(rng.choice(ALPHABET + [" "] * 6, size=n))
        out.append(s.lstrip(" "))
    return out


class RefTokenizer:
    """The reference's tokenizer through oracle/ref_tokenizer_shim.c."""

    def __init__(self, path: str, lib_path: str):
        self.L = C.CDLL(lib_path)
        self.L.ref_tok_create.argtypes = [C.c_char_p]
        self.L.ref_tok_create.restype = C.c_int
        self.L.ref_tok_encode.argtypes = [C.c_int, C.c_char_p, C.c_void_p, C.c_long]
        self.L.ref_tok_encode.restype = C.c_long
        self.L.ref_tok_destroy.argtypes = [C.c_int]
        self.h = self.L.ref_tok_create(os.fsencode(path))
        assert self.h >= 0

    def encode(self, text: str) -> list[int]:
        raw = text.encode()
        out = np.zeros(len(raw) + 1, dtype=np.uint32)
        n = self.L.ref_tok_encode(self.h, raw, out.ctypes.data, out.size)
        assert 0 <= n <= out.size
        return out[:n].tolist()

    def close(self):
        self.L.ref_tok_destroy(self.h)


def main() -> int:
    lib = os.path.join(ROOT, "oracle", "_ref", "libref_tokenizer.so")
    if not os.path.exists(lib):
        print("build the reference tokenizer first: make -C oracle ref", file=sys.stderr)
        return 1
    rng = np.random.default_rng(20261202)
    tok, lex = build_tokenizer(rng)
    tok_path = os.path.join(HERE, "tokenizer_synth.json")
    with open(tok_path, "w", encoding="utf-8") as f:
        json.dump(tok, f, ensure_ascii=False, separators=(",", ":"))
    ref = RefTokenizer(tok_path, lib)
    cases = [{"text": t, "ids": ref.encode(t)} for t in texts(rng, lex)]
    ref.close()
    with open(os.path.join(HERE, "tokenizer_golden.json"), "w", encoding="utf-8") as f:
        json.dump({"tokenizer": "tokenizer_synth.json", "cases": cases}, f, ensure_ascii=False, separators=(",", ":"))
    print(f"{len(tok['model']['vocab'])} pieces, {len(tok['model']['merges'])} merges, {len(cases)} cases")
    return 0


if __name__ == "__main__":
    sys.exit(main())
