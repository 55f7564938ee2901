"""The host tokenizer (inf_tokenizer_*) against the reference's own tokenizer_encode
(src/tokenizer.c:39-183): the committed golden ids (tests/golden/gen_tokenizer.py ran the
reference, compiled from its sources, on a synthetic BPE tokenizer.json) and, where
oracle/_ref/libref_tokenizer.so is built, the live reference on further seeded texts.  Then the
deliberate differences (byte fallback for unknown pieces instead of dropping them, defect D13;
a leading space), the decoder the reference declares but never defines (src/tokenizer.h:38),
and malformed files."""
import json
import os

import numpy as np
import pytest

import infb200 as I

HERE = os.path.dirname(os.path.abspath(__file__))
GOLD = os.path.join(HERE, "golden")
TOK = os.path.join(GOLD, "tokenizer_synth.json")
REF_LIB = os.path.join(os.path.dirname(HERE), "oracle", "_ref", "libref_tokenizer.so")
SP = "▁"
E_IO, E_INVALID, E_TOKEN, E_UNSUPPORTED = 14, 4, 10, 15


@pytest.fixture(scope="module")
def tok():
    t = I.Tokenizer(TOK)
    yield t
    t.close()


@pytest.fixture(scope="module")
def spec():
    with open(TOK, encoding="utf-8") as f:
        return json.load(f)


def test_golden_ids_from_the_reference(tok):
    with open(os.path.join(GOLD, "tokenizer_golden.json"), encoding="utf-8") as f:
        cases = json.load(f)["cases"]
    assert len(cases) > 100
    for c in cases:
        np.testing.assert_array_equal(tok.encode(c["text"]), np.array(c["ids"], np.uint32), err_msg=repr(c["text"]))


def seeded_texts(spec, n, seed):
    """Texts over the vocabulary's characters with random spacing (no leading space)."""
    rng = np.random.default_rng(seed)
    chars = [p for p in spec["model"]["vocab"] if len(p) == 1 and p != SP]
    words = [p.replace(SP, "") for p in spec["model"]["vocab"] if len(p) > 1 and not p.startswith("<")]
    words = [w for w in words if w]
    out = []
    for _ in range(n):
        kind = rng.integers(0, 3)
        if kind == 0:
            s = " ".join(rng.choice(words, size=int(rng.integers(1, 60))))
        elif kind == 1:
            s = "".join(rng.choice(words, size=int(rng.integers(1, 400))))
        else:
            s = "".join(rng.choice(chars + [" "] * 5, size=int(rng.integers(1, 500))))
        out.append(s.lstrip(" "))
    return out


@pytest.mark.skipif(not os.path.exists(REF_LIB), reason="reference tokenizer not built (make -C oracle ref)")
def test_live_reference_on_seeded_texts(tok, spec):
    import sys
    sys.path.insert(0, GOLD)
    from gen_tokenizer import RefTokenizer
    ref = RefTokenizer(TOK, REF_LIB)
    try:
        for s in seeded_texts(spec, 300, 7):
            np.testing.assert_array_equal(tok.encode(s), np.array(ref.encode(s), np.uint32), err_msg=repr(s))
    finally:
        ref.close()


def decode_expect(s: str) -> str:
    """What decode(encode(s)) gives back: a final space ends the text and is dropped."""
    return s[:-1] if s.endswith(" ") else s


def test_round_trip(tok, spec):
    for s in seeded_texts(spec, 200, 8) + ["", "a", "a  b", " lead", "  two lead", "tail  ", "é中🦙 x"]:
        assert tok.decode(tok.encode(s)) == decode_expect(s), repr(s)


def test_leading_space_is_an_empty_word(tok):
    """The reference indexes past its piece array for a leading space; here the empty first
    word produces nothing and the next word carries its "▁"."""
    assert list(tok.encode(" e")) == list(tok.encode("a e"))[len(tok.encode("a")):]


def test_unknown_characters_fall_back_to_bytes(tok, spec):
    """Defect D13: the reference drops pieces outside the vocabulary (and still counts them);
    with byte_fallback they become their UTF-8 bytes as <0xXX> tokens."""
    vocab = spec["model"]["vocab"]
    ids = tok.encode("aω")  # U+03C9 is not in the vocabulary
    want_tail = [vocab["<0xCF>"], vocab["<0x89>"]]
    assert list(ids[-2:]) == want_tail
    assert tok.decode(ids) == "aω"
    ids = tok.encode("x \U0001F600")  # a 4-byte character after a space: "▁" stays a piece
    assert tok.decode(ids) == "x \U0001F600"


def write_spec(tmp_path, spec, name="t.json"):
    p = str(tmp_path / name)
    with open(p, "w", encoding="utf-8") as f:
        f.write(spec if isinstance(spec, str) else json.dumps(spec, ensure_ascii=False))
    return p


def test_unk_and_no_fallback(tmp_path, spec):
    s = json.loads(json.dumps(spec))
    s["model"]["byte_fallback"] = False
    with I.Tokenizer(write_spec(tmp_path, s)) as t:
        assert list(t.encode("aω"))[-1] == spec["model"]["vocab"]["<unk>"]
    s["model"]["unk_token"] = None
    with I.Tokenizer(write_spec(tmp_path, s, "n.json")) as t:
        with pytest.raises(I.InfError) as ei:
            t.encode("aω")
        assert ei.value.code == E_INVALID and "ω" in str(ei.value)


def test_legacy_string_merges(tmp_path, spec, tok):
    s = json.loads(json.dumps(spec))
    s["model"]["merges"] = [f"{a} {b}" for a, b in spec["model"]["merges"]]
    with I.Tokenizer(write_spec(tmp_path, s)) as t:
        for text in seeded_texts(spec, 50, 9):
            np.testing.assert_array_equal(t.encode(text), tok.encode(text))


def test_merge_order_is_rank_not_frequency(tmp_path):
    """Hand-built: ranks decide, all occurrences of the best pair merge in one left-to-right
    round, a pair a round creates waits for the next round."""
    vocab = {c: i for i, c in enumerate(["a", "b", "c", "ab", "bc", "abc", "aa", "aaa", "aaaa", SP])}
    merges = [["a", "a"], ["b", "c"], ["a", "b"], ["a", "bc"], ["aa", "aa"], ["aa", "a"]]
    spec = {"model": {"type": "BPE", "vocab": vocab, "merges": merges}}
    import tempfile
    with tempfile.TemporaryDirectory() as d:
        with I.Tokenizer(write_spec(__import__("pathlib").Path(d), spec)) as t:
            enc = lambda s: [list(vocab)[i] for i in t.encode(s)]
            assert enc("abc") == ["abc"]          # (b,c) rank 1 before (a,b) rank 2, then (a,bc)
            assert enc("aaa") == ["aaa"]          # first merge pass: (a,a) at 0 only -> aa a; second: (aa,a)
            assert enc("aaaa") == ["aaaa"]        # (a,a) twice in one round, then (aa,aa)
            assert enc("aaaaa") == ["aaaa", "a"]  # first pass: aa aa a; second: (aa,aa) rank 4 < (aa,a) rank 5


def test_buffers_and_counts(tok):
    n = I.u64()
    with pytest.raises(I.InfError) as ei:
        small = np.zeros(1, np.uint32)
        I.check(I.lib().inf_tokenizer_encode(tok.h, b"the end of it", small.ctypes.data_as(I.vp), 1, I.C.byref(n)), "enc")
    assert ei.value.code == E_INVALID and n.value == len(tok.encode("the end of it"))
    ids = tok.encode("the end")
    with pytest.raises(I.InfError) as ei:
        buf = I.C.create_string_buffer(3)
        I.check(I.lib().inf_tokenizer_decode(tok.h, ids.ctypes.data_as(I.vp), ids.size, buf, 3, I.C.byref(n)), "dec")
    assert ei.value.code == E_INVALID and n.value == len("the end")
    with pytest.raises(I.InfError) as ei:
        tok.decode([tok.vocab_size + 5])
    assert ei.value.code == E_TOKEN


def test_added_tokens_decode(tok, spec):
    added = {a["content"]: a["id"] for a in spec["added_tokens"]}
    assert tok.vocab_size == max(added.values()) + 1
    assert tok.decode([added["<start_of_turn>"], spec["model"]["vocab"]["e"]]) == "<start_of_turn>e"
    assert tok.decode_bytes([spec["model"]["vocab"]["<0x41>"]]) == b"A"


@pytest.mark.parametrize("doc,code", [
    ("{", E_INVALID),
    ({"version": "1.0"}, E_INVALID),
    ({"model": {"vocab": [], "merges": []}}, E_INVALID),
    ({"model": {"vocab": {"a": 0}}}, E_INVALID),
    ({"model": {"vocab": {"a": -1}, "merges": []}}, E_INVALID),
    ({"model": {"vocab": {"a": 0}, "merges": [["a"]]}}, E_INVALID),
    ({"model": {"vocab": {"a": 0}, "merges": ["ab"]}}, E_INVALID),
    ({"model": {"type": "Unigram", "vocab": {"a": 0}, "merges": []}}, E_UNSUPPORTED),
    ({"pre_tokenizer": {"type": "ByteLevel", "add_prefix_space": False},
      "model": {"type": "BPE", "vocab": {"a": 0}, "merges": []}}, E_UNSUPPORTED),
    ({"pre_tokenizer": {"type": "Sequence", "pretokenizers": [{"type": "Split"}, {"type": "ByteLevel"}]},
      "model": {"type": "BPE", "vocab": {"a": 0}, "merges": []}}, E_UNSUPPORTED),
])
def test_malformed_tokenizer_json(tmp_path, doc, code):
    with pytest.raises(I.InfError) as ei:
        I.Tokenizer(write_spec(tmp_path, doc))
    assert ei.value.code == code


def test_missing_tokenizer_file(tmp_path):
    with pytest.raises(I.InfError) as ei:
        I.Tokenizer(str(tmp_path / "none.json"))
    assert ei.value.code == E_IO


def test_long_unspaced_text_is_fast(tok, spec):
    """A 200,000-character word (no spaces): the heap-ordered merge rounds keep it fast; the
    reference rescans the word every round."""
    import time
    s = "".join(seeded_texts(spec, 1, 10)[0].split(" ")) * 1
    s = (s * (200_000 // max(1, len(s)) + 1))[:200_000]
    t0 = time.perf_counter()
    ids = tok.encode(s)
    assert time.perf_counter() - t0 < 5.0
    assert tok.decode(ids) == s


def test_special_tokens_are_cut_out_when_asked(tok, spec):
    """inf_tokenizer_encode_special: added tokens marked special match whole (longest first) and
    each text piece between them encodes as a whole text; the plain encode (the reference's)
    splits them into characters."""
    added = {a["content"]: a["id"] for a in spec["added_tokens"]}
    sot, bos = added["<start_of_turn>"], added["<bos>"]
    text = "<bos><start_of_turn>the end<start_of_turn> a b"
    got = list(tok.encode(text, special=True))
    want = [bos, sot] + list(tok.encode("the end")) + [sot] + list(tok.encode(" a b"))
    assert got == want
    assert sot not in list(tok.encode(text))  # the reference's encoding has no special tokens
    assert list(tok.encode("no specials here", special=True)) == list(tok.encode("no specials here"))
    assert tok.decode(got) == text
