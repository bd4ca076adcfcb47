"""Tokenizer (tokenizer.bin format, encode / decode, exporter, prompt
templates) against the reference's own tokenizer.h: token ids recorded by
tests/golden/make_tokenizer_golden.py on a seeded synthetic vocabulary.  Host
code only (no GPU)."""
import json
import math
import os
import struct
import sys

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
sys.path.insert(0, os.path.join(HERE, "golden"))
import make_tokenizer_golden as G  # noqa: E402

GOLDEN = json.load(open(os.path.join(HERE, "golden", "tokenizer_cases.json"), encoding="utf-8"))


def _tokmod():
    import importlib.util
    spec = importlib.util.spec_from_file_location("qwen_tokenizer", os.path.join(REPO, "qwen600-rocm-inference_b200", "tokenizer.py"))
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    return m


T = _tokmod()


@pytest.fixture(scope="module")
def model_dir(tmp_path_factory):
    d = str(tmp_path_factory.mktemp("tok"))
    G.write_model_dir(d)
    return d


@pytest.fixture(scope="module")
def tok(model_dir):
    t = T.Tokenizer(os.path.join(model_dir, "tokenizer.bin"))
    yield t
    t.close()


def test_fixture_file_is_the_one_the_golden_ids_came_from(model_dir):
    assert G.sha256(os.path.join(model_dir, "tokenizer.bin")) == GOLDEN["tokenizer_bin_sha256"]


def test_writer_matches_the_format(tmp_path, model_dir):
    pieces, scores, bos, eos = G.build_vocab(0)
    p = str(tmp_path / "tokenizer.bin")
    T.write_tokenizer_bin(p, pieces, scores, bos, eos)
    assert G.sha256(p) == GOLDEN["tokenizer_bin_sha256"]


def test_header(tok):
    assert tok.vocab_size == 151936          # the reference reads VOCAB_SIZE entries
    assert (tok.bos_token_id, tok.eos_token_id) == (GOLDEN["bos"], GOLDEN["eos"])
    pieces, _, _, _ = G.build_vocab(0)
    assert tok.max_token_length == max(len(p) for p in pieces)


@pytest.mark.parametrize("i", range(len(GOLDEN["cases"])))
def test_encode_matches_reference(tok, i):
    case = GOLDEN["cases"][i]
    ids, unk = tok.encode(case["text"], return_unknown=True)
    assert ids == case["ids"]
    assert unk == 0
    assert tok.decode_all(ids) == case["text"].encode("utf-8")


def test_duplicate_entry_resolves_to_lowest_id(tok):
    pieces, _, _, _ = G.build_vocab(0)
    dup = len(pieces) - 1
    assert pieces[dup] == pieces[256]
    assert tok.encode(pieces[256]) == [256]
    assert tok.decode(dup) == pieces[256]


def test_entries_past_the_file_are_empty(tok):
    assert tok.decode(151935) == b""
    assert tok.decode(GOLDEN["entries"]) == b""


def test_errors(tmp_path, model_dir, tok):
    with pytest.raises(T._lib()[0].QwenError) as e:
        T.Tokenizer(str(tmp_path / "missing.bin"))
    assert e.value.code == -2
    p = tmp_path / "short.bin"
    p.write_bytes(b"\x01\x00")
    with pytest.raises(T._lib()[0].QwenError) as e:
        T.Tokenizer(str(p))
    assert e.value.code == -3
    p.write_bytes(struct.pack("<III", 4, 0, 0) + struct.pack("<fI", 0.0, 10) + b"ab")   # entry cut short
    with pytest.raises(T._lib()[0].QwenError) as e:
        T.Tokenizer(str(p))
    assert e.value.code == -3
    with pytest.raises(T._lib()[0].QwenError) as e:
        tok.decode(151936)
    assert e.value.code == -1


def test_unknown_bytes_are_skipped_and_counted(tmp_path):
    pieces = [b"a", b"b", b"ab"]
    p = str(tmp_path / "tokenizer.bin")
    T.write_tokenizer_bin(p, pieces, [-1e6, -1e6, 0.0], 0, 1)
    t = T.Tokenizer(p, vocab_size=3)
    ids, unk = t.encode("zabz b", return_unknown=True)
    assert ids == [2, 1] and unk == 3
    t.close()


def test_merge_order_follows_scores(tmp_path):
    # "abc": pair scores ab -> -1, bc -> 0 (higher): bc merges first, then a+bc
    pieces = [b"a", b"b", b"c", b"ab", b"bc", b"abc"]
    scores = [-1e6, -1e6, -1e6, -1.0, 0.0, -2.0]
    p = str(tmp_path / "tokenizer.bin")
    T.write_tokenizer_bin(p, pieces, scores, 0, 1)
    t = T.Tokenizer(p, vocab_size=len(pieces))
    assert t.encode("abc") == [5]
    assert t.encode("abab") == [3, 3]
    assert t.encode("bcab") == [4, 3]
    t.close()


def test_export_from_tokenizer_json(tmp_path):
    b2u = T.bytes_to_unicode()
    assert len(set(b2u.values())) == 256 and b2u[ord(" ")] == "Ġ" and b2u[ord("a")] == "a"
    sp = b2u[ord(" ")]
    tj = {"model": {"vocab": {"a": 0, "b": 1, sp: 2, "ab": 3, sp + "ab": 4}, "merges": ["a b", sp + " ab"]},
          "added_tokens": [{"id": 5, "content": "<|x|>"}]}
    jp = tmp_path / "tokenizer.json"
    jp.write_text(json.dumps(tj), encoding="utf-8")
    out = str(tmp_path / "tokenizer.bin")
    assert T.export_from_tokenizer_json(str(jp), 5, 5, out) == 6
    raw = open(out, "rb").read()
    assert struct.unpack_from("<III", raw, 0) == (5, 5, 5)     # longest token: "<|x|>" (5 characters)
    t = T.Tokenizer(out, vocab_size=6)
    assert [t.decode(i) for i in range(6)] == [b"a", b"b", b" ", b"ab", b" ab", b"<|x|>"]
    assert t.encode(" ab<|x|>") == [4, 5]
    t.close()
    # scores: merge rank r -> -log(r + 1); others -1e6
    off, sc = 12, []
    for _ in range(6):
        s, n = struct.unpack_from("<fI", raw, off)
        sc.append(s)
        off += 8 + n
    assert sc[3] == 0.0 and abs(sc[4] + 0.6931472) < 1e-6 and sc[0] == sc[5] == pytest.approx(-1e6)


def test_export_duplicate_merge_takes_last_rank(tmp_path):
    """Two merges that produce the same string ("a bc" and "ab c" both give
    "abc"): the score comes from the later one, rank 2 -> -log(3), the way
    export.py:186's dict comprehension keeps the last rank."""
    tj = {"model": {"vocab": {"a": 0, "b": 1, "c": 2, "ab": 3, "bc": 4, "abc": 5},
                    "merges": ["b c", "a bc", "ab c", "a b"]}}
    jp = tmp_path / "tokenizer.json"
    jp.write_text(json.dumps(tj), encoding="utf-8")
    out = str(tmp_path / "tokenizer.bin")
    assert T.export_from_tokenizer_json(str(jp), 0, 0, out) == 6
    raw = open(out, "rb").read()
    off, sc = 12, []
    for _ in range(6):
        s, n = struct.unpack_from("<fI", raw, off)
        sc.append(s)
        off += 8 + n
    assert sc[5] == pytest.approx(-math.log(3))      # "abc": rank 2 ("ab c"), not rank 1
    assert sc[3] == pytest.approx(-math.log(4))      # "ab": rank 3
    assert sc[4] == 0.0                              # "bc": rank 0


def test_templates(model_dir):
    user, system = T.load_templates(model_dir, enable_thinking=False)
    assert T.render(user, "hi") == "<|start|>user\nhi<|end|>\n<|start|>assistant\n"
    assert T.render(system, "S", "U").startswith("<|start|>system\nS<|end|>\n<|start|>user\nU")
    user_t, _ = T.load_templates(model_dir, enable_thinking=True)
    assert T.render(user_t, "q").endswith("<think>\n")
    assert T.render("100%% %s", "x") == "100% x"
    with pytest.raises(ValueError):
        T.render("%s %s", "one")
