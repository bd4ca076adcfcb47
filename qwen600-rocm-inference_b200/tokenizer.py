"""Tokenizer of the chat driver: the reference's tokenizer.bin format and its
encode / decode, plus the exporter that writes the format.

    tok = Tokenizer("model_dir/tokenizer.bin")
    ids = tok.encode("text")          # tokenizer.h:104-185, through qwen_tokenizer_encode
    tok.decode(ids[0])                # tokenizer.h:80-82 -> bytes
    user_t, system_t = load_templates("model_dir", enable_thinking=False)
    render(user_t, "question")        # main.cu:129-131 (sprintf with %s)

Format (export.py:168-212 writes it, tokenizer.h:38-70 reads it), little
endian: u32 max_token_length, u32 bos_token_id, u32 eos_token_id, then for
every token id in order: f32 merge score, u32 byte length, the bytes.
Scores: a token that is the result of BPE merge rank r scores -log(r + 1), any
other token -1e6 (export.py:186-197); encode merges the highest-scoring pair
first, so merges apply in rank order.
"""
import ctypes
import json
import math
import os
import struct

import importlib.util

HERE = os.path.dirname(os.path.abspath(__file__))


def _qb():
    spec = importlib.util.spec_from_file_location("qwen_b200", os.path.join(HERE, "qwen_b200.py"))
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    return m


_QB = None


def _lib():
    global _QB
    if _QB is None:
        _QB = _qb()
    return _QB, _QB.load_library()


class Tokenizer:
    """A loaded tokenizer.bin (qwen_tokenizer_load); vocab_size <= 0 reads the
    model's 151936 entries, as the reference does."""

    def __init__(self, path, vocab_size=0):
        qb, lib = _lib()
        self._qb, self._lib = qb, lib
        h = ctypes.c_void_p()
        qb._check(lib.qwen_tokenizer_load(os.fsencode(path), int(vocab_size), ctypes.byref(h)))
        self._h = h
        v, m, b, e = (ctypes.c_int() for _ in range(4))
        qb._check(lib.qwen_tokenizer_info(h, ctypes.byref(v), ctypes.byref(m), ctypes.byref(b), ctypes.byref(e)))
        self.vocab_size, self.max_token_length, self.bos_token_id, self.eos_token_id = v.value, m.value, b.value, e.value

    def encode(self, text, return_unknown=False):
        """Token ids of `text` (str: UTF-8 encoded; or bytes without NUL).  Bytes
        with no one-byte entry are skipped; return_unknown=True also returns
        their count."""
        data = text.encode("utf-8") if isinstance(text, str) else bytes(text)
        cap = len(data) + 1
        buf = (ctypes.c_int * cap)()
        n, unk = ctypes.c_int(), ctypes.c_int()
        self._qb._check(self._lib.qwen_tokenizer_encode(self._h, data, buf, cap, ctypes.byref(n), ctypes.byref(unk)))
        ids = list(buf[:n.value])
        return (ids, unk.value) if return_unknown else ids

    def decode(self, token):
        """The token's bytes (a C string: up to its first NUL)."""
        p = ctypes.c_char_p()
        self._qb._check(self._lib.qwen_tokenizer_decode(self._h, int(token), ctypes.byref(p)))
        return p.value

    def decode_all(self, ids):
        return b"".join(self.decode(t) for t in ids)

    def close(self):
        if self._h:
            self._lib.qwen_tokenizer_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ---------------------------------------------------------------------------
# writing the format (export.py:168-212)
# ---------------------------------------------------------------------------
def write_tokenizer_bin(path, pieces, scores, bos_token_id, eos_token_id, max_token_length=None):
    """pieces: the bytes of every token id in order; scores: their f32 merge
    scores.  max_token_length defaults to the longest piece in bytes."""
    if len(pieces) != len(scores):
        raise ValueError("pieces and scores differ in length")
    if max_token_length is None:
        max_token_length = max((len(p) for p in pieces), default=0)
    with open(path, "wb") as f:
        f.write(struct.pack("<III", max_token_length, bos_token_id, eos_token_id))
        for p, sc in zip(pieces, scores):
            f.write(struct.pack("<fI", sc, len(p)))
            f.write(p)


def bytes_to_unicode():
    """The byte-level BPE alphabet (published with GPT-2's tokenizer): the
    printable bytes '!'..'~', 0xA1..0xAC and 0xAE..0xFF stand for themselves;
    the other 68 bytes, in increasing order, map to code points 256, 257, ...
    Returns {byte: character}."""
    keep = list(range(ord("!"), ord("~") + 1)) + list(range(0xA1, 0xAC + 1)) + list(range(0xAE, 0xFF + 1))
    out, extra = {}, 0
    for b in range(256):
        if b in keep:
            out[b] = chr(b)
        else:
            out[b] = chr(256 + extra)
            extra += 1
    return out


def export_from_tokenizer_json(tokenizer_json, bos_token_id, eos_token_id, out_path):
    """export.py:168-212 for a Hugging Face tokenizer.json (byte-level BPE):
    every id of model.vocab and added_tokens in order, each token's characters
    mapped back to bytes (characters outside the byte alphabet as UTF-8), scores
    -log(rank + 1) for tokens that are the result of merge `rank`, -1e6 for the
    rest (a merge result produced by several merges scores by the last one);
    max_token_length = the longest token in characters.  Returns the number of
    tokens written."""
    with open(tokenizer_json, encoding="utf-8") as f:
        data = json.load(f)
    id_to_token = {int(i): t for t, i in data["model"]["vocab"].items()}
    for a in data.get("added_tokens", []):
        id_to_token[int(a["id"])] = a["content"]
    tokens = [id_to_token[i] for i in sorted(id_to_token)]
    # A string that several merges produce takes the rank of the LAST of them,
    # as export.py:186 builds its table (a dict comprehension overwrites).
    rank = {}
    for r, m in enumerate(data["model"].get("merges", [])):
        rank["".join(m if isinstance(m, list) else m.split())] = r
    u2b = {c: b for b, c in bytes_to_unicode().items()}
    pieces = [b"".join(bytes([u2b[ch]]) if ch in u2b else ch.encode("utf-8") for ch in t) for t in tokens]
    scores = [-math.log(rank[t] + 1) if t in rank else -1e6 for t in tokens]
    write_tokenizer_bin(out_path, pieces, scores, bos_token_id, eos_token_id, max((len(t) for t in tokens), default=0))
    return len(tokens)


# ---------------------------------------------------------------------------
# prompt templates (tokenizer.h:58-68, main.cu:129-131)
# ---------------------------------------------------------------------------
TEMPLATE_FILES = {False: ("template_user.txt", "template_system.txt"),
                  True: ("template_user_thinking.txt", "template_system_thinking.txt")}


def load_templates(model_dir, enable_thinking=False):
    """(user template, system + user template) as text, read as the reference
    does (at most 1023 bytes each)."""
    out = []
    for name in TEMPLATE_FILES[bool(enable_thinking)]:
        with open(os.path.join(model_dir, name), "rb") as f:
            out.append(f.read(1023).decode("utf-8", errors="replace"))
    return tuple(out)


def render(template, *args):
    """sprintf(template, args...) for a template whose conversions are %s (and
    %% for a literal percent sign)."""
    out, i, k = [], 0, 0
    while i < len(template):
        c = template[i]
        if c == "%" and i + 1 < len(template):
            n = template[i + 1]
            if n == "s":
                if k >= len(args):
                    raise ValueError("template has more %s than arguments")
                out.append(str(args[k]))
                k += 1
                i += 2
                continue
            if n == "%":
                out.append("%")
                i += 2
                continue
        out.append(c)
        i += 1
    return "".join(out)
