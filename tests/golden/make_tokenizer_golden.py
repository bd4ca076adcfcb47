"""Golden vectors for the tokenizer: token ids from the reference's own
tokenizer.h (compiled into oracle/_ref/libref_tokenizer.so by
oracle/build_oracle.py) on a synthetic vocabulary.

    python tests/golden/make_tokenizer_golden.py     # writes tests/golden/tokenizer_cases.json

No real Qwen tokenizer files are available offline, so the vocabulary is built
here from a seed: ids 0..255 are the single bytes, then byte-level BPE merges
learnt on seeded pseudo-text (merge rank r scores -log(r + 1), as export.py
scores them), then special "<|...|>"-style entries, then one entry that repeats
the bytes of an earlier merge (the reference's lookup returns the lowest id).
build_vocab() is imported by the tests to rebuild the same file; the fixture
records its SHA-256.
"""
import ctypes
import hashlib
import json
import math
import os
import random
import struct
import sys
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.abspath(os.path.join(HERE, "..", ".."))
N_MERGES = 400
SPECIALS = ["<|start|>", "<|end|>", "<think>", "</think>", "<|pad|>"]
TEMPLATES = {
    "template_user.txt": "<|start|>user\n%s<|end|>\n<|start|>assistant\n",
    "template_system.txt": "<|start|>system\n%s<|end|>\n<|start|>user\n%s<|end|>\n<|start|>assistant\n",
    "template_user_thinking.txt": "<|start|>user\n%s<|end|>\n<|start|>assistant\n<think>\n",
    "template_system_thinking.txt": "<|start|>system\n%s<|end|>\n<|start|>user\n%s<|end|>\n<|start|>assistant\n<think>\n",
}


def corpus(seed):
    rng = random.Random(seed)
    syl = ["ka", "to", "ri", "se", "an", "on", "er", "th", "in", "qu", "ei", "ou", "st", "ng", "é", "ü", "日本", "ß"]
    words = ["".join(rng.choice(syl) for _ in range(rng.randint(1, 4))) for _ in range(300)]
    out = []
    for _ in range(4000):
        out.append(rng.choice(words))
        out.append(rng.choice([" ", " ", " ", ", ", ". ", "\n", " - ", "  "]))
    return "".join(out).encode("utf-8")


def build_vocab(seed=0):
    """(pieces, scores, bos, eos): the synthetic vocabulary in id order."""
    pieces = [bytes([b]) for b in range(256)]
    scores = [-1e6] * 256
    seq = list(corpus(seed))          # byte ids
    for r in range(N_MERGES):
        counts = {}
        for a, b in zip(seq, seq[1:]):
            counts[(a, b)] = counts.get((a, b), 0) + 1
        if not counts:
            break
        best = max(counts.items(), key=lambda kv: (kv[1], -kv[0][0], -kv[0][1]))[0]
        new = len(pieces)
        pieces.append(pieces[best[0]] + pieces[best[1]])
        scores.append(-math.log(r + 1))
        out, i = [], 0
        while i < len(seq):
            if i + 1 < len(seq) and (seq[i], seq[i + 1]) == best:
                out.append(new)
                i += 2
            else:
                out.append(seq[i])
                i += 1
        seq = out
    for s in SPECIALS:
        pieces.append(s.encode())
        scores.append(-1e6)
    pieces.append(pieces[256])        # a repeat of the first merge, scored higher: never chosen by lookup
    scores.append(0.0)
    bos = pieces.index(b"<|start|>")
    eos = pieces.index(b"<|end|>")
    return pieces, scores, bos, eos


def write_bin(path, pieces, scores, bos, eos):
    with open(path, "wb") as f:
        f.write(struct.pack("<III", max(len(p) for p in pieces), bos, eos))
        for p, s in zip(pieces, scores):
            f.write(struct.pack("<fI", s, len(p)))
            f.write(p)


def write_model_dir(d, seed=0):
    pieces, scores, bos, eos = build_vocab(seed)
    write_bin(os.path.join(d, "tokenizer.bin"), pieces, scores, bos, eos)
    for name, text in TEMPLATES.items():
        with open(os.path.join(d, name), "w", encoding="utf-8", newline="") as f:
            f.write(text)
    return pieces, scores, bos, eos


def sha256(path):
    with open(path, "rb") as f:
        return hashlib.sha256(f.read()).hexdigest()


# Every '<' is followed by a '>' within 64 bytes (the reference's special-token
# scan reads past the end of the text otherwise) and every byte has an entry.
CASES = [
    "",
    "k",
    "kato rise",
    "anon erth inqu, eiou stng.",
    "qukatori seanon. thin\nstér üka",
    "日本ka 日本日本 toß",
    "<|start|>user\nhello there<|end|>",
    "<|start|><|end|><think></think>",
    "<b>bold</b> <|nope|> <think>x</think>",
    "tokens <|pad|><|pad|> end",
    "   multiple   spaces\n\n\nand lines",
    "ka" * 24,
    "1234 + 5678 = 6912; !?#$%&*()[]{}",
    "<|start|>system\nbe brief<|end|>\n<|start|>user\nwhy? <|end|>\n<|start|>assistant\n<think>\n",
]


def main():
    lib_path = os.path.join(REPO, "oracle", "_ref", "libref_tokenizer.so")
    if not os.path.exists(lib_path):
        sys.exit("build the reference tokenizer first: python oracle/build_oracle.py")
    lib = ctypes.CDLL(lib_path)
    lib.ref_tokenizer_encode.restype = ctypes.c_int
    lib.ref_tokenizer_encode.argtypes = [ctypes.c_char_p, ctypes.c_char_p, ctypes.POINTER(ctypes.c_int), ctypes.c_int]
    with tempfile.TemporaryDirectory() as d:
        pieces, scores, bos, eos = write_model_dir(d)
        digest = sha256(os.path.join(d, "tokenizer.bin"))
        cases = []
        for text in CASES:
            data = text.encode("utf-8")
            buf = (ctypes.c_int * (len(data) + 8))()
            n = lib.ref_tokenizer_encode(d.encode(), data, buf, len(data) + 8)
            cases.append({"text": text, "ids": list(buf[:n])})
            print(f"{len(data):4d} bytes -> {n:3d} tokens", flush=True)
    out = {"generator": "tests/golden/make_tokenizer_golden.py (reference tokenizer.h via oracle/_ref/libref_tokenizer.so)",
           "seed": 0, "entries": len(pieces), "bos": bos, "eos": eos, "tokenizer_bin_sha256": digest, "cases": cases}
    with open(os.path.join(HERE, "tokenizer_cases.json"), "w", encoding="utf-8") as f:
        json.dump(out, f, ensure_ascii=False, indent=1)


if __name__ == "__main__":
    main()
