"""Checkpoint layout, safetensors parsing and the C-ABI surface (CPU only).

The canonical tensor table must equal the reference's TENSOR_METADATA
(static_loader.h:83-400, recorded in golden/tensor_table.json); the header
parser must reject the damaged files the reference would misread (it never
parses the header: static_loader.h:421-427) and accept any tensor order."""
import json
import os
import re
import struct

import pytest

from conftest import GOLDEN, REPO


def test_tensor_table_matches_reference(qb):
    gold = json.load(open(os.path.join(GOLDEN, "tensor_table.json")))
    mine = qb.tensor_table()
    assert len(mine) == len(gold["tensors"]) == 311
    for (n, o, b), (gn, go, gb) in zip(mine, gold["tensors"]):
        assert (n, o, b) == (gn, go, gb)
    assert qb.load_library().qwen_total_weight_bytes() == gold["total_bytes"] == 1503264768


def test_abi_exports_every_declared_symbol(qb):
    hdr = open(os.path.join(REPO, "include", "qwen_b200.h")).read()
    hdr = re.sub(r"/\*.*?\*/", "", hdr, flags=re.S)
    names = set(re.findall(r"\b(qwen_[a-z0-9_]+)\s*\(", hdr))
    assert len(names) >= 25
    lib = qb.load_library()
    for n in sorted(names):
        assert hasattr(lib, n), n
    # the ctypes signature table covers the whole header
    assert names == set(qb._SIGS), names ^ set(qb._SIGS)


def _header(entries, meta=True):
    d = {"__metadata__": {"format": "pt"}} if meta else {}
    d.update(entries)
    js = json.dumps(d).encode()
    return struct.pack("<Q", len(js)) + js


def _valid_entries(qb, swap=None):
    ents = {}
    for n, o, b in qb.tensor_table():
        shape = None
        ents[n] = {"dtype": "BF16", "data_offsets": [o, o + b]}
    # shapes from the canonical derivation
    import numpy as np  # noqa: F401
    dims = {"lm_head.weight": [151936, 1024], "model.embed_tokens.weight": [151936, 1024], "model.norm.weight": [1024]}
    per = {"input_layernorm.weight": [1024], "post_attention_layernorm.weight": [1024], "mlp.down_proj.weight": [1024, 3072],
           "mlp.gate_proj.weight": [3072, 1024], "mlp.up_proj.weight": [3072, 1024], "self_attn.k_norm.weight": [128],
           "self_attn.q_norm.weight": [128], "self_attn.k_proj.weight": [1024, 1024], "self_attn.v_proj.weight": [1024, 1024],
           "self_attn.o_proj.weight": [1024, 2048], "self_attn.q_proj.weight": [2048, 1024]}
    for n in ents:
        if n in dims:
            shape = dims[n]
        else:
            shape = per[n.split(".", 3)[3]]
        ents[n]["shape"] = shape
    if swap:
        a, b = swap
        ents[a]["data_offsets"], ents[b]["data_offsets"] = ents[b]["data_offsets"], ents[a]["data_offsets"]
    return ents


def _sparse_file(path, header, data_bytes):
    with open(path, "wb") as f:
        f.write(header)
        f.truncate(len(header) + data_bytes)


def test_checkpoint_header_validation(qb, tmp_path):
    total = 1503264768
    good = _valid_entries(qb)
    p = str(tmp_path / "ok.safetensors")
    _sparse_file(p, _header(good), total)
    qb.checkpoint_validate(p)
    # tensors in another order (same sizes swapped) are accepted
    sw = _valid_entries(qb, swap=("model.layers.3.self_attn.q_norm.weight", "model.layers.7.self_attn.k_norm.weight"))
    _sparse_file(p, _header(sw), total)
    qb.checkpoint_validate(p)

    def expect(code, path):
        with pytest.raises(qb.QwenError) as e:
            qb.checkpoint_validate(path)
        assert e.value.code == code, str(e.value)

    # truncated data section
    _sparse_file(p, _header(good), total - 4096)
    expect(-3, p)
    # header length that overruns the file
    with open(p, "wb") as f:
        f.write(struct.pack("<Q", 10 ** 6) + b"{}")
    expect(-3, p)
    # shorter than the 8-byte length field
    with open(p, "wb") as f:
        f.write(b"\x01\x02")
    expect(-3, p)
    # wrong dtype
    bad = _valid_entries(qb)
    bad["model.norm.weight"]["dtype"] = "F16"
    _sparse_file(p, _header(bad), total)
    expect(-3, p)
    # wrong shape
    bad = _valid_entries(qb)
    bad["model.layers.0.mlp.up_proj.weight"]["shape"] = [1024, 3072]
    _sparse_file(p, _header(bad), total)
    expect(-3, p)
    # missing tensor
    bad = _valid_entries(qb)
    del bad["model.layers.27.self_attn.v_proj.weight"]
    _sparse_file(p, _header(bad), total)
    expect(-3, p)
    # overlapping tensors
    bad = _valid_entries(qb)
    bad["model.layers.5.self_attn.k_norm.weight"]["data_offsets"] = list(bad["model.layers.5.self_attn.q_norm.weight"]["data_offsets"])
    _sparse_file(p, _header(bad), total)
    expect(-3, p)
    # unknown tensor
    bad = _valid_entries(qb)
    bad["model.layers.28.mlp.up_proj.weight"] = dict(bad["model.layers.0.mlp.up_proj.weight"])
    _sparse_file(p, _header(bad), total)
    expect(-3, p)
    # not JSON
    with open(p, "wb") as f:
        f.write(struct.pack("<Q", 4) + b"nope")
        f.truncate(8 + 4 + 16)
    expect(-3, p)
    # missing file
    expect(-2, str(tmp_path / "absent.safetensors"))


def test_synthetic_checkpoint(qb, checkpoint):
    qb.checkpoint_validate(checkpoint)
    import numpy as np
    tab = {n: (o, b) for n, o, b in qb.tensor_table()}
    with open(checkpoint, "rb") as f:
        hl = struct.unpack("<Q", f.read(8))[0]
        base = 8 + hl
        assert base % 256 == 0

        def read(name, n=4096):
            o, b = tab[name]
            f.seek(base + o)
            return np.frombuffer(f.read(min(n, b)), dtype=np.uint16)
        # gains are 1.0; lm_head is the embedding; matrices are N(0, 0.02)
        assert (read("model.layers.4.input_layernorm.weight") == 0x3F80).all()
        assert (read("model.layers.9.self_attn.k_norm.weight", 256) == 0x3F80).all()
        assert (read("lm_head.weight", 1 << 20) == read("model.embed_tokens.weight", 1 << 20)).all()
        w = (read("model.layers.11.mlp.gate_proj.weight", 1 << 21).astype(np.uint32) << 16).view(np.float32)
        assert abs(float(w.mean())) < 1e-3 and abs(float(w.std()) - 0.02) < 5e-4


def _permuted_copy(src, dst):
    """The same checkpoint with its tensors stored in reverse name order (the
    header lists them in that order too)."""
    hl = struct.unpack("<Q", open(src, "rb").read(8))[0]
    meta = json.loads(open(src, "rb").read(8 + hl)[8:])
    names = sorted((k for k in meta if k != "__metadata__"), reverse=True)
    ents, off = {"__metadata__": meta.get("__metadata__", {})}, 0
    for n in names:
        a, b = meta[n]["data_offsets"]
        ents[n] = {"dtype": meta[n]["dtype"], "shape": meta[n]["shape"], "data_offsets": [off, off + b - a]}
        off += b - a
    js = json.dumps(ents).encode()
    with open(src, "rb") as f, open(dst, "wb") as g:
        g.write(struct.pack("<Q", len(js)) + js)
        for n in names:
            a, b = meta[n]["data_offsets"]
            f.seek(8 + hl + a)
            g.write(f.read(b - a))


def test_ordered_blob_round_trip(qb, checkpoint, tmp_path):
    """qwen_write_ordered_blob writes export.py:80-146's weights_qwen600.bin: each
    tensor's bytes at the offset of that order; the loaders accept the blob
    directly, and prefer one lying beside a safetensors file
    (static_loader.hip.h:185-202)."""
    import numpy as np
    blob = str(tmp_path / "weights_qwen600.bin")
    qb.write_ordered_blob(checkpoint, blob)
    assert os.path.getsize(blob) == 1503264768
    qb.checkpoint_validate(blob)
    hl = struct.unpack("<Q", open(checkpoint, "rb").read(8))[0]
    meta = json.loads(open(checkpoint, "rb").read(8 + hl)[8:])
    order = ["model.embed_tokens.weight", "lm_head.weight", "model.norm.weight"]
    for i in range(28):
        p = f"model.layers.{i}."
        order += [p + "self_attn.q_proj.weight", p + "self_attn.k_proj.weight", p + "self_attn.v_proj.weight", p + "self_attn.o_proj.weight",
                  p + "self_attn.q_norm.weight", p + "self_attn.k_norm.weight", p + "mlp.gate_proj.weight", p + "mlp.up_proj.weight",
                  p + "mlp.down_proj.weight", p + "input_layernorm.weight", p + "post_attention_layernorm.weight"]
    assert len(order) == 311
    b = np.memmap(blob, dtype=np.uint8, mode="r")
    c = np.memmap(checkpoint, dtype=np.uint8, mode="r")
    off = 0
    for n in order:
        lo, hi = meta[n]["data_offsets"]
        if n.endswith(("norm.weight", "q_proj.weight")) or n.startswith("model.layers.27"):
            assert np.array_equal(b[off:off + hi - lo], c[8 + hl + lo:8 + hl + hi]), n
        off += hi - lo
    assert off == b.shape[0]
    # a blob of the wrong size is a (headerless) file the parser rejects
    bad = str(tmp_path / "short.bin")
    with open(bad, "wb") as f:
        f.write(b"\0" * 4096)
    with pytest.raises(qb.QwenError):
        qb.checkpoint_validate(bad)


def test_permuted_checkpoint_validates(qb, checkpoint, tmp_path):
    p = str(tmp_path / "permuted.safetensors")
    _permuted_copy(checkpoint, p)
    qb.checkpoint_validate(p)
