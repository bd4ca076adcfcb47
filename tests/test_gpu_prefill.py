"""qwen_prefill on the tensor cores (whole-prompt passes: tcgen05 GEMMs with the
activations split into bf16 parts, causal attention over the KV cache on the
tcgen05/TMEM kernel or on the mma.sync kernel) against the one-launch-per-token
path and the fp32 oracle.  Tolerances as in test_gpu_decode: max-abs <= 2e-2
and relative RMS <= 2.5e-3 on the logits against the other paths; the two
attention kernels agree to 1e-3."""
import numpy as np
import pytest

from conftest import rel_rms

pytestmark = pytest.mark.gpu

VOCAB = 151936


def _prompt(n, seed):
    return np.random.default_rng(seed).integers(0, VOCAB, n).tolist()


def _both(qb, checkpoint, chunks):
    """Prefill the chunks (list of token lists, consecutive) on a GEMM-path and
    a per-token-path handle; returns both final logits and both handles."""
    a, b = qb.Engine(checkpoint, 0), qb.Engine(checkpoint, 0)
    b.set_prefill_mode(False)
    pos = 0
    for ch in chunks:
        la = a.prefill(ch, pos, want_logits=True)
        lb = b.prefill(ch, pos, want_logits=True)
        pos += len(ch)
    return la, lb, a, b, pos


def test_prefill_300_matches_per_token_path_and_oracle(qb, O, checkpoint):
    toks = _prompt(300, 11)
    la, lb, a, b, pos = _both(qb, checkpoint, [toks])
    try:
        assert np.abs(la - lb).max() <= 2e-2 and rel_rms(la, lb) <= 2.5e-3
        assert int(np.argmax(la)) == int(np.argmax(lb))
        of = O.Oracle(checkpoint, O.FP32, 320)
        for p, t in enumerate(toks[:-1]):
            of.forward(t, p, want_logits=False)
        lo = of.forward(toks[-1], len(toks) - 1)
        assert np.abs(la - lo).max() <= 2e-2 and rel_rms(la, lo) <= 2.5e-3, (np.abs(la - lo).max(), rel_rms(la, lo))
        # decoding continues from the cache the pass wrote
        ga, _ = a.generate(int(np.argmax(la)), pos, 8)
        gb, _ = b.generate(int(np.argmax(lb)), pos, 8)
        assert ga == gb
    finally:
        a.close(); b.close()


def test_prefill_two_passes_and_continuation(qb, checkpoint):
    # 2100 tokens: a 2048-row pass plus a 51-row pass; then 200 more at pos0 = 2100
    la, lb, a, b, pos = _both(qb, checkpoint, [_prompt(2100, 12), _prompt(200, 13)])
    try:
        assert pos == 2300 and a.cached == 2300
        assert np.abs(la - lb).max() <= 2e-2 and rel_rms(la, lb) <= 2.5e-3, (np.abs(la - lb).max(), rel_rms(la, lb))
        assert int(np.argmax(la)) == int(np.argmax(lb))
    finally:
        a.close(); b.close()


# Prompt lengths at the path boundaries: 65 (the smallest prompt of the tensor-core
# path; 63 padding rows in the 128-row tiles), 129 (127 padding rows), 1281 (a pass
# whose gate|up GEMM carries SwiGLU in its epilogue while 127 of its rows are
# padding), 2049 (a full 2048-row pass plus a one-row pass).
@pytest.mark.parametrize("n", [65, 129, 1281, 2049])
def test_prefill_edge_lengths(qb, checkpoint, n):
    la, lb, a, b, pos = _both(qb, checkpoint, [_prompt(n, 20 + n)])
    try:
        assert a.cached == n
        assert np.abs(la - lb).max() <= 2e-2 and rel_rms(la, lb) <= 2.5e-3, (n, np.abs(la - lb).max(), rel_rms(la, lb))
        assert int(np.argmax(la)) == int(np.argmax(lb))
        ga, _ = a.generate(int(np.argmax(la)), pos, 4)
        gb, _ = b.generate(int(np.argmax(lb)), pos, 4)
        assert ga == gb
    finally:
        a.close(); b.close()


def _pair_attention(qb, checkpoint, chunks):
    """Prefill the chunks on a handle with the mma.sync prompt-pass attention
    and on one with the tcgen05/TMEM kernel (the default); returns both final
    logits and both handles."""
    a, t = qb.Engine(checkpoint, 0), qb.Engine(checkpoint, 0)
    a.set_prefill_attention(0)
    t.set_prefill_attention(1)
    pos = 0
    for ch in chunks:
        la = a.prefill(ch, pos, want_logits=True)
        lt = t.prefill(ch, pos, want_logits=True)
        pos += len(ch)
    return la, lt, a, t, pos


def test_prefill_tcgen05_attention_300_against_oracle(qb, O, checkpoint):
    toks = _prompt(300, 11)
    la, lt, a, t, pos = _pair_attention(qb, checkpoint, [toks])
    try:
        of = O.Oracle(checkpoint, O.FP32, 320)
        for p, tok in enumerate(toks[:-1]):
            of.forward(tok, p, want_logits=False)
        lo = of.forward(toks[-1], len(toks) - 1)
        assert np.abs(lt - lo).max() <= 2e-2 and rel_rms(lt, lo) <= 2.5e-3, (np.abs(lt - lo).max(), rel_rms(lt, lo))
        assert rel_rms(lt, la) <= 1e-3 and int(np.argmax(lt)) == int(np.argmax(la))
        ga, _ = a.generate(int(np.argmax(la)), pos, 8)
        gt, _ = t.generate(int(np.argmax(lt)), pos, 8)
        assert ga == gt
    finally:
        a.close(); t.close()


# 65 and 129: one 128-row pass with 63 / 127 padding rows; 2049: a full pass
# plus a one-row pass; 2100 + 200: a second prefill call at pos0 = 2100 whose
# key tiles start in the first call's cache.
@pytest.mark.parametrize("lens", [(65,), (129,), (2049,), (2100, 200)])
def test_prefill_tcgen05_attention_matches_mma(qb, checkpoint, lens):
    chunks = [_prompt(n, 40 + i + n) for i, n in enumerate(lens)]
    la, lt, a, t, pos = _pair_attention(qb, checkpoint, chunks)
    try:
        assert t.cached == sum(lens)
        assert np.abs(lt - la).max() <= 2e-2 and rel_rms(lt, la) <= 1e-3, (lens, np.abs(lt - la).max(), rel_rms(lt, la))
        assert int(np.argmax(lt)) == int(np.argmax(la))
        ga, _ = a.generate(int(np.argmax(la)), pos, 4)
        gt, _ = t.generate(int(np.argmax(lt)), pos, 4)
        assert ga == gt
    finally:
        a.close(); t.close()


def test_prefill_attention_kind_rejects_unknown(qb, checkpoint):
    e = qb.Engine(checkpoint, 0)
    try:
        with pytest.raises(Exception):
            qb._check(e._lib.qwen_set_prefill_attention(e._h, 2))
    finally:
        e.close()


def test_prefill_programmatic_launch_matches_normal_launch(qb, checkpoint, tmp_path):
    """The prompt pass's kernels start early under programmatic dependent launch
    and wait for their predecessors on the device; launched normally
    (QWEN_B200_PDL=0, read once per process, so in a child process) the same
    kernels must give bit-identical logits, over two passes (2100 + 200 tokens)."""
    import os
    import subprocess
    import sys
    from conftest import PKG
    chunks = [_prompt(2100, 61), _prompt(200, 62)]
    script = (
        "import importlib.util, sys, numpy as np\n"
        f"spec = importlib.util.spec_from_file_location('qwen_b200', {os.path.join(PKG, 'qwen_b200.py')!r})\n"
        "qb = importlib.util.module_from_spec(spec); spec.loader.exec_module(qb)\n"
        f"e = qb.Engine({checkpoint!r}, 0)\n"
        f"chunks = {chunks!r}\n"
        "pos = 0\n"
        "for ch in chunks:\n"
        "    lg = e.prefill(ch, pos, want_logits=True); pos += len(ch)\n"
        f"np.save({str(tmp_path / 'normal.npy')!r}, lg)\n"
        "e.close()\n")
    env = dict(os.environ, QWEN_B200_PDL="0")
    r = subprocess.run([sys.executable, "-c", script], env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    e = qb.Engine(checkpoint, 0)
    try:
        pos = 0
        for ch in chunks:
            lg = e.prefill(ch, pos, want_logits=True)
            pos += len(ch)
    finally:
        e.close()
    normal = np.load(tmp_path / "normal.npy")
    assert np.array_equal(lg, normal), np.abs(lg.astype(np.float64) - normal).max()


def test_prefill_qkv_epilogue_matches_separate_kernel(qb, checkpoint, monkeypatch):
    """QK-norm, RoPE, the K/V append and V's transposed copy in the q|k|v GEMM's
    epilogue (passes of 768 rows and more) against the fp32-output GEMM plus
    qkv_post_kernel (QWEN_B200_QKV_EPILOGUE=0, read when a handle is created)
    and against the per-token path.  Chunks: 1000 rows at position 0, 1001 rows
    at 1000 (an odd last row), 999 rows at 2001 (an odd first position: the
    transposed-V stores go one position at a time)."""
    chunks = [_prompt(1000, 71), _prompt(1001, 72), _prompt(999, 73)]
    fused = qb.Engine(checkpoint, 0)
    monkeypatch.setenv("QWEN_B200_QKV_EPILOGUE", "0")
    sep = qb.Engine(checkpoint, 0)
    monkeypatch.delenv("QWEN_B200_QKV_EPILOGUE")
    tok = qb.Engine(checkpoint, 0)
    tok.set_prefill_mode(False)
    try:
        pos = 0
        for ch in chunks:
            lf = fused.prefill(ch, pos, want_logits=True)
            ls = sep.prefill(ch, pos, want_logits=True)
            lt = tok.prefill(ch, pos, want_logits=True)
            pos += len(ch)
            assert np.abs(lf - ls).max() <= 2e-2 and rel_rms(lf, ls) <= 1e-3, (pos, np.abs(lf - ls).max(), rel_rms(lf, ls))
            assert np.abs(lf - lt).max() <= 2e-2 and rel_rms(lf, lt) <= 2.5e-3, (pos, np.abs(lf - lt).max(), rel_rms(lf, lt))
            assert int(np.argmax(lf)) == int(np.argmax(ls)) == int(np.argmax(lt))
        gf, _ = fused.generate(int(np.argmax(lf)), pos, 8)
        gs, _ = sep.generate(int(np.argmax(ls)), pos, 8)
        assert gf == gs
    finally:
        fused.close(); sep.close(); tok.close()


@pytest.mark.parametrize("parts,tol,abs_tol", [(3, 2.5e-3, 2e-2), (1, 1e-2, 1e-1)])
def test_prefill_activation_parts(qb, checkpoint, parts, tol, abs_tol):
    """The tensor-core passes with three bf16 parts per activation (fp32-exact
    operands: one GEMM stage holds three A boxes and the B box) and with one
    (plain bf16 activations, ~5e-3 relative RMS from the fp32 chain, hence the
    looser bound) against the per-token path: a 2048-row pass (SM-pair GEMMs,
    the q|k|v epilogue) and a 300-row pass (single-CTA GEMMs)."""
    for n, seed in ((2048, 81), (300, 82)):
        toks = _prompt(n, seed)
        a, b = qb.Engine(checkpoint, 0), qb.Engine(checkpoint, 0)
        a.set_prefill_parts(parts)
        b.set_prefill_mode(False)
        try:
            la = a.prefill(toks, 0, want_logits=True)
            lb = b.prefill(toks, 0, want_logits=True)
            assert np.abs(la - lb).max() <= abs_tol and rel_rms(la, lb) <= tol, (parts, n, np.abs(la - lb).max(), rel_rms(la, lb))
            assert int(np.argmax(la)) == int(np.argmax(lb))
        finally:
            a.close(); b.close()
