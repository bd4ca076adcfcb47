"""Parity at the lengths of the long-context and prefill workloads, against the
fp32 oracle (qwen_model.cuh:772-851 restated) on the seed-0 synthetic
checkpoint, one oracle pass over a seeded 4,600-token sequence:

* prefill workload: the first 2,048 tokens through qwen_prefill (tensor-core
  passes), logits of position 2,047;
* long-context workload: the first 4,096 tokens through qwen_prefill (logits of
  position 4,095), then positions 4,096 .. 4,599 one launch each (logits at
  4,096 .. 4,099 and 4,599: context 4,600, the KV cache split over every CTA of
  a group in many chunks), then 32 sampled tokens (temperature 0.6, top-k 20,
  top-p 0.95) each equal to the oracle sampler, in the reference's candidate
  order, on the device's own logits.

Tolerances: max-abs <= 2e-2 and relative RMS <= 1e-3 at every compared
position (the stated contract).  At these depths the oracle with float
instead of double accumulation differs from itself by 1.7-1.9e-4 and the
engine from the oracle by ~4.5e-4; only the first positions of a sequence sit
near 2e-3 (see test_gpu_decode, which allows 2.5e-3 per position there)."""
import numpy as np
import pytest

from conftest import rel_rms

pytestmark = pytest.mark.gpu

VOCAB = 151936
N = 4600
TOKS = np.random.default_rng(4600).integers(0, VOCAB, N).tolist()
CHECK = [2047, 4095, 4096, 4097, 4098, 4099, 4599]


@pytest.fixture(scope="module")
def oracle_long(O, checkpoint):
    o = O.Oracle(checkpoint, O.FP32, N + 1)
    out = {}
    try:
        for p in range(N):
            lg = o.forward(TOKS[p], p, want_logits=p in CHECK)
            if p in CHECK:
                out[p] = lg
    finally:
        o.close()
    return out


def _check(got, want, where):
    d, r = float(np.abs(got - want).max()), rel_rms(got, want)
    assert d <= 2e-2, (where, d)
    assert r <= 1e-3, (where, r)
    assert int(np.argmax(got)) == int(np.argmax(want)), where
    return r


def test_prefill_2048_against_oracle(qb, checkpoint, oracle_long):
    eng = qb.Engine(checkpoint, 0)
    try:
        lg = eng.prefill(TOKS[:2048], 0, want_logits=True)
        r = _check(lg, oracle_long[2047], 2047)
        assert r <= 1e-3, r
    finally:
        eng.close()


def test_long_context_4600_against_oracle(qb, O, checkpoint, oracle_long):
    eng = qb.Engine(checkpoint, 0)
    try:
        rr = [_check(eng.prefill(TOKS[:4096], 0, want_logits=True), oracle_long[4095], 4095)]
        for p in range(4096, N):
            lg = eng.forward(TOKS[p], p)
            if p in oracle_long:
                rr.append(_check(lg, oracle_long[p], p))
        assert np.mean(rr) <= 1e-3, rr
        # 32 sampled tokens from context 4,600 on
        sp = qb.Sampling(0.6, 0.95, 20)
        tok, rng = int(np.argmax(lg)), 0x5EED
        for p in range(N, N + 32):
            nxt, rng2 = eng.decode_step(tok, p, sp, rng)
            want, want_rng = O.sample(eng.read_logits(), 0.6, 0.95, 20, rng, order_mode=0)
            assert (nxt, rng2) == (want, want_rng), p
            tok, rng = nxt, rng2
    finally:
        eng.close()
