"""Batched decode (qwen_batch_*), prompts of different lengths so the slots sit
at different positions:
  - greedy: each slot's token stream equals the batch-1 engine's for the same
    prompt, and the prompt logits are within the decode tolerances (max-abs
    <= 2e-2, relative RMS <= 2.5e-3);
  - sampled: each slot's stream equals the same prompt run alone in a
    one-slot batch, bit for bit (rows of a step do not interact: every GEMM
    output keeps its accumulation order whatever the other rows hold).  Against
    the batch-1 engine, sampled streams may part where a coin lands within the
    fp32-level logit difference of a CDF boundary; the sampler math itself is
    pinned in the sampler tests."""
import numpy as np
import pytest

from conftest import rel_rms

pytestmark = pytest.mark.gpu

VOCAB = 151936
LENGTHS = [70, 5, 130, 33]


def _prompts():
    return [np.random.default_rng(100 + i).integers(0, VOCAB, n).tolist() for i, n in enumerate(LENGTHS)]


def _single(qb, checkpoint, prompt, n_tokens, sp, seed):
    eng = qb.Engine(checkpoint, 0)
    try:
        lg = eng.prefill(prompt, 0, want_logits=True)
        tok, rng = qb.sample_host(lg, sp, seed)
        out, pos = [tok], len(prompt)
        while len(out) < n_tokens:
            tok, rng = eng.decode_step(tok, pos, sp, rng)
            out.append(tok)
            pos += 1
        return lg, out
    finally:
        eng.close()


def test_batch_greedy_matches_single_sequences(qb, checkpoint):
    sp = qb.Sampling(0.0, 1.0, 1)
    prompts, n_tokens = _prompts(), 8
    seeds = [11, 22, 33, 44]
    singles = [_single(qb, checkpoint, p, n_tokens, sp, s) for p, s in zip(prompts, seeds)]
    b = qb.Engine(checkpoint, 0)
    try:
        b.batch_init(len(prompts))
        toks, rngs = [], []
        for slot, (p, s) in enumerate(zip(prompts, seeds)):
            lg = b.batch_prefill(slot, p, want_logits=True)
            ref = singles[slot][0]
            assert np.abs(lg - ref).max() <= 2e-2 and rel_rms(lg, ref) <= 2.5e-3, (slot, np.abs(lg - ref).max(), rel_rms(lg, ref))
            t, r = qb.sample_host(lg, sp, s)
            toks.append(t)
            rngs.append(r)
        outs = [[t] for t in toks]
        pos = [len(p) for p in prompts]
        for _ in range(n_tokens - 1):
            toks, rngs = b.batch_step(toks, pos, sp, rngs)
            for slot, t in enumerate(toks):
                outs[slot].append(t)
            pos = [q + 1 for q in pos]
        for slot in range(len(prompts)):
            assert outs[slot] == singles[slot][1], slot
    finally:
        b.close()


def _batch_stream(qb, eng, prompts, seeds, sp, n_tokens):
    toks, rngs = [], []
    for slot, (p, s) in enumerate(zip(prompts, seeds)):
        lg = eng.batch_prefill(slot, p, want_logits=True)
        t, r = qb.sample_host(lg, sp, s)
        toks.append(t)
        rngs.append(r)
    outs = [[t] for t in toks]
    pos = [len(p) for p in prompts]
    for _ in range(n_tokens - 1):
        toks, rngs = eng.batch_step(toks, pos, sp, rngs)
        for slot, t in enumerate(toks):
            outs[slot].append(t)
        pos = [q + 1 for q in pos]
    return outs


def test_batch_sampled_slots_are_independent(qb, checkpoint):
    sp = qb.Sampling(0.6, 0.95, 20)
    prompts, seeds, n_tokens = _prompts(), [11, 22, 33, 44], 12
    b = qb.Engine(checkpoint, 0)
    try:
        b.batch_init(len(prompts))
        together = _batch_stream(qb, b, prompts, seeds, sp, n_tokens)
    finally:
        b.close()
    for slot in range(len(prompts)):
        one = qb.Engine(checkpoint, 0)
        try:
            one.batch_init(1)
            alone = _batch_stream(qb, one, [prompts[slot]], [seeds[slot]], sp, n_tokens)[0]
        finally:
            one.close()
        assert together[slot] == alone, slot


@pytest.mark.parametrize("T,p,k", [(0.8, 1.0, 20), (0.7, 1.0, 0), (0.6, 0.95, 20)])
def test_batch_sampled_tokens_follow_reference_order(qb, O, checkpoint, T, p, k):
    """Every sampled batch token equals the oracle sampler in the reference's
    candidate order (order_mode=0) on that row's logits: with the nucleus cut
    off or k = 0 the step draws over the whole row on the host; with it on,
    over the device top-k."""
    sp = qb.Sampling(T, p, k)
    prompts, seeds = _prompts(), [5, 6, 7, 8]
    b = qb.Engine(checkpoint, 0)
    try:
        b.batch_init(len(prompts))
        for slot, pr in enumerate(prompts):
            b.batch_prefill(slot, pr[:-1])
        toks, pos = [pr[-1] for pr in prompts], [len(pr) - 1 for pr in prompts]
        rngs = list(seeds)
        for _ in range(6):
            nxt, rngs2 = b.batch_step(toks, pos, sp, rngs)
            lg = b.batch_read_logits(len(prompts))
            for r in range(len(prompts)):
                want, want_rng = O.sample(lg[r], T, p, k, rngs[r], order_mode=0)
                assert (nxt[r], rngs2[r]) == (want, want_rng), r
            toks, rngs, pos = nxt, rngs2, [q + 1 for q in pos]
    finally:
        b.close()


@pytest.mark.parametrize("batch,slots", [(32, [0, 13, 31]), (128, [0, 77, 127])])
def test_batch_greedy_at_scale_matches_single_sequences(qb, checkpoint, batch, slots):
    """B = 32 and 128 at 1K context (the split-K / short-pass GEMM paths of
    the benchmark's batched steps): the greedy streams of sample slots equal
    the batch-1 engine's for the same prompts."""
    sp, n_prompt, n_tokens = qb.Sampling(0.0, 1.0, 1), 1024, 6
    prompts = [np.random.default_rng(7000 + s).integers(0, VOCAB, n_prompt).tolist() for s in range(batch)]
    b = qb.Engine(checkpoint, 0)
    try:
        b.batch_init(batch)
        toks = []
        for slot, pr in enumerate(prompts):
            b.batch_prefill(slot, pr[:-1])
            toks.append(pr[-1])
        pos = [n_prompt - 1] * batch
        outs = [[] for _ in range(batch)]
        for _ in range(n_tokens):
            toks, _ = b.batch_step(toks, pos, sp)
            for slot in range(batch):
                outs[slot].append(toks[slot])
            pos = [q + 1 for q in pos]
    finally:
        b.close()
    for slot in slots:
        one = qb.Engine(checkpoint, 0)
        try:
            one.prefill(prompts[slot][:-1], 0)
            want, _ = one.generate(prompts[slot][-1], n_prompt - 1, n_tokens)
        finally:
            one.close()
        assert outs[slot] == want, slot


def test_batch_errors(qb, checkpoint):
    b = qb.Engine(checkpoint, 0)
    try:
        with pytest.raises(qb.QwenError) as e:
            b.batch_step([1], [0])
        assert e.value.code == -7                       # not initialised
        b.batch_init(2)
        with pytest.raises(qb.QwenError) as e:
            b.batch_init(2)
        assert e.value.code == -7
        b.batch_prefill(0, [5, 6, 7])
        with pytest.raises(qb.QwenError) as e:
            b.batch_step([1, 2], [3, 1])                # slot 1 holds no positions yet
        assert e.value.code == -7
        with pytest.raises(qb.QwenError) as e:
            b.batch_step([1, 2, 3], [3, 0, 0])          # batch larger than max_batch
        assert e.value.code == -1
        nxt, _ = b.batch_step([1], [3])                 # slot 0 continues at position 3
        assert 0 <= nxt[0] < VOCAB
    finally:
        b.close()
