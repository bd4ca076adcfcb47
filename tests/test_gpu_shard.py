"""The vocabulary-sharded head's device loop on one GPU: two handles, each
with half of the LM-head rows, exchange their shard top-k through a device
buffer (the stand-in for the ranks' NCCL all-gather) and each merges them with
qwen_shard_merge.  Both must produce the token stream, and the RNG state, of
one full-vocabulary handle's device sampler: the trunk is bit-reproducible
for a given grid, so the union of the shards' top-k holds the full top-k."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

VOCAB = 151936
PROMPT = np.random.default_rng(33).integers(0, VOCAB, 20).tolist()
N = 12


@pytest.mark.parametrize("T,p,k", [(0.0, 1.0, 1), (0.6, 0.95, 20), (1.0, 0.9, 64)])
def test_sharded_head_merge_matches_full_vocab(qb, checkpoint, T, p, k):
    import torch
    sp = qb.Sampling(T, p, k)
    full = qb.Engine(checkpoint, 0)
    shards = [qb.Engine(checkpoint, 0), qb.Engine(checkpoint, 0)]
    try:
        shards[0].set_vocab_shard(0, VOCAB // 2)
        shards[1].set_vocab_shard(VOCAB // 2, VOCAB)
        for e in [full] + shards:
            e.prefill(PROMPT[:-1], 0)
        want, want_rng = full.generate(PROMPT[-1], len(PROMPT) - 1, N, sp, 0xABC)
        kk = [s.shard_begin(PROMPT[-1], len(PROMPT) - 1, sp, 0xABC) for s in shards]
        assert kk[0] == kk[1] == (1 if T == 0.0 else k)
        kk = kk[0]
        buf = torch.zeros(2 * 2 * kk, dtype=torch.int32, device="cuda")
        base = buf.data_ptr()
        for _ in range(N):
            for s in shards:
                s.shard_decode()
            for r, s in enumerate(shards):
                s.shard_candidates(base + 8 * kk * r, base + 8 * kk * r + 4 * kk)
            torch.cuda.synchronize()
            for s in shards:
                s.shard_merge(base, base + 4 * kk, 2, 2 * kk)
            torch.cuda.synchronize()
        got = [s.shard_finish(N) for s in shards]
        assert got[0] == got[1] == (want, want_rng)
        assert all(s.cached == len(PROMPT) - 1 + N for s in shards)
    finally:
        for e in [full] + shards:
            e.close()


def test_sharded_head_rejects_host_order_settings(qb, checkpoint, engine):
    engine.prefill(PROMPT[:4], 0)
    with pytest.raises(qb.QwenError) as e:
        engine.shard_begin(PROMPT[4], 4, qb.Sampling(0.7, 1.0, 20), 1)     # top-p off: the reference's order is host-only
    assert e.value.code == -6
    with pytest.raises(qb.QwenError) as e:
        engine.shard_decode()                                                 # no loop begun
    assert e.value.code == -7
