"""Two GPUs, one process each, NCCL: the vocabulary-sharded LM head.

Each rank runs the full trunk and half of the 151936 LM-head rows; per token
the ranks all-gather their shard's top-k (logit, id) lists over NCCL on the
engine's stream and merge them on the device with the same sampler math and
RNG state (sharding.ShardedHead: no host round trip per token).  The merged
token stream must equal the single-GPU full-vocabulary stream (the trunk is
bit-reproducible for a given grid size, so the candidates are exactly the full
top-k).  Skipped unless two GPUs are visible.
"""
import datetime
import importlib.util
import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from conftest import PKG, REPO

pytestmark = pytest.mark.gpu

N_STEPS = 16
PROMPT = np.random.default_rng(21).integers(0, 151936, 12).tolist()


def _load(name):
    spec = importlib.util.spec_from_file_location(name, os.path.join(PKG, name + ".py"))
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    return m


def _worker(rank, world, port, ck, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    qb, sh = _load("qwen_b200"), _load("sharding")
    sp = qb.Sampling(0.6, 0.95, 20)
    eng = qb.Engine(ck, rank)
    try:
        eng.set_vocab_shard(*sh.shard_range(rank, world))
        eng.prefill(PROMPT[:-1], 0)
        head = sh.ShardedHead(eng)
        out = head.generate(PROMPT[-1], len(PROMPT) - 1, N_STEPS, sp, 0x1234)
    finally:
        eng.close()
    q.put((rank, out))
    dist.barrier()
    dist.destroy_process_group()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_vocab_sharded_head_two_gpus(qb, checkpoint):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, checkpoint, q)) for r in range(2)]
    for p in ps:
        p.start()
    got = dict(q.get(timeout=600) for _ in ps)
    for p in ps:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert got[0] == got[1]
    # one GPU, full vocabulary, the device sampler
    sp = qb.Sampling(0.6, 0.95, 20)
    eng = qb.Engine(checkpoint, 0)
    try:
        eng.prefill(PROMPT[:-1], 0)
        want = eng.generate(PROMPT[-1], len(PROMPT) - 1, N_STEPS, sp, 0x1234)
    finally:
        eng.close()
    assert got[0] == want
