"""World-size-2 gloo tests of the multi-GPU host logic (CPU only).

* the vocabulary-sharded head's candidate exchange and merge: every rank must
  pick the token the full-vocabulary sampler picks;
* failure detection on the host: a rank that leaves before a collective makes
  the other rank's collective fail within the process group's timeout.
"""
import datetime
import importlib.util
import os
import sys

import numpy as np
import pytest
import torch.multiprocessing as mp

from conftest import PKG, REPO

VOCAB = 151936


def _load(name):
    spec = importlib.util.spec_from_file_location(name, os.path.join(PKG, name + ".py"))
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    return m


def _init(rank, world, port):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
    return dist


def _merge_worker(rank, world, port, out):
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    qb, sh = _load("qwen_b200"), _load("sharding")
    dist = _init(rank, world, port)
    g = np.random.default_rng(4)
    res = []
    for step in range(12):
        lg = (g.standard_normal(VOCAB) * 0.64).astype(np.float32)   # same on every rank
        k = int([1, 5, 20, 64][step % 4])
        sp = qb.Sampling(0.0 if step % 3 == 0 else 0.6, 0.95, k)
        seed = 1000 + step
        b, e = sh.shard_range(rank, world)
        top = b + np.argsort(-lg[b:e], kind="stable")[:k]
        v, i = sh.gather_candidates(lg[top], top.astype(np.int32))
        res.append(sh.merge_and_sample(qb, v, i, sp, seed))
    out.put((rank, res))
    dist.destroy_process_group()


def _free_port():
    import socket
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_sharded_merge_two_ranks(O):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_merge_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    got = dict(q.get(timeout=120) for _ in ps)
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert got[0] == got[1]
    # the single-process sampler over the full vocabulary agrees
    g = np.random.default_rng(4)
    for step in range(12):
        lg = (g.standard_normal(VOCAB) * 0.64).astype(np.float32)
        k = int([1, 5, 20, 64][step % 4])
        T = 0.0 if step % 3 == 0 else 0.6
        assert got[0][step] == O.sample(lg, T, 0.95, k, 1000 + step, order_mode=1), step


def _leaver_worker(rank, world, port, out):
    dist = _init(rank, world, port)
    import torch
    if rank == 1:
        out.put((rank, "left"))
        out.close(); out.join_thread()
        os._exit(0)          # leaves between steps, never joins the collective
    try:
        t = torch.zeros(4)
        dist.all_reduce(t)
        out.put((rank, "no error"))
    except Exception as e:   # the collective must fail, not hang
        out.put((rank, "error: " + type(e).__name__))
    out.close(); out.join_thread()
    os._exit(0)


def test_rank_loss_is_detected():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_leaver_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    got = dict(q.get(timeout=120) for _ in ps)
    for p in ps:
        p.join(timeout=60)
    assert got[1] == "left"
    assert got[0].startswith("error"), got[0]
