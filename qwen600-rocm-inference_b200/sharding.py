"""Multi-GPU coordination for the decode engine (one process per GPU).

Two modes (no reference counterpart: the reference is single-GPU):

* replicas -- every rank runs an independent batch-1 sequence on its own GPU;
  there is no data-path collective.
* vocabulary-sharded LM head -- every rank runs the same trunk, but serves
  only rows [begin, end) of the 151936-row LM head.  Each rank reports its
  shard's top-k (logit, global id) list; the lists are all-gathered (NCCL over
  NVLink on GPUs, gloo in the CPU tests) and every rank merges them with the
  same sampler math and the same RNG state, so all ranks pick the same token
  with no second exchange.  Exact for argmax and for 1 <= top_k <= 64.
"""
import numpy as np

VOCAB_SIZE = 151936


def shard_range(rank, world, n=VOCAB_SIZE):
    """Rows [begin, end) of rank `rank` out of `world` (contiguous, balanced)."""
    return n * rank // world, n * (rank + 1) // world


def gather_candidates(values, ids, group=None, device=None):
    """All-gather every rank's k candidates; returns (values[world*k], ids[world*k])."""
    import torch
    import torch.distributed as dist
    world = dist.get_world_size(group)
    v = torch.as_tensor(np.ascontiguousarray(values, np.float32), device=device)
    i = torch.as_tensor(np.ascontiguousarray(ids, np.int32), device=device)
    vs = [torch.empty_like(v) for _ in range(world)]
    is_ = [torch.empty_like(i) for _ in range(world)]
    dist.all_gather(vs, v, group=group)
    dist.all_gather(is_, i, group=group)
    return torch.cat(vs).cpu().numpy(), torch.cat(is_).cpu().numpy()


def merge_and_sample(qb, values, ids, sampling, rng):
    """The device sampler's math over the gathered candidates (host side)."""
    return qb.sample_candidates(values, ids, sampling, rng)
