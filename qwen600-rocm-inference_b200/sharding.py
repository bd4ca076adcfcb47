"""Multi-GPU modes of the decode engine (one process per GPU).

Two modes (no reference counterpart: the reference is single-GPU):

* replicas -- every rank runs an independent batch-1 sequence on its own GPU;
  there is no data-path collective (bench.py --gpus N).
* vocabulary-sharded LM head (ShardedHead) -- every rank runs the same trunk
  but only rows [begin, end) of the 151936-row LM head.  Per token each rank's
  launch leaves its shard's top-k (logit, global id) list on the device; one
  NCCL all-gather on the engine's stream exchanges the lists (k x 8 bytes per
  rank: 160 B for top-k 20); a one-CTA kernel on every rank merges them in
  descending order, ties by id, and samples with the same math and RNG state,
  so all ranks pick the same token and feed it to their next launch without a
  host round trip.  Exact for argmax and for top-p in (0, 1) with 1 <= top_k
  <= 64 (the device sampler's settings).

The host-side helpers (gather_candidates, merge_and_sample) do the same merge
through host memory; the CPU tests use them with gloo ranks.
"""
import numpy as np

VOCAB_SIZE = 151936
MAX_K = 64


def shard_range(rank, world, n=VOCAB_SIZE):
    """Rows [begin, end) of rank `rank` out of `world` (contiguous, balanced)."""
    return n * rank // world, n * (rank + 1) // world


class ShardedHead:
    """The device-resident decode loop of a vocabulary-sharded head on one rank.

    `engine` is this rank's qwen_b200.Engine (prefilled with the same prompt on
    every rank); the process group must be NCCL with this rank's GPU current.
    generate() runs n steps: per step qwen_shard_decode, the candidate copy,
    one all-gather (values and ids packed in one int32 buffer) and
    qwen_shard_merge, all on the engine's stream; the host waits once, at the
    end.  step_times() measures the per-token device latency."""

    def __init__(self, engine, group=None):
        import torch
        import torch.distributed as dist
        self.eng = engine
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.dev = torch.device("cuda", engine.device)
        self.stream = torch.cuda.ExternalStream(engine.stream, device=self.dev)
        # per rank: k values (fp32 bits) then k ids, 2 * MAX_K int32 slots
        self.mine = torch.zeros(2 * MAX_K, dtype=torch.int32, device=self.dev)
        self.all = torch.zeros(self.world * 2 * MAX_K, dtype=torch.int32, device=self.dev)
        self.k = 1

    def _step(self):
        import torch.distributed as dist
        k = self.k
        self.eng.shard_decode()
        self.eng.shard_candidates(self.mine.data_ptr(), self.mine.data_ptr() + 4 * k)
        dist.all_gather_into_tensor(self.all[: self.world * 2 * k], self.mine[: 2 * k], group=self.group)
        self.eng.shard_merge(self.all.data_ptr(), self.all.data_ptr() + 4 * k, self.world, 2 * k)

    def generate(self, token, pos, n_steps, sampling, rng=0):
        """n_steps tokens after `token` at `pos`; returns (tokens, rng state)."""
        import torch
        self.k = self.eng.shard_begin(token, pos, sampling, rng)
        with torch.cuda.stream(self.stream):
            for _ in range(n_steps):
                self._step()
        return self.eng.shard_finish(n_steps)

    def timed(self, token, pos, n_steps, sampling, rng=0):
        """generate() with the steps bracketed by CUDA events on the engine's
        stream; returns (tokens, rng state, device ms per token)."""
        import torch
        self.k = self.eng.shard_begin(token, pos, sampling, rng)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(self.stream):
            e0.record(self.stream)
            for _ in range(n_steps):
                self._step()
            e1.record(self.stream)
        toks, r = self.eng.shard_finish(n_steps)
        return toks, r, e0.elapsed_time(e1) / n_steps


def gather_candidates(values, ids, group=None, device=None):
    """All-gather every rank's k candidates through host memory; returns
    (values[world*k], ids[world*k])."""
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
    """The device sampler's math over gathered candidates, on the host."""
    return qb.sample_candidates(values, ids, sampling, rng)
