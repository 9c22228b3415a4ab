"""Vocabulary-sharded sampling over ranks (one process per GPU).

A row's logits are split by vocabulary across the ranks of a process group:
rank g holds columns [offset_g, offset_g + width_g). Each step every rank

  1. streams only its columns through rl_sample_partial (penalties, mask,
     temperature, the shard's sorted top-min(top_k, 128) list and its
     softmax sum relative to the shard's max),
  2. all-gathers the partial results (1056 bytes per row and rank),
  3. merges the G results with rl_sample_merge.

Every rank then holds the same tokens, equal to sampling the whole row in
one piece up to the order in which the softmax sums are added. The exchange
is the only collective on the path; it runs on torch.distributed (NCCL on
GPUs, gloo in the CPU tests of the gather layout).
"""
from __future__ import annotations

import numpy as np

import rlsampler

# columns per shard boundary: 8 bf16 / 4 f32 logits keep each shard's row
# start on a 16-byte boundary when the full row is
SHARD_ALIGN = 8


def shard_bounds(V: int, world: int, align: int = SHARD_ALIGN):
    """Contiguous split of V columns into `world` shards whose offsets are
    multiples of `align`; returns [(offset, width)] per rank."""
    if world < 1 or V < 1:
        raise ValueError(f"shard_bounds: V={V} world={world}")
    step = -(-V // world)
    step = -(-step // align) * align
    out = []
    for g in range(world):
        lo = min(g * step, V)
        hi = min(lo + step, V)
        if hi <= lo:
            raise ValueError(f"shard_bounds: V={V} leaves rank {g} of {world} without columns")
        out.append((lo, hi - lo))
    return out


def gather_partials(keys, stats, group=None):
    """All-gather of the ranks' partial results into the shard-major layout
    rl_sample_merge reads: keys [B, 128] int64 and stats [B, 32] uint8 per
    rank -> ([G, B, 128], [G, B, 32]), rank g's result at index g."""
    import torch
    import torch.distributed as dist

    G = dist.get_world_size(group)
    B = keys.shape[0]
    kall = torch.empty((G * B, keys.shape[1]), dtype=keys.dtype, device=keys.device)
    sall = torch.empty((G * B, stats.shape[1]), dtype=stats.dtype, device=stats.device)
    dist.all_gather_into_tensor(kall, keys.contiguous(), group=group)
    dist.all_gather_into_tensor(sall, stats.contiguous(), group=group)
    return kall.view(G, B, keys.shape[1]), sall.view(G, B, stats.shape[1])


class ShardedSampler:
    """Samples rows whose vocabulary is split across the ranks of `group`."""

    def __init__(self, V: int, max_batch: int, group=None, device=None, max_history: int = 1024):
        import torch
        import torch.distributed as dist

        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if self.world > 16:
            raise ValueError("rl_sample_merge takes at most 16 shards")
        self.V = V
        self.bounds = shard_bounds(V, self.world)
        self.offset, self.width = self.bounds[self.rank]
        dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self.device = dev
        self.sampler = rlsampler.Sampler(dev.index or 0, max_batch=max_batch, max_vocab=self.width,
                                         max_history=max_history)
        self.keys = torch.empty((max_batch, rlsampler.PART_KEYS), dtype=torch.int64, device=dev)
        self.stats = torch.empty((max_batch, rlsampler.PART_STATS_DTYPE.itemsize), dtype=torch.uint8, device=dev)

    def sample(self, logits_shard, params, uniforms, hist=None, hist_len=None, mask_shard=None, stream=None):
        """logits_shard [B, width] (this rank's columns, f32 or bf16);
        params / uniforms / hist as rlsampler.Sampler.sample (history ids
        global). Returns (tokens, probs, row_status) with global ids."""
        B = logits_shard.shape[0]
        if logits_shard.shape[1] != self.width:
            raise ValueError(f"rank {self.rank}: shard has {logits_shard.shape[1]} columns, expected {self.width}")
        k, s = self.keys[:B], self.stats[:B]
        self.sampler.sample_partial(logits_shard, self.offset, params, hist, hist_len, mask_shard, out_keys=k,
                                    out_stats=s, stream=stream)
        kall, sall = gather_partials(k, s, self.group)
        return self.sampler.sample_merge(kall, sall, params, uniforms, stream=stream)

    def close(self):
        self.sampler.close()


def stats_view(stats) -> np.ndarray:
    """Host view of gathered stats bytes [..., 32] as rl_part_stats records."""
    a = np.ascontiguousarray(stats.cpu().numpy() if hasattr(stats, "cpu") else stats)
    return a.view(rlsampler.PART_STATS_DTYPE).reshape(a.shape[:-1])
