"""One long sequence decoded across the GPUs of a node (BASELINE config 4's
single-sequence variant).

* Gated DeltaNet: heads-parallel.  Rank r owns value heads
  [r*Hv/N, (r+1)*Hv/N) (and the key heads they read), their conv channels and
  recurrent state; its in_proj shard produces exactly those channels.  The
  per-rank outputs [Hv/N * 128] are all-gathered into the [Hv * 128] input of
  out_proj.
* Gated GQA: the KV cache is split along its length (there are only 2 KV
  heads).  Rank r holds a contiguous key range; the last rank holds the tail
  and receives the appended token.  Every rank computes softmax partials
  (o, m, l) for all query heads over its keys (q35_gqa_decode_partial); the
  partials are all-gathered and merged locally (q35_gqa_combine_partials).

The compute and the collective are injected, so the same orchestration runs
with the CUDA kernels over NCCL and, in the CPU tests, with a numpy stand-in
over gloo.
"""
from __future__ import annotations

from dataclasses import dataclass


def split_range(n: int, world: int, rank: int):
    """Contiguous near-even split of [0, n) -- rank r gets [lo, hi)."""
    base, rem = divmod(n, world)
    lo = rank * base + min(rank, rem)
    return lo, lo + base + (1 if rank < rem else 0)


@dataclass
class ShardPlan:
    world: int
    rank: int
    num_k_heads: int
    num_v_heads: int
    kv_len: int  # tokens cached before the first decode step

    def __post_init__(self):
        if self.num_k_heads % self.world:
            raise ValueError("the world size must divide the number of GDN key heads")
        if self.num_v_heads % self.num_k_heads:
            raise ValueError("num_v_heads must be a multiple of num_k_heads")

    @property
    def gdn_k_heads(self):
        return split_range(self.num_k_heads, self.world, self.rank)

    @property
    def gdn_v_heads(self):
        rf = self.num_v_heads // self.num_k_heads
        k0, k1 = self.gdn_k_heads
        return k0 * rf, k1 * rf

    @property
    def kv_tokens(self):
        """This rank's slice [lo, hi) of the initial cache."""
        return split_range(self.kv_len, self.world, self.rank)

    @property
    def holds_tail(self):
        return self.rank == self.world - 1

    def channel_slices(self, head_dim=128):
        """Channel ranges of this rank's heads inside the full q | k | v layout
        (in_proj_qkv output, text_modules.rs:554-567): (q, k, v) slices."""
        k0, k1 = self.gdn_k_heads
        v0, v1 = self.gdn_v_heads
        kd = self.num_k_heads * head_dim
        return (slice(k0 * head_dim, k1 * head_dim), slice(kd + k0 * head_dim, kd + k1 * head_dim),
                slice(2 * kd + v0 * head_dim, 2 * kd + v1 * head_dim))


def decode_step(plan: ShardPlan, gdn_local, gqa_partial, all_gather, combine):
    """One decode step of one sequence on this rank.

    gdn_local()      -> this rank's GDN output [Hv/N * 128]
    gqa_partial()    -> this rank's GQA partial [Hq, 258]
    all_gather(x)    -> list of every rank's x (rank order)
    combine(parts)   -> merged GQA output [Hq * 256] from the stacked partials
    Returns (gdn_out_full, gqa_out_full), identical on every rank."""
    g_local = gdn_local()
    p_local = gqa_partial()
    g_all = all_gather(g_local)
    p_all = all_gather(p_local)
    return g_all, combine(p_all)
