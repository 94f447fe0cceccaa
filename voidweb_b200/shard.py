"""Placement of the decode work on N GPUs (one process per GPU).

The (sequence, KV head) segments of a decode step are independent: append,
decode, block copies and the host bookkeeping never read another segment's
pages.  Two placements follow from that, and neither needs a collective on the
data path:

* ``"sequences"``: rank r holds a contiguous slice of the batch with every KV
  head (its own pool, block tables and block manager).  Per-GPU work is fixed
  as ranks are added when each rank brings its own sequences (weak scaling).
* ``"kv_heads"``: rank r holds a contiguous slice of the KV heads, with the
  query heads of their GQA groups, for every sequence; every rank keeps the
  same block ids (the host block manager and radix tree run replicated, and a
  block-copy list is replayed on every rank).  This is the placement for a
  model too large for one GPU's HBM (Llama-3-70B: one KV head per GPU on 8).
* ``"kv_heads_seqs"``: both at once, for more ranks than KV heads: the ranks
  form gcd(world, KV heads) head groups of world / that many ranks each; rank
  r takes head slice r // seq_groups and sequence slice r % seq_groups
  (Qwen2.5-7B's 4 KV heads on 8 GPUs: one KV head and half the batch each).
  Ranks of one head group keep the block ids of their own sequences; the
  ranks that share a sequence slice keep the same ones.

Outputs stay on the rank that computed them (the next operation of a
tensor-parallel layer consumes its own heads); ``gather_outputs`` assembles
the whole [B][Hq][D] tensor when a caller wants it, with one all-gather.
"""
from __future__ import annotations

from dataclasses import dataclass
from math import gcd

MODES = ("sequences", "kv_heads", "kv_heads_seqs")


def shard_range(n: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous [lo, hi) of n items for `rank`; sizes differ by at most one,
    the larger slices first."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    base, extra = divmod(n, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


@dataclass(frozen=True)
class ShardPlan:
    mode: str            # one of MODES
    world: int
    rank: int
    num_seqs: int
    num_q_heads: int
    num_kv_heads: int

    def __post_init__(self):
        if self.mode not in MODES:
            raise ValueError(f"unknown placement {self.mode!r}")
        if self.num_kv_heads <= 0 or self.num_q_heads % self.num_kv_heads:
            raise ValueError("num_q_heads must be a positive multiple of num_kv_heads")
        if self.mode == "kv_heads" and self.num_kv_heads < self.world:
            raise ValueError(f"{self.num_kv_heads} KV heads cannot cover {self.world} ranks")

    @property
    def group(self) -> int:
        return self.num_q_heads // self.num_kv_heads

    @property
    def head_groups(self) -> int:
        """How many slices the KV heads are cut into."""
        if self.mode == "kv_heads":
            return self.world
        if self.mode == "kv_heads_seqs":
            return gcd(self.world, self.num_kv_heads)
        return 1

    @property
    def seq_groups(self) -> int:
        """How many slices the batch is cut into."""
        return self.world // self.head_groups

    def seqs(self) -> tuple[int, int]:
        return shard_range(self.num_seqs, self.seq_groups, self.rank % self.seq_groups)

    def kv_heads(self) -> tuple[int, int]:
        return shard_range(self.num_kv_heads, self.head_groups, self.rank // self.seq_groups)

    def q_heads(self) -> tuple[int, int]:
        h0, h1 = self.kv_heads()
        return h0 * self.group, h1 * self.group

    def local_pool_kv_heads(self) -> int:
        h0, h1 = self.kv_heads()
        return h1 - h0

    def slice_inputs(self, q, k_new=None, v_new=None, block_tables=None, seq_lens=None):
        """This rank's part of one layer's inputs: q [B][Hq][D], k_new/v_new
        [B][Hkv][D], block_tables [B][stride], seq_lens [B] (arrays or tensors)."""
        s0, s1 = self.seqs()
        h0, h1 = self.kv_heads()
        g0, g1 = self.q_heads()
        pick = lambda a, heads: None if a is None else (a[s0:s1, heads[0]:heads[1]])
        return (pick(q, (g0, g1)), pick(k_new, (h0, h1)), pick(v_new, (h0, h1)),
                None if block_tables is None else block_tables[s0:s1],
                None if seq_lens is None else seq_lens[s0:s1])


def gather_outputs(plan: ShardPlan, local_out, group=None):
    """Assemble [B][Hq][D] on every rank from each rank's local output (one
    all-gather over the process group; slices of uneven size are padded)."""
    import torch
    import torch.distributed as dist

    world = plan.world
    if world == 1:
        return local_out
    D = local_out.shape[-1]
    n_seq = -(-plan.num_seqs // plan.seq_groups)
    n_head = -(-plan.num_kv_heads // plan.head_groups) * plan.group
    pad = torch.zeros((n_seq, n_head, D), dtype=local_out.dtype, device=local_out.device)
    pad[:local_out.shape[0], :local_out.shape[1]] = local_out
    parts = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(parts, pad.contiguous(), group=group)
    out = torch.empty((plan.num_seqs, plan.num_q_heads, D), dtype=local_out.dtype,
                      device=local_out.device)
    for r in range(world):
        p = ShardPlan(plan.mode, world, r, plan.num_seqs, plan.num_q_heads, plan.num_kv_heads)
        s0, s1 = p.seqs()
        g0, g1 = p.q_heads()
        out[s0:s1, g0:g1] = parts[r][:s1 - s0, :g1 - g0]
    return out
