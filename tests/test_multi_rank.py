"""The N>1 placement logic on CPU: two (or four) gloo ranks, each running the
oracle on its shard (append + decode + a block-copy list), must reproduce the
single-process result bit for bit once the shards are gathered."""
import os
import socket
import zlib

import numpy as np
import pytest

import oracle
from tests import kvgen
from tests.kvgen import BF16, FP8

torch = pytest.importorskip("torch")


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _case(kv, hkv=4):
    return kvgen.make_case(77 + kv, 2, hkv, 128, 4 * hkv, 7, 1, 400, kv, BF16)


def _full_result(c, pairs):
    data = c.data.copy()
    scales = None if c.scales is None else c.scales.copy()
    slots = kvgen.new_token_slots(c)
    outs = []
    for l in range(c.L):
        oracle.kv_append(c.geom, data, scales, l, c.k_new[l], c.v_new[l], slots)
        outs.append(oracle.paged_decode_f32(c.geom, data, scales, l, c.q[l], c.Hq,
                                            c.block_tables, c.seq_lens, 1.0 / np.sqrt(c.D)))
    oracle.block_copy(c.geom, data, scales, pairs)
    return np.stack(outs), data, scales


def _rank_main(rank, world, port, mode, kv, hkv=4):
    import torch.distributed as dist
    from voidweb_b200.shard import ShardPlan, gather_outputs
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        c = _case(kv, hkv)
        pairs = np.array([[int(c.block_tables[0, 0]), c.NB - 1]], dtype=np.uint32)
        plan = ShardPlan(mode, world, rank, c.B, c.Hq, c.Hkv)
        s0, s1 = plan.seqs()
        h0, h1 = plan.kv_heads()
        # this rank's pool: every block id, its own KV heads
        g = oracle.geom(c.L, h1 - h0, c.D, c.NB, c.kv, c.io, c.fp8_mode)
        # copies: a slice over every head would otherwise alias the case's pages
        data = c.data[:, :, h0:h1].copy()
        scales = None if c.scales is None else c.scales[:, :, h0:h1].copy()
        slots = kvgen.new_token_slots(c)[s0:s1]
        outs = []
        for l in range(c.L):
            q, kn, vn, bt, sl = plan.slice_inputs(c.q[l], c.k_new[l], c.v_new[l],
                                                  c.block_tables, c.seq_lens)
            oracle.kv_append(g, data, scales, l, np.ascontiguousarray(kn),
                             np.ascontiguousarray(vn), slots)
            local = oracle.paged_decode_f32(g, data, scales, l, q, q.shape[1], bt, sl,
                                            1.0 / np.sqrt(c.D))
            # gloo has no 16-bit integer type: carry the bf16 bits in int32
            outs.append(gather_outputs(plan, torch.from_numpy(local.astype(np.int32))))
        # block-copy lists are replayed on every rank
        oracle.block_copy(g, data, scales, pairs)
        ref_out, ref_data, ref_scales = _full_result(c, pairs)
        got = torch.stack(outs).numpy().astype(np.uint16)
        assert np.array_equal(got, ref_out), f"rank {rank}: gathered outputs differ"
        if mode == "kv_heads":
            assert np.array_equal(data, ref_data[:, :, h0:h1]), f"rank {rank}: pool shard differs"
            crc = torch.tensor([zlib.crc32(data.tobytes())], dtype=torch.int64)
            crcs = [torch.zeros_like(crc) for _ in range(world)]
            dist.all_gather(crcs, crc)
            for r in range(world):
                rp = ShardPlan(mode, world, r, c.B, c.Hq, c.Hkv)
                a, b = rp.kv_heads()
                want = zlib.crc32(np.ascontiguousarray(ref_data[:, :, a:b]).tobytes())
                assert int(crcs[r]) == want, f"rank {r}: pool checksum differs"
        else:
            # sequence shards append only their own rows: the rows they own match
            for b in range(s0, s1):
                p = int(c.seq_lens[b]) - 1
                blk = int(c.block_tables[b, p // 16])
                assert np.array_equal(data[:, blk, :, :, p % 16], ref_data[:, blk, h0:h1, :, p % 16])
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("mode,kv", [("sequences", BF16), ("kv_heads", BF16), ("kv_heads", FP8)])
def test_two_rank_shards_match_single_process(mode, kv):
    import torch.multiprocessing as mp
    mp.spawn(_rank_main, args=(2, _free_port(), mode, kv), nprocs=2, join=True)


def test_four_rank_heads_and_sequences_match_single_process():
    """Two head groups of two sequence slices each (2 KV heads on 4 ranks)."""
    import torch.multiprocessing as mp
    mp.spawn(_rank_main, args=(4, _free_port(), "kv_heads_seqs", BF16, 2), nprocs=4, join=True)


def test_placements_cover_every_segment_once():
    from voidweb_b200.shard import MODES, ShardPlan
    for mode in MODES:
        for world in (1, 2, 4, 8):
            for hkv in (1, 2, 4, 8):
                if mode == "kv_heads" and hkv < world:
                    with pytest.raises(ValueError):
                        ShardPlan(mode, world, 0, 16, 4 * hkv, hkv)
                    continue
                seen = np.zeros((16, hkv), dtype=int)
                for r in range(world):
                    p = ShardPlan(mode, world, r, 16, 4 * hkv, hkv)
                    s0, s1 = p.seqs()
                    h0, h1 = p.kv_heads()
                    seen[s0:s1, h0:h1] += 1
                    assert p.q_heads() == (h0 * 4, h1 * 4)
                assert (seen == 1).all(), (mode, world, hkv)


def test_shard_range_covers_everything():
    from voidweb_b200.shard import shard_range
    for n in range(0, 40):
        for world in (1, 2, 3, 8):
            spans = [shard_range(n, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(spans[i][1] == spans[i + 1][0] for i in range(world - 1))
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1
