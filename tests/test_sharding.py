"""Multi-GPU partition of the independent (batch, head) units: host logic, and a
world_size-2 gloo run where each rank evaluates its shard with the oracle and the
gathered shards equal the single-process result."""
import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from flash_attention_sm75.sharding import batch_range, shard_units


@pytest.mark.parametrize("B,Hq,Hkv,world", [(4, 32, 32, 8), (2, 32, 8, 8), (4, 12, 12, 5),
                                            (1, 1, 1, 2), (2, 32, 8, 3)])
def test_partition_covers_each_unit_once(B, Hq, Hkv, world):
    seen = []
    for r in range(world):
        sh = shard_units(B, Hq, Hkv, world, r)
        seen += sh.query_units
        # GQA: a rank owns whole groups of query heads sharing one KV head
        for (b, h) in sh.query_units:
            assert (b, h // (Hq // Hkv)) in sh.groups
    assert sorted(seen) == [(b, h) for b in range(B) for h in range(Hq)]
    sizes = [len(shard_units(B, Hq, Hkv, world, r).groups) for r in range(world)]
    assert max(sizes) - min(sizes) <= 1


def test_bad_arguments():
    with pytest.raises(ValueError):
        shard_units(1, 6, 4, 2, 0)
    with pytest.raises(ValueError):
        shard_units(1, 4, 4, 2, 2)
    assert batch_range(4, 3) == (12, 16)


def _worker(rank, world, port, out_path):
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path[:0] = [os.path.dirname(here), os.path.join(os.path.dirname(here),
                                                         "flash-attention-sm75-register-fused_b200")]
    from oracle import attention_oracle as orc
    from flash_attention_sm75.sharding import shard_units as su
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg = orc.AttnConfig("t", 2, 8, 2, 96, 64, True)
        q, k, v = orc.make_inputs(cfg, seed=5)
        sh = su(cfg.B, cfg.Hq, cfg.Hkv, world, rank)
        out = torch.zeros(cfg.B, cfg.Hq, cfg.N, cfg.d)
        g = cfg.Hq // cfg.Hkv
        for (b, hk) in sh.groups:
            o, _ = orc.attention_fp32(q[b:b + 1, hk * g:(hk + 1) * g], k[b:b + 1, hk:hk + 1],
                                      v[b:b + 1, hk:hk + 1], causal=True)
            out[b, hk * g:(hk + 1) * g] = o[0]
        dist.all_reduce(out)  # shards are disjoint: the sum assembles the full output
        if rank == 0:
            torch.save(out, out_path)
    finally:
        dist.destroy_process_group()


def test_gloo_two_ranks_assemble_full_output(tmp_path):
    import socket
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    out_path = str(tmp_path / "out.pt")
    mp.start_processes(_worker, args=(2, port, out_path), nprocs=2, start_method="spawn", join=True)
    from oracle import attention_oracle as orc
    cfg = orc.AttnConfig("t", 2, 8, 2, 96, 64, True)
    q, k, v = orc.make_inputs(cfg, seed=5)
    full, _ = orc.attention_fp32(q, k, v, causal=True)
    got = torch.load(out_path)
    assert torch.allclose(got, full, atol=1e-6)


def _bench_worker(rank, world, port, out_path):
    """One rank of bench.py's strong-scaling path on CPU: its RankShard views
    of the global tensors, the oracle in place of the kernel, then the
    all-gather that brings every rank's O / LSE to rank 0."""
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path[:0] = [os.path.dirname(here), os.path.join(os.path.dirname(here),
                                                         "flash-attention-sm75-register-fused_b200")]
    import bench
    from oracle import attention_oracle as orc
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg = orc.AttnConfig("t", 3, 8, 2, 80, 64, True)
        q, k, v = orc.make_inputs(cfg, seed=6)
        o = torch.zeros(q.shape, dtype=torch.float32)
        lse = torch.zeros(q.shape[:3])
        sh = bench.RankShard(cfg, world, rank, "strong")
        qs, ks, vs, os_, ls = sh.views(cfg, q, k, v, o, lse)
        if sh.units:
            oo, ll = orc.attention_fp32(qs[None], ks[None], vs[None], causal=True)
            os_.copy_(oo[0])
            ls.copy_(ll[0])
        max_heads = -(-cfg.B * cfg.Hkv // world) * sh.G
        go = bench.gather_to_rank0(dist, os_, sh.q_heads, max_heads, world, "cpu")
        gl = bench.gather_to_rank0(dist, ls, sh.q_heads, max_heads, world, "cpu")
        counts = bench.units_per_rank(cfg, world, "strong")
        if rank == 0:
            o_full = torch.cat([go[r, :c * sh.G] for r, c in enumerate(counts)]).view_as(o)
            l_full = torch.cat([gl[r, :c * sh.G] for r, c in enumerate(counts)]).view_as(lse)
            torch.save((o_full, l_full), out_path)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_bench_strong_scaling_shards_reassemble(tmp_path, world):
    """bench.py's strong-scaling split (6 KV-head groups over 2 or 4 ranks, the
    latter uneven) gathers back to exactly the single-process result."""
    import socket
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    out_path = str(tmp_path / "out.pt")
    mp.start_processes(_bench_worker, args=(world, port, out_path), nprocs=world,
                       start_method="spawn", join=True)
    from oracle import attention_oracle as orc
    cfg = orc.AttnConfig("t", 3, 8, 2, 80, 64, True)
    q, k, v = orc.make_inputs(cfg, seed=6)
    full, full_l = orc.attention_fp32(q, k, v, causal=True)
    got, got_l = torch.load(out_path)
    assert torch.allclose(got, full, atol=1e-6)
    assert torch.allclose(got_l, full_l, atol=1e-6)
