"""Host-side logic of the multi-GPU path (strong and weak plans), on CPU.

Every config partitions into independent units (batch rows; (batch, head);
(batch, kv group)); a rank owns a contiguous range of global units and draws
each unit's inputs from its own seed, so a unit's data never depends on the
world size.  The only collectives are the barrier and the max-over-ranks time
reduction of bench.py, exercised here on a world_size-2 gloo group.
"""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from edifice_b200 import shard


def test_plan_units_weak_scaling():
    for world in (1, 2, 4, 8):
        seen = []
        for r in range(world):
            u = shard.plan_units(3, r, world)
            assert u == list(range(3 * r, 3 * r + 3))
            seen += u
        assert seen == list(range(3 * world))
    with pytest.raises(ValueError):
        shard.plan_units(3, 2, 2)
    with pytest.raises(ValueError):
        shard.plan_units(3, 0, 0)


def test_split_units_strong_scaling():
    for n, w in ((64, 8), (10, 4), (3, 8)):
        parts = shard.split_units(n, w)
        assert sum(c for _, c in parts) == n
        assert max(c for _, c in parts) - min(c for _, c in parts) <= 1
        starts = [s for s, _ in parts]
        assert starts == sorted(starts) and starts[0] == 0


def test_unit_inputs_do_not_depend_on_world_size():
    cfg = shard.ScanConfig(batch=4, seq_len=16, hidden=32, dtype=torch.float32)
    a_all, b_all, dy_all = shard.scan_inputs(cfg, [0, 1, 2, 3], "cpu")
    a_r1, b_r1, dy_r1 = shard.scan_inputs(cfg, shard.plan_units(2, 1, 2), "cpu")
    assert torch.equal(a_all[2:], a_r1) and torch.equal(b_all[2:], b_r1)
    assert torch.equal(dy_all[2:], dy_r1)
    dcfg = shard.DeltaConfig(batch=2, heads=2, seq_len=8, head_dim=16, dtype=torch.float32)
    full = shard.delta_inputs(dcfg, [0, 1, 2, 3], "cpu")
    upper = shard.delta_inputs(dcfg, [2, 3], "cpu")  # (b=1, h=0..1) of the full problem
    for f, u in zip(full, upper):
        assert torch.equal(f[1:], u)


def test_units_for_strong_and_weak():
    # strong: the fixed configs[4] batch of 64 rows, 64/N rows per rank
    for world in (1, 2, 4, 8):
        seen = []
        for r in range(world):
            u = shard.units_for(64, r, world, "strong")
            assert len(u) == 64 // world
            seen += u
        assert seen == list(range(64))
        assert shard.units_for(64, 1, world, "weak") == list(range(64, 128)) if world > 1 \
            else True
    # more ranks than units: the surplus ranks get none
    assert [len(shard.units_for(2, r, 8, "strong")) for r in range(8)] == [1, 1] + [0] * 6
    with pytest.raises(ValueError):
        shard.units_for(4, 0, 2, "sideways")


def test_strong_split_layouts_match_the_full_problem():
    """A rank's share of a strong split holds exactly the full problem's values of
    its units, in the layout the kernels take: attention units of part of a batch
    become a [U, G, L, d] batch (byte for byte the [B, Hq, L, d] layout), delta-rule
    units of part of a batch a [1, L, U, d] batch."""
    acfg = shard.AttnConfig(batch=2, q_heads=8, kv_heads=4, seq_len=8, head_dim=16,
                            dtype=torch.float32)
    full = shard.attn_inputs(acfg, list(range(8)), "cpu")
    assert full[0].shape == (2, 8, 8, 16) and full[1].shape == (2, 4, 8, 16)
    part = shard.attn_inputs(acfg, shard.units_for(8, 3, 4, "strong"), "cpu")  # units 6, 7
    assert part[0].shape == (2, 2, 8, 16) and part[1].shape == (2, 1, 8, 16)
    assert torch.equal(part[0].reshape(2 * 2, 8, 16), full[0][1, 4:8])
    assert torch.equal(part[1].reshape(2, 8, 16), full[1][1, 2:4])
    dcfg = shard.DeltaConfig(batch=2, heads=4, seq_len=8, head_dim=16, dtype=torch.float32)
    dfull = shard.delta_inputs(dcfg, list(range(8)), "cpu")
    dpart = shard.delta_inputs(dcfg, shard.units_for(8, 3, 4, "strong"), "cpu")  # (1, 2..3)
    assert dpart[0].shape == (1, 8, 2, 16) and dpart[3].shape == (1, 8, 2)
    for f, u in zip(dfull, dpart):
        assert torch.equal(f[1:, :, 2:4], u)
    gfull = shard.gated_alpha(dcfg, list(range(8)), "cpu")
    assert torch.equal(gfull[1:, :, 2:4], shard.gated_alpha(dcfg, [6, 7], "cpu"))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg = shard.ScanConfig(batch=2, seq_len=16, hidden=32, dtype=torch.float32)
        units = shard.plan_units(cfg.batch, rank, world)
        a, b, _ = shard.scan_inputs(cfg, units, "cpu")
        # this rank's "elapsed time": the bench takes the max over ranks
        t = torch.tensor([1.5 + rank], dtype=torch.float64)
        dist.barrier()
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        sums = [torch.zeros(2, dtype=torch.float64) for _ in range(world)]
        dist.all_gather(sums, torch.tensor([a.double().sum(), b.double().sum()]))
        if rank == 0:
            torch.save({"tmax": float(t), "sums": torch.stack(sums)}, out_path)
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_two_rank_gloo_plan_and_max_time(tmp_path):
    world = 2
    out = str(tmp_path / "r0.pt")
    mp.spawn(_rank_main, args=(world, _free_port(), out), nprocs=world, join=True)
    res = torch.load(out)
    assert res["tmax"] == 1.5 + (world - 1)
    cfg = shard.ScanConfig(batch=2, seq_len=16, hidden=32, dtype=torch.float32)
    a, b, _ = shard.scan_inputs(cfg, list(range(cfg.batch * world)), "cpu")
    for r in range(world):
        sl = slice(r * cfg.batch, (r + 1) * cfg.batch)
        assert torch.allclose(res["sums"][r],
                              torch.tensor([a[sl].double().sum(), b[sl].double().sum()]))


def _gather_main(rank, world, port, out_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg = shard.ScanConfig(batch=2, seq_len=16, hidden=32, dtype=torch.float32)
        a, _, _ = shard.scan_inputs(cfg, shard.plan_units(cfg.batch, rank, world), "cpu")
        dcfg = shard.DeltaConfig(batch=1, heads=2, seq_len=8, head_dim=16, dtype=torch.float32)
        q = shard.delta_inputs(dcfg, shard.plan_units(dcfg.batch * dcfg.heads, rank, world),
                               "cpu")[0]
        ga = shard.all_gather_units(a)
        gq = shard.all_gather_units(q)
        if rank == 0:
            torch.save({"a": ga, "q": gq}, out_path)
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_two_rank_gloo_replicated_output(tmp_path):
    """all_gather_units rebuilds the whole problem's tensor on every rank from the
    ranks' unit shards (batch rows; (batch, head) units of whole batch rows)."""
    world = 2
    out = str(tmp_path / "g0.pt")
    mp.spawn(_gather_main, args=(world, _free_port(), out), nprocs=world, join=True)
    res = torch.load(out)
    cfg = shard.ScanConfig(batch=2, seq_len=16, hidden=32, dtype=torch.float32)
    a, _, _ = shard.scan_inputs(cfg, list(range(cfg.batch * world)), "cpu")
    assert torch.equal(res["a"], a)
    dcfg = shard.DeltaConfig(batch=1, heads=2, seq_len=8, head_dim=16, dtype=torch.float32)
    q = shard.delta_inputs(dcfg, list(range(dcfg.batch * dcfg.heads * world)), "cpu")[0]
    assert torch.equal(res["q"], q)


def test_gated_alpha_per_unit():
    """GatedDeltaNet decays: in (0, 1), identical for a unit wherever it lands."""
    cfg = shard.DeltaConfig(batch=2, heads=2, seq_len=16, head_dim=8, dtype=torch.float32)
    a_all = shard.gated_alpha(cfg, [0, 1, 2, 3], torch.device("cpu"))
    a_hi = shard.gated_alpha(cfg, [2, 3], torch.device("cpu"))
    assert a_all.shape == (2, 16, 2)
    assert torch.equal(a_all[1], a_hi[0])
    assert float(a_all.min()) > 0.0 and float(a_all.max()) < 1.0
