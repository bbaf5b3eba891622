"""Shard planning and seeded synthetic inputs for the fused sequence-mixing configs.

One process per GPU.  Every config partitions into independent units (batch
rows for the scans and Mamba, (batch, head) pairs for DeltaNet, (batch,
kv-group) for GQA attention); ranks never exchange data on the kernel path.
Weak scaling: every rank processes a full config-sized shard of its own units,
so the global problem at N GPUs is N shards of units [rank*U, (rank+1)*U).

Inputs of unit u are drawn from a generator seeded with (base_seed, u), so a
unit's data are identical whatever the world size.
"""
import dataclasses
import math

import torch


@dataclasses.dataclass(frozen=True)
class ScanConfig:
    """diagonal linear-RNN scan fwd+bwd, bf16 io, f32 state."""
    name: str = "linear_scan_cfg1"
    batch: int = 8
    seq_len: int = 4096
    hidden: int = 2048
    dtype: torch.dtype = torch.bfloat16
    mingru: bool = False

    @property
    def units(self):
        return self.batch

    @property
    def tokens(self):
        return self.batch * self.seq_len

    def bytes_fwd(self):
        e = self.batch * self.seq_len * self.hidden
        es = torch.finfo(self.dtype).bits // 8
        return 3 * e * es  # read a, b; write h

    def bytes_bwd(self):
        e = self.batch * self.seq_len * self.hidden
        es = torch.finfo(self.dtype).bits // 8
        n_in = 4 if self.mingru else 3   # a|z, (c), h, dY
        return (n_in + 2) * e * es + self.batch * self.hidden * es


def unit_seed(base_seed, unit):
    return (int(base_seed) * 1_000_003 + int(unit)) & 0x7FFFFFFFFFFF


def plan_units(n_units_per_rank, rank, world_size):
    """Weak-scaling plan: rank r owns global units [r*U, (r+1)*U)."""
    if world_size < 1 or not (0 <= rank < world_size):
        raise ValueError("bad rank/world_size")
    lo = rank * n_units_per_rank
    return list(range(lo, lo + n_units_per_rank))


def split_units(n_units, world_size):
    """Strong-scaling split of n_units over world_size ranks (contiguous, sizes
    differ by at most one).  Returns a list of (start, count)."""
    base, rem = divmod(n_units, world_size)
    out, s = [], 0
    for r in range(world_size):
        c = base + (1 if r < rem else 0)
        out.append((s, c))
        s += c
    return out


def scan_inputs(cfg, units, device, base_seed=0):
    """a = sigmoid(N(0,1)), b ~ N(0,1), dY ~ N(0,1) for each batch-row unit,
    drawn in f32 and rounded to cfg.dtype.  Returns (a, b, dy) [U, L, H]."""
    L, H = cfg.seq_len, cfg.hidden
    a = torch.empty((len(units), L, H), dtype=cfg.dtype, device=device)
    b = torch.empty_like(a)
    dy = torch.empty_like(a)
    for i, u in enumerate(units):
        g = torch.Generator(device=device).manual_seed(unit_seed(base_seed, u))
        a[i].copy_(torch.sigmoid(torch.randn((L, H), generator=g, device=device)))
        b[i].copy_(torch.randn((L, H), generator=g, device=device))
        dy[i].copy_(torch.randn((L, H), generator=g, device=device))
    return a, b, dy


def ceil_div(a, b):
    return -(-a // b)


def grid_waves(ctas, sms=148, per_sm=1):
    return math.ceil(ctas / (sms * per_sm))
