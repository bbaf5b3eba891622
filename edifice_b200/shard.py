"""Shard planning and seeded synthetic inputs for the fused sequence-mixing configs.

One process per GPU.  Every config partitions into independent units (batch
rows for the scans and Mamba, (batch, head) pairs for DeltaNet, (batch,
kv-group) for GQA attention); ranks never exchange data on the kernel path.
Two plans:
  strong  the config's fixed problem is split over the ranks: rank r owns the
          contiguous units split_units(U, N)[r] (configs[4]: 64 batch rows ->
          8 per GPU at N = 8);
  weak    every rank processes a full config-sized shard of its own units, so
          the global problem at N GPUs is N shards of units [r*U, (r+1)*U).

Inputs of unit u are drawn from a generator seeded with (base_seed, u), so a
unit's data are identical whatever the world size and plan.
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


@dataclasses.dataclass(frozen=True)
class SsmConfig:
    """Mamba selective scan fwd+bwd, bf16 io, f32 state."""
    name: str = "selective_scan_cfg4"
    batch: int = 64
    seq_len: int = 8192
    d_inner: int = 4096
    d_state: int = 16
    dtype: torch.dtype = torch.bfloat16

    @property
    def units(self):
        return self.batch

    @property
    def tokens(self):
        return self.batch * self.seq_len

    def bytes_fwd(self):
        """read x, dt, B, C, A; write y"""
        es = torch.finfo(self.dtype).bits // 8
        e = self.batch * self.seq_len * self.d_inner
        bc = self.batch * self.seq_len * self.d_state
        return 3 * e * es + 2 * bc * es + self.d_inner * self.d_state * es

    def bytes_bwd(self):
        """read x, dt, dY, B, C, A; write dx, ddt (io dtype), dB, dC (f32)"""
        es = torch.finfo(self.dtype).bits // 8
        e = self.batch * self.seq_len * self.d_inner
        bc = self.batch * self.seq_len * self.d_state
        return 5 * e * es + 2 * bc * es + 2 * bc * 4 + self.d_inner * self.d_state * es

    def exps_fwd(self):
        """exp(dt A) evaluations of the forward: one per (b, t, d, n)."""
        return self.batch * self.seq_len * self.d_inner * self.d_state

    def exps_bwd(self):
        """Of the recompute-not-store backward: one per element to rebuild the
        sub-chunk start states from the chunk checkpoint, one to recompute each
        sub-chunk (its exp(dt A) then serves the reverse walk)."""
        return 2 * self.exps_fwd()


def ssm_cfg0():
    """the Mamba selective-scan forward the reference runs on
    its CPU host backend, f32, batch 2 x seq 256 x d_inner 512, d_state 16."""
    return SsmConfig(name="selective_scan_cfg0", batch=2, seq_len=256, d_inner=512, d_state=16,
                     dtype=torch.float32)


@dataclasses.dataclass(frozen=True)
class AttnConfig:
    """causal GQA attention fwd+bwd, bf16."""
    name: str = "flash_attention_cfg3"
    batch: int = 4
    q_heads: int = 32
    kv_heads: int = 8
    seq_len: int = 8192
    head_dim: int = 128
    causal: bool = True
    dtype: torch.dtype = torch.bfloat16

    @property
    def units(self):
        return self.batch * self.kv_heads  # (batch, kv-group) pairs

    @property
    def tokens(self):
        return self.batch * self.seq_len

    def flops_fwd(self):
        f = 4.0 * self.batch * self.q_heads * self.seq_len ** 2 * self.head_dim
        return f / 2 if self.causal else f

    def flops_bwd(self):
        return 2.5 * self.flops_fwd()


@dataclasses.dataclass(frozen=True)
class DeltaConfig:
    """DeltaNet fwd+bwd, bf16 io, f32 state, chunk 64,
    one beta per (token, head)."""
    name: str = "delta_net_cfg2"
    batch: int = 4
    heads: int = 16
    seq_len: int = 4096
    head_dim: int = 128
    chunk: int = 64
    dtype: torch.dtype = torch.bfloat16

    @property
    def units(self):
        return self.batch * self.heads  # (batch, head) pairs

    @property
    def tokens(self):
        return self.batch * self.seq_len

    def flops_fwd(self):
        # chunked WY form, dense-tile count: 10 C^2 d + 6 C d^2 per chunk
        C, d = self.chunk, self.head_dim
        n_chunks = self.batch * self.heads * self.seq_len // C
        return (10 * C * C * d + 6 * C * d * d) * n_chunks

    def flops_bwd(self):
        return 2 * self.flops_fwd()

    def bytes_fwd(self):
        e = self.batch * self.seq_len * self.heads * self.head_dim
        return 4 * e * 2 + self.batch * self.seq_len * self.heads * 2  # q k v o + beta

    def bytes_bwd(self):
        e = self.batch * self.seq_len * self.heads * self.head_dim
        return 8 * e * 2 + 2 * self.batch * self.seq_len * self.heads * 2


def unit_seed(base_seed, unit):
    return (int(base_seed) * 1_000_003 + int(unit)) & 0x7FFFFFFFFFFF


def plan_units(n_units_per_rank, rank, world_size):
    """Weak-scaling plan: rank r owns global units [r*U, (r+1)*U)."""
    if world_size < 1 or not (0 <= rank < world_size):
        raise ValueError("bad rank/world_size")
    lo = rank * n_units_per_rank
    return list(range(lo, lo + n_units_per_rank))


def units_for(n_units, rank, world_size, scaling="strong"):
    """The global unit indices rank `rank` processes under `scaling` ("strong":
    its contiguous share of the config's n_units; "weak": a full config of its
    own).  A strong split may leave a rank with no units (world > n_units)."""
    if scaling == "weak":
        return plan_units(n_units, rank, world_size)
    if scaling != "strong":
        raise ValueError("scaling must be 'strong' or 'weak'")
    if world_size < 1 or not (0 <= rank < world_size):
        raise ValueError("bad rank/world_size")
    start, count = split_units(n_units, world_size)[rank]
    return list(range(start, start + count))


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


def ssm_inputs(cfg, units, device, base_seed=0):
    """configs[0]/[4] distributions per batch-row unit: x ~ N(0,1);
    dt = softplus(0.5 N(0,1) - 2); B, C, dY ~ N(0,1); A = -exp(U(log 1, log 16))
    shared by all units (its own seed).  Returns x, dt, A, B, C, dy."""
    L, D, N = cfg.seq_len, cfg.d_inner, cfg.d_state
    U = len(units)
    x = torch.empty((U, L, D), dtype=cfg.dtype, device=device)
    dt, dy = torch.empty_like(x), torch.empty_like(x)
    Bm = torch.empty((U, L, N), dtype=cfg.dtype, device=device)
    Cm = torch.empty_like(Bm)
    for i, u in enumerate(units):
        g = torch.Generator(device=device).manual_seed(unit_seed(base_seed, u))
        x[i].copy_(torch.randn((L, D), generator=g, device=device))
        dt[i].copy_(torch.nn.functional.softplus(
            torch.randn((L, D), generator=g, device=device) * 0.5 - 2))
        Bm[i].copy_(torch.randn((L, N), generator=g, device=device))
        Cm[i].copy_(torch.randn((L, N), generator=g, device=device))
        dy[i].copy_(torch.randn((L, D), generator=g, device=device))
    g = torch.Generator(device=device).manual_seed(unit_seed(base_seed, 1 << 40))
    A = (-torch.exp(torch.rand((D, N), generator=g, device=device) * math.log(16.0))).to(cfg.dtype)
    return x, dt, A, Bm, Cm, dy


def attn_inputs(cfg, units, device, base_seed=0):
    """configs[3] per (batch, kv-group) unit: q, k, v, dO ~ N(0,1).  The rank's
    units are laid out unit-major, q/dO [U, G, L, d] and k/v [U, 1, L, d] (G query
    heads per kv head), which is byte for byte the reference's [B, Hq, L, d] /
    [B, Hkv, L, d] layout of whole batches; when the units make whole batches the
    tensors are returned in that [U/Hkv, Hq, L, d] / [U/Hkv, Hkv, L, d] form."""
    G = cfg.q_heads // cfg.kv_heads
    L, d = cfg.seq_len, cfg.head_dim
    U = len(units)
    q = torch.empty((U, G, L, d), dtype=cfg.dtype, device=device)
    do = torch.empty_like(q)
    k = torch.empty((U, 1, L, d), dtype=cfg.dtype, device=device)
    v = torch.empty_like(k)
    for i, u in enumerate(units):
        g = torch.Generator(device=device).manual_seed(unit_seed(base_seed, u))
        q[i].copy_(torch.randn((G, L, d), generator=g, device=device))
        k[i, 0].copy_(torch.randn((L, d), generator=g, device=device))
        v[i, 0].copy_(torch.randn((L, d), generator=g, device=device))
        do[i].copy_(torch.randn((G, L, d), generator=g, device=device))
    if U % cfg.kv_heads == 0 and all(u % cfg.kv_heads == i % cfg.kv_heads
                                     for i, u in enumerate(units)):
        nb = U // cfg.kv_heads
        q, do = (t.view(nb, cfg.q_heads, L, d) for t in (q, do))
        k, v = (t.view(nb, cfg.kv_heads, L, d) for t in (k, v))
    return q, k, v, do


def _delta_heads(cfg, units):
    """Heads per batch entry of a rank's (batch, head) units: whole batches keep
    cfg.heads; a run of consecutive heads of one batch becomes one batch entry."""
    U, H = len(units), cfg.heads
    if U % H == 0:
        return H
    if H % U == 0 and units[0] // H == units[-1] // H:
        return U
    raise ValueError("a rank's (batch, head) units must be whole batches or part of one")


def delta_inputs(cfg, units, device, base_seed=0):
    """configs[2] per (batch, head) unit: q, k ~ N(0,1), k L2-normalised over d;
    v ~ N(0,1); beta = sigmoid(N(0,1)) per token; dO ~ N(0,1).  The rank's units
    are laid out as a [len(units)/Hl, L, Hl, d] batch, Hl = heads for whole
    batches, else the number of units (consecutive heads of one batch)."""
    L, d = cfg.seq_len, cfg.head_dim
    H = _delta_heads(cfg, units)
    nb = len(units) // H
    q = torch.empty((nb, L, H, d), dtype=cfg.dtype, device=device)
    k, v, do = torch.empty_like(q), torch.empty_like(q), torch.empty_like(q)
    beta = torch.empty((nb, L, H), dtype=cfg.dtype, device=device)
    for i, u in enumerate(units):
        b, h = divmod(i, H)
        g = torch.Generator(device=device).manual_seed(unit_seed(base_seed, u))
        q[b, :, h].copy_(torch.randn((L, d), generator=g, device=device))
        kk = torch.randn((L, d), generator=g, device=device)
        k[b, :, h].copy_(kk / torch.sqrt((kk * kk).sum(-1, keepdim=True) + 1e-6))
        v[b, :, h].copy_(torch.randn((L, d), generator=g, device=device))
        beta[b, :, h].copy_(torch.sigmoid(torch.randn((L,), generator=g, device=device)))
        do[b, :, h].copy_(torch.randn((L, d), generator=g, device=device))
    return q, k, v, beta, do


def gated_alpha(cfg, units, device, base_seed=0):
    """The decay of GatedDeltaNet per (batch, head) unit, alpha [len(units)/heads, L,
    heads]: the mean over head_dim of sigmoid(N(0,1)) gates, the model's form
    (lib/edifice/recurrent/gated_delta_net.ex:382-389), drawn after that unit's
    delta_inputs stream (a separate generator offset, so the q/k/v/beta/dO draws
    are the configs[2] ones).  Laid out as delta_inputs lays out the units."""
    L, d = cfg.seq_len, cfg.head_dim
    H = _delta_heads(cfg, units)
    nb = len(units) // H
    alpha = torch.empty((nb, L, H), dtype=cfg.dtype, device=device)
    for i, u in enumerate(units):
        b, h = divmod(i, H)
        g = torch.Generator(device=device).manual_seed(unit_seed(base_seed + 1, u))
        gates = torch.sigmoid(torch.randn((L, d), generator=g, device=device))
        alpha[b, :, h].copy_(gates.mean(-1))
    return alpha


def all_gather_units(local, group=None):
    """A replicated output, when the caller asks for one: every rank's shard
    (dim 0 unit-major over its contiguous units, e.g. batch rows) gathered in rank
    order along dim 0, so each rank holds the whole problem's tensor.  NCCL over
    NVLink on GPUs, gloo on CPU.  The kernel path never calls it; it is the one
    collective the sharded configs have, and it moves only outputs."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    local = local.contiguous()
    out = torch.empty((world * local.shape[0],) + tuple(local.shape[1:]), dtype=local.dtype,
                      device=local.device)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(out, local, group=group)
    else:
        dist.all_gather(list(out.chunk(world)), local, group=group)
    return out


def ceil_div(a, b):
    return -(-a // b)


def grid_waves(ctas, sms=148, per_sm=1):
    return math.ceil(ctas / (sms * per_sm))
