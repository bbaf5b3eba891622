"""GPU parity of the DeltaNet delta rule (forward + backward) against the oracle,
the golden DeltaNet vectors, and the reference's own delta-rule CUDA kernels."""
import ctypes
import os

import numpy as np
import pytest
import torch

import oracle as O
from oracle import build as ob
from edifice_b200 import fused_scan as fs
from edifice_b200 import build, device_errors

pytestmark = pytest.mark.gpu

TOL = {torch.float32: 1e-4, torch.bfloat16: 2e-2}
GOLD = os.path.join(os.path.dirname(__file__), "golden")


def _np(t):
    return t.detach().float().cpu().numpy()


def delta_inputs(B, L, H, d, dtype, seed, scalar_beta):
    """configs[2] distributions: q, k ~ N(0,1), k L2-normalised per head; v ~ N(0,1);
    beta = sigmoid(N(0,1)); dO ~ N(0,1)."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    q = torch.randn(B, L, H, d, generator=g)
    k = torch.randn(B, L, H, d, generator=g)
    k = k / torch.sqrt((k * k).sum(-1, keepdim=True) + 1e-6)
    v = torch.randn(B, L, H, d, generator=g)
    beta = torch.sigmoid(torch.randn((B, L, H) if scalar_beta else (B, L, H, d), generator=g))
    do = torch.randn(B, L, H, d, generator=g)
    return [t.to(dtype).cuda() for t in (q, k, v, beta, do)]


CASES = [
    (1, 3, 2, 2),       # the reference's backward test shape
    (2, 8, 4, 8),
    (2, 100, 3, 16),
    (1, 300, 2, 64),    # several checkpoint chunks
    (1, 130, 2, 128),
]


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("case", CASES)
@pytest.mark.parametrize("scalar_beta", [False, True])
@pytest.mark.parametrize("use_ckpt", [False, True])
def test_delta_rule_parity(cuda, dtype, case, scalar_beta, use_ckpt):
    q, k, v, beta, do = delta_inputs(*case, dtype, seed=51, scalar_beta=scalar_beta)
    if use_ckpt:
        o, ck = fs.delta_net_scan(q, k, v, beta, with_ckpt=True)
    else:
        o, ck = fs.delta_net_scan(q, k, v, beta), None
    grads = fs.delta_rule_backward(q, k, v, beta, do, ck)
    torch.cuda.synchronize()
    args = [_np(t) for t in (q, k, v, beta)]
    assert O.norm_rel(_np(o), O.delta_net_fwd(*args)) <= TOL[dtype]
    ref = O.delta_net_bwd(*args, _np(do))
    for got, r in zip(grads, ref):
        assert got.shape == torch.Size(r.shape)
        assert O.norm_rel(_np(got), r) <= TOL[dtype], O.norm_rel(_np(got), r)
    assert device_errors() == 0


CHUNKED_CASES = [
    (1, 1, 1, 128),     # one token
    (1, 64, 1, 128),    # exactly one chunk
    (2, 200, 3, 128),   # ragged last chunk
    (1, 1000, 2, 128),  # many chunks
]


@pytest.mark.parametrize("case", CHUNKED_CASES)
def test_delta_chunked_forward(cuda, case):
    """bf16 io, one beta per token, head_dim 128: the chunked tensor-core
    forward and backward.  Outputs and gradients against the oracle; the
    chunk-start states (stored transposed by this path) against the token
    recurrence's, [B][H][nchunks + 1][d][d], from the f32 path run on the same
    bf16-rounded inputs."""
    B, L, H, d = case
    q, k, v, beta, do = delta_inputs(*case, torch.bfloat16, seed=54, scalar_beta=True)
    o, ck = fs.delta_net_scan(q, k, v, beta, with_ckpt=True)
    of, ckf = fs.delta_net_scan(q.float(), k.float(), v.float(), beta.float(), with_ckpt=True)
    torch.cuda.synchronize()
    assert device_errors() == 0
    args = [_np(t) for t in (q, k, v, beta)]
    ref = O.delta_net_fwd(*args)
    assert O.norm_rel(_np(o), ref) <= 2e-2
    assert O.norm_rel(_np(of), ref) <= 1e-4
    nc = (L + 63) // 64
    states = ck[:B * H * (nc + 1) * d * d].view(B, H, nc + 1, d, d).transpose(-1, -2)
    assert ck.numel() == B * H * (nc + 1) * d * d + B * H * nc * 64 * d
    # the token recurrence checkpoints every 16 tokens: its 64-token chunk starts are
    # every 4th slot, its final state the last
    ncp = (L + 15) // 16
    tok = ckf.view(B, H, ncp + 1, d, d)
    tok = torch.cat([tok[:, :, 0:4 * nc:4], tok[:, :, ncp:]], dim=2)
    assert O.norm_rel(_np(states), _np(tok)) <= 5e-3
    rg = O.delta_net_bwd(*args, _np(do))
    for ckpt in (ck, None):  # residuals from the forward, or recomputed inside
        grads = fs.delta_rule_backward(q, k, v, beta, do, ckpt)
        torch.cuda.synchronize()
        assert device_errors() == 0
        for got, r in zip(grads, rg):
            assert got.shape == torch.Size(r.shape)
            assert O.norm_rel(_np(got), r) <= 2e-2, O.norm_rel(_np(got), r)


@pytest.mark.parametrize("layer", [0, 1])
def test_delta_golden(cuda, layer):
    g = np.load(os.path.join(GOLD, "delta_net_fixture.npz"))
    q, k, v, beta, do = (torch.tensor(g["%s%d" % (n, layer)]).cuda()
                         for n in ("q", "k", "v", "beta", "do"))
    o = fs.delta_net_scan(q, k, v, beta)
    grads = fs.delta_rule_backward(q, k, v, beta, do)
    torch.cuda.synchronize()
    np.testing.assert_allclose(_np(o), g["o%d" % layer], atol=2e-5)
    for got, n in zip(grads, ("gq", "gk", "gv", "gbeta")):
        np.testing.assert_allclose(_np(got), g["%s%d" % (n, layer)], atol=5e-5)


def test_config2_full_size_sampled_heads(cuda):
    """B4 H16 L4096 d128, scalar beta, bf16.  Heads are
    independent, so two sampled (b, h) pairs are checked against the oracle."""
    B, L, H, d = 4, 4096, 16, 128
    q, k, v, beta, do = delta_inputs(B, L, H, d, torch.bfloat16, seed=0, scalar_beta=True)
    o, ck = fs.delta_net_scan(q, k, v, beta, with_ckpt=True)
    grads = fs.delta_rule_backward(q, k, v, beta, do, ck)
    torch.cuda.synchronize()
    assert device_errors() == 0
    for b, h in ((0, 0), (3, 11)):
        sl = lambda t: _np(t[b:b + 1, :, h:h + 1])
        args = [sl(q), sl(k), sl(v), _np(beta[b:b + 1, :, h:h + 1])]
        assert O.norm_rel(sl(o), O.delta_net_fwd(*args)) <= 2e-2
        ref = O.delta_net_bwd(*args, sl(do))
        got = [sl(grads[0]), sl(grads[1]), sl(grads[2]), _np(grads[3][b:b + 1, :, h:h + 1])]
        for gg, r in zip(got, ref):
            assert O.norm_rel(gg, r) <= 2e-2


@pytest.mark.skipif(not os.path.exists(ob.REF_KERNELS_SO["f32"]), reason="oracle/_ref not built")
def test_oracle_matches_reference_cuda_delta(cuda):
    """Pin the oracle's delta rule (per-element beta, forward and backward)
    against the reference's own fused_delta_net_scan_launch and
    fused_delta_rule_scan_backward_launch (f32 build for sm_100a)."""
    lib = ctypes.CDLL(ob.REF_KERNELS_SO["f32"])
    B, L, H, d = 2, 40, 3, 16
    q, k, v, beta, do = delta_inputs(B, L, H, d, torch.float32, seed=52, scalar_beta=False)
    P = lambda t: ctypes.c_void_p(t.data_ptr())
    o = torch.empty_like(q)
    assert lib.fused_delta_net_scan_launch(None, P(q), P(k), P(v), P(beta), P(o), B, L, H, d) == 0
    cat = torch.empty(4 * q.numel(), dtype=torch.float32, device="cuda")
    assert lib.fused_delta_rule_scan_backward_launch(None, P(q), P(k), P(v), P(beta), P(o), P(do),
                                                     P(cat), B, L, H, d) == 0
    torch.cuda.synchronize()
    args = [_np(t) for t in (q, k, v, beta)]
    assert O.norm_rel(_np(o), O.delta_net_fwd(*args)) <= 1e-5
    ref = O.delta_net_bwd(*args, _np(do))
    n = q.numel()
    for idx, r in enumerate(ref):
        assert O.norm_rel(_np(cat[idx * n:(idx + 1) * n]).reshape(r.shape), r) <= 1e-4


@pytest.mark.parametrize("prec,dtype", [("f32", torch.float32), ("bf16", torch.bfloat16)])
def test_legacy_shim(cuda, prec, dtype):
    lib = ctypes.CDLL(build.SHIMS[prec])
    B, L, H, d = 2, 70, 2, 32
    q, k, v, beta, do = delta_inputs(B, L, H, d, dtype, seed=53, scalar_beta=False)
    P = lambda t: ctypes.c_void_p(t.data_ptr())
    o = torch.empty_like(q)
    assert lib.fused_delta_net_scan_launch(None, P(q), P(k), P(v), P(beta), P(o), B, L, H, d) == 0
    cat = torch.empty(4 * q.numel(), dtype=dtype, device="cuda")
    assert lib.fused_delta_rule_scan_backward_launch(None, P(q), P(k), P(v), P(beta), P(o), P(do),
                                                     P(cat), B, L, H, d) == 0
    torch.cuda.synchronize()
    assert torch.equal(o, fs.delta_net_scan(q, k, v, beta))
    ref = fs.delta_rule_backward(q, k, v, beta, do)
    torch.cuda.synchronize()
    n = q.numel()
    for idx, r in enumerate(ref):
        assert torch.equal(cat[idx * n:(idx + 1) * n].view(r.shape), r)


def test_autograd_fn(cuda):
    q, k, v, beta, do = delta_inputs(2, 50, 2, 32, torch.float32, seed=54, scalar_beta=True)
    leaves = [t.clone().requires_grad_(True) for t in (q, k, v, beta)]
    o = fs.DeltaNetFn.apply(*leaves)
    o.backward(do)
    ref = O.delta_net_bwd(*[_np(t) for t in (q, k, v, beta)], _np(do))
    for leaf, r in zip(leaves, ref):
        assert O.norm_rel(_np(leaf.grad), r) <= 1e-4


@pytest.mark.parametrize("dtype,scalar_beta,d", [(torch.bfloat16, True, 128),
                                                 (torch.bfloat16, False, 64),
                                                 (torch.float32, True, 32)])
@pytest.mark.parametrize("B,L,H", [(4, 130, 2), (7, 70, 3)])
def test_delta_rule_train_host(cuda, dtype, scalar_beta, d, B, L, H):
    """Forward + backward over pinned host tensors (batch-row chunks through a ring of
    three slots, each on its own compute stream) equals the device entry points on the
    whole batch bit for bit: every (batch, head) recurrence is independent."""
    q, k, v, beta, do = delta_inputs(B, L, H, d, dtype, seed=80 + L, scalar_beta=scalar_beta)
    o_r, ck = fs.delta_net_scan(q, k, v, beta, with_ckpt=True)
    ref = (o_r,) + tuple(fs.delta_rule_backward(q, k, v, beta, do, ck))
    pin = [t.cpu().pin_memory() for t in (q, k, v, beta, do)]
    for _ in range(2):
        out = fs.delta_rule_train_host(*pin)
        torch.cuda.synchronize()
        for o, r in zip(out, ref):
            assert o.dtype == r.dtype and o.shape == r.shape
            assert torch.equal(o, r.cpu())
    assert device_errors() == 0
