"""GPU parity of GatedDeltaNet (the delta rule with a per-token decay alpha),
forward + backward, against the oracle (gated_delta_net_scan_fallback,
fused_scan.ex:2256-2284, and its backward :1347-1431 with the exact key
gradient), through the C-ABI, the legacy reference-named shims and the
autograd wrapper."""
import ctypes

import pytest
import torch

import oracle as O
from edifice_b200 import fused_scan as fs
from edifice_b200 import build, device_errors

pytestmark = pytest.mark.gpu

TOL = {torch.float32: 1e-4, torch.bfloat16: 2e-2}


def _np(t):
    return t.detach().float().cpu().numpy()


def gated_inputs(B, L, H, d, dtype, seed, scalar_beta, alpha_lo=0.05):
    """q, k ~ N(0,1), k L2-normalised per head; v ~ N(0,1); beta = sigmoid(N(0,1));
    alpha ~ U(alpha_lo, 1) (the model's mean of sigmoids lies in (0, 1)); dO ~ N(0,1)."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    q = torch.randn(B, L, H, d, generator=g)
    k = torch.randn(B, L, H, d, generator=g)
    k = k / torch.sqrt((k * k).sum(-1, keepdim=True) + 1e-6)
    v = torch.randn(B, L, H, d, generator=g)
    beta = torch.sigmoid(torch.randn((B, L, H) if scalar_beta else (B, L, H, d), generator=g))
    alpha = alpha_lo + (1.0 - alpha_lo) * torch.rand(B, L, H, generator=g)
    do = torch.randn(B, L, H, d, generator=g)
    return [t.to(dtype).cuda() for t in (q, k, v, beta, alpha, do)]


CASES = [
    (1, 3, 2, 2),       # the reference's backward test shape
    (2, 8, 4, 8),
    (2, 100, 3, 16),
    (1, 300, 2, 64),    # several checkpoint chunks, ragged last chunk
    (1, 130, 2, 128),
]


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("case", CASES)
@pytest.mark.parametrize("scalar_beta", [False, True])
@pytest.mark.parametrize("use_ckpt", [False, True])
def test_gated_delta_net_parity(cuda, dtype, case, scalar_beta, use_ckpt):
    q, k, v, beta, alpha, do = gated_inputs(*case, dtype, seed=61, scalar_beta=scalar_beta)
    if use_ckpt:
        o, ck = fs.gated_delta_net_scan(q, k, v, beta, alpha, with_ckpt=True)
    else:
        o, ck = fs.gated_delta_net_scan(q, k, v, beta, alpha), None
    grads = fs.gated_delta_net_backward(q, k, v, beta, alpha, do, ck)
    torch.cuda.synchronize()
    args = [_np(t) for t in (q, k, v, beta, alpha)]
    assert O.norm_rel(_np(o), O.gated_delta_net_fwd(*args)) <= TOL[dtype]
    ref = O.gated_delta_net_bwd(*args, _np(do))
    for got, r in zip(grads, ref):
        assert got.shape == torch.Size(r.shape)
        assert O.norm_rel(_np(got), r) <= TOL[dtype], O.norm_rel(_np(got), r)
    assert device_errors() == 0


def test_alpha_one_is_the_delta_rule(cuda):
    """alpha == 1 reduces to the (token-recurrence) delta rule."""
    q, k, v, beta, alpha, do = gated_inputs(2, 150, 2, 32, torch.float32, seed=62,
                                            scalar_beta=False)
    one = torch.ones_like(alpha)
    o = fs.gated_delta_net_scan(q, k, v, beta, one)
    g = fs.gated_delta_net_backward(q, k, v, beta, one, do)
    o_ref = fs.delta_net_scan(q, k, v, beta)
    g_ref = fs.delta_rule_backward(q, k, v, beta, do)
    torch.cuda.synchronize()
    assert O.norm_rel(_np(o), _np(o_ref)) <= 1e-5
    for a, b_ in zip(g[:4], g_ref):
        assert O.norm_rel(_np(a), _np(b_)) <= 1e-5


def test_long_sequence_small_alpha(cuda):
    """Strong decay over many chunks (alpha down to 0.01): the backward reads
    stored states, so nothing is amplified by 1/alpha."""
    q, k, v, beta, alpha, do = gated_inputs(1, 700, 2, 64, torch.float32, seed=63,
                                            scalar_beta=True, alpha_lo=0.01)
    o = fs.gated_delta_net_scan(q, k, v, beta, alpha)
    grads = fs.gated_delta_net_backward(q, k, v, beta, alpha, do)
    torch.cuda.synchronize()
    args = [_np(t) for t in (q, k, v, beta, alpha)]
    assert O.norm_rel(_np(o), O.gated_delta_net_fwd(*args)) <= 1e-4
    for got, r in zip(grads, O.gated_delta_net_bwd(*args, _np(do))):
        assert O.norm_rel(_np(got), r) <= 1e-4


@pytest.mark.parametrize("prec,dtype", [("f32", torch.float32), ("bf16", torch.bfloat16)])
def test_gated_legacy_shim(cuda, prec, dtype):
    lib = ctypes.CDLL(build.SHIMS[prec])
    B, L, H, d = 2, 70, 2, 32
    q, k, v, beta, alpha, do = gated_inputs(B, L, H, d, dtype, seed=64, scalar_beta=False)
    P = lambda t: ctypes.c_void_p(t.data_ptr())
    o = torch.empty_like(q)
    assert lib.fused_gated_delta_net_scan_launch(None, P(q), P(k), P(v), P(beta), P(alpha), P(o),
                                                 B, L, H, d) == 0
    o2 = torch.empty_like(q)
    assert lib.fused_delta_rule_scan_launch(None, P(q), P(k), P(v), P(beta), P(alpha), P(o2),
                                            B, L, H, d) == 0
    o3 = torch.empty_like(q)
    assert lib.fused_delta_rule_scan_launch(None, P(q), P(k), P(v), P(beta), None, P(o3),
                                            B, L, H, d) == 0
    n = q.numel()
    cat = torch.empty(4 * n + alpha.numel(), dtype=dtype, device="cuda")
    assert lib.fused_gated_delta_net_scan_backward_launch(None, P(q), P(k), P(v), P(beta),
                                                          P(alpha), P(o), P(do), P(cat), B, L, H,
                                                          d) == 0
    torch.cuda.synchronize()
    assert torch.equal(o, fs.gated_delta_net_scan(q, k, v, beta, alpha))
    assert torch.equal(o2, o)
    assert torch.equal(o3, fs.delta_net_scan(q, k, v, beta))
    ref = fs.gated_delta_net_backward(q, k, v, beta, alpha, do)
    torch.cuda.synchronize()
    for idx, r in enumerate(ref):
        assert torch.equal(cat[idx * n:idx * n + r.numel()].view(r.shape), r)


def test_gated_autograd_fn(cuda):
    q, k, v, beta, alpha, do = gated_inputs(2, 50, 2, 32, torch.float32, seed=65,
                                            scalar_beta=True)
    leaves = [t.clone().requires_grad_(True) for t in (q, k, v, beta, alpha)]
    o = fs.GatedDeltaNetFn.apply(*leaves)
    o.backward(do)
    ref = O.gated_delta_net_bwd(*[_np(t) for t in (q, k, v, beta, alpha)], _np(do))
    for leaf, r in zip(leaves, ref):
        assert O.norm_rel(_np(leaf.grad), r) <= 1e-4


# ---------------------------------------------------------------- chunked form
# bf16, one beta per (token, head), head_dim 128: the chunked tensor-core kernels
# with the decay folded into the chunk products (tf32 operands, f32 accumulation).
CHUNKED = [
    (1, 1, 1),      # one token
    (1, 65, 2),     # one token past a chunk
    (1, 64, 1),     # one full chunk
    (2, 130, 3),    # ragged last chunk
    (1, 300, 2),
    (2, 1000, 2),   # sixteen chunks per (batch, head)
]


def _chunked(B, L, H):
    from edifice_b200 import _lib
    return _lib.load().edb_gated_delta_net_fwd_workspace(1, 0, B, L, H, 128) > 0


@pytest.mark.parametrize("case", CHUNKED)
@pytest.mark.parametrize("alpha_lo", [0.05, 0.01])
@pytest.mark.parametrize("use_ckpt", [False, True])
def test_chunked_gated_parity(cuda, case, alpha_lo, use_ckpt):
    B, L, H = case
    assert _chunked(B, L, H)
    q, k, v, beta, alpha, do = gated_inputs(B, L, H, 128, torch.bfloat16, seed=70 + L,
                                            scalar_beta=True, alpha_lo=alpha_lo)
    if use_ckpt:
        o, ck = fs.gated_delta_net_scan(q, k, v, beta, alpha, with_ckpt=True)
    else:
        o, ck = fs.gated_delta_net_scan(q, k, v, beta, alpha), None
    grads = fs.gated_delta_net_backward(q, k, v, beta, alpha, do, ck)
    torch.cuda.synchronize()
    args = [_np(t) for t in (q, k, v, beta, alpha)]
    assert O.norm_rel(_np(o), O.gated_delta_net_fwd(*args)) <= TOL[torch.bfloat16]
    ref = O.gated_delta_net_bwd(*args, _np(do))
    for name, got, r in zip(("q", "k", "v", "beta", "alpha"), grads, ref):
        assert got.shape == torch.Size(r.shape)
        assert torch.isfinite(got.float()).all(), name
        err = O.norm_rel(_np(got), r)
        assert err <= TOL[torch.bfloat16], (name, err)
    assert device_errors() == 0


def test_chunked_gated_alpha_one_is_the_delta_rule(cuda):
    """alpha == 1 through the chunked gated kernels equals the chunked delta rule
    (gamma = 1 everywhere, so every product matches up to summation order)."""
    q, k, v, beta, alpha, do = gated_inputs(2, 200, 2, 128, torch.bfloat16, seed=71,
                                            scalar_beta=True)
    one = torch.ones_like(alpha)
    o = fs.gated_delta_net_scan(q, k, v, beta, one)
    g = fs.gated_delta_net_backward(q, k, v, beta, one, do)
    o_ref = fs.delta_net_scan(q, k, v, beta)
    g_ref = fs.delta_rule_backward(q, k, v, beta, do)
    torch.cuda.synchronize()
    assert O.norm_rel(_np(o), _np(o_ref)) <= 1e-2
    for a, b_ in zip(g[:4], g_ref):
        assert O.norm_rel(_np(a), _np(b_)) <= 1e-2


def test_chunked_gated_no_workspace_entry(cuda):
    """edb_gated_delta_net_fwd (no workspace argument, stream-ordered scratch) gives
    the same bits as the workspace entry point."""
    from edifice_b200 import _lib
    lib = _lib.load()
    B, L, H, d = 1, 150, 2, 128
    q, k, v, beta, alpha, do = gated_inputs(B, L, H, d, torch.bfloat16, seed=72,
                                            scalar_beta=True)
    o_ref, ck_ref = fs.gated_delta_net_scan(q, k, v, beta, alpha, with_ckpt=True)
    o = torch.empty_like(q)
    ck = torch.empty_like(ck_ref)
    P = lambda t: ctypes.c_void_p(t.data_ptr())
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert lib.edb_gated_delta_net_fwd(1, P(q), P(k), P(v), P(beta), 0, P(alpha), P(o), P(ck),
                                       B, L, H, d, st) == 0
    torch.cuda.synchronize()
    assert torch.equal(o, o_ref)
    assert torch.equal(ck, ck_ref)


@pytest.mark.parametrize("dtype,scalar_beta,d", [(torch.bfloat16, True, 128),
                                                 (torch.bfloat16, False, 64)])
def test_gated_train_host(cuda, dtype, scalar_beta, d):
    """GatedDeltaNet over pinned host tensors (the delta rule's row ring) equals the
    device entry points on the whole batch bit for bit."""
    B, L, H = 5, 150, 2
    q, k, v, beta, alpha, do = gated_inputs(B, L, H, d, dtype, seed=73, scalar_beta=scalar_beta)
    o_r, ck = fs.gated_delta_net_scan(q, k, v, beta, alpha, with_ckpt=True)
    ref = (o_r,) + tuple(fs.gated_delta_net_backward(q, k, v, beta, alpha, do, ck))
    pin = [t.cpu().pin_memory() for t in (q, k, v, beta, alpha, do)]
    out = fs.gated_delta_net_train_host(*pin)
    torch.cuda.synchronize()
    for o, r in zip(out, ref):
        assert o.dtype == r.dtype and o.shape == r.shape
        assert torch.equal(o, r.cpu())
    assert device_errors() == 0
