"""GPU parity of the native-recurrence scans (elu_gru, real_gru, diag_linear:
lib/edifice/recurrent/native_recurrence.ex, FusedScan.elu_gru/real_gru/diag_linear)
against the CPU oracle, against the reference's own kernels built for sm_100a
(native/cuda/fused_native_rec_scan.cu and the three backward files, oracle/_ref),
through the reference-named shim symbols, and through the autograd wiring.

Bar (north_star): norm-relative error <= 1e-4 for f32 io and <= 2e-2 for bf16 io.
"""
import ctypes
import os

import pytest
import torch

import oracle as O
from oracle import build as ob
from edifice_b200 import build, device_errors
from edifice_b200 import fused_scan as fs

pytestmark = pytest.mark.gpu

TOL = {torch.float32: 1e-4, torch.bfloat16: 2e-2}

SHAPES = [
    (2, 37, 45),     # odd hidden -> generic kernel
    (2, 300, 128),   # TMA path, partial last tile
    (3, 1000, 96),   # f32: 3 full blocks; bf16: partial channel block
    (1, 4096, 256),  # long sequence
]

KINDS = {
    "elu_gru": (fs.elu_gru, O.elu_gru_fwd),
    "real_gru": (fs.real_gru, O.real_gru_fwd),
    "diag_linear": (fs.diag_linear, O.diag_linear_fwd),
}


def _np(t):
    return t.detach().float().cpu().numpy()


def _inputs(shape, dtype, seed):
    """Raw pre-activations ~ N(0, 1) (the dense projections' outputs), dY ~ N(0, 1)."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    x0 = torch.randn(shape, generator=g)
    x1 = torch.randn(shape, generator=g)
    dy = torch.randn(shape, generator=g)
    h0 = torch.randn((shape[0], shape[2]), generator=g)
    return [t.to(dtype).cuda() for t in (x0, x1, dy, h0)]


def _activated(kind, x0, x1):
    """The post-activation tensors the reference's backward launches take."""
    if kind == "elu_gru":
        return torch.sigmoid(x0), 1.0 + torch.where(x1 > 0, x1, torch.expm1(x1))
    if kind == "real_gru":
        return torch.sigmoid(x0), x1
    return torch.sigmoid(x0), x1


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("kind", sorted(KINDS))
@pytest.mark.parametrize("use_h0", [False, True])
def test_native_rec_forward_parity(cuda, dtype, shape, kind, use_h0):
    x0, x1, _, h0 = _inputs(shape, dtype, 41)
    h0 = h0 if use_h0 else None
    fn, ref = KINDS[kind]
    h = fn(x0, x1, h0)
    torch.cuda.synchronize()
    r = ref(_np(x0), _np(x1), None if h0 is None else _np(h0))
    assert O.norm_rel(_np(h), r) <= TOL[dtype], O.norm_rel(_np(h), r)
    assert device_errors() == 0


@pytest.mark.parametrize("kind", sorted(KINDS))
def test_native_rec_autograd(cuda, kind):
    """Gradients w.r.t. the raw inputs equal torch autograd of the reference's
    scan loop (native_recurrence.ex) in f64."""
    B, L, H = 2, 150, 64
    x0, x1, dy, _ = _inputs((B, L, H), torch.float32, 42)
    fnc = {"elu_gru": fs.EluGRUFn, "real_gru": fs.RealGRUFn, "diag_linear": fs.DiagLinearFn}[kind]
    a = x0.clone().requires_grad_(True)
    b = x1.clone().requires_grad_(True)
    fnc.apply(a, b).backward(dy)
    ra = x0.double().cpu().requires_grad_(True)
    rb = x1.double().cpu().requires_grad_(True)
    if kind == "diag_linear":
        A, Bv = torch.sigmoid(ra), rb
    else:
        z = torch.sigmoid(ra)
        c = (1.0 + torch.nn.functional.elu(rb)) if kind == "elu_gru" else rb
        A, Bv = 1 - z, z * c
    s, outs = torch.zeros(B, H, dtype=torch.float64), []
    for t in range(L):
        s = A[:, t] * s + Bv[:, t]
        outs.append(s)
    torch.stack(outs, 1).backward(dy.double().cpu())
    assert O.norm_rel(_np(a.grad), ra.grad.numpy()) <= 1e-4
    assert O.norm_rel(_np(b.grad), rb.grad.numpy()) <= 1e-4


@pytest.mark.parametrize("prec,dtype", [("f32", torch.float32), ("bf16", torch.bfloat16)])
@pytest.mark.parametrize("kind", sorted(KINDS))
def test_shim_symbols_match_edb_entry_points(cuda, prec, dtype, kind):
    """fused_<kind>_scan_launch and fused_<kind>_scan_backward_launch (NULL stream,
    concatenated [g0 | g1 | gh0]) give the same bits as the edb_* entry points."""
    lib = ctypes.CDLL(build.SHIMS[prec])
    B, L, H = 2, 200, 128
    x0, x1, dy, h0 = _inputs((B, L, H), dtype, 43)
    P = lambda t: ctypes.c_void_p(t.data_ptr())
    out = torch.empty_like(x0)
    assert getattr(lib, "fused_%s_scan_launch" % kind)(None, P(x0), P(x1), P(h0), P(out),
                                                       B, L, H) == 0
    torch.cuda.synchronize()
    ref_h = KINDS[kind][0](x0, x1, h0)
    torch.cuda.synchronize()
    assert torch.equal(out, ref_h)
    v0, v1 = _activated(kind, x0, x1)
    v0, v1 = v0.contiguous(), v1.contiguous()
    n = B * L * H
    cat = torch.empty(2 * n + B * H, dtype=dtype, device="cuda")
    bwd = getattr(lib, "fused_%s_scan_backward_launch" % kind)
    if kind == "diag_linear":
        assert bwd(None, P(v0), P(h0), P(ref_h), P(dy), P(cat), B, L, H) == 0
        want = fs.linear_scan_backward(v0, h0, ref_h, dy)
    else:
        assert bwd(None, P(v0), P(v1), P(h0), P(ref_h), P(dy), P(cat), B, L, H) == 0
        want = fs.mingru_backward(v0, v1, h0, ref_h, dy)
    torch.cuda.synchronize()
    assert torch.equal(cat[:n].view(B, L, H), want[0])
    assert torch.equal(cat[n:2 * n].view(B, L, H), want[1])
    assert torch.equal(cat[2 * n:].view(B, H), want[2])


@pytest.mark.skipif(not os.path.exists(ob.REF_KERNELS_SO["f32"]), reason="oracle/_ref not built")
@pytest.mark.parametrize("kind", sorted(KINDS))
def test_against_reference_cuda_kernels(cuda, kind):
    """The reference's own fused_native_rec_scan.cu forward and backward launches
    (f32 build, sm_100a) against the oracle and this library on the same inputs."""
    lib = ctypes.CDLL(ob.REF_KERNELS_SO["f32"])
    B, L, H = 2, 257, 96
    x0, x1, dy, h0 = _inputs((B, L, H), torch.float32, 44)
    P = lambda t: ctypes.c_void_p(t.data_ptr())
    ref_out = torch.empty_like(x0)
    assert getattr(lib, "fused_%s_scan_launch" % kind)(None, P(x0), P(x1), P(h0), P(ref_out),
                                                       B, L, H) == 0
    torch.cuda.synchronize()
    orc = KINDS[kind][1](_np(x0), _np(x1), _np(h0))
    assert O.norm_rel(_np(ref_out), orc) <= 1e-5
    ours = KINDS[kind][0](x0, x1, h0)
    torch.cuda.synchronize()
    assert O.norm_rel(_np(ours), _np(ref_out)) <= 1e-5
    v0, v1 = [t.contiguous() for t in _activated(kind, x0, x1)]
    n = B * L * H
    cat = torch.zeros(2 * n + B * H, dtype=torch.float32, device="cuda")
    bwd = getattr(lib, "fused_%s_scan_backward_launch" % kind)
    if kind == "diag_linear":
        assert bwd(None, P(v0), P(h0), P(ours), P(dy), P(cat), B, L, H) == 0
        want = fs.linear_scan_backward(v0, h0, ours, dy)
    else:
        assert bwd(None, P(v0), P(v1), P(h0), P(ours), P(dy), P(cat), B, L, H) == 0
        want = fs.mingru_backward(v0, v1, h0, ours, dy)
    torch.cuda.synchronize()
    for i, w in enumerate(want[:2]):
        assert O.norm_rel(_np(w), _np(cat[i * n:(i + 1) * n].view(B, L, H))) <= 1e-5
    assert O.norm_rel(_np(want[2]), _np(cat[2 * n:].view(B, H))) <= 1e-5
