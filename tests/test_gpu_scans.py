"""GPU parity of the diagonal scans (linear scan, MinGRU) against the CPU oracle.

Bar (north_star): norm-relative error <= 1e-4 for f32 io and <= 2e-2 for bf16
io, for outputs and every gradient, against the f64 oracle run on the identical
(bf16-rounded) inputs.  Also reported/checked: max-abs error.
"""
import ctypes

import numpy as np
import pytest
import torch

import oracle as O
from edifice_b200 import fused_scan as fs
from edifice_b200 import build, device_errors

pytestmark = pytest.mark.gpu

TOL = {torch.float32: 1e-4, torch.bfloat16: 2e-2}

SHAPES = [
    (2, 37, 45),     # odd hidden -> generic kernel
    (1, 1, 64),      # single step
    (2, 300, 128),   # TMA path, partial last tile
    (3, 1000, 96),   # f32: 3 full blocks; bf16: partial channel block
    (2, 130, 200),   # partial channel block, partial tile
    (1, 4096, 256),  # long sequence
    (40, 64, 512),   # >= 2 CTAs per SM of 128-byte channel blocks (the wide-block path)
]


def _np(t):
    return t.detach().float().cpu().numpy()


def _inputs(shape, dtype, seed, mingru=False):
    g = torch.Generator(device="cpu").manual_seed(seed)
    a = torch.sigmoid(torch.randn(shape, generator=g))
    b = torch.randn(shape, generator=g)
    dy = torch.randn(shape, generator=g)
    h0 = torch.randn((shape[0], shape[2]), generator=g)
    return [x.to(dtype).cuda() for x in (a, b, dy, h0)]


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("use_h0", [False, True])
def test_linear_scan_parity(cuda, dtype, shape, use_h0):
    a, b, dy, h0 = _inputs(shape, dtype, 11)
    h0 = h0 if use_h0 else None
    h = fs.linear_scan(a, b, h0)
    ga, gb, gh0 = fs.linear_scan_backward(a, h0, h, dy)
    torch.cuda.synchronize()
    h0n = None if h0 is None else _np(h0)
    ref_h = O.linear_scan_fwd(_np(a), _np(b), h0n)
    assert O.norm_rel(_np(h), ref_h) <= TOL[dtype]
    rga, rgb, rgh0 = O.linear_scan_bwd(_np(a), h0n, _np(h), _np(dy))
    assert O.norm_rel(_np(ga), rga) <= TOL[dtype]
    assert O.norm_rel(_np(gb), rgb) <= TOL[dtype]
    assert O.norm_rel(_np(gh0), rgh0) <= TOL[dtype]
    assert device_errors() == 0


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("use_h0", [False, True])
def test_mingru_parity(cuda, dtype, shape, use_h0):
    z, c, dy, h0 = _inputs(shape, dtype, 12)
    h0 = h0 if use_h0 else None
    h = fs.mingru_scan(z, c, h0)
    gz, gc, gh0 = fs.mingru_backward(z, c, h0, h, dy)
    torch.cuda.synchronize()
    h0n = None if h0 is None else _np(h0)
    assert O.norm_rel(_np(h), O.mingru_fwd(_np(z), _np(c), h0n)) <= TOL[dtype]
    rgz, rgc, rgh0 = O.mingru_bwd(_np(z), _np(c), h0n, _np(h), _np(dy))
    assert O.norm_rel(_np(gz), rgz) <= TOL[dtype]
    assert O.norm_rel(_np(gc), rgc) <= TOL[dtype]
    assert O.norm_rel(_np(gh0), rgh0) <= TOL[dtype]


def test_config1_full_size_bf16(cuda):
    """B8 L4096 H2048 bf16, a = sigmoid(N(0,1)), b, dY ~ N(0,1)."""
    shape = (8, 4096, 2048)
    a, b, dy, _ = _inputs(shape, torch.bfloat16, 0)
    h = fs.linear_scan(a, b)
    ga, gb, gh0 = fs.linear_scan_backward(a, None, h, dy)
    torch.cuda.synchronize()
    ref_h = O.linear_scan_fwd(_np(a), _np(b))
    assert O.norm_rel(_np(h), ref_h) <= 2e-2
    rga, rgb, rgh0 = O.linear_scan_bwd(_np(a), None, _np(h), _np(dy))
    for x, r in ((ga, rga), (gb, rgb), (gh0, rgh0)):
        assert O.norm_rel(_np(x), r) <= 2e-2
    # MinGRU form on the same shape
    hm = fs.mingru_scan(a, b)
    gz, gc, _ = fs.mingru_backward(a, b, None, hm, dy)
    torch.cuda.synchronize()
    assert O.norm_rel(_np(hm), O.mingru_fwd(_np(a), _np(b))) <= 2e-2
    rgz, rgc, _ = O.mingru_bwd(_np(a), _np(b), None, _np(hm), _np(dy))
    assert O.norm_rel(_np(gz), rgz) <= 2e-2
    assert O.norm_rel(_np(gc), rgc) <= 2e-2
    assert device_errors() == 0


@pytest.mark.parametrize("prec,dtype", [("f32", torch.float32), ("bf16", torch.bfloat16)])
def test_legacy_shim_symbols(cuda, prec, dtype):
    """The reference-named fused_*_launch symbols (NULL stream, concatenated
    backward outputs) give the same results as the edb_* entry points."""
    lib = ctypes.CDLL(build.SHIMS[prec])
    B, L, H = 2, 200, 128
    a, b, dy, h0 = _inputs((B, L, H), dtype, 13)
    out = torch.empty_like(a)
    st = lib.fused_linear_scan_launch(None, ctypes.c_void_p(a.data_ptr()),
                                      ctypes.c_void_p(b.data_ptr()), ctypes.c_void_p(h0.data_ptr()),
                                      ctypes.c_void_p(out.data_ptr()), B, L, H)
    assert st == 0
    cat = torch.empty(2 * B * L * H + B * H, dtype=dtype, device="cuda")
    st = lib.fused_linear_scan_backward_launch(
        None, ctypes.c_void_p(a.data_ptr()), ctypes.c_void_p(h0.data_ptr()),
        ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(dy.data_ptr()),
        ctypes.c_void_p(cat.data_ptr()), B, L, H)
    assert st == 0
    torch.cuda.synchronize()
    ref = fs.linear_scan(a, b, h0)
    ga, gb, gh0 = fs.linear_scan_backward(a, h0, ref, dy)
    torch.cuda.synchronize()
    assert torch.equal(out, ref)
    n = B * L * H
    assert torch.equal(cat[:n].view(B, L, H), ga)
    assert torch.equal(cat[n:2 * n].view(B, L, H), gb)
    assert torch.equal(cat[2 * n:].view(B, H), gh0)
    zc = torch.empty_like(a)
    st = lib.fused_mingru_scan_launch(None, ctypes.c_void_p(a.data_ptr()),
                                      ctypes.c_void_p(b.data_ptr()), ctypes.c_void_p(h0.data_ptr()),
                                      ctypes.c_void_p(zc.data_ptr()), B, L, H)
    assert st == 0
    torch.cuda.synchronize()
    assert torch.equal(zc, fs.mingru_scan(a, b, h0))


def test_autograd_functions(cuda):
    B, L, H = 2, 77, 64
    g = torch.Generator(device="cpu").manual_seed(5)
    gates = torch.randn(B, L, H, generator=g).cuda().requires_grad_(True)
    cand = torch.randn(B, L, H, generator=g).cuda().requires_grad_(True)
    dy = torch.randn(B, L, H, generator=g).cuda()
    out = fs.MinGRUFn.apply(gates, cand)
    out.backward(dy)
    # same through plain torch autograd of the recurrence
    g2 = gates.detach().clone().requires_grad_(True)
    c2 = cand.detach().clone().requires_grad_(True)
    z = torch.sigmoid(g2)
    s, outs = torch.zeros(B, H, device="cuda"), []
    for t in range(L):
        s = (1 - z[:, t]) * s + z[:, t] * c2[:, t]
        outs.append(s)
    torch.stack(outs, 1).backward(dy)
    assert O.norm_rel(_np(gates.grad), _np(g2.grad)) < 1e-4
    assert O.norm_rel(_np(cand.grad), _np(c2.grad)) < 1e-4


def test_rejects_cpu_tensors(cuda):
    a = torch.rand(1, 4, 8)
    with pytest.raises(RuntimeError):
        fs.linear_scan(a, a)


HOST_SHAPES = [
    (8, 300, 128),   # 4 chunks of 2 rows through 3 slots (slot reuse)
    (9, 50, 45),     # odd hidden -> generic kernel; ragged last chunk
    (1, 1000, 256),  # one row, one chunk
    (2, 4096, 2048), # 16 MiB rows: one row per chunk
]


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("shape", HOST_SHAPES)
@pytest.mark.parametrize("op", ["linear", "mingru"])
def test_train_host_matches_device_path(cuda, dtype, shape, op):
    """Forward + backward over pinned host tensors (copies overlapped with the
    kernels chunk by chunk) equals the device entry points on the whole batch,
    bit for bit (every kernel is independent per batch row), for two calls in a
    row through the same workspace, and agrees with the oracle."""
    a, b, dy, h0 = _inputs(shape, dtype, 21)
    for use_h0 in (False, True):
        hh0 = h0 if use_h0 else None
        if op == "linear":
            ref_h = fs.linear_scan(a, b, hh0)
            ref = (ref_h,) + tuple(fs.linear_scan_backward(a, hh0, ref_h, dy))
            fn = fs.linear_scan_train_host
        else:
            ref_h = fs.mingru_scan(a, b, hh0)
            ref = (ref_h,) + tuple(fs.mingru_backward(a, b, hh0, ref_h, dy))
            fn = fs.mingru_train_host
        pin = [x.cpu().pin_memory() for x in (a, b, dy)]
        ph0 = hh0.cpu().pin_memory() if use_h0 else None
        for _ in range(2):
            out = fn(pin[0], pin[1], pin[2], h0=ph0)
            torch.cuda.synchronize()
            for o, r in zip(out, ref):
                assert torch.equal(o, r.cpu())
    if op == "linear":
        ref_o = O.linear_scan_fwd(_np(a), _np(b), _np(h0))
    else:
        ref_o = O.mingru_fwd(_np(a), _np(b), _np(h0))
    assert O.norm_rel(out[0].float().numpy(), ref_o) <= TOL[dtype]
    assert device_errors() == 0


def test_train_host_rejects_device_tensors(cuda):
    a = torch.rand(1, 4, 8, device="cuda")
    with pytest.raises(RuntimeError):
        fs.linear_scan_train_host(a, a, a)


@pytest.mark.parametrize("op", ["linear", "mingru"])
def test_bounded_wait_gives_up_reports_and_recovers(cuda, op):
    """A wait of the TMA pipeline that runs out (limit 0: the first probe of a
    tile that has not landed gives up) makes the kernel flag EDB_DEVERR_SCAN_PIPE
    in the device error word and exit -- after its in-flight copies land -- rather
    than hang; the next call with the default limit is exact."""
    import edifice_b200
    lib = edifice_b200.load()
    a, b, dy, _ = _inputs((2, 512, 256), torch.bfloat16, 5, mingru=op == "mingru")
    fwd = fs.linear_scan if op == "linear" else fs.mingru_scan
    ref = fwd(a, b)
    torch.cuda.synchronize()
    assert device_errors() == 0
    assert lib.edb_set_wait_limit_ns(0) == 0
    try:
        fwd(a, b)
        torch.cuda.synchronize()  # the kernel has exited: the call did not hang
        flags = device_errors()
    finally:
        assert lib.edb_set_wait_limit_ns(-1) == 0
    assert flags & 0x1, flags  # EDB_DEVERR_SCAN_PIPE
    again = fwd(a, b)
    torch.cuda.synchronize()
    assert torch.equal(again, ref)
    assert device_errors() == 0
