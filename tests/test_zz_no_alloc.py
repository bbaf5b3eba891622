"""edb_selective_scan_bwd_noalloc: the selective-scan backward for callers that
cannot allocate device memory (an XLA/EXLA custom-call handler, whose process
has handed most of the GPU to XLA's own allocator and which gets no scratch
buffer from XLA).  Its scratch is a fixed array inside the library.

Checked through the C ABI against the workspace-taking entry point
(edb_selective_scan_bwd) on the same inputs, on two calls in a row: the second
call reuses the array with the first call's contents still in it.  This file
sorts last so a failure here comes after every other test has run; it also
passes alone in a fresh process (the first call does the per-device set-up).
"""
import ctypes
import math

import pytest
import torch

import oracle as O
import edifice_b200
from edifice_b200 import fused_scan as fs

pytestmark = pytest.mark.gpu

P = lambda t: ctypes.c_void_p(None if t is None else t.data_ptr())


def _inputs(Bsz, L, D, N, dtype, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    x = torch.randn(Bsz, L, D, generator=g)
    dt = torch.nn.functional.softplus(torch.randn(Bsz, L, D, generator=g) * 0.5 - 2)
    A = -torch.exp(torch.rand(D, N, generator=g) * math.log(16.0))
    Bm, Cm, dy = (torch.randn(*s, generator=g) for s in ((Bsz, L, N), (Bsz, L, N), (Bsz, L, D)))
    return [t.to(dtype).cuda() for t in (x, dt, A, Bm, Cm, dy)]


def _noalloc(lib, dtype_code, x, dt, A, Bm, Cm, dy, ck=None):
    Bsz, L, D = x.shape
    N = A.shape[1]
    gx, gdt = torch.empty_like(x), torch.empty_like(x)
    gB = torch.empty(Bsz, L, N, dtype=torch.float32, device=x.device)
    gC = torch.empty_like(gB)
    st = lib.edb_selective_scan_bwd_noalloc(dtype_code, P(x), P(dt), P(A), P(Bm), P(Cm), P(dy),
                                            P(ck), P(gx), P(gdt), P(gB), P(gC), Bsz, L, D, N,
                                            0.001, 0.1, None)
    return st, (gx, gdt, gB, gC)


@pytest.mark.parametrize("dtype,code,tol", [(torch.float32, 0, 1e-4), (torch.bfloat16, 1, 2e-2)])
def test_noalloc_matches_workspace_entry_point_twice(cuda, dtype, code, tol):
    lib = edifice_b200.load()
    x, dt, A, Bm, Cm, dy = _inputs(2, 300, 256, 16, dtype, seed=31)
    ref = fs.selective_scan_backward(x, dt, A, Bm, Cm, dy)
    torch.cuda.synchronize()
    for _ in range(2):
        st, got = _noalloc(lib, code, x, dt, A, Bm, Cm, dy)
        assert st == 0, edifice_b200._lib.status_string(st)
        torch.cuda.synchronize()
        for g, r in zip(got, ref):
            assert O.norm_rel(g.float().cpu().numpy(), r.float().cpu().numpy()) <= tol
    # with the forward's checkpoints as an extra input
    _, ck = fs.selective_scan(x, dt, A, Bm, Cm, with_ckpt=True)
    st, got = _noalloc(lib, code, x, dt, A, Bm, Cm, dy, ck)
    assert st == 0
    torch.cuda.synchronize()
    for g, r in zip(got, ref):
        assert O.norm_rel(g.float().cpu().numpy(), r.float().cpu().numpy()) <= tol


def test_noalloc_rejects_problems_beyond_its_scratch(cuda):
    lib = edifice_b200.load()
    Bsz, L, D, N = 8, 4096, 2048, 16
    need = lib.edb_selective_scan_bwd_workspace(Bsz, L, D, N, 0)
    assert need > 16 * 2 ** 20
    dummy = torch.empty(16, dtype=torch.bfloat16, device="cuda")
    p = P(dummy)
    st = lib.edb_selective_scan_bwd_noalloc(1, p, p, p, p, p, p, None, p, p, p, p, Bsz, L, D, N,
                                            0.001, 0.1, None)
    assert st == 1004  # EDB_ERR_WORKSPACE_TOO_SMALL, returned before any GPU work


@pytest.mark.parametrize("D", [130, 256])
def test_noalloc_odd_width_on_a_side_stream(cuda, D):
    """An odd channel count (the unstaged kernels, no 16-byte copies) and a
    non-default stream passed through the C ABI, twice in a row, against the
    workspace entry point."""
    lib = edifice_b200.load()
    x, dt, A, Bm, Cm, dy = _inputs(2, 97, D, 16, torch.bfloat16, seed=5)
    ref = fs.selective_scan_backward(x, dt, A, Bm, Cm, dy)
    torch.cuda.synchronize()
    side = torch.cuda.Stream()
    for _ in range(2):
        Bsz, L, _ = x.shape
        gx, gdt = torch.empty_like(x), torch.empty_like(x)
        gB = torch.empty(Bsz, L, 16, dtype=torch.float32, device=x.device)
        gC = torch.empty_like(gB)
        st = lib.edb_selective_scan_bwd_noalloc(1, P(x), P(dt), P(A), P(Bm), P(Cm), P(dy), P(None),
                                                P(gx), P(gdt), P(gB), P(gC), Bsz, L, D, 16, 0.001,
                                                0.1, ctypes.c_void_p(side.cuda_stream))
        assert st == 0, edifice_b200._lib.status_string(st)
        side.synchronize()
        for g, r in zip((gx, gdt, gB, gC), ref):
            assert O.norm_rel(g.float().cpu().numpy(), r.float().cpu().numpy()) <= 2e-2
