"""GPU parity of causal/full GQA attention against the CPU oracle (f64), the
golden GQA vectors, and the reference's own flash-attention CUDA kernels."""
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


def attn_inputs(B, Hq, Hkv, L, d, dtype, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    q = torch.randn(B, Hq, L, d, generator=g)
    k = torch.randn(B, Hkv, L, d, generator=g)
    v = torch.randn(B, Hkv, L, d, generator=g)
    do = torch.randn(B, Hq, L, d, generator=g)
    return [t.to(dtype).cuda() for t in (q, k, v, do)]


FWD_CASES = [
    # (B, Hq, Hkv, L, d)
    (1, 2, 2, 128, 128),
    (2, 4, 2, 256, 128),
    (1, 8, 2, 300, 128),   # partial last tile
    (2, 4, 4, 64, 128),    # L < tile
    (1, 2, 1, 1000, 64),   # head_dim 64
    (1, 1, 1, 1, 128),     # single token
    (2, 4, 2, 37, 8),      # small head_dim: SIMT path
    (1, 4, 1, 200, 96),    # other head_dim: SIMT path
]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("case", FWD_CASES)
@pytest.mark.parametrize("causal", [True, False])
def test_attention_forward(cuda, dtype, case, causal):
    q, k, v, _ = attn_inputs(*case, dtype, seed=41)
    o, lse = fs.flash_attention(q, k, v, causal=causal, return_lse=True)
    torch.cuda.synchronize()
    ro, rl = O.attention_fwd(_np(q), _np(k), _np(v), causal=causal, want_lse=True)
    assert O.norm_rel(_np(o), ro) <= TOL[dtype]
    assert O.norm_rel(_np(lse), rl) <= 1e-4
    assert device_errors() == 0


@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("d", [64, 128])
def test_attention_forward_large_scores(cuda, causal, d):
    """Scores of standard deviation ~12: the running row max grows by more than
    8 between kv tiles in some rows of a warp and not in others, so the lazy O
    rescale is taken by part of each warp's rows (the warp rescales together,
    the other rows with factor 1)."""
    q, k, v, do = attn_inputs(2, 4, 2, 448, d, torch.bfloat16, seed=47)
    q = (q.float() * 12.0).to(torch.bfloat16)
    o, lse = fs.flash_attention(q, k, v, causal=causal, return_lse=True)
    torch.cuda.synchronize()
    assert device_errors() == 0
    ro, rl = O.attention_fwd(_np(q), _np(k), _np(v), causal=causal, want_lse=True)
    assert O.norm_rel(_np(o), ro) <= TOL[torch.bfloat16]
    assert O.norm_rel(_np(lse), rl) <= 1e-4
    dq, dk, dv = fs.flash_attention_backward(q, k, v, causal, o, do, lse)
    torch.cuda.synchronize()
    assert device_errors() == 0
    ref = O.attention_bwd(_np(q), _np(k), _np(v), _np(do), causal=causal)
    for name, got, r in zip(("dq", "dk", "dv"), (dq, dk, dv), ref):
        assert O.norm_rel(_np(got), r) <= 3e-2, (name, O.norm_rel(_np(got), r))


@pytest.mark.parametrize("layer", [0, 1])
def test_attention_golden_gqa(cuda, layer):
    g = np.load(os.path.join(GOLD, "gqa_fixture.npz"))
    q, k, v = (torch.tensor(g["%s%d" % (n, layer)]).cuda() for n in ("q", "k", "v"))
    o = fs.flash_attention(q, k, v, causal=True)
    torch.cuda.synchronize()
    np.testing.assert_allclose(_np(o), g["o%d" % layer], atol=2e-5)


def test_config3_forward_rows(cuda):
    """B4 Hq32 Hkv8 L8192 d128 causal bf16; a sample of
    query rows (first and last 96 of three heads) against the f64 oracle."""
    B, Hq, Hkv, L, d = 4, 32, 8, 8192, 128
    q, k, v, _ = attn_inputs(B, Hq, Hkv, L, d, torch.bfloat16, seed=0)
    o = fs.flash_attention(q, k, v, causal=True)
    torch.cuda.synchronize()
    assert device_errors() == 0
    kn, vn = _np(k), _np(v)
    for (b, h) in ((0, 0), (1, 13), (3, 31)):
        hk = h // (Hq // Hkv)
        for sl in (slice(0, 96), slice(L - 96, L)):
            rows = np.arange(L)[sl]
            # oracle on the needed prefix of keys for these rows
            qq = _np(q[b:b + 1, h:h + 1, sl])
            kk = kn[b:b + 1, hk:hk + 1, :rows[-1] + 1]
            vv = vn[b:b + 1, hk:hk + 1, :rows[-1] + 1]
            ref = _ref_rows(qq, kk, vv, rows)
            assert O.norm_rel(_np(o[b, h, sl]), ref) <= 2e-2


def _ref_rows(q, k, v, rows):
    """causal attention for query rows `rows` (f64 numpy)."""
    qd, kd, vd = (x[0, 0].astype(np.float64) for x in (q, k, v))
    s = qd @ kd.T / np.sqrt(qd.shape[-1])
    s[rows[:, None] < np.arange(kd.shape[0])[None, :]] = -np.inf
    s -= s.max(-1, keepdims=True)
    p = np.exp(s)
    p /= p.sum(-1, keepdims=True)
    return p @ vd


@pytest.mark.skipif(not os.path.exists(ob.REF_KERNELS_SO["f32"]), reason="oracle/_ref not built")
@pytest.mark.parametrize("causal", [0, 1])
def test_oracle_matches_reference_cuda_flash(cuda, causal):
    """Pin the oracle's attention against the reference's own
    fused_flash_attention_launch (f32 build for sm_100a, equal heads).
    L is a multiple of the reference's 32-row tile: for other L the reference
    kernel's threads past the end skip the cooperative K/V tile load and the
    block barrier (native/cuda/fused_flash_attention.cu:75-77, `continue`
    before the loads), so its output is wrong there (seen at L = 70)."""
    lib = ctypes.CDLL(ob.REF_KERNELS_SO["f32"])
    B, H, L, d = 2, 3, 96, 32
    q, k, v, _ = attn_inputs(B, H, H, L, d, torch.float32, seed=7)
    o = torch.empty_like(q)
    P = lambda t: ctypes.c_void_p(t.data_ptr())
    assert lib.fused_flash_attention_launch(None, P(q), P(k), P(v), P(o), B, H, L, d, causal) == 0
    torch.cuda.synchronize()
    assert O.norm_rel(_np(o), O.attention_fwd(_np(q), _np(k), _np(v), causal=bool(causal))) <= 1e-5


@pytest.mark.parametrize("prec,dtype", [("f32", torch.float32), ("bf16", torch.bfloat16)])
def test_legacy_shim_forward(cuda, prec, dtype):
    lib = ctypes.CDLL(build.SHIMS[prec])
    B, H, L, d = 2, 4, 256, 128
    q, k, v, _ = attn_inputs(B, H, H, L, d, dtype, seed=9)
    o = torch.empty_like(q)
    P = lambda t: ctypes.c_void_p(t.data_ptr())
    assert lib.fused_flash_attention_launch(None, P(q), P(k), P(v), P(o), B, H, L, d, 1) == 0
    torch.cuda.synchronize()
    assert torch.equal(o, fs.flash_attention(q, k, v, causal=True))


# ------------------------------------------------------------------ backward
BWD_CASES = [
    (1, 2, 2, 128, 128),
    (2, 4, 2, 256, 128),
    (1, 8, 2, 300, 128),   # partial tiles
    (2, 4, 4, 64, 128),
    (1, 2, 1, 1000, 64),
    (2, 4, 2, 37, 8),      # SIMT path
    (1, 4, 1, 130, 96),    # SIMT path
]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("case", BWD_CASES)
@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("with_lse", [True, False])
def test_attention_backward(cuda, dtype, case, causal, with_lse):
    q, k, v, do = attn_inputs(*case, dtype, seed=43)
    o, lse = fs.flash_attention(q, k, v, causal=causal, return_lse=True)
    dq, dk, dv = fs.flash_attention_backward(q, k, v, causal, o, do, lse if with_lse else None)
    torch.cuda.synchronize()
    ref = O.attention_bwd(_np(q), _np(k), _np(v), _np(do), causal=causal)
    for got, r in zip((dq, dk, dv), ref):
        assert O.norm_rel(_np(got), r) <= TOL[dtype], O.norm_rel(_np(got), r)
    assert device_errors() == 0


@pytest.mark.parametrize("layer", [0, 1])
def test_attention_backward_golden_gqa(cuda, layer):
    g = np.load(os.path.join(GOLD, "gqa_fixture.npz"))
    q, k, v, do = (torch.tensor(g["%s%d" % (n, layer)]).cuda() for n in ("q", "k", "v", "do"))
    o = fs.flash_attention(q, k, v, causal=True)
    dq, dk, dv = fs.flash_attention_backward(q, k, v, True, o, do)
    torch.cuda.synchronize()
    for got, n in zip((dq, dk, dv), ("dq", "dk", "dv")):
        np.testing.assert_allclose(_np(got), g["%s%d" % (n, layer)], atol=5e-5)


def test_attention_backward_mid_size_full_oracle(cuda):
    """B1 Hq8 Hkv2 L2048 d128 causal bf16: every gradient against the f64 oracle."""
    q, k, v, do = attn_inputs(1, 8, 2, 2048, 128, torch.bfloat16, seed=44)
    o, lse = fs.flash_attention(q, k, v, causal=True, return_lse=True)
    dq, dk, dv = fs.flash_attention_backward(q, k, v, True, o, do, lse)
    torch.cuda.synchronize()
    O.set_threads(os.cpu_count() or 8)
    ref = O.attention_bwd(_np(q), _np(k), _np(v), _np(do), causal=True)
    for got, r in zip((dq, dk, dv), ref):
        assert O.norm_rel(_np(got), r) <= 2e-2


def test_config3_backward_vs_torch_fp32(cuda):
    """BASELINE configs[3] at full size (B4 Hq32 Hkv8 L8192 d128, causal):
    forward + backward against torch's fp32 SDPA (memory-efficient backend, K/V
    repeated over the group, dK/dV summed back) on the same bf16-rounded inputs."""
    from torch.nn.attention import SDPBackend, sdpa_kernel
    B, Hq, Hkv, L, d = 4, 32, 8, 8192, 128
    q, k, v, do = attn_inputs(B, Hq, Hkv, L, d, torch.bfloat16, seed=0)
    o, lse = fs.flash_attention(q, k, v, causal=True, return_lse=True)
    dq, dk, dv = fs.flash_attention_backward(q, k, v, True, o, do, lse)
    torch.cuda.synchronize()
    assert device_errors() == 0
    G = Hq // Hkv
    qf = q.float().requires_grad_(True)
    kf = k.float().requires_grad_(True)
    vf = v.float().requires_grad_(True)
    with sdpa_kernel(SDPBackend.EFFICIENT_ATTENTION):
        of = torch.nn.functional.scaled_dot_product_attention(
            qf, kf.repeat_interleave(G, 1), vf.repeat_interleave(G, 1), is_causal=True)
    of.backward(do.float())
    rel = lambda a, b: ((a.float() - b).norm() / b.norm()).item()
    assert rel(o, of.detach()) <= 2e-2
    assert rel(dq, qf.grad) <= 2e-2
    assert rel(dk, kf.grad) <= 2e-2
    assert rel(dv, vf.grad) <= 2e-2


@pytest.mark.parametrize("prec,dtype", [("f32", torch.float32), ("bf16", torch.bfloat16)])
def test_legacy_shim_backward(cuda, prec, dtype):
    lib = ctypes.CDLL(build.SHIMS[prec])
    B, H, L, d = 2, 4, 256, 128
    q, k, v, do = attn_inputs(B, H, H, L, d, dtype, seed=45)
    o = fs.flash_attention(q, k, v, causal=True)
    cat = torch.empty(3 * q.numel(), dtype=dtype, device="cuda")
    P = lambda t: ctypes.c_void_p(t.data_ptr())
    assert lib.fused_flash_attention_backward_launch(None, P(q), P(k), P(v), P(o), P(do), P(cat),
                                                     B, H, L, d, 1) == 0
    torch.cuda.synchronize()
    ref = O.attention_bwd(_np(q), _np(k), _np(v), _np(do), causal=True)
    n = q.numel()
    for idx, r in enumerate(ref):
        assert O.norm_rel(_np(cat[idx * n:(idx + 1) * n]).reshape(r.shape), r) <= TOL[dtype]


def test_autograd_fn(cuda):
    q, k, v, do = attn_inputs(1, 4, 2, 200, 128, torch.bfloat16, seed=46)
    leaves = [t.clone().requires_grad_(True) for t in (q, k, v)]
    o = fs.FlashAttentionFn.apply(*leaves, True)
    o.backward(do)
    ref = O.attention_bwd(_np(q), _np(k), _np(v), _np(do), causal=True)
    for leaf, r in zip(leaves, ref):
        assert O.norm_rel(_np(leaf.grad), r) <= 2e-2


# ----------------------------------------- the reference's attention callers
def _dense_reference(q, k, v, heads, kv_heads, d, causal):
    """SDPA.compute / GQA.gqa_attention_impl as the reference writes them
    (sdpa.ex:74-118, gqa.ex:192-306): reshape [B, L, H*d] -> [B, H, L, d], repeat
    K/V over the group, scores / sqrt(d), -1e9 causal fill, softmax, P V; in f64."""
    B, L, _ = q.shape
    qh = q.double().reshape(B, L, heads, d).transpose(1, 2)
    kh = k.double().reshape(B, L, kv_heads, d).transpose(1, 2)
    vh = v.double().reshape(B, L, kv_heads, d).transpose(1, 2)
    g = heads // kv_heads
    kh = kh[:, :, None].expand(B, kv_heads, g, L, d).reshape(B, heads, L, d)
    vh = vh[:, :, None].expand(B, kv_heads, g, L, d).reshape(B, heads, L, d)
    s = qh @ kh.transpose(-1, -2) / d ** 0.5
    if causal:
        tri = torch.ones(L, L, dtype=torch.bool, device=q.device).tril()
        s = torch.where(tri, s, torch.full_like(s, -1.0e9))
    o = torch.softmax(s, -1) @ vh
    return o.transpose(1, 2).reshape(B, L, heads * d)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("heads,kv_heads,d,L", [(8, 2, 128, 300), (4, 4, 64, 129), (4, 1, 96, 77)])
def test_gqa_attention_routes_to_flash(cuda, dtype, heads, kv_heads, d, L):
    """GQA.gqa_attention_impl's numbers (K/V repeated, -1e9 causal fill) from the
    flash kernel with native grouped heads, forward and gradients."""
    B = 2
    g = torch.Generator(device="cpu").manual_seed(61)
    q = torch.randn(B, L, heads * d, generator=g).to(dtype).cuda().requires_grad_(True)
    k = torch.randn(B, L, kv_heads * d, generator=g).to(dtype).cuda().requires_grad_(True)
    v = torch.randn(B, L, kv_heads * d, generator=g).to(dtype).cuda().requires_grad_(True)
    do = torch.randn(B, L, heads * d, generator=g).to(dtype).cuda()
    o = fs.gqa_attention(q, k, v, heads, kv_heads, d)
    o.backward(do)
    rq, rk, rv = (t.detach().double().requires_grad_(True) for t in (q, k, v))
    ro = _dense_reference(rq, rk, rv, heads, kv_heads, d, causal=True)
    ro.backward(do.double())
    assert O.norm_rel(_np(o), _np(ro)) <= TOL[dtype]
    for got, ref in ((q.grad, rq.grad), (k.grad, rk.grad), (v.grad, rv.grad)):
        assert O.norm_rel(_np(got), _np(ref)) <= TOL[dtype]


@pytest.mark.parametrize("causal", [False, True])
def test_sdpa_compute_and_multi_head_sdpa(cuda, causal):
    """SDPA.compute/6 (causal = mask given) and Primitives.multi_head_sdpa/4
    (mask None, or the causal lower triangle) against the dense formulation;
    a non-causal mask is refused rather than silently ignored."""
    B, L, H, d = 2, 200, 4, 128
    g = torch.Generator(device="cpu").manual_seed(62)
    q, k, v = (torch.randn(B, L, H * d, generator=g).to(torch.bfloat16).cuda() for _ in range(3))
    o = fs.sdpa_compute(q, k, v, H, d, causal=causal)
    ref = _dense_reference(q, k, v, H, H, d, causal)
    assert O.norm_rel(_np(o), _np(ref)) <= 2e-2
    qh, kh, vh = (t.reshape(B, L, H, d).transpose(1, 2) for t in (q, k, v))
    mask = torch.ones(L, L, dtype=torch.bool, device="cuda").tril() if causal else None
    oh = fs.multi_head_sdpa(qh, kh, vh, mask=mask)
    assert O.norm_rel(_np(oh.transpose(1, 2).reshape(B, L, H * d)), _np(ref)) <= 2e-2
    band = torch.ones(L, L, dtype=torch.bool, device="cuda").triu(-4).tril()
    with pytest.raises(RuntimeError):
        fs.multi_head_sdpa(qh, kh, vh, mask=band)


# ---------------------------------------------------------------- LASER attention
LASER_CASES = [
    # (B, Hq, Hkv, L, d)
    (2, 4, 4, 200, 128),   # equal heads (the reference's form), tcgen05 path in bf16
    (1, 8, 2, 300, 128),   # grouped heads, partial last tile
    (2, 2, 2, 129, 64),    # head_dim 64
    (1, 4, 1, 77, 96),     # SIMT path
]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("case", LASER_CASES)
@pytest.mark.parametrize("causal", [True, False])
def test_laser_attention(cuda, dtype, case, causal):
    """LASER (fused_scan.ex:3593-3611, 3667-3766) forward and backward against the
    oracle on the same rounded inputs."""
    q, k, v, do = attn_inputs(*case, dtype, seed=71)
    o, resid = fs.laser_attention(q, k, v, causal=causal, return_resid=True)
    dq, dk, dv = fs.laser_attention_backward(q, k, v, do, resid, causal=causal)
    torch.cuda.synchronize()
    ro, _ = O.laser_fwd(_np(q), _np(k), _np(v), causal=causal)
    assert O.norm_rel(_np(o), ro) <= TOL[dtype]
    for got, ref in zip((dq, dk, dv), O.laser_bwd(_np(q), _np(k), _np(v), _np(do),
                                                  causal=causal)):
        assert O.norm_rel(_np(got), ref) <= TOL[dtype], O.norm_rel(_np(got), ref)
    assert device_errors() == 0


def test_laser_given_v_max_and_autograd(cuda):
    """A caller-given v_max (the reference's argument) equal to the computed one
    gives the same bits; the autograd wiring matches the explicit backward."""
    q, k, v, do = attn_inputs(2, 4, 2, 150, 128, torch.bfloat16, seed=72)
    vmax = v.amax(dim=2)
    o1 = fs.laser_attention(q, k, v)
    o2 = fs.laser_attention(q, k, v, v_max=vmax.contiguous())
    torch.cuda.synchronize()
    assert torch.equal(o1, o2)
    leaves = [t.clone().requires_grad_(True) for t in (q, k, v)]
    fs.LaserAttentionFn.apply(*leaves, True).backward(do)
    _, resid = fs.laser_attention(q, k, v, return_resid=True)
    want = fs.laser_attention_backward(q, k, v, do, resid)
    for leaf, w in zip(leaves, want):
        assert torch.equal(leaf.grad, w)


@pytest.mark.parametrize("prec,dtype", [("f32", torch.float32), ("bf16", torch.bfloat16)])
def test_laser_shim_symbols(cuda, prec, dtype):
    """fused_laser_attention_launch / _backward_launch (equal heads, NULL stream,
    [dq | dk | dv] concatenated) match the edb_* path."""
    lib = ctypes.CDLL(build.SHIMS[prec])
    B, H, L, d = 2, 2, 96, 64
    q, k, v, do = attn_inputs(B, H, H, L, d, dtype, seed=73)
    vmax = v.amax(dim=2).contiguous()
    P = lambda t: ctypes.c_void_p(t.data_ptr())
    out = torch.empty_like(q)
    assert lib.fused_laser_attention_launch(None, P(q), P(k), P(v), P(vmax), P(out), B, H, L, d,
                                            1) == 0
    cat = torch.empty(3 * q.numel(), dtype=dtype, device="cuda")
    assert lib.fused_laser_attention_backward_launch(None, P(q), P(k), P(v), P(vmax), P(out),
                                                     P(do), P(cat), B, H, L, d, 1) == 0
    torch.cuda.synchronize()
    o, resid = fs.laser_attention(q, k, v, return_resid=True)
    want = fs.laser_attention_backward(q, k, v, do, resid)
    torch.cuda.synchronize()
    assert torch.equal(out, o)
    n = q.numel()
    for i, w in enumerate(want):
        assert torch.equal(cat[i * n:(i + 1) * n].view_as(w), w)


# ------------------------------------------------------------------ FoX attention
def fox_cs(B, H, L, seed):
    """cs = cumsum(log(sigmoid(f))), f ~ N(0, 1) (the model's forget gates)."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    f = torch.randn(B, H, L, generator=g)
    return torch.cumsum(torch.nn.functional.logsigmoid(f), -1).cuda()


FOX_CASES = [
    # (B, Hq, Hkv, L, d)
    (2, 4, 4, 200, 128),   # equal heads (the reference's form)
    (1, 8, 2, 300, 128),   # grouped heads
    (2, 2, 2, 132, 64),    # head_dim 64
    (1, 2, 2, 77, 64),     # odd length
    (1, 4, 1, 64, 96),     # other head_dim
]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("case", FOX_CASES)
def test_fox_attention(cuda, dtype, case):
    """FoX (fused_scan.ex:3796-3984) forward and backward, grad_cs included, against
    the oracle on the same rounded inputs."""
    B, Hq, Hkv, L, d = case
    q, k, v, do = attn_inputs(*case, dtype, seed=81)
    cs = fox_cs(B, Hq, L, 82)
    o, lse = fs.fox_attention(q, k, v, cs, return_lse=True)
    dq, dk, dv, dcs = fs.fox_attention_backward(q, k, v, cs, o, do, lse)
    torch.cuda.synchronize()
    assert O.norm_rel(_np(o), O.fox_fwd(_np(q), _np(k), _np(v), _np(cs))) <= TOL[dtype]
    ref = O.fox_bwd(_np(q), _np(k), _np(v), _np(cs), _np(do))
    for name, got, r in zip(("dq", "dk", "dv", "dcs"), (dq, dk, dv, dcs), ref):
        assert O.norm_rel(_np(got), r) <= TOL[dtype], (name, O.norm_rel(_np(got), r))
    assert device_errors() == 0


def test_fox_zero_gates_is_causal_attention(cuda):
    """cs = 0 (no forgetting) is causal attention."""
    q, k, v, _ = attn_inputs(2, 4, 2, 256, 128, torch.bfloat16, seed=83)
    cs = torch.zeros(2, 4, 256, device="cuda")
    o = fs.fox_attention(q, k, v, cs)
    ref = fs.flash_attention(q, k, v, causal=True)
    torch.cuda.synchronize()
    assert O.norm_rel(_np(o), _np(ref)) <= 2e-2


@pytest.mark.parametrize("prec,dtype", [("f32", torch.float32), ("bf16", torch.bfloat16)])
def test_fox_shim_symbols(cuda, prec, dtype):
    """fused_fox_attention_launch / _backward_launch (io-typed cs, [dq|dk|dv|dcs])
    match the edb_* path on the io-rounded cs."""
    lib = ctypes.CDLL(build.SHIMS[prec])
    B, H, L, d = 2, 2, 96, 64
    q, k, v, do = attn_inputs(B, H, H, L, d, dtype, seed=84)
    cs_io = fox_cs(B, H, L, 85).to(dtype)
    cs = cs_io.float()
    P = lambda t: ctypes.c_void_p(t.data_ptr())
    out = torch.empty_like(q)
    assert lib.fused_fox_attention_launch(None, P(q), P(k), P(v), P(cs_io), P(out), B, H, L, d) == 0
    n = q.numel()
    cat = torch.empty(3 * n + B * H * L, dtype=dtype, device="cuda")
    assert lib.fused_fox_attention_backward_launch(None, P(q), P(k), P(v), P(cs_io), P(out),
                                                   P(do), P(cat), B, H, L, d) == 0
    torch.cuda.synchronize()
    o, lse = fs.fox_attention(q, k, v, cs, return_lse=True)
    want = fs.fox_attention_backward(q, k, v, cs, o, do, lse)
    torch.cuda.synchronize()
    assert torch.equal(out, o)
    for i, w in enumerate(want[:3]):
        assert torch.equal(cat[i * n:(i + 1) * n].view_as(w), w)
    assert torch.equal(cat[3 * n:].view(B, H, L), want[3].to(dtype))


@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("B,Hq,Hkv,L,d", [(2, 4, 2, 256, 64), (3, 8, 2, 384, 128),
                                          (4, 8, 4, 200, 128), (1, 2, 1, 130, 64)])
def test_flash_attention_train_host(cuda, causal, B, Hq, Hkv, L, d):
    """The host-tensor entry point ((batch, kv head) units streamed through a ring of
    three device slots, copies overlapped with the kernels) against the device entry
    points on the same inputs: four to eight chunks, so the ring wraps."""
    q, k, v, do = attn_inputs(B, Hq, Hkv, L, d, torch.bfloat16, seed=90 + L)
    pin = [t.cpu().pin_memory() for t in (q, k, v, do)]
    o, dq, dk, dv = fs.flash_attention_train_host(*pin, causal=causal)
    torch.cuda.synchronize()
    o_r, lse = fs.flash_attention(q, k, v, causal=causal, return_lse=True)
    dq_r, dk_r, dv_r = fs.flash_attention_backward(q, k, v, causal, o_r, do, lse)
    torch.cuda.synchronize()
    assert torch.equal(o, o_r.cpu())
    for got, ref in ((dq, dq_r), (dk, dk_r), (dv, dv_r)):
        ref = ref.cpu().double()
        assert ((got.double() - ref).norm() / ref.norm()).item() <= 1e-3
    assert device_errors() == 0


@pytest.mark.parametrize("B,Hq,Hkv,L,d", [(2, 4, 2, 256, 128), (3, 8, 2, 384, 64)])
def test_fox_and_laser_train_host(cuda, B, Hq, Hkv, L, d):
    """FoX and LASER over host tensors (the same unit ring as flash attention)
    against their device entry points on the same inputs."""
    q, k, v, do = attn_inputs(B, Hq, Hkv, L, d, torch.bfloat16, seed=95 + L)
    g = torch.Generator(device="cpu").manual_seed(96 + L)
    cs = torch.cumsum(torch.nn.functional.logsigmoid(torch.randn(B, Hq, L, generator=g)), -1)
    pin = [t.cpu().pin_memory() for t in (q, k, v, do)]
    cs_p = cs.pin_memory()
    cs = cs.cuda()
    # FoX
    got = fs.fox_attention_train_host(pin[0], pin[1], pin[2], cs_p, pin[3])
    torch.cuda.synchronize()
    o_r, lse = fs.fox_attention(q, k, v, cs, return_lse=True)
    ref = (o_r,) + tuple(fs.fox_attention_backward(q, k, v, cs, o_r, do, lse))
    torch.cuda.synchronize()
    assert torch.equal(got[0], ref[0].cpu())
    for a, r in zip(got[1:], ref[1:]):
        r = r.cpu().double()
        assert ((a.double() - r).norm() / r.norm()).item() <= 1e-3
    # LASER
    got = fs.laser_attention_train_host(*pin, causal=True)
    torch.cuda.synchronize()
    o_r, resid = fs.laser_attention(q, k, v, causal=True, return_resid=True)
    ref = (o_r,) + tuple(fs.laser_attention_backward(q, k, v, do, resid, causal=True))
    torch.cuda.synchronize()
    assert torch.equal(got[0], ref[0].cpu())
    for a, r in zip(got[1:], ref[1:]):
        r = r.cpu().double()
        assert ((a.double() - r).norm() / r.norm()).item() <= 1e-3
    assert device_errors() == 0
