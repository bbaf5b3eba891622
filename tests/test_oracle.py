"""Pin the CPU oracle (test infrastructure) before trusting it.

1. Golden vectors: op-level inputs/outputs captured from the reference's own
   fixtures and model classes (tests/golden/make_golden.py).
2. The reference's own C CPU references (native/cuda/test_kernels.cu), compiled
   from the reference sources into oracle/_ref/ (skipped where absent).
3. Backward = autograd of the forward (the reference's own test strategy,
   test/edifice/cuda/backward_kernels_test.exs), in f64 torch, at small shapes.
"""
import os

import numpy as np
import pytest
import torch

import oracle as O

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def _g(name):
    return np.load(os.path.join(GOLD, name))


# ------------------------------------------------------------------ golden
def test_golden_replays_matched_fixtures():
    for f in ("mingru_fixture.npz", "delta_net_fixture.npz", "mamba_fixture.npz", "gqa_fixture.npz"):
        assert float(_g(f)["model_replay_err"]) <= 1e-5


@pytest.mark.parametrize("layer", [0, 1])
def test_mingru_golden(layer):
    g = _g("mingru_fixture.npz")
    z, c, h = g["z%d" % layer], g["c%d" % layer], g["h%d" % layer]
    np.testing.assert_allclose(O.mingru_fwd(z, c), h, atol=1e-5)
    gz, gc, _ = O.mingru_bwd(z, c, None, h, g["dy%d" % layer])
    np.testing.assert_allclose(gz, g["gz%d" % layer], atol=1e-5)
    np.testing.assert_allclose(gc, g["gc%d" % layer], atol=1e-5)


@pytest.mark.parametrize("layer", [0, 1])
def test_delta_net_golden(layer):
    g = _g("delta_net_fixture.npz")
    q, k, v, beta = (g["%s%d" % (n, layer)] for n in ("q", "k", "v", "beta"))
    np.testing.assert_allclose(O.delta_net_fwd(q, k, v, beta), g["o%d" % layer], atol=1e-5)
    got = O.delta_net_bwd(q, k, v, beta, g["do%d" % layer])
    for x, n in zip(got, ("gq", "gk", "gv", "gbeta")):
        np.testing.assert_allclose(x, g["%s%d" % (n, layer)], atol=1e-5)


@pytest.mark.parametrize("layer", [0, 1])
def test_mamba_model_semantics_golden(layer):
    g = _g("mamba_fixture.npz")
    y = O.selective_scan_model_fwd(g["x%d" % layer], g["dt%d" % layer], g["B%d" % layer],
                                   g["C%d" % layer])
    np.testing.assert_allclose(y, g["y%d" % layer], atol=1e-6)


@pytest.mark.parametrize("layer", [0, 1])
def test_gqa_golden(layer):
    g = _g("gqa_fixture.npz")
    q, k, v = (g["%s%d" % (n, layer)] for n in ("q", "k", "v"))
    np.testing.assert_allclose(O.attention_fwd(q, k, v, causal=True), g["o%d" % layer], atol=1e-5)
    got = O.attention_bwd(q, k, v, g["do%d" % layer], causal=True)
    for x, n in zip(got, ("dq", "dk", "dv")):
        np.testing.assert_allclose(x, g["%s%d" % (n, layer)], atol=1e-5)


# ------------------------------------------- the reference's own C CPU refs
need_ref = pytest.mark.skipif(O.ref_cpu_lib() is None, reason="oracle/_ref not built")


@need_ref
def test_against_reference_c_linear_and_mingru():
    rng = np.random.default_rng(1)
    a = rng.random((3, 37, 45), dtype=np.float32)
    b = rng.standard_normal((3, 37, 45), dtype=np.float32)
    h0 = rng.standard_normal((3, 45), dtype=np.float32)
    np.testing.assert_allclose(O.linear_scan_fwd(a, b, h0), O.ref_linear_scan_cpu(a, b, h0),
                               rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(O.mingru_fwd(a, b, h0), O.ref_mingru_scan_cpu(a, b, h0),
                               rtol=1e-5, atol=1e-5)


@need_ref
def test_against_reference_c_delta_net():
    rng = np.random.default_rng(2)
    q, k, v = (rng.standard_normal((2, 19, 3, 16), dtype=np.float32) for _ in range(3))
    k /= np.sqrt((k * k).sum(-1, keepdims=True) + 1e-6)
    beta = rng.random((2, 19, 3, 16), dtype=np.float32)
    np.testing.assert_allclose(O.delta_net_fwd(q, k, v, beta),
                               O.ref_delta_net_scan_cpu(q, k, v, beta), rtol=1e-4, atol=1e-5)


# --------------------------------------------- backward = autograd(forward)
def _t(x):
    return torch.tensor(np.asarray(x, np.float64), requires_grad=True)


def test_linear_scan_bwd_autograd():
    rng = np.random.default_rng(3)
    a = rng.random((2, 11, 5)).astype(np.float32)
    b = rng.standard_normal((2, 11, 5)).astype(np.float32)
    h0 = rng.standard_normal((2, 5)).astype(np.float32)
    dy = rng.standard_normal((2, 11, 5)).astype(np.float32)
    ta, tb, th0 = _t(a), _t(b), _t(h0)
    s, outs = th0, []
    for t in range(11):
        s = ta[:, t] * s + tb[:, t]
        outs.append(s)
    h = torch.stack(outs, 1)
    h.backward(torch.tensor(dy, dtype=torch.float64))
    ga, gb, gh0 = O.linear_scan_bwd(a, h0, O.linear_scan_fwd(a, b, h0), dy)
    np.testing.assert_allclose(ga, ta.grad.numpy(), rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(gb, tb.grad.numpy(), rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(gh0, th0.grad.numpy(), rtol=1e-5, atol=1e-6)


def _ssm_torch(x, dt, A, Bm, Cm):
    dtc = dt.clamp(0.001, 0.1)
    Bsz, L, D = x.shape
    N = A.shape[1]
    h = torch.zeros(Bsz, D, N, dtype=x.dtype)
    ys = []
    for t in range(L):
        abar = torch.exp(dtc[:, t, :, None] * A[None])
        h = abar * h + dtc[:, t, :, None] * Bm[:, t, None, :] * x[:, t, :, None]
        ys.append((h * Cm[:, t, None, :]).sum(-1))
    return torch.stack(ys, 1)


def test_selective_scan_kernel_semantics_autograd():
    """Kernel semantics: given A, per-channel clamped dt (fused_selective_scan.cu:68-96);
    backward fused_scan.ex:1453-1531 (A gets no gradient, gdt masked outside the clamp)."""
    rng = np.random.default_rng(4)
    Bsz, L, D, N = 2, 13, 6, 4
    x = rng.standard_normal((Bsz, L, D)).astype(np.float32)
    dt = np.log1p(np.exp(rng.standard_normal((Bsz, L, D)) * 0.5 - 2)).astype(np.float32)
    dt[0, 3, 2] = 0.5      # clamped high: gdt must be 0 there
    dt[1, 5, 1] = 0.0005   # clamped low
    A = (-np.exp(rng.uniform(0, np.log(16), (D, N)))).astype(np.float32)
    Bm = rng.standard_normal((Bsz, L, N)).astype(np.float32)
    Cm = rng.standard_normal((Bsz, L, N)).astype(np.float32)
    dy = rng.standard_normal((Bsz, L, D)).astype(np.float32)
    tx, tdt, tB, tC = _t(x), _t(dt), _t(Bm), _t(Cm)
    y = _ssm_torch(tx, tdt, torch.tensor(A, dtype=torch.float64), tB, tC)
    np.testing.assert_allclose(O.selective_scan_fwd(x, dt, A, Bm, Cm), y.detach().numpy(),
                               rtol=1e-5, atol=1e-6)
    y.backward(torch.tensor(dy, dtype=torch.float64))
    gx, gdt, gB, gC = O.selective_scan_bwd(x, dt, A, Bm, Cm, dy)
    np.testing.assert_allclose(gx, tx.grad.numpy(), rtol=1e-5, atol=1e-6)
    # torch's clamp passes no gradient outside [lo, hi] -- the same mask as the fallback
    np.testing.assert_allclose(gdt, tdt.grad.numpy(), rtol=1e-5, atol=1e-6)
    assert gdt[0, 3, 2] == 0 and gdt[1, 5, 1] == 0
    np.testing.assert_allclose(gB, tB.grad.numpy(), rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(gC, tC.grad.numpy(), rtol=1e-5, atol=1e-6)


def _ssm_model_torch(x, dt, A, Bm, Cm, lo=O.DT_MIN, hi=O.DT_MAX):
    """discretize_ssm + sequential_scan + compute_ssm_output (common.ex:402-515)
    written in torch f64; A None is the fixed -(1..N) diagonal."""
    D, N = x.shape[2], Bm.shape[2]
    if A is None:
        A = -(torch.arange(N, dtype=torch.float64) + 1).expand(D, N)
    dtc = dt.clamp(lo, hi)
    mean = dtc.mean(2, keepdim=True)
    abar = torch.exp(dtc[..., None] * A)
    bx = (mean * x)[..., None] * Bm[:, :, None, :]
    h = torch.zeros(x.shape[0], D, N, dtype=torch.float64)
    ys = []
    for t in range(x.shape[1]):
        h = abar[:, t] * h + bx[:, t]
        ys.append((h * Cm[:, t, None, :]).sum(-1))
    return torch.stack(ys, 1)


@pytest.mark.parametrize("given_a", [False, True])
def test_selective_scan_model_semantics_autograd(given_a):
    """Model semantics (Edifice.build(:mamba) fallback): forward against a torch
    restatement and the golden-pinned oracle forward, backward against its
    autograd (A gets no gradient; gdt masked outside the clamp, and it carries
    the channel-mean term of B_bar)."""
    rng = np.random.default_rng(5)
    Bsz, L, D, N = 2, 11, 7, 5
    x = rng.standard_normal((Bsz, L, D)).astype(np.float32)
    dt = np.log1p(np.exp(rng.standard_normal((Bsz, L, D)) * 0.5 - 2)).astype(np.float32)
    dt[0, 3, 2] = 0.5
    dt[1, 5, 1] = 0.0005
    A = (-np.exp(rng.uniform(0, np.log(16), (D, N)))).astype(np.float32) if given_a else None
    Bm = rng.standard_normal((Bsz, L, N)).astype(np.float32)
    Cm = rng.standard_normal((Bsz, L, N)).astype(np.float32)
    dy = rng.standard_normal((Bsz, L, D)).astype(np.float32)
    tx, tdt, tB, tC = _t(x), _t(dt), _t(Bm), _t(Cm)
    tA = None if A is None else torch.tensor(A, dtype=torch.float64)
    y = _ssm_model_torch(tx, tdt, tA, tB, tC)
    np.testing.assert_allclose(O.selective_scan_model_fwd(x, dt, Bm, Cm, A=A),
                               y.detach().numpy(), rtol=1e-5, atol=1e-6)
    y.backward(torch.tensor(dy, dtype=torch.float64))
    gx, gdt, gB, gC = O.selective_scan_model_bwd(x, dt, Bm, Cm, dy, A=A)
    np.testing.assert_allclose(gx, tx.grad.numpy(), rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(gdt, tdt.grad.numpy(), rtol=1e-5, atol=1e-6)
    assert gdt[0, 3, 2] == 0 and gdt[1, 5, 1] == 0
    np.testing.assert_allclose(gB, tB.grad.numpy(), rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(gC, tC.grad.numpy(), rtol=1e-5, atol=1e-6)
    if not given_a:
        # the fixed diagonal passed explicitly gives the same numbers
        fixed = np.broadcast_to(-(np.arange(N, dtype=np.float32) + 1), (D, N))
        np.testing.assert_array_equal(O.selective_scan_model_fwd(x, dt, Bm, Cm, A=fixed),
                                      O.selective_scan_model_fwd(x, dt, Bm, Cm))


@pytest.mark.parametrize("causal", [True, False])
def test_laser_attention_autograd(causal):
    """LASER (fused_scan.ex:3667-3703 forward, :3723-3766 backward) in torch f64:
    the oracle's composition matches the restated fallback and its autograd (v_max
    held constant, as the reference captures it)."""
    rng = np.random.default_rng(9)
    B, H, L, d = 2, 3, 21, 8
    q, k, v, do = (rng.standard_normal((B, H, L, d)).astype(np.float32) for _ in range(4))
    tq, tk, tv = _t(q), _t(k), _t(v)
    vm = tv.detach().amax(2, keepdim=True)
    s = tq @ tk.transpose(-1, -2) / np.sqrt(d)
    if causal:
        s = s.masked_fill(~torch.ones(L, L, dtype=torch.bool).tril(), float("-inf"))
    A = torch.softmax(s, -1) @ torch.exp(tv - vm)
    o = torch.log(A.clamp_min(1e-7)) + vm
    o.backward(torch.tensor(do, dtype=torch.float64))
    got_o, got_a = O.laser_fwd(q, k, v, causal=causal)
    np.testing.assert_allclose(got_o, o.detach().numpy(), rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(got_a, A.detach().numpy(), rtol=1e-5, atol=1e-6)
    for got, ref in zip(O.laser_bwd(q, k, v, do, causal=causal), (tq, tk, tv)):
        np.testing.assert_allclose(got, ref.grad.numpy(), rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("hkv", [3, 1])
def test_fox_attention_autograd(hkv):
    """FoX (fused_scan.ex:3863-3912 forward, :3926-3984 backward): the oracle's
    backward equals torch f64 autograd of the forward (grad_cs included)."""
    rng = np.random.default_rng(10)
    B, H, L, d = 2, 3, 17, 8
    q = rng.standard_normal((B, H, L, d)).astype(np.float32)
    k, v = (rng.standard_normal((B, hkv, L, d)).astype(np.float32) for _ in range(2))
    cs = np.cumsum(np.log(1 / (1 + np.exp(-rng.standard_normal((B, H, L))))), -1).astype(
        np.float32)
    do = rng.standard_normal((B, H, L, d)).astype(np.float32)
    tq, tk, tv, tcs = _t(q), _t(k), _t(v), _t(cs)
    ke = tk.repeat_interleave(H // hkv, 1)
    ve = tv.repeat_interleave(H // hkv, 1)
    s = tq @ ke.transpose(-1, -2) / np.sqrt(d) + (tcs[..., :, None] - tcs[..., None, :])
    s = s.masked_fill(~torch.ones(L, L, dtype=torch.bool).tril(), float("-inf"))
    o = torch.softmax(s, -1) @ ve
    o.backward(torch.tensor(do, dtype=torch.float64))
    np.testing.assert_allclose(O.fox_fwd(q, k, v, cs), o.detach().numpy(), rtol=1e-5, atol=1e-6)
    for got, ref in zip(O.fox_bwd(q, k, v, cs, do), (tq, tk, tv, tcs)):
        np.testing.assert_allclose(got, ref.grad.numpy(), rtol=1e-4, atol=1e-6)


@pytest.mark.parametrize("scalar_beta", [False, True])
def test_delta_net_bwd_autograd(scalar_beta):
    rng = np.random.default_rng(5)
    Bsz, L, H, d = 2, 21, 2, 8
    q, k, v = (rng.standard_normal((Bsz, L, H, d)).astype(np.float32) for _ in range(3))
    k /= np.sqrt((k * k).sum(-1, keepdims=True) + 1e-6)
    beta = rng.random((Bsz, L, H) if scalar_beta else (Bsz, L, H, d)).astype(np.float32)
    do = rng.standard_normal((Bsz, L, H, d)).astype(np.float32)
    tq, tk, tv, tb = _t(q), _t(k), _t(v), _t(beta)
    bb = tb[..., None] if scalar_beta else tb
    S = torch.zeros(Bsz, H, d, d, dtype=torch.float64)
    outs = []
    for t in range(L):
        r = torch.einsum("bhij,bhj->bhi", S, tk[:, t])
        S = S + torch.einsum("bhi,bhj->bhij", bb[:, t] * (tv[:, t] - r), tk[:, t])
        outs.append(torch.einsum("bhij,bhj->bhi", S, tq[:, t]))
    o = torch.stack(outs, 1)
    np.testing.assert_allclose(O.delta_net_fwd(q, k, v, beta), o.detach().numpy(), rtol=1e-5,
                               atol=1e-6)
    o.backward(torch.tensor(do, dtype=torch.float64))
    got = O.delta_net_bwd(q, k, v, beta, do)
    for x, t_ in zip(got, (tq, tk, tv, tb)):
        np.testing.assert_allclose(x, t_.grad.numpy(), rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("scalar_beta", [False, True])
def test_gated_delta_net_bwd_autograd(scalar_beta):
    """GatedDeltaNet: the forward restates gated_delta_net_scan_fallback
    (fused_scan.ex:2256-2284); the backward is checked against autograd of that
    forward, the reference's own test strategy for it
    (test/edifice/cuda/backward_kernels_test.exs:1003-1060), at alpha in [0.8, 0.99]
    as there and at alpha in [0.05, 1) (decays a division-based backward could
    not undo)."""
    rng = np.random.default_rng(7)
    Bsz, L, H, d = 2, 37, 2, 8
    for lo in (0.8, 0.05):
        q, k, v = (rng.standard_normal((Bsz, L, H, d)).astype(np.float32) for _ in range(3))
        k /= np.sqrt((k * k).sum(-1, keepdims=True) + 1e-6)
        beta = rng.uniform(0.1, 0.9, (Bsz, L, H) if scalar_beta else (Bsz, L, H, d)).astype(
            np.float32)
        alpha = rng.uniform(lo, 0.99, (Bsz, L, H)).astype(np.float32)
        do = rng.standard_normal((Bsz, L, H, d)).astype(np.float32)
        tq, tk, tv, tb, ta = _t(q), _t(k), _t(v), _t(beta), _t(alpha)
        bb = tb[..., None] if scalar_beta else tb
        S = torch.zeros(Bsz, H, d, d, dtype=torch.float64)
        outs = []
        for t in range(L):
            Sd = ta[:, t, :, None, None] * S
            r = torch.einsum("bhij,bhj->bhi", Sd, tk[:, t])
            S = Sd + torch.einsum("bhi,bhj->bhij", bb[:, t] * (tv[:, t] - r), tk[:, t])
            outs.append(torch.einsum("bhij,bhj->bhi", S, tq[:, t]))
        o = torch.stack(outs, 1)
        np.testing.assert_allclose(O.gated_delta_net_fwd(q, k, v, beta, alpha),
                                   o.detach().numpy(), rtol=1e-5, atol=1e-6)
        o.backward(torch.tensor(do, dtype=torch.float64))
        got = O.gated_delta_net_bwd(q, k, v, beta, alpha, do)
        for x, t_ in zip(got, (tq, tk, tv, tb, ta)):
            np.testing.assert_allclose(x, t_.grad.numpy(), rtol=1e-5, atol=1e-5)
        # alpha == 1 is the plain delta rule
        one = np.ones_like(alpha)
        np.testing.assert_allclose(O.gated_delta_net_fwd(q, k, v, beta, one),
                                   O.delta_net_fwd(q, k, v, beta), rtol=1e-6, atol=1e-6)
        g1 = O.gated_delta_net_bwd(q, k, v, beta, one, do)
        for x, y in zip(g1[:4], O.delta_net_bwd(q, k, v, beta, do)):
            np.testing.assert_allclose(x, y, rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("causal,hq,hkv", [(True, 4, 2), (False, 4, 4), (True, 8, 2)])
def test_attention_bwd_autograd(causal, hq, hkv):
    rng = np.random.default_rng(6)
    Bsz, L, d = 2, 17, 8
    q = rng.standard_normal((Bsz, hq, L, d)).astype(np.float32)
    k, v = (rng.standard_normal((Bsz, hkv, L, d)).astype(np.float32) for _ in range(2))
    do = rng.standard_normal((Bsz, hq, L, d)).astype(np.float32)
    tq, tk, tv = _t(q), _t(k), _t(v)
    g = hq // hkv
    kr = tk.repeat_interleave(g, dim=1)
    vr = tv.repeat_interleave(g, dim=1)
    o = torch.nn.functional.scaled_dot_product_attention(tq, kr, vr, is_causal=causal)
    ours, lse = O.attention_fwd(q, k, v, causal=causal, want_lse=True)
    np.testing.assert_allclose(ours, o.detach().numpy(), rtol=1e-5, atol=1e-6)
    s = torch.einsum("bhid,bhjd->bhij", tq, kr) / np.sqrt(d)
    if causal:
        s = s.masked_fill(torch.triu(torch.ones(L, L, dtype=torch.bool), 1), float("-inf"))
    np.testing.assert_allclose(lse, torch.logsumexp(s, -1).detach().numpy(), rtol=1e-5, atol=1e-5)
    o.backward(torch.tensor(do, dtype=torch.float64))
    got = O.attention_bwd(q, k, v, do, causal=causal)
    for x, t_ in zip(got, (tq, tk, tv)):
        np.testing.assert_allclose(x, t_.grad.numpy(), rtol=1e-5, atol=1e-6)


def test_f32_variant_tracks_f64():
    rng = np.random.default_rng(7)
    a = (1 / (1 + np.exp(-rng.standard_normal((2, 300, 64))))).astype(np.float32)
    b = rng.standard_normal((2, 300, 64)).astype(np.float32)
    assert O.norm_rel(O.linear_scan_fwd(a, b, prec="f32"), O.linear_scan_fwd(a, b)) < 1e-6
