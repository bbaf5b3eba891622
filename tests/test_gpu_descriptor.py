"""GPU checks of the descriptor form of the C ABI (edb_<op>_{fwd,bwd}_desc).

Every case feeds the descriptor entry points strided views -- transposed
layouts, slices of packed buffers, broadcasts, unaligned pointers -- for inputs
and outputs, and compares with the positional entry points run on contiguous
copies of the same values.  The descriptor form gathers into dense copies and
runs the same kernels, so results agree bit for bit wherever the kernels are
deterministic (every path here but the flash-attention dQ and the chunked
DeltaNet, whose f32 reductions may land in a different order before the bf16
rounding, so a few elements move by one bf16 ulp: checked to 1e-3
norm-relative, a quarter of bf16's relative resolution).  Absolute correctness of those kernels is the oracle
parity tests' job.
"""
import pytest
import torch

from edifice_b200 import descriptor as D
from edifice_b200 import device_errors
from edifice_b200 import fused_scan as fs

pytestmark = pytest.mark.gpu


def _g(seed):
    return torch.Generator(device="cpu").manual_seed(seed)


def _exact(a, b):
    assert a.shape == b.shape and a.dtype == b.dtype
    assert torch.equal(a, b), (a.float() - b.float()).abs().max().item()


def _close(a, b, tol=1e-3):
    a, b = a.double(), b.double()
    assert ((a - b).norm() / b.norm().clamp_min(1e-30)).item() <= tol


def _transposed(x, dims):
    """A non-contiguous view equal to x: x's values stored with `dims` permuted."""
    inv = [dims.index(i) for i in range(len(dims))]
    return x.permute(*dims).contiguous().permute(*inv)


def _unaligned(x):
    """A dense view of x's values starting 2 bytes past a 16-byte boundary."""
    flat = torch.empty(x.numel() + 8, dtype=x.dtype, device=x.device)
    v = flat[1:1 + x.numel()].view(x.shape)
    v.copy_(x)
    return v


def _out_view(shape, dtype, dims):
    """An uninitialised output view with a permuted storage order."""
    inv = [dims.index(i) for i in range(len(dims))]
    store = torch.full([shape[d] for d in dims], float("nan"), dtype=dtype, device="cuda")
    return store.permute(*inv)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_linear_scan_desc_strided(cuda, dtype):
    g = _g(1)
    B, L, H = 3, 300, 96
    a = torch.sigmoid(torch.randn(B, L, H, generator=g)).to(dtype).cuda()
    b = torch.randn(B, L, H, generator=g).to(dtype).cuda()
    dy = torch.randn(B, L, H, generator=g).to(dtype).cuda()
    h0row = torch.randn(1, H, generator=g).to(dtype).cuda()
    h0 = h0row.expand(B, H)                        # broadcast, stride 0
    h_ref = fs.linear_scan(a, b, h0.contiguous())
    ga_r, gb_r, gh0_r = fs.linear_scan_backward(a, h0.contiguous(), h_ref, dy)

    a_v, b_v = _transposed(a, [0, 2, 1]), _unaligned(b)
    h = _out_view((B, L, H), dtype, [2, 0, 1])
    args = D.make_args("linear_scan", dtype, a=a_v, b=b_v, h0=h0, h=h)
    D.run("linear_scan", "fwd", args)
    ga = _out_view((B, L, H), dtype, [1, 0, 2])
    gb = torch.empty(B, L, 2 * H, dtype=dtype, device="cuda")[..., H:]   # slice of a wider row
    gh0 = torch.empty(H, B, dtype=dtype, device="cuda").t()
    args = D.make_args("linear_scan", dtype, a=a_v, h0=h0, h=_transposed(h_ref, [1, 0, 2]),
                       dy=_unaligned(dy), ga=ga, gb=gb, gh0=gh0)
    D.run("linear_scan", "bwd", args)
    torch.cuda.synchronize()
    _exact(h.contiguous(), h_ref)
    for u, r in ((ga, ga_r), (gb, gb_r), (gh0, gh0_r)):
        _exact(u.contiguous(), r)
    assert device_errors() == 0


def test_linear_scan_desc_dense_runs_in_place(cuda):
    g = _g(2)
    B, L, H = 2, 256, 128
    a = torch.sigmoid(torch.randn(B, L, H, generator=g)).bfloat16().cuda()
    b = torch.randn(B, L, H, generator=g).bfloat16().cuda()
    h = torch.empty_like(a)
    args = D.make_args("linear_scan", torch.bfloat16, a=a, b=b, h=h)
    assert D.workspace_bytes("linear_scan", "fwd", args) == 0
    D.run("linear_scan", "fwd", args)
    _exact(h, fs.linear_scan(a, b))


def test_mingru_desc_strided(cuda):
    g = _g(3)
    B, L, H = 2, 200, 130
    z = torch.sigmoid(torch.randn(B, L, H, generator=g)).bfloat16().cuda()
    c = torch.randn(B, L, H, generator=g).bfloat16().cuda()
    dy = torch.randn(B, L, H, generator=g).bfloat16().cuda()
    h_ref = fs.mingru_scan(z, c)
    gz_r, gc_r, gh0_r = fs.mingru_backward(z, c, None, h_ref, dy)
    # z and c interleaved in one [B, L, 2, H] buffer, as a fused projection leaves them
    zc = torch.stack([z, c], dim=2)
    h = _out_view((B, L, H), torch.bfloat16, [1, 2, 0])
    D.run("mingru", "fwd", D.make_args("mingru", torch.bfloat16, z=zc[:, :, 0], c=zc[:, :, 1],
                                       h=h))
    gz, gc = _out_view((B, L, H), torch.bfloat16, [2, 1, 0]), torch.empty_like(z)
    gh0 = torch.empty(B, H, dtype=torch.bfloat16, device="cuda")
    D.run("mingru", "bwd", D.make_args("mingru", torch.bfloat16, z=zc[:, :, 0], c=zc[:, :, 1],
                                       h=h, dy=_transposed(dy, [2, 1, 0]), gz=gz, gc=gc,
                                       gh0=gh0))
    torch.cuda.synchronize()
    _exact(h.contiguous(), h_ref)
    for u, r in ((gz, gz_r), (gc, gc_r), (gh0, gh0_r)):
        _exact(u.contiguous(), r)


@pytest.mark.parametrize("semantics", [D.SSM_KERNEL, D.SSM_MODEL])
def test_selective_scan_desc_strided(cuda, semantics):
    g = _g(4)
    B, L, Dn, N = 2, 160, 256, 16
    dtype = torch.bfloat16
    x = torch.randn(B, L, Dn, generator=g).to(dtype).cuda()
    dt = torch.nn.functional.softplus(0.5 * torch.randn(B, L, Dn, generator=g) - 2).to(dtype).cuda()
    A = (-torch.exp(torch.rand(Dn, N, generator=g) * 2.77)).to(dtype).cuda()
    Bm = torch.randn(B, L, N, generator=g).to(dtype).cuda()
    Cm = torch.randn(B, L, N, generator=g).to(dtype).cuda()
    dy = torch.randn(B, L, Dn, generator=g).to(dtype).cuda()
    model = semantics == D.SSM_MODEL
    if model:
        y_r, dtm_r = fs.selective_scan_model(x, dt, Bm, Cm)
        gx_r, gdt_r, gB_r, gC_r = fs.selective_scan_model_backward(x, dt, Bm, Cm, dy, dtm_r)
    else:
        y_r = fs.selective_scan(x, dt, A, Bm, Cm)
        gx_r, gdt_r, gB_r, gC_r = fs.selective_scan_backward(x, dt, A, Bm, Cm, dy)
    # B and C as the two halves of one dense(2N) projection output (common.ex:333-396)
    BC = torch.cat([Bm, Cm], dim=-1)
    dt_mean = torch.empty(B, L, dtype=torch.float32, device="cuda")
    y = _out_view((B, L, Dn), dtype, [2, 0, 1])
    common = dict(semantics=semantics, dt_min=1e-3, dt_max=0.1, x=_transposed(x, [1, 0, 2]),
                  dt=_unaligned(dt), A=None if model else _transposed(A, [1, 0]),
                  B=BC[..., :N], C=BC[..., N:], dt_mean=dt_mean)
    D.run("selective_scan", "fwd", D.make_args("selective_scan", dtype, y=y, **common))
    gx, gdt = _out_view((B, L, Dn), dtype, [1, 2, 0]), torch.empty_like(x)
    gBC = torch.empty(B, L, 2 * N, dtype=torch.float32, device="cuda")
    D.run("selective_scan", "bwd",
          D.make_args("selective_scan", dtype, dy=dy, gx=gx, gdt=gdt, gB=gBC[..., :N],
                      gC=gBC[..., N:], **common))
    torch.cuda.synchronize()
    _exact(y.contiguous(), y_r)
    if model:
        _exact(dt_mean, dtm_r)
    for u, r in ((gx, gx_r), (gdt, gdt_r), (gBC[..., :N], gB_r), (gBC[..., N:], gC_r)):
        _exact(u.contiguous(), r)
    assert device_errors() == 0


def _delta_inputs(B, L, H, d, dtype, seed, per_element=False):
    g = _g(seed)
    q, k, v, do = (torch.randn(B, L, H, d, generator=g) for _ in range(4))
    k = k / torch.sqrt((k * k).sum(-1, keepdim=True) + 1e-6)
    beta = torch.sigmoid(torch.randn(*((B, L, H, d) if per_element else (B, L, H)), generator=g))
    alpha = 0.5 + 0.5 * torch.rand(B, L, H, generator=g)
    return [t.to(dtype).cuda() for t in (q, k, v, beta, alpha, do)]


@pytest.mark.parametrize("form", ["chunked", "token_per_element", "gated", "gated_chunked"])
def test_delta_rule_desc_packed_qkv(cuda, form):
    B, L, H, d = 2, 192, 2, (128 if form in ("chunked", "gated_chunked") else 64)
    dtype = torch.bfloat16
    q, k, v, beta, alpha, do = _delta_inputs(B, L, H, d, dtype, 5,
                                             per_element=form == "token_per_element")
    gated = form.startswith("gated")
    if gated:
        o_r = fs.gated_delta_net_scan(q, k, v, beta, alpha)
        grads_r = fs.gated_delta_net_backward(q, k, v, beta, alpha, do)
    else:
        o_r = fs.delta_net_scan(q, k, v, beta)
        grads_r = fs.delta_rule_backward(q, k, v, beta, do)
    # q, k, v as slices of one packed [B, L, 3, H, d] projection
    qkv = torch.stack([q, k, v], dim=2)
    mode = D.BETA_PER_ELEMENT if beta.dim() == 4 else D.BETA_PER_TOKEN
    common = dict(beta_mode=mode, q=qkv[:, :, 0], k=qkv[:, :, 1], v=qkv[:, :, 2],
                  beta=_unaligned(beta), alpha=alpha if gated else None)
    o = _out_view((B, L, H, d), dtype, [0, 2, 1, 3])
    D.run("delta_rule", "fwd", D.make_args("delta_rule", dtype, o=o, **common))
    gqkv = torch.empty(B, L, 3, H, d, dtype=dtype, device="cuda")
    gbeta = torch.empty_like(beta)
    galpha = torch.empty(H, B, L, dtype=dtype, device="cuda").permute(1, 2, 0) if gated else None
    D.run("delta_rule", "bwd",
          D.make_args("delta_rule", dtype, dO=_transposed(do, [0, 2, 1, 3]), gq=gqkv[:, :, 0],
                      gk=gqkv[:, :, 1], gv=gqkv[:, :, 2], gbeta=gbeta, galpha=galpha, **common))
    torch.cuda.synchronize()
    got = [gqkv[:, :, 0], gqkv[:, :, 1], gqkv[:, :, 2], gbeta] + ([galpha] if gated else [])
    cmp = _close if form in ("chunked", "gated_chunked") else _exact
    cmp(o.contiguous(), o_r)
    for u, r in zip(got, grads_r):
        cmp(u.contiguous(), r)
    assert device_errors() == 0


@pytest.mark.parametrize("causal", [True, False])
def test_flash_attention_desc_blhd_layout(cuda, causal):
    g = _g(6)
    B, Hq, Hkv, L, d = 2, 4, 2, 320, 128
    dtype = torch.bfloat16
    # the usual projection layout [B, L, H, d], read as [B, H, L, d] views
    q_blhd = torch.randn(B, L, Hq, d, generator=g).to(dtype).cuda()
    k_blhd = torch.randn(B, L, Hkv, d, generator=g).to(dtype).cuda()
    v_blhd = torch.randn(B, L, Hkv, d, generator=g).to(dtype).cuda()
    do_blhd = torch.randn(B, L, Hq, d, generator=g).to(dtype).cuda()
    q, k, v, do = (t.transpose(1, 2) for t in (q_blhd, k_blhd, v_blhd, do_blhd))
    o_r, lse_r = fs.flash_attention(q.contiguous(), k.contiguous(), v.contiguous(), causal=causal,
                                    return_lse=True)
    dq_r, dk_r, dv_r = fs.flash_attention_backward(q.contiguous(), k.contiguous(), v.contiguous(),
                                                   causal, o_r, do.contiguous(), lse_r)
    lse = torch.empty(B, Hq, L, dtype=torch.float32, device="cuda")
    o = torch.empty(B, L, Hq, d, dtype=dtype, device="cuda").transpose(1, 2)
    common = dict(causal=int(causal), num_kv_heads=Hkv, scale=0.0, q=q, k=k, v=v, lse=lse)
    D.run("flash_attention", "fwd", D.make_args("flash_attention", dtype, o=o, **common))
    dq = torch.empty(B, L, Hq, d, dtype=dtype, device="cuda").transpose(1, 2)
    dk = torch.empty(B, L, Hkv, d, dtype=dtype, device="cuda").transpose(1, 2)
    dv = torch.empty(B, L, Hkv, d, dtype=dtype, device="cuda").transpose(1, 2)
    D.run("flash_attention", "bwd",
          D.make_args("flash_attention", dtype, o=o, dO=do, dq=dq, dk=dk, dv=dv, **common))
    torch.cuda.synchronize()
    _exact(o.contiguous(), o_r)
    _exact(lse, lse_r)
    _close(dq.contiguous(), dq_r)
    _exact(dk.contiguous(), dk_r)
    _exact(dv.contiguous(), dv_r)
    assert device_errors() == 0


@pytest.mark.parametrize("kind", [0, 1, 2])
def test_native_rec_desc_strided(cuda, kind):
    g = _g(7)
    B, L, H = 2, 257, 192
    x0 = torch.randn(B, L, H, generator=g).bfloat16().cuda()
    x1 = torch.randn(B, L, H, generator=g).bfloat16().cuda()
    h0 = torch.randn(B, H, generator=g).bfloat16().cuda()
    ref = [fs.elu_gru, fs.real_gru, fs.diag_linear][kind](x0, x1, h0)
    h = _out_view((B, L, H), torch.bfloat16, [1, 0, 2])
    D.run("native_rec", "fwd", D.make_args("native_rec", torch.bfloat16, kind=kind,
                                           x0=_transposed(x0, [2, 1, 0]), x1=_unaligned(x1),
                                           h0=_transposed(h0, [1, 0]), h=h))
    torch.cuda.synchronize()
    _exact(h.contiguous(), ref)


def _attn_blhd(B, Hq, Hkv, L, d, seed):
    g = _g(seed)
    mk = lambda h: torch.randn(B, L, h, d, generator=g).bfloat16().cuda().transpose(1, 2)
    return mk(Hq), mk(Hkv), mk(Hkv), mk(Hq)


def test_laser_attention_desc_blhd_layout(cuda):
    B, Hq, Hkv, L, d = 1, 4, 2, 256, 128
    q, k, v, do = _attn_blhd(B, Hq, Hkv, L, d, 8)
    qc, kc, vc, doc = (t.contiguous() for t in (q, k, v, do))
    o_r, resid_r = fs.laser_attention(qc, kc, vc, causal=True, return_resid=True)
    dq_r, dk_r, dv_r = fs.laser_attention_backward(qc, kc, vc, doc, resid_r, causal=True)
    resid = torch.empty_like(resid_r)
    o = torch.empty(B, L, Hq, d, dtype=torch.bfloat16, device="cuda").transpose(1, 2)
    common = dict(causal=1, scale=0.0, q=q, k=k, resid=resid)
    D.run("laser_attention", "fwd",
          D.make_args("laser_attention", torch.bfloat16, v=v, o=o, **common))
    dq = torch.empty(B, L, Hq, d, dtype=torch.bfloat16, device="cuda").transpose(1, 2)
    dk, dv = torch.empty_like(kc), _out_view((B, Hkv, L, d), torch.bfloat16, [0, 2, 1, 3])
    D.run("laser_attention", "bwd",
          D.make_args("laser_attention", torch.bfloat16, dO=do, dq=dq, dk=dk, dv=dv, **common))
    torch.cuda.synchronize()
    _exact(o.contiguous(), o_r)
    _close(dq.contiguous(), dq_r)
    _exact(dk, dk_r)
    _exact(dv.contiguous(), dv_r)
    assert device_errors() == 0


def test_fox_attention_desc_blhd_layout(cuda):
    B, Hq, Hkv, L, d = 1, 4, 2, 192, 64
    q, k, v, do = _attn_blhd(B, Hq, Hkv, L, d, 9)
    qc, kc, vc, doc = (t.contiguous() for t in (q, k, v, do))
    g = _g(10)
    cs = torch.cumsum(torch.nn.functional.logsigmoid(torch.randn(B, L, Hq, generator=g)), 1)
    cs = cs.cuda().transpose(1, 2)                       # [B, Hq, L] view of [B, L, Hq]
    o_r, lse_r = fs.fox_attention(qc, kc, vc, cs.contiguous(), return_lse=True)
    dq_r, dk_r, dv_r, dcs_r = fs.fox_attention_backward(qc, kc, vc, cs.contiguous(), o_r, doc,
                                                        lse_r)
    lse = torch.empty_like(lse_r)
    o = torch.empty(B, L, Hq, d, dtype=torch.bfloat16, device="cuda").transpose(1, 2)
    common = dict(scale=0.0, q=q, k=k, v=v, cs=cs, lse=lse)
    D.run("fox_attention", "fwd", D.make_args("fox_attention", torch.bfloat16, o=o, **common))
    dq = torch.empty(B, L, Hq, d, dtype=torch.bfloat16, device="cuda").transpose(1, 2)
    dk, dv = torch.empty_like(kc), torch.empty_like(vc)
    dcs = torch.empty(B, L, Hq, dtype=torch.float32, device="cuda").transpose(1, 2)
    D.run("fox_attention", "bwd",
          D.make_args("fox_attention", torch.bfloat16, o=o, dO=do, dq=dq, dk=dk, dv=dv,
                      dcs=dcs, **common))
    torch.cuda.synchronize()
    _exact(o.contiguous(), o_r)
    _exact(lse, lse_r)
    for u, r in ((dq, dq_r), (dk, dk_r), (dv, dv_r), (dcs, dcs_r)):
        _close(u.contiguous(), r)
    assert device_errors() == 0


def test_all_zero_strides_are_a_broadcast(cuda):
    """A one-element tensor expanded to the full shape has every stride zero: as an
    input it is gathered as the broadcast it is (never read as a dense array past
    its one element), as an output it is rejected before any GPU work."""
    g = _g(7)
    B, L, H = 2, 130, 64
    dtype = torch.bfloat16
    a1 = torch.tensor(0.75, dtype=dtype, device="cuda").expand(B, L, H)
    assert a1.stride() == (0, 0, 0)
    b = torch.randn(B, L, H, generator=g).to(dtype).cuda()
    h_ref = fs.linear_scan(a1.contiguous(), b)
    h = torch.empty(B, L, H, dtype=dtype, device="cuda")
    D.run("linear_scan", "fwd", D.make_args("linear_scan", dtype, a=a1, b=b, h=h))
    _exact(h, h_ref)
    out1 = torch.empty((), dtype=dtype, device="cuda").expand(B, L, H)
    with pytest.raises(Exception):
        D.run("linear_scan", "fwd", D.make_args("linear_scan", dtype, a=a1, b=b, h=out1))
    torch.cuda.synchronize()
    assert device_errors() == 0
