"""Host-side mirror of ``Edifice.CUDA.FusedScan`` for the fused sequence-mixing path.

Same op names, argument meaning and error behaviour as the reference module
(lib/edifice/cuda/fused_scan.ex), over torch CUDA tensors as the device-memory
plumbing, calling libedifice_b200.so through its C ABI.  There is no fallback
tier: a missing library, a CPU tensor or a failed launch raises, the way the
reference's NIF tier raises ``"CUDA fused ... failed: reason"``
(e.g. fused_scan.ex:2804-2806).

Forward ops return new tensors; ``*_backward`` functions return the gradient
tuple of the reference's backward dispatch; the ``*_fn`` autograd Functions
reproduce the reference's ``custom_grad`` wiring (which inputs get gradients,
and the sigmoid chain rule applied outside the kernel for MinGRU).
"""
import torch

from . import _lib

_DT = {torch.float32: _lib.EDB_F32, torch.bfloat16: _lib.EDB_BF16}


def _dtype_code(t, what):
    if t.dtype not in _DT:
        raise _lib.EdbError("%s: unsupported dtype %s (f32 or bf16)" % (what, t.dtype))
    return _DT[t.dtype]


def _dev(*ts, what="op"):
    for t in ts:
        if t is not None and (not t.is_cuda or not t.is_contiguous()):
            raise _lib.EdbError("%s: inputs must be contiguous CUDA tensors "
                                "(there is no CPU path)" % what)


def _p(t):
    return None if t is None else t.data_ptr()


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _same(shape_a, shape_b, what):
    if tuple(shape_a) != tuple(shape_b):
        raise _lib.EdbError("%s: shape mismatch %s vs %s" % (what, tuple(shape_a), tuple(shape_b)))


# ------------------------------------------------------------------ linear scan
def linear_scan(a_vals, b_vals, h0=None):
    """h_t = a_t * h_{t-1} + b_t, h_{-1} = h0 (zeros if None).  [B, L, H] -> [B, L, H].
    Mirrors FusedScan.linear_scan/2 (fused_scan.ex:171-185)."""
    _dev(a_vals, b_vals, h0, what="linear_scan")
    _same(a_vals.shape, b_vals.shape, "linear_scan")
    B, L, H = a_vals.shape
    out = torch.empty_like(a_vals)
    lib = _lib.load()
    _lib.check(lib.edb_linear_scan_fwd(_dtype_code(a_vals, "linear_scan"), _p(a_vals), _p(b_vals),
                                       _p(h0), _p(out), B, L, H, _stream()), "CUDA linear scan")
    return out


def linear_scan_backward(a_vals, h0, forward_out, grad_output):
    """Returns (grad_a, grad_b, grad_h0).  Mirrors linear_scan_backward_dispatch/4
    (fused_scan.ex:852-867); h0 None means zeros."""
    _dev(a_vals, h0, forward_out, grad_output, what="linear_scan_backward")
    B, L, H = a_vals.shape
    ga, gb = torch.empty_like(a_vals), torch.empty_like(a_vals)
    gh0 = torch.empty((B, H), dtype=a_vals.dtype, device=a_vals.device)
    lib = _lib.load()
    _lib.check(lib.edb_linear_scan_bwd(_dtype_code(a_vals, "linear_scan_backward"), _p(a_vals),
                                       _p(h0), _p(forward_out), _p(grad_output), _p(ga), _p(gb),
                                       _p(gh0), B, L, H, _stream()), "CUDA linear scan backward")
    return ga, gb, gh0


class LinearScanFn(torch.autograd.Function):
    """custom_grad wiring of linear_scan_custom_call/2 (fused_scan.ex:834-850):
    gradients flow to a_vals and b_vals."""

    @staticmethod
    def forward(ctx, a_vals, b_vals):
        out = linear_scan(a_vals, b_vals)
        ctx.save_for_backward(a_vals, out)
        return out

    @staticmethod
    def backward(ctx, grad_output):
        a_vals, out = ctx.saved_tensors
        ga, gb, _ = linear_scan_backward(a_vals, None, out, grad_output.contiguous())
        return ga, gb


# ------------------------------------------------------------------------ MinGRU
def mingru_scan(z, candidates, h0=None):
    """Kernel-level MinGRU on post-sigmoid gates: h = (1 - z) h + z c."""
    _dev(z, candidates, h0, what="mingru")
    _same(z.shape, candidates.shape, "mingru")
    B, L, H = z.shape
    out = torch.empty_like(z)
    lib = _lib.load()
    _lib.check(lib.edb_mingru_fwd(_dtype_code(z, "mingru"), _p(z), _p(candidates), _p(h0),
                                  _p(out), B, L, H, _stream()), "CUDA fused MinGRU scan")
    return out


def mingru(gates, candidates):
    """FusedScan.mingru/2 (fused_scan.ex:60-74): z = sigmoid(gates) is computed
    outside the kernel (as the reference does on the XLA side, :2777), h0 = 0."""
    return mingru_scan(torch.sigmoid(gates), candidates)


def mingru_backward(z, candidates, h0, forward_out, grad_output):
    """Returns (grad_z, grad_cand, grad_h0) w.r.t. post-sigmoid z.  Mirrors
    mingru_backward_dispatch/5 (fused_scan.ex:530-545)."""
    _dev(z, candidates, h0, forward_out, grad_output, what="mingru_backward")
    B, L, H = z.shape
    gz, gc = torch.empty_like(z), torch.empty_like(z)
    gh0 = torch.empty((B, H), dtype=z.dtype, device=z.device)
    lib = _lib.load()
    _lib.check(lib.edb_mingru_bwd(_dtype_code(z, "mingru_backward"), _p(z), _p(candidates), _p(h0),
                                  _p(forward_out), _p(grad_output), _p(gz), _p(gc), _p(gh0), B, L,
                                  H, _stream()), "CUDA fused MinGRU scan backward")
    return gz, gc, gh0


class MinGRUFn(torch.autograd.Function):
    """custom_grad wiring of mingru_custom_call/2 (fused_scan.ex:454-481):
    gradients to the raw gates (sigmoid chain rule applied outside the kernel,
    :477-479) and to the candidates."""

    @staticmethod
    def forward(ctx, gates, candidates):
        z = torch.sigmoid(gates)
        out = mingru_scan(z, candidates)
        ctx.save_for_backward(z, candidates, out)
        return out

    @staticmethod
    def backward(ctx, grad_output):
        z, cand, out = ctx.saved_tensors
        gz, gc, _ = mingru_backward(z, cand, None, out, grad_output.contiguous())
        return gz * z * (1 - z), gc


# ------------------------------------------------- native-recurrence scans
def _native_rec(kind, x0, x1, h0, what):
    _dev(x0, x1, h0, what=what)
    _same(x0.shape, x1.shape, what)
    B, L, H = x0.shape
    out = torch.empty_like(x0)
    lib = _lib.load()
    _lib.check(lib.edb_native_rec_fwd(kind, _dtype_code(x0, what), _p(x0), _p(x1), _p(h0),
                                      _p(out), B, L, H, _stream()), "CUDA fused %s" % what)
    return out


def elu_gru(gates, candidates, h0=None):
    """FusedScan.elu_gru/2 (fused_scan.ex:94-108; NativeRecurrence.elu_gru_scan,
    native_recurrence.ex:146-172): z = sigmoid(gates), c = 1 + elu(candidates),
    h = (1 - z) h + z c, activations inside the kernel."""
    return _native_rec(_lib.EDB_NATIVE_ELU_GRU, gates, candidates, h0, "elu_gru")


def real_gru(gates, candidates, h0=None):
    """FusedScan.real_gru/2 (fused_scan.ex:111-125; native_recurrence.ex:193-213):
    z = sigmoid(gates), h = (1 - z) h + z candidates."""
    return _native_rec(_lib.EDB_NATIVE_REAL_GRU, gates, candidates, h0, "real_gru")


def diag_linear(a_vals, b_vals, h0=None):
    """FusedScan.diag_linear/2 (fused_scan.ex:128-142; native_recurrence.ex:232-250):
    h = sigmoid(a_vals) h + b_vals."""
    return _native_rec(_lib.EDB_NATIVE_DIAG_LINEAR, a_vals, b_vals, h0, "diag_linear")


class EluGRUFn(torch.autograd.Function):
    """custom_grad wiring of elu_gru_custom_call (fused_scan.ex:679-706): the
    MinGRU backward on z = sigmoid(gates), c = 1 + elu(candidates), then the
    sigmoid and elu chain rules (elu'(x) = 1 for x > 0, exp(x) otherwise)."""

    @staticmethod
    def forward(ctx, gates, candidates):
        out = elu_gru(gates, candidates)
        ctx.save_for_backward(gates, candidates, out)
        return out

    @staticmethod
    def backward(ctx, grad_output):
        gates, cand, out = ctx.saved_tensors
        z = torch.sigmoid(gates)
        c_act = 1.0 + torch.where(cand > 0, cand, torch.expm1(cand))
        gz, gc, _ = mingru_backward(z, c_act, None, out, grad_output.contiguous())
        elu_d = torch.where(cand > 0, torch.ones_like(cand), torch.exp(cand))
        return gz * z * (1 - z), gc * elu_d


class RealGRUFn(torch.autograd.Function):
    """custom_grad wiring of real_gru (the MinGRU backward, fused_scan.ex:995-998,
    and the sigmoid chain rule)."""

    @staticmethod
    def forward(ctx, gates, candidates):
        out = real_gru(gates, candidates)
        ctx.save_for_backward(gates, candidates, out)
        return out

    @staticmethod
    def backward(ctx, grad_output):
        gates, cand, out = ctx.saved_tensors
        z = torch.sigmoid(gates)
        gz, gc, _ = mingru_backward(z, cand, None, out, grad_output.contiguous())
        return gz * z * (1 - z), gc


class DiagLinearFn(torch.autograd.Function):
    """custom_grad wiring of diag_linear (the linear-scan backward on
    a = sigmoid(a_vals), fused_scan.ex:1019-1023, and the sigmoid chain rule)."""

    @staticmethod
    def forward(ctx, a_vals, b_vals):
        out = diag_linear(a_vals, b_vals)
        ctx.save_for_backward(a_vals, out)
        return out

    @staticmethod
    def backward(ctx, grad_output):
        a_vals, out = ctx.saved_tensors
        a = torch.sigmoid(a_vals)
        ga, gb, _ = linear_scan_backward(a, None, out, grad_output.contiguous())
        return ga * a * (1 - a), gb


# --------------------------------------------- scans over host-resident tensors
def _host_ws(device, nbytes):
    """Device workspace for one host-entry call, from torch's caching allocator on
    the current stream: stream-ordered, so concurrent calls on different streams
    never share a ring (a reused block comes back only after its stream is done)."""
    return torch.empty(nbytes, dtype=torch.uint8, device=device)


def _host_train(op, x0, x1, dy, h0, out, device, what):
    for t in (x0, x1, dy, h0):
        if t is not None and (t.is_cuda or not t.is_contiguous()):
            raise _lib.EdbError("%s: inputs must be contiguous host tensors" % what)
    _same(x0.shape, x1.shape, what)
    _same(x0.shape, dy.shape, what)
    B, L, H = x0.shape
    if h0 is not None:
        _same(h0.shape, (B, H), what)
    if out is None:
        out = tuple(torch.empty(x0.shape, dtype=x0.dtype, pin_memory=True) for _ in range(3)) + (
            torch.empty((B, H), dtype=x0.dtype, pin_memory=True),)
    for o in out:
        if o is not None and (o.is_cuda or not o.is_contiguous() or o.dtype != x0.dtype):
            raise _lib.EdbError("%s: outputs must be contiguous host tensors of the input dtype"
                                % what)
    device = torch.device(device if device is not None else "cuda")
    dt_code = _dtype_code(x0, what)
    lib = _lib.load()
    with torch.cuda.device(device):
        nbytes = lib.edb_scan_train_host_workspace(dt_code, B, L, H)
        ws = _host_ws(device, nbytes)
        fn = lib.edb_linear_scan_train_host if op == "linear" else lib.edb_mingru_train_host
        _lib.check(fn(dt_code, _p(x0), _p(x1), _p(h0), _p(dy), _p(out[0]), _p(out[1]),
                      _p(out[2]), _p(out[3]), B, L, H, _p(ws), nbytes, _stream()),
                   "CUDA %s over host tensors" % what)
    return out


def linear_scan_train_host(a_vals, b_vals, grad_output, h0=None, out=None, device=None):
    """Forward and backward of the linear scan for host-resident tensors, copies
    overlapped with the kernels batch-row chunk by chunk.  Returns host tensors
    (h, grad_a, grad_b, grad_h0), written into ``out`` when given (four
    contiguous host tensors; the last may be None).  Asynchronous on the current
    stream of ``device``: synchronise it before reading the results.  Inputs and
    outputs should be pinned for the copies to overlap."""
    return _host_train("linear", a_vals, b_vals, grad_output, h0, out, device,
                       "linear_scan_train_host")


def mingru_train_host(z, candidates, grad_output, h0=None, out=None, device=None):
    """As linear_scan_train_host for MinGRU on post-sigmoid z: returns
    (h, grad_z, grad_cand, grad_h0) on the host."""
    return _host_train("mingru", z, candidates, grad_output, h0, out, device,
                       "mingru_train_host")


# ---------------------------------------------------------------- selective scan
DT_MIN, DT_MAX = 0.001, 0.1  # lib/edifice/ssm/common.ex:58-63


def _ssm_shapes(x, a, b):
    Bsz, L, D = x.shape
    if a.shape[0] != D or tuple(b.shape[:2]) != (Bsz, L) or b.shape[2] != a.shape[1]:
        raise _lib.EdbError("selective_scan: shape mismatch x%s A%s B%s"
                            % (tuple(x.shape), tuple(a.shape), tuple(b.shape)))
    return Bsz, L, D, a.shape[1]


def selective_scan(x, dt, a, b, c, with_ckpt=False):
    """FusedScan.selective_scan/5 (fused_scan.ex:370-384), kernel semantics:
    x, dt [B, L, D]; A [D, N]; B, C [B, L, N] -> y [B, L, D].
    with_ckpt=True also returns the f32 chunk-start states the backward can reuse."""
    _dev(x, dt, a, b, c, what="selective_scan")
    Bsz, L, D, N = _ssm_shapes(x, a, b)
    y = torch.empty_like(x)
    lib = _lib.load()
    ck = None
    if with_ckpt:
        nbytes = lib.edb_selective_scan_ckpt_bytes(Bsz, L, D, N)
        ck = torch.empty(nbytes // 4, dtype=torch.float32, device=x.device)
    _lib.check(lib.edb_selective_scan_fwd(_dtype_code(x, "selective_scan"), _p(x), _p(dt), _p(a),
                                          _p(b), _p(c), _p(y), _p(ck), Bsz, L, D, N, DT_MIN,
                                          DT_MAX, _stream()), "CUDA fused selective scan")
    return (y, ck) if with_ckpt else y


def selective_scan_backward(x, dt, a, b, c, grad_output, h_ckpt=None):
    """Returns (grad_x, grad_dt, grad_B, grad_C); grad_B/grad_C are f32 as in
    selective_scan_backward_dispatch/7 (fused_scan.ex:1433-1450)."""
    _dev(x, dt, a, b, c, grad_output, h_ckpt, what="selective_scan_backward")
    Bsz, L, D, N = _ssm_shapes(x, a, b)
    lib = _lib.load()
    gx, gdt = torch.empty_like(x), torch.empty_like(x)
    gB = torch.empty((Bsz, L, N), dtype=torch.float32, device=x.device)
    gC = torch.empty_like(gB)
    wsb = lib.edb_selective_scan_bwd_workspace(Bsz, L, D, N, int(h_ckpt is not None))
    ws = torch.empty(max(wsb, 16), dtype=torch.uint8, device=x.device)
    _lib.check(lib.edb_selective_scan_bwd(_dtype_code(x, "selective_scan_backward"), _p(x), _p(dt),
                                          _p(a), _p(b), _p(c), _p(grad_output), _p(h_ckpt),
                                          _p(gx), _p(gdt), _p(gB), _p(gC), Bsz, L, D, N, DT_MIN,
                                          DT_MAX, _p(ws), wsb, _stream()),
               "CUDA fused selective scan backward")
    return gx, gdt, gB, gC


def selective_scan_train_host(x, dt, a, b, c, grad_output, out=None, device=None):
    """Forward and backward of the selective scan (kernel semantics) for
    host-resident tensors, the copies overlapped with the kernels batch-row chunk
    by chunk.  Returns host tensors (y, grad_x, grad_dt, grad_B, grad_C), written
    into ``out`` when given (y, grad_x, grad_dt in the input dtype, grad_B and
    grad_C f32).  Asynchronous on the current stream of ``device``: synchronise it
    before reading the results.  Inputs and outputs should be pinned for the
    copies to overlap."""
    what = "selective_scan_train_host"
    for t in (x, dt, a, b, c, grad_output):
        if t.is_cuda or not t.is_contiguous():
            raise _lib.EdbError("%s: inputs must be contiguous host tensors" % what)
    Bsz, L, D, N = _ssm_shapes(x, a, b)
    _same(x.shape, dt.shape, what)
    _same(x.shape, grad_output.shape, what)
    _same(b.shape, c.shape, what)
    if out is None:
        out = tuple(torch.empty(x.shape, dtype=x.dtype, pin_memory=True) for _ in range(3)) + \
            tuple(torch.empty((Bsz, L, N), dtype=torch.float32, pin_memory=True)
                  for _ in range(2))
    dts = (x.dtype,) * 3 + (torch.float32,) * 2
    for o, want in zip(out, dts):
        if o.is_cuda or not o.is_contiguous() or o.dtype != want:
            raise _lib.EdbError("%s: outputs must be contiguous host tensors (y, gx, gdt in "
                                "the input dtype, gB, gC f32)" % what)
    device = torch.device(device if device is not None else "cuda")
    dt_code = _dtype_code(x, what)
    lib = _lib.load()
    with torch.cuda.device(device):
        nbytes = lib.edb_selective_scan_train_host_workspace(dt_code, Bsz, L, D, N)
        ws = _host_ws(device, nbytes)
        _lib.check(lib.edb_selective_scan_train_host(
            dt_code, _p(x), _p(dt), _p(a), _p(b), _p(c), _p(grad_output), _p(out[0]),
            _p(out[1]), _p(out[2]), _p(out[3]), _p(out[4]), Bsz, L, D, N, DT_MIN, DT_MAX,
            _p(ws), nbytes, _stream()), "CUDA fused selective scan over host tensors")
    return out


def selective_scan_model_train_host(x, dt, b, c, grad_output, a=None, out=None,
                                    device=None):
    """Forward and backward of the model semantics (selective_scan_model) for
    host-resident tensors, as selective_scan_train_host: batch-row chunks with the
    copies overlapped with the kernels; ``a`` None is the model's fixed -(1..N)
    diagonal.  Returns host tensors (y, grad_x, grad_dt, grad_B, grad_C)."""
    what = "selective_scan_model_train_host"
    for t in (x, dt, a, b, c, grad_output):
        if t is not None and (t.is_cuda or not t.is_contiguous()):
            raise _lib.EdbError("%s: inputs must be contiguous host tensors" % what)
    Bsz, L, D, N = _model_shapes(x, a, b)
    _same(x.shape, dt.shape, what)
    _same(x.shape, grad_output.shape, what)
    _same(b.shape, c.shape, what)
    if out is None:
        out = tuple(torch.empty(x.shape, dtype=x.dtype, pin_memory=True) for _ in range(3)) + \
            tuple(torch.empty((Bsz, L, N), dtype=torch.float32, pin_memory=True)
                  for _ in range(2))
    dts = (x.dtype,) * 3 + (torch.float32,) * 2
    for o, want in zip(out, dts):
        if o.is_cuda or not o.is_contiguous() or o.dtype != want:
            raise _lib.EdbError("%s: outputs must be contiguous host tensors (y, gx, gdt in "
                                "the input dtype, gB, gC f32)" % what)
    device = torch.device(device if device is not None else "cuda")
    code = _dtype_code(x, what)
    lib = _lib.load()
    with torch.cuda.device(device):
        nbytes = lib.edb_selective_scan_model_train_host_workspace(code, Bsz, L, D, N)
        ws = _host_ws(device, nbytes)
        _lib.check(lib.edb_selective_scan_model_train_host(
            code, _p(x), _p(dt), _p(a), _p(b), _p(c), _p(grad_output), _p(out[0]), _p(out[1]),
            _p(out[2]), _p(out[3]), _p(out[4]), Bsz, L, D, N, DT_MIN, DT_MAX, _p(ws), nbytes,
            _stream()), "CUDA selective scan (model semantics) over host tensors")
    return out


def _model_shapes(x, a, b):
    Bsz, L, D = x.shape
    N = b.shape[2]
    if tuple(b.shape[:2]) != (Bsz, L) or (a is not None and tuple(a.shape) != (D, N)):
        raise _lib.EdbError("selective_scan_model: shape mismatch x%s B%s A%s"
                            % (tuple(x.shape), tuple(b.shape),
                               None if a is None else tuple(a.shape)))
    return Bsz, L, D, N


def selective_scan_model(x, dt, b, c, a=None, with_ckpt=False):
    """Model semantics of Edifice.build(:mamba): Common.selective_scan_fallback/5
    (lib/edifice/ssm/common.ex:661-670 -> discretize_ssm :402-444): B_bar is the
    channel mean of the clamped dt times B, A the fixed -(1..N) diagonal when
    ``a`` is None (common.ex:409; Mamba.parallel_scan_ssm_impl builds the same
    matrix, mamba.ex:187-193).  Returns (y, dt_mean) or (y, dt_mean, h_ckpt);
    dt_mean [B, L] f32 is what the backward needs."""
    _dev(x, dt, a, b, c, what="selective_scan_model")
    Bsz, L, D, N = _model_shapes(x, a, b)
    y = torch.empty_like(x)
    dtm = torch.empty((Bsz, L), dtype=torch.float32, device=x.device)
    lib = _lib.load()
    ck = None
    if with_ckpt:
        nbytes = lib.edb_selective_scan_ckpt_bytes(Bsz, L, D, N)
        ck = torch.empty(nbytes // 4, dtype=torch.float32, device=x.device)
    _lib.check(lib.edb_selective_scan_model_fwd(_dtype_code(x, "selective_scan_model"), _p(x),
                                                _p(dt), _p(a), _p(b), _p(c), _p(y), _p(dtm),
                                                _p(ck), Bsz, L, D, N, DT_MIN, DT_MAX, _stream()),
               "CUDA fused selective scan (model semantics)")
    return (y, dtm, ck) if with_ckpt else (y, dtm)


def selective_scan_model_backward(x, dt, b, c, grad_output, dt_mean, a=None, h_ckpt=None):
    """Returns (grad_x, grad_dt, grad_B, grad_C) of selective_scan_model;
    grad_B/grad_C f32, A gets none."""
    _dev(x, dt, a, b, c, grad_output, dt_mean, h_ckpt, what="selective_scan_model_backward")
    Bsz, L, D, N = _model_shapes(x, a, b)
    lib = _lib.load()
    gx, gdt = torch.empty_like(x), torch.empty_like(x)
    gB = torch.empty((Bsz, L, N), dtype=torch.float32, device=x.device)
    gC = torch.empty_like(gB)
    wsb = lib.edb_selective_scan_bwd_workspace(Bsz, L, D, N, int(h_ckpt is not None))
    ws = torch.empty(max(wsb, 16), dtype=torch.uint8, device=x.device)
    _lib.check(lib.edb_selective_scan_model_bwd(
        _dtype_code(x, "selective_scan_model_backward"), _p(x), _p(dt), _p(a), _p(b), _p(c),
        _p(grad_output), _p(dt_mean), _p(h_ckpt), _p(gx), _p(gdt), _p(gB), _p(gC), Bsz, L, D, N,
        DT_MIN, DT_MAX, _p(ws), wsb, _stream()),
        "CUDA fused selective scan backward (model semantics)")
    return gx, gdt, gB, gC


class SelectiveScanModelFn(torch.autograd.Function):
    """The Mamba layer's SSM core with gradients to x, dt, B and C (A is the
    fixed diagonal, as Edifice.build(:mamba) uses it)."""

    @staticmethod
    def forward(ctx, x, dt, b, c):
        y, dtm, ck = selective_scan_model(x, dt, b, c, with_ckpt=True)
        ctx.save_for_backward(x, dt, b, c, dtm, ck)
        return y

    @staticmethod
    def backward(ctx, grad_output):
        x, dt, b, c, dtm, ck = ctx.saved_tensors
        return selective_scan_model_backward(x, dt, b, c, grad_output.contiguous(), dtm,
                                             h_ckpt=ck)


def _delta_shapes(q, k, v, beta):
    if q.dim() != 4 or q.shape != k.shape or q.shape != v.shape:
        raise _lib.EdbError("delta_net_scan: q, k, v must share one [B, L, H, d] shape")
    B, L, H, d = q.shape
    if tuple(beta.shape) == (B, L, H, d):
        return B, L, H, d, 1
    if tuple(beta.shape) == (B, L, H):
        return B, L, H, d, 0
    raise _lib.EdbError("delta_net_scan: beta must be [B, L, H, d] or [B, L, H], got %s"
                        % (tuple(beta.shape),))


def delta_net_scan(q, k, v, beta, with_ckpt=False):
    """FusedScan.delta_net_scan/4 (fused_scan.ex:195-209): q, k (L2-normalised),
    v [B, L, H, d]; beta (post-sigmoid) [B, L, H, d] or [B, L, H] -> o [B, L, H, d].
    with_ckpt=True also returns the f32 chunk-start states the backward can reuse."""
    _dev(q, k, v, beta, what="delta_net_scan")
    B, L, H, d, per_el = _delta_shapes(q, k, v, beta)
    o = torch.empty_like(q)
    lib = _lib.load()
    dt = _dtype_code(q, "delta_net_scan")
    ck = None
    if with_ckpt:
        ck = torch.empty(lib.edb_delta_rule_ckpt_bytes(dt, per_el, B, L, H, d) // 4,
                         dtype=torch.float32, device=q.device)
    wsb = lib.edb_delta_rule_fwd_workspace(dt, per_el, B, L, H, d)
    ws = torch.empty(wsb, dtype=torch.uint8, device=q.device) if wsb else None
    _lib.check(lib.edb_delta_rule_fwd(dt, _p(q), _p(k), _p(v), _p(beta), per_el, _p(o), _p(ck),
                                      B, L, H, d, _p(ws), wsb, _stream()),
               "CUDA fused DeltaNet scan")
    return (o, ck) if with_ckpt else o


def delta_rule_backward(q, k, v, beta, grad_output, s_ckpt=None):
    """Returns (grad_q, grad_k, grad_v, grad_beta).  Mirrors
    delta_rule_backward_dispatch/6 (fused_scan.ex:1241-1255)."""
    _dev(q, k, v, beta, grad_output, s_ckpt, what="delta_rule_backward")
    B, L, H, d, per_el = _delta_shapes(q, k, v, beta)
    lib = _lib.load()
    gq, gk, gv, gb = (torch.empty_like(q), torch.empty_like(k), torch.empty_like(v),
                      torch.empty_like(beta))
    dt = _dtype_code(q, "delta_rule_backward")
    wsb = lib.edb_delta_rule_bwd_workspace(dt, per_el, B, L, H, d, int(s_ckpt is not None))
    ws = torch.empty(max(wsb, 16), dtype=torch.uint8, device=q.device)
    _lib.check(lib.edb_delta_rule_bwd(dt, _p(q), _p(k), _p(v),
                                      _p(beta), per_el, _p(grad_output), _p(s_ckpt), _p(gq),
                                      _p(gk), _p(gv), _p(gb), B, L, H, d, _p(ws), wsb, _stream()),
               "CUDA fused DeltaNet scan backward")
    return gq, gk, gv, gb


class DeltaNetFn(torch.autograd.Function):
    """custom_grad wiring of delta_net_custom_call/4 (fused_scan.ex:2195-2210):
    gradients to q, k, v, beta."""

    @staticmethod
    def forward(ctx, q, k, v, beta):
        o, ck = delta_net_scan(q, k, v, beta, with_ckpt=True)
        ctx.save_for_backward(q, k, v, beta, ck)
        return o

    @staticmethod
    def backward(ctx, grad_output):
        q, k, v, beta, ck = ctx.saved_tensors
        return delta_rule_backward(q, k, v, beta, grad_output.contiguous(), ck)


def _delta_host(q, k, v, beta, alpha, grad_output, out, device):
    """Shared body of delta_rule_train_host / gated_delta_net_train_host."""
    gated = alpha is not None
    what = "gated_delta_net_train_host" if gated else "delta_rule_train_host"
    for t in (q, k, v, beta, alpha, grad_output):
        if t is not None and (t.is_cuda or not t.is_contiguous()):
            raise _lib.EdbError("%s: inputs must be contiguous host tensors" % what)
    B, L, H, d, per_el = _gated_shapes(q, k, v, beta, alpha) if gated else \
        _delta_shapes(q, k, v, beta)
    _same(q.shape, grad_output.shape, what)
    want = [q, q, k, v, beta] + ([alpha] if gated else [])
    if out is None:
        out = tuple(torch.empty(t.shape, dtype=t.dtype, pin_memory=True) for t in want)
    if len(out) != len(want):
        raise _lib.EdbError("%s: expected %d outputs" % (what, len(want)))
    for o_, t in zip(out, want):
        if o_.is_cuda or not o_.is_contiguous() or o_.shape != t.shape or o_.dtype != t.dtype:
            raise _lib.EdbError("%s: outputs must be contiguous host tensors shaped like "
                                "(q, q, k, v, beta%s)" % (what, ", alpha" if gated else ""))
    device = torch.device(device if device is not None else "cuda")
    code = _dtype_code(q, what)
    lib = _lib.load()
    with torch.cuda.device(device):
        if gated:
            nbytes = lib.edb_gated_delta_net_train_host_workspace(code, per_el, B, L, H, d)
            ws = _host_ws(device, nbytes)
            st = lib.edb_gated_delta_net_train_host(
                code, _p(q), _p(k), _p(v), _p(beta), per_el, _p(alpha), _p(grad_output),
                _p(out[0]), _p(out[1]), _p(out[2]), _p(out[3]), _p(out[4]), _p(out[5]), B, L,
                H, d, _p(ws), nbytes, _stream())
        else:
            nbytes = lib.edb_delta_rule_train_host_workspace(code, per_el, B, L, H, d)
            ws = _host_ws(device, nbytes)
            st = lib.edb_delta_rule_train_host(
                code, _p(q), _p(k), _p(v), _p(beta), per_el, _p(grad_output), _p(out[0]),
                _p(out[1]), _p(out[2]), _p(out[3]), _p(out[4]), B, L, H, d, _p(ws), nbytes,
                _stream())
        _lib.check(st, "CUDA %s over host tensors" % what)
    return out


def delta_rule_train_host(q, k, v, beta, grad_output, out=None, device=None):
    """Forward and backward of the delta rule (DeltaNet) for host-resident q, k, v,
    beta and grad_output: batch-row chunks stream through the device with the copies
    overlapped with the kernels.  Returns host tensors (o, grad_q, grad_k, grad_v,
    grad_beta), written into ``out`` when given.  Asynchronous on the current stream
    of ``device``: synchronise it before reading the results."""
    return _delta_host(q, k, v, beta, None, grad_output, out, device)


def gated_delta_net_train_host(q, k, v, beta, alpha, grad_output, out=None, device=None):
    """GatedDeltaNet over host tensors, as delta_rule_train_host; returns
    (o, grad_q, grad_k, grad_v, grad_beta, grad_alpha)."""
    return _delta_host(q, k, v, beta, alpha, grad_output, out, device)


def _gated_shapes(q, k, v, beta, alpha):
    B, L, H, d, per_el = _delta_shapes(q, k, v, beta)
    if tuple(alpha.shape) != (B, L, H) or alpha.dtype != q.dtype:
        raise _lib.EdbError("gated_delta_net: alpha must be [B, L, H] of the q dtype, got %s %s"
                            % (tuple(alpha.shape), alpha.dtype))
    return B, L, H, d, per_el


def gated_delta_net_scan(q, k, v, beta, alpha, with_ckpt=False):
    """FusedScan.gated_delta_net_scan/5 (fused_scan.ex:219-233): q, k (L2-normalised),
    v [B, L, H, d]; beta (post-sigmoid) [B, L, H, d] or [B, L, H]; alpha (decay)
    [B, L, H] -> o [B, L, H, d].  with_ckpt=True also returns the f32 residuals the
    backward can reuse (the chunk-start states; for the chunked form, bf16 with a
    per-token beta and d = 128, transposed and followed by the chunk errors)."""
    _dev(q, k, v, beta, alpha, what="gated_delta_net_scan")
    B, L, H, d, per_el = _gated_shapes(q, k, v, beta, alpha)
    o = torch.empty_like(q)
    lib = _lib.load()
    dt = _dtype_code(q, "gated_delta_net_scan")
    ck = None
    if with_ckpt:
        ck = torch.empty(lib.edb_gated_delta_net_ckpt_bytes(dt, per_el, B, L, H, d) // 4,
                         dtype=torch.float32, device=q.device)
    # the chunked tensor-core form (bf16, one beta per token, d = 128) takes a workspace
    wsb = lib.edb_gated_delta_net_fwd_workspace(dt, per_el, B, L, H, d)
    ws = torch.empty(wsb, dtype=torch.uint8, device=q.device) if wsb else None
    _lib.check(lib.edb_gated_delta_net_fwd_ws(dt, _p(q), _p(k), _p(v), _p(beta), per_el,
                                              _p(alpha), _p(o), _p(ck), B, L, H, d, _p(ws), wsb,
                                              _stream()),
               "CUDA fused GatedDeltaNet scan")
    return (o, ck) if with_ckpt else o


def gated_delta_net_backward(q, k, v, beta, alpha, grad_output, s_ckpt=None):
    """Returns (grad_q, grad_k, grad_v, grad_beta, grad_alpha).  Mirrors
    gated_delta_net_backward_dispatch/7 (fused_scan.ex:1330-1345)."""
    _dev(q, k, v, beta, alpha, grad_output, s_ckpt, what="gated_delta_net_backward")
    B, L, H, d, per_el = _gated_shapes(q, k, v, beta, alpha)
    lib = _lib.load()
    gq, gk, gv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    gb, ga = torch.empty_like(beta), torch.empty_like(alpha)
    dt = _dtype_code(q, "gated_delta_net_backward")
    wsb = lib.edb_gated_delta_net_bwd_workspace(dt, per_el, B, L, H, d, int(s_ckpt is not None))
    ws = torch.empty(max(wsb, 16), dtype=torch.uint8, device=q.device)
    _lib.check(lib.edb_gated_delta_net_bwd(dt, _p(q), _p(k), _p(v), _p(beta), per_el, _p(alpha),
                                           _p(grad_output), _p(s_ckpt), _p(gq), _p(gk), _p(gv),
                                           _p(gb), _p(ga), B, L, H, d, _p(ws), wsb, _stream()),
               "CUDA fused GatedDeltaNet scan backward")
    return gq, gk, gv, gb, ga


class GatedDeltaNetFn(torch.autograd.Function):
    """custom_grad wiring of gated_delta_net_custom_call/5 (fused_scan.ex:2239-2254):
    gradients to q, k, v, beta, alpha."""

    @staticmethod
    def forward(ctx, q, k, v, beta, alpha):
        o, ck = gated_delta_net_scan(q, k, v, beta, alpha, with_ckpt=True)
        ctx.save_for_backward(q, k, v, beta, alpha, ck)
        return o

    @staticmethod
    def backward(ctx, grad_output):
        q, k, v, beta, alpha, ck = ctx.saved_tensors
        return gated_delta_net_backward(q, k, v, beta, alpha, grad_output.contiguous(), ck)


def _attn_shapes(q, k, v):
    if q.dim() != 4 or k.dim() != 4 or k.shape != v.shape:
        raise _lib.EdbError("flash_attention: expected [B, H, L, d] q and equal k/v shapes")
    B, Hq, L, d = q.shape
    if k.shape[0] != B or k.shape[2] != L or k.shape[3] != d or Hq % k.shape[1] != 0:
        raise _lib.EdbError("flash_attention: q %s incompatible with k/v %s"
                            % (tuple(q.shape), tuple(k.shape)))
    return B, Hq, k.shape[1], L, d


def flash_attention(q, k, v, causal=False, scale=None, return_lse=False):
    """FusedScan.flash_attention/4 (fused_scan.ex:3398-3414) with GQA:
    q [B, Hq, L, d], k/v [B, Hkv, L, d] -> o [B, Hq, L, d].  `causal` masks
    j > i; scale defaults to 1/sqrt(d).  return_lse adds the f32 [B, Hq, L]
    row log-sum-exp the backward can reuse."""
    _dev(q, k, v, what="flash_attention")
    B, Hq, Hkv, L, d = _attn_shapes(q, k, v)
    o = torch.empty_like(q)
    lse = torch.empty((B, Hq, L), dtype=torch.float32, device=q.device) if return_lse else None
    lib = _lib.load()
    _lib.check(lib.edb_flash_attention_fwd(_dtype_code(q, "flash_attention"), _p(q), _p(k), _p(v),
                                           _p(o), _p(lse), B, Hq, Hkv, L, d, int(bool(causal)),
                                           float(scale or 0.0), _stream()),
               "CUDA flash attention")
    return (o, lse) if return_lse else o


def flash_attention_backward(q, k, v, causal, forward_out, grad_output, lse=None, scale=None):
    """Returns (grad_q, grad_k, grad_v).  Mirrors flash_attention_backward_dispatch/6
    (fused_scan.ex:3510-3525); lse (from flash_attention(return_lse=True)) is
    optional and recomputed when absent."""
    _dev(q, k, v, forward_out, grad_output, lse, what="flash_attention_backward")
    B, Hq, Hkv, L, d = _attn_shapes(q, k, v)
    lib = _lib.load()
    code = _dtype_code(q, "flash_attention_backward")
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    wsb = lib.edb_flash_attention_bwd_workspace(code, B, Hq, Hkv, L, d, int(lse is not None))
    ws = torch.empty(max(wsb, 16), dtype=torch.uint8, device=q.device)
    _lib.check(lib.edb_flash_attention_bwd(code, _p(q), _p(k), _p(v), _p(forward_out),
                                           _p(grad_output), _p(lse), _p(dq), _p(dk), _p(dv), B,
                                           Hq, Hkv, L, d, int(bool(causal)), float(scale or 0.0),
                                           _p(ws), wsb, _stream()),
               "CUDA flash attention backward")
    return dq, dk, dv


def _attn_host(kind, q, k, v, cs, grad_output, causal, scale, out, device):
    """Shared body of the three host-tensor attention entry points (kind: "flash",
    "fox", "laser")."""
    what = "%s_attention_train_host" % kind
    for t in (q, k, v, cs, grad_output):
        if t is not None and (t.is_cuda or not t.is_contiguous()):
            raise _lib.EdbError("%s: inputs must be contiguous host tensors" % what)
    B, Hq, Hkv, L, d = _attn_shapes(q, k, v)
    _same(q.shape, grad_output.shape, what)
    fox = kind == "fox"
    if fox and (cs is None or tuple(cs.shape) != (B, Hq, L) or cs.dtype != torch.float32):
        raise _lib.EdbError("%s: cs must be f32 [B, Hq, L]" % what)
    want = [(q.shape, q.dtype), (q.shape, q.dtype), (k.shape, k.dtype), (v.shape, v.dtype)]
    if fox:
        want.append((cs.shape, torch.float32))
    if out is None:
        out = tuple(torch.empty(sh, dtype=dt, pin_memory=True) for sh, dt in want)
    if len(out) != len(want):
        raise _lib.EdbError("%s: expected %d outputs" % (what, len(want)))
    for o_, (sh, dt) in zip(out, want):
        if o_.is_cuda or not o_.is_contiguous() or o_.shape != sh or o_.dtype != dt:
            raise _lib.EdbError("%s: outputs must be contiguous host tensors shaped like "
                                "(q, q, k, v%s)" % (what, ", cs" if fox else ""))
    device = torch.device(device if device is not None else "cuda")
    code = _dtype_code(q, what)
    lib = _lib.load()
    sc = float(scale or 0.0)
    with torch.cuda.device(device):
        nbytes = getattr(lib, "edb_%s_attention_train_host_workspace" % kind)(code, B, Hq, Hkv,
                                                                              L, d)
        ws = _host_ws(device, nbytes)
        if fox:
            st = lib.edb_fox_attention_train_host(
                code, _p(q), _p(k), _p(v), _p(cs), _p(grad_output), _p(out[0]), _p(out[1]),
                _p(out[2]), _p(out[3]), _p(out[4]), B, Hq, Hkv, L, d, sc, _p(ws), nbytes,
                _stream())
        else:
            st = getattr(lib, "edb_%s_attention_train_host" % kind)(
                code, _p(q), _p(k), _p(v), _p(grad_output), _p(out[0]), _p(out[1]), _p(out[2]),
                _p(out[3]), B, Hq, Hkv, L, d, int(bool(causal)), sc, _p(ws), nbytes, _stream())
        _lib.check(st, "CUDA %s attention over host tensors" % kind)
    return out


def flash_attention_train_host(q, k, v, grad_output, causal=True, scale=None, out=None,
                               device=None):
    """Forward and backward of flash attention for host-resident q, k, v [B, Hq, L, d] /
    [B, Hkv, L, d] and grad_output [B, Hq, L, d]: (batch, kv head) units stream through
    the device with their copies overlapped with the kernels.  Returns host tensors
    (o, grad_q, grad_k, grad_v), written into ``out`` when given.  Asynchronous on the
    current stream of ``device``: synchronise it before reading the results.  Inputs
    and outputs should be pinned for the copies to overlap."""
    return _attn_host("flash", q, k, v, None, grad_output, causal, scale, out, device)


def laser_attention_train_host(q, k, v, grad_output, causal=True, scale=None, out=None,
                               device=None):
    """LASER attention over host tensors, as flash_attention_train_host: returns
    (o, grad_q, grad_k, grad_v) (v_max computed per (batch, kv head))."""
    return _attn_host("laser", q, k, v, None, grad_output, causal, scale, out, device)


def fox_attention_train_host(q, k, v, cs, grad_output, scale=None, out=None, device=None):
    """FoX attention over host tensors, as flash_attention_train_host; cs f32
    [B, Hq, L].  Returns (o, grad_q, grad_k, grad_v, grad_cs)."""
    return _attn_host("fox", q, k, v, cs, grad_output, True, scale, out, device)


class FlashAttentionFn(torch.autograd.Function):
    """custom_grad wiring of flash_attention_custom_call/4 (fused_scan.ex:3427-3443):
    gradients to q, k, v."""

    @staticmethod
    def forward(ctx, q, k, v, causal=False):
        o, lse = flash_attention(q, k, v, causal=causal, return_lse=True)
        ctx.causal = causal
        ctx.save_for_backward(q, k, v, o, lse)
        return o

    @staticmethod
    def backward(ctx, grad_output):
        q, k, v, o, lse = ctx.saved_tensors
        dq, dk, dv = flash_attention_backward(q, k, v, ctx.causal, o, grad_output.contiguous(), lse)
        return dq, dk, dv, None


# --------------------------------------------------------------- LASER attention
def laser_attention(q, k, v, causal=True, v_max=None, scale=None, return_resid=False):
    """FusedScan.laser_attention/4 (fused_scan.ex:3593-3611): attention over
    exp(V - v_max), O = log(max(A, 1e-7)) + v_max, with v_max the max over the
    sequence of v (computed when None, else [B, Hkv, d] as the reference passes it).
    q [B, Hq, L, d], k / v [B, Hkv, L, d].  return_resid adds the buffer
    laser_attention_backward reads."""
    _dev(q, k, v, v_max, what="laser_attention")
    B, Hq, Hkv, L, d = _attn_shapes(q, k, v)
    code = _dtype_code(q, "laser_attention")
    lib = _lib.load()
    o = torch.empty_like(q)
    resid = torch.empty(lib.edb_laser_attention_resid_bytes(code, B, Hq, Hkv, L, d),
                        dtype=torch.uint8, device=q.device)
    _lib.check(lib.edb_laser_attention_fwd(code, _p(q), _p(k), _p(v), _p(v_max), _p(o),
                                           _p(resid), B, Hq, Hkv, L, d, int(bool(causal)),
                                           float(scale or 0.0), _stream()),
               "CUDA LASER attention")
    return (o, resid) if return_resid else o


def laser_attention_backward(q, k, v, grad_output, resid, causal=True, scale=None):
    """Returns (grad_q, grad_k, grad_v) of laser_attention from its resid; mirrors
    laser_attention_backward_dispatch (fused_scan.ex:3705-3721, 3723-3766)."""
    _dev(q, k, v, grad_output, resid, what="laser_attention_backward")
    B, Hq, Hkv, L, d = _attn_shapes(q, k, v)
    code = _dtype_code(q, "laser_attention_backward")
    lib = _lib.load()
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    wsb = lib.edb_laser_attention_bwd_workspace(code, B, Hq, Hkv, L, d)
    ws = torch.empty(wsb, dtype=torch.uint8, device=q.device)
    _lib.check(lib.edb_laser_attention_bwd(code, _p(q), _p(k), _p(grad_output), _p(resid),
                                           _p(dq), _p(dk), _p(dv), B, Hq, Hkv, L, d,
                                           int(bool(causal)), float(scale or 0.0), _p(ws), wsb,
                                           _stream()),
               "CUDA LASER attention backward")
    return dq, dk, dv


class LaserAttentionFn(torch.autograd.Function):
    """custom_grad wiring of laser_attention_custom_call (fused_scan.ex:3615-3633):
    gradients to q, k, v (v_max held constant)."""

    @staticmethod
    def forward(ctx, q, k, v, causal=True):
        o, resid = laser_attention(q, k, v, causal=causal, return_resid=True)
        ctx.causal = causal
        ctx.save_for_backward(q, k, v, resid)
        return o

    @staticmethod
    def backward(ctx, grad_output):
        q, k, v, resid = ctx.saved_tensors
        dq, dk, dv = laser_attention_backward(q, k, v, grad_output.contiguous(), resid,
                                              causal=ctx.causal)
        return dq, dk, dv, None


# ----------------------------------------------------------------- FoX attention
def fox_attention(q, k, v, cs, scale=None, return_lse=False):
    """FusedScan.fox_attention/4 (fused_scan.ex:3796-3861): causal attention with
    the forget bias cs_i - cs_j, cs [B, Hq, L] the cumulative log forget gates (f32).
    q [B, Hq, L, d], k / v [B, Hkv, L, d].  return_lse adds the f32 row
    log-sum-exp (without the row's own cs_i) the backward reads."""
    _dev(q, k, v, cs, what="fox_attention")
    B, Hq, Hkv, L, d = _attn_shapes(q, k, v)
    if cs.dtype != torch.float32 or tuple(cs.shape) != (B, Hq, L):
        raise _lib.EdbError("fox_attention: cs must be f32 [B, Hq, L]")
    o = torch.empty_like(q)
    lse = torch.empty((B, Hq, L), dtype=torch.float32, device=q.device)
    lib = _lib.load()
    _lib.check(lib.edb_fox_attention_fwd(_dtype_code(q, "fox_attention"), _p(q), _p(k), _p(v),
                                         _p(cs), _p(o), _p(lse), B, Hq, Hkv, L, d,
                                         float(scale or 0.0), _stream()),
               "CUDA FoX attention")
    return (o, lse) if return_lse else o


def fox_attention_backward(q, k, v, cs, forward_out, grad_output, lse, scale=None):
    """Returns (grad_q, grad_k, grad_v, grad_cs) as fox_attention_backward_dispatch
    (fused_scan.ex:3914-3924); grad_cs f32."""
    _dev(q, k, v, cs, forward_out, grad_output, lse, what="fox_attention_backward")
    B, Hq, Hkv, L, d = _attn_shapes(q, k, v)
    code = _dtype_code(q, "fox_attention_backward")
    lib = _lib.load()
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    dcs = torch.empty((B, Hq, L), dtype=torch.float32, device=q.device)
    wsb = lib.edb_fox_attention_bwd_workspace(code, B, Hq, Hkv, L, d)
    ws = torch.empty(wsb, dtype=torch.uint8, device=q.device)
    _lib.check(lib.edb_fox_attention_bwd(code, _p(q), _p(k), _p(v), _p(cs), _p(forward_out),
                                         _p(grad_output), _p(lse), _p(dq), _p(dk), _p(dv),
                                         _p(dcs), B, Hq, Hkv, L, d, float(scale or 0.0), _p(ws),
                                         wsb, _stream()),
               "CUDA FoX attention backward")
    return dq, dk, dv, dcs


class FoxAttentionFn(torch.autograd.Function):
    """custom_grad wiring of fox_attention_custom_call (fused_scan.ex:3796-3861):
    gradients to q, k, v and cs."""

    @staticmethod
    def forward(ctx, q, k, v, cs):
        o, lse = fox_attention(q, k, v, cs, return_lse=True)
        ctx.save_for_backward(q, k, v, cs, o, lse)
        return o

    @staticmethod
    def backward(ctx, grad_output):
        q, k, v, cs, o, lse = ctx.saved_tensors
        return fox_attention_backward(q, k, v, cs, o, grad_output.contiguous(), lse)


# ------------------------------------------- attention callers routed to flash
def _attend(q, k, v, causal):
    """[B, H, L, d] attention through the flash kernel, with gradients when any
    input requires them."""
    if torch.is_grad_enabled() and any(t.requires_grad for t in (q, k, v)):
        return FlashAttentionFn.apply(q, k, v, causal)
    return flash_attention(q, k, v, causal=causal)


def sdpa_compute(q, k, v, num_heads, head_dim, causal=False, num_kv_heads=None):
    """Blocks.SDPA.compute/6 (lib/edifice/blocks/sdpa.ex:74-118) on the flash
    kernel: q [B, L, num_heads * head_dim], k / v [B, L, num_kv_heads * head_dim]
    (num_kv_heads defaults to num_heads) -> [B, L, num_heads * head_dim].  The
    reference takes this branch for self-attention (equal lengths) and passes
    causal = (mask != nil); K/V heads are grouped natively, never repeated."""
    B, L, _ = q.shape
    hkv = num_kv_heads or num_heads
    if k.shape[1] != L or v.shape[1] != L:
        raise _lib.EdbError("sdpa_compute: the flash path takes self-attention "
                            "(equal query and key lengths)")
    qh = q.reshape(B, L, num_heads, head_dim).transpose(1, 2).contiguous()
    kh = k.reshape(B, L, hkv, head_dim).transpose(1, 2).contiguous()
    vh = v.reshape(B, L, hkv, head_dim).transpose(1, 2).contiguous()
    o = _attend(qh, kh, vh, causal)
    return o.transpose(1, 2).reshape(B, L, num_heads * head_dim)


def gqa_attention(q, k, v, num_heads, num_kv_heads, head_dim):
    """GQA.gqa_attention_impl (lib/edifice/attention/gqa.ex:192-306, rope / yarn
    off): causal grouped-query attention.  The reference repeats K/V to
    num_heads and masks with -1e9; the kernel reads each K/V head once per group
    and masks with -inf, which is identical here because every causal row keeps
    its diagonal."""
    if num_heads % num_kv_heads:
        raise _lib.EdbError("gqa_attention: num_heads must be a multiple of num_kv_heads")
    return sdpa_compute(q, k, v, num_heads, head_dim, causal=True, num_kv_heads=num_kv_heads)


def multi_head_sdpa(query, key, value, mask=None):
    """Primitives.multi_head_sdpa/4 (lib/edifice/attention/primitives.ex:307-341):
    [B, H, L, d] in and out.  mask None is full attention; a [L, L] (or
    broadcastable [B, H, L, L]) boolean mask equal to the causal lower triangle
    runs the causal kernel (the reference's -1e9 fill equals -inf there).  Any
    other mask has no kernel on this path and raises."""
    causal = False
    if mask is not None:
        L = query.shape[2]
        tri = torch.ones(L, L, dtype=torch.bool, device=mask.device).tril()
        if not bool((mask.bool() == tri).all()):
            raise _lib.EdbError("multi_head_sdpa: only a causal mask runs on the flash path")
        causal = True
    return _attend(query.contiguous(), key.contiguous(), value.contiguous(), causal)


class SelectiveScanFn(torch.autograd.Function):
    """custom_grad wiring of selective_scan_custom_call/5 (fused_scan.ex:2595-2611):
    gradients to x, dt, B, C; A gets none."""

    @staticmethod
    def forward(ctx, x, dt, a, b, c):
        y, ck = selective_scan(x, dt, a, b, c, with_ckpt=True)
        ctx.save_for_backward(x, dt, a, b, c, ck)
        return y

    @staticmethod
    def backward(ctx, grad_output):
        x, dt, a, b, c, ck = ctx.saved_tensors
        gx, gdt, gB, gC = selective_scan_backward(x, dt, a, b, c, grad_output.contiguous(), ck)
        return gx, gdt, None, gB.to(b.dtype), gC.to(c.dtype)
