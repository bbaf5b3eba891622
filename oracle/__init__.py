"""CPU oracle for the fused sequence-mixing path -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference
arm import this package, and only as the checker (or the timed CPU baseline).
The product library never routes through it.

Every function takes numpy arrays (any float dtype; they are widened to f32,
which is exact for bf16-rounded values) and returns f32 numpy arrays.
``prec="f64"`` (default) is the parity oracle with f64 accumulation;
``prec="f32"`` is the Nx-like f32 arithmetic used for the timed CPU baseline.

Reference citations (edifice project paths) live beside each C function in
oracle_body.h.
"""
import ctypes
import os

import numpy as np

from . import build as _build

_lib = None
_ref_cpu = None

_F = ctypes.POINTER(ctypes.c_float)
_I = ctypes.c_int


def lib():
    global _lib
    if _lib is None:
        path = _build.ORACLE_SO
        if not os.path.exists(path):
            _build.build_oracle()
        _lib = ctypes.CDLL(path)
    return _lib


def ref_cpu_lib():
    """The reference's own CPU references (oracle/_ref), or None when absent."""
    global _ref_cpu
    if _ref_cpu is None and os.path.exists(_build.REF_CPU_SO):
        _ref_cpu = ctypes.CDLL(_build.REF_CPU_SO)
    return _ref_cpu


def set_threads(n):
    lib().orc_set_num_threads(int(n))


def num_threads():
    return int(lib().orc_num_threads())


def _f32(x):
    return np.ascontiguousarray(np.asarray(x, dtype=np.float32))


def _p(x):
    return None if x is None else x.ctypes.data_as(_F)


def _fn(name, prec):
    return getattr(lib(), "orc_%s_%s" % (name, prec))


# ----------------------------------------------------------------- scans
def linear_scan_fwd(a, b, h0=None, prec="f64"):
    a, b = _f32(a), _f32(b)
    B, L, H = a.shape
    h0 = None if h0 is None else _f32(h0)
    out = np.empty_like(a)
    _fn("linear_scan_fwd", prec)(_p(a), _p(b), _p(h0), _p(out), _I(B), _I(L), _I(H))
    return out


def linear_scan_bwd(a, h0, fwd, dy, prec="f64"):
    a, fwd, dy = _f32(a), _f32(fwd), _f32(dy)
    B, L, H = a.shape
    h0 = None if h0 is None else _f32(h0)
    ga, gb = np.empty_like(a), np.empty_like(a)
    gh0 = np.empty((B, H), np.float32)
    _fn("linear_scan_bwd", prec)(_p(a), _p(h0), _p(fwd), _p(dy), _p(ga), _p(gb), _p(gh0),
                                 _I(B), _I(L), _I(H))
    return ga, gb, gh0


def mingru_fwd(z, c, h0=None, prec="f64"):
    z, c = _f32(z), _f32(c)
    B, L, H = z.shape
    h0 = None if h0 is None else _f32(h0)
    out = np.empty_like(z)
    _fn("mingru_fwd", prec)(_p(z), _p(c), _p(h0), _p(out), _I(B), _I(L), _I(H))
    return out


def mingru_bwd(z, c, h0, fwd, dy, prec="f64"):
    z, c, fwd, dy = _f32(z), _f32(c), _f32(fwd), _f32(dy)
    B, L, H = z.shape
    h0 = None if h0 is None else _f32(h0)
    gz, gc = np.empty_like(z), np.empty_like(z)
    gh0 = np.empty((B, H), np.float32)
    _fn("mingru_bwd", prec)(_p(z), _p(c), _p(h0), _p(fwd), _p(dy), _p(gz), _p(gc), _p(gh0),
                            _I(B), _I(L), _I(H))
    return gz, gc, gh0


# ------------------------------------------ native-recurrence scans
# lib/edifice/recurrent/native_recurrence.ex: elu_gru_scan :146-172 (z = sigmoid(g),
# c = 1 + elu(x)), real_gru_scan :193-213 (z = sigmoid(g)), diag_linear_scan
# :232-250 (a = sigmoid(a_pre)).  The activations are taken in f64 and the
# recurrences run through the MinGRU / linear-scan restatements above (the
# activated values are rounded to f32 on the way, ~6e-8 relative).
def sigmoid64(x):
    x = np.asarray(x, np.float64)
    return 1.0 / (1.0 + np.exp(-x))


def one_plus_elu64(x):
    x = np.asarray(x, np.float64)
    return 1.0 + np.where(x > 0, x, np.expm1(np.minimum(x, 0.0)))


def elu_gru_fwd(gates, cand, h0=None, prec="f64"):
    return mingru_fwd(sigmoid64(gates), one_plus_elu64(cand), h0, prec)


def real_gru_fwd(gates, cand, h0=None, prec="f64"):
    return mingru_fwd(sigmoid64(gates), cand, h0, prec)


def diag_linear_fwd(a_pre, b, h0=None, prec="f64"):
    return linear_scan_fwd(sigmoid64(a_pre), b, h0, prec)


# ------------------------------------------------------- selective scan
DT_MIN, DT_MAX = 0.001, 0.1


def selective_scan_fwd(x, dt, A, Bm, Cm, prec="f64", dt_min=DT_MIN, dt_max=DT_MAX):
    x, dt, A, Bm, Cm = map(_f32, (x, dt, A, Bm, Cm))
    B, L, D = x.shape
    N = A.shape[1]
    if N > 64:
        raise ValueError("oracle supports d_state <= 64")
    y = np.empty_like(x)
    _fn("selective_scan_fwd", prec)(_p(x), _p(dt), _p(A), _p(Bm), _p(Cm), _p(y), _I(B), _I(L),
                                    _I(D), _I(N), ctypes.c_float(dt_min), ctypes.c_float(dt_max))
    return y


def selective_scan_bwd(x, dt, A, Bm, Cm, dy, prec="f64", dt_min=DT_MIN, dt_max=DT_MAX):
    x, dt, A, Bm, Cm, dy = map(_f32, (x, dt, A, Bm, Cm, dy))
    B, L, D = x.shape
    N = A.shape[1]
    gx, gdt = np.empty_like(x), np.empty_like(x)
    gB, gC = np.empty((B, L, N), np.float32), np.empty((B, L, N), np.float32)
    _fn("selective_scan_bwd", prec)(_p(x), _p(dt), _p(A), _p(Bm), _p(Cm), _p(dy), _p(gx),
                                    _p(gdt), _p(gB), _p(gC), _I(B), _I(L), _I(D), _I(N),
                                    ctypes.c_float(dt_min), ctypes.c_float(dt_max))
    return gx, gdt, gB, gC


def selective_scan_model_fwd(x, dt, Bm, Cm, prec="f64", dt_min=DT_MIN, dt_max=DT_MAX, A=None):
    """Model semantics (common.ex:661-670); A=None is the fixed -(1..N) diagonal."""
    x, dt, Bm, Cm = map(_f32, (x, dt, Bm, Cm))
    A = None if A is None else _f32(A)
    B, L, D = x.shape
    N = Bm.shape[2]
    y = np.empty_like(x)
    _fn("selective_scan_model_fwd", prec)(_p(x), _p(dt), _p(A), _p(Bm), _p(Cm), _p(y), _I(B),
                                          _I(L), _I(D), _I(N), ctypes.c_float(dt_min),
                                          ctypes.c_float(dt_max))
    return y


def selective_scan_model_bwd(x, dt, Bm, Cm, dy, prec="f64", dt_min=DT_MIN, dt_max=DT_MAX,
                             A=None):
    """Gradients (gx, gdt, gB, gC) of the model semantics; A gets none."""
    x, dt, Bm, Cm, dy = map(_f32, (x, dt, Bm, Cm, dy))
    A = None if A is None else _f32(A)
    B, L, D = x.shape
    N = Bm.shape[2]
    gx, gdt = np.empty_like(x), np.empty_like(x)
    gB, gC = np.empty((B, L, N), np.float32), np.empty((B, L, N), np.float32)
    _fn("selective_scan_model_bwd", prec)(_p(x), _p(dt), _p(A), _p(Bm), _p(Cm), _p(dy), _p(gx),
                                          _p(gdt), _p(gB), _p(gC), _I(B), _I(L), _I(D), _I(N),
                                          ctypes.c_float(dt_min), ctypes.c_float(dt_max))
    return gx, gdt, gB, gC


# ------------------------------------------------------------ delta rule
def delta_net_fwd(q, k, v, beta, prec="f64"):
    q, k, v, beta = map(_f32, (q, k, v, beta))
    B, L, H, d = q.shape
    scalar = int(beta.ndim == 3)
    o = np.empty_like(q)
    _fn("delta_net_fwd", prec)(_p(q), _p(k), _p(v), _p(beta), _p(o), _I(B), _I(L), _I(H),
                               _I(d), _I(scalar))
    return o


def delta_net_bwd(q, k, v, beta, dO, prec="f64"):
    q, k, v, beta, dO = map(_f32, (q, k, v, beta, dO))
    B, L, H, d = q.shape
    scalar = int(beta.ndim == 3)
    gq, gk, gv = np.empty_like(q), np.empty_like(q), np.empty_like(q)
    gbeta = np.empty_like(beta)
    _fn("delta_net_bwd", prec)(_p(q), _p(k), _p(v), _p(beta), _p(dO), _p(gq), _p(gk), _p(gv),
                               _p(gbeta), _I(B), _I(L), _I(H), _I(d), _I(scalar))
    return gq, gk, gv, gbeta


# ------------------------------------------------------ gated delta rule
def gated_delta_net_fwd(q, k, v, beta, alpha, prec="f64"):
    q, k, v, beta, alpha = map(_f32, (q, k, v, beta, alpha))
    B, L, H, d = q.shape
    scalar = int(beta.ndim == 3)
    o = np.empty_like(q)
    _fn("gated_delta_net_fwd", prec)(_p(q), _p(k), _p(v), _p(beta), _p(alpha), _p(o), _I(B),
                                     _I(L), _I(H), _I(d), _I(scalar))
    return o


def gated_delta_net_bwd(q, k, v, beta, alpha, dO, prec="f64"):
    q, k, v, beta, alpha, dO = map(_f32, (q, k, v, beta, alpha, dO))
    B, L, H, d = q.shape
    scalar = int(beta.ndim == 3)
    gq, gk, gv = np.empty_like(q), np.empty_like(q), np.empty_like(q)
    gbeta, galpha = np.empty_like(beta), np.empty_like(alpha)
    _fn("gated_delta_net_bwd", prec)(_p(q), _p(k), _p(v), _p(beta), _p(alpha), _p(dO), _p(gq),
                                     _p(gk), _p(gv), _p(gbeta), _p(galpha), _I(B), _I(L), _I(H),
                                     _I(d), _I(scalar))
    return gq, gk, gv, gbeta, galpha


# ------------------------------------------------------------- attention
def attention_fwd(q, k, v, causal=True, prec="f64", want_lse=False):
    q, k, v = map(_f32, (q, k, v))
    B, Hq, L, d = q.shape
    Hkv = k.shape[1]
    o = np.empty_like(q)
    lse = np.empty((B, Hq, L), np.float32) if want_lse else None
    _fn("attention_fwd", prec)(_p(q), _p(k), _p(v), _p(o), _p(lse), _I(B), _I(Hq), _I(Hkv),
                               _I(L), _I(d), _I(int(bool(causal))))
    return (o, lse) if want_lse else o


def attention_bwd(q, k, v, dO, causal=True, prec="f64"):
    q, k, v, dO = map(_f32, (q, k, v, dO))
    B, Hq, L, d = q.shape
    Hkv = k.shape[1]
    dq, dk, dv = np.empty_like(q), np.empty_like(k), np.empty_like(v)
    _fn("attention_bwd", prec)(_p(q), _p(k), _p(v), _p(dO), _p(dq), _p(dk), _p(dv), _I(B),
                               _I(Hq), _I(Hkv), _I(L), _I(d), _I(int(bool(causal))))
    return dq, dk, dv


# ------------------------------------------------------------- LASER attention
# lib/edifice/cuda/fused_scan.ex:3593-3611 (v_max = max over the sequence of v),
# laser_attention_fallback :3667-3703 and laser_attention_backward_fallback
# :3723-3766, composed from the attention restatement above: the values are
# exp(V - v_max) (taken in f64, rounded to f32 on the way in), the log and the
# gradient pre/post-scaling in f64.  v_max is a constant for the gradient, as in
# the reference.
def _laser_parts(v, v_max):
    v64 = np.asarray(v, np.float64)
    vm = v64.max(axis=2, keepdims=True) if v_max is None else \
        np.asarray(v_max, np.float64)[:, :, None, :]
    return vm, np.exp(v64 - vm)


def _expand_heads(x, hq):
    """[B, Hkv, ...] -> [B, Hq, ...] (each kv head repeated over its query group)."""
    return np.repeat(x, hq // x.shape[1], axis=1)


def laser_fwd(q, k, v, causal=True, v_max=None, prec="f64"):
    """Returns (O, A): the output and the attention output before the log."""
    vm, ev = _laser_parts(v, v_max)
    A = attention_fwd(q, k, ev, causal=causal, prec=prec).astype(np.float64)
    O = np.log(np.maximum(A, 1e-7)) + _expand_heads(vm, A.shape[1])
    return O.astype(np.float32), A


def laser_bwd(q, k, v, dO, causal=True, v_max=None, prec="f64"):
    vm, ev = _laser_parts(v, v_max)
    A = attention_fwd(q, k, ev, causal=causal, prec=prec).astype(np.float64)
    dR = np.asarray(dO, np.float64) / np.maximum(A, 1e-7)
    dq, dk, dev = attention_bwd(q, k, ev, dR, causal=causal, prec=prec)
    return dq, dk, (dev.astype(np.float64) * ev).astype(np.float32)


# --------------------------------------------------------------- FoX attention
# fox_attention_fallback (fused_scan.ex:3863-3912) and its backward (:3926-3984),
# dense in f64 numpy (small cases): scores q k^T / sqrt(d) + (cs_i - cs_j) with the
# diagonal bias zeroed, causal, softmax; grad_cs = rowsum(dS) - colsum(dS) of the
# unscaled score gradient with the diagonal excluded.  Grouped kv heads are expanded
# to the query heads (gqa.ex:257-271), their gradients summed back.
def _fox_parts(q, k, v, cs):
    q, k, v, cs = (np.asarray(x, np.float64) for x in (q, k, v, cs))
    B, Hq, L, d = q.shape
    ke, ve = _expand_heads(k, Hq), _expand_heads(v, Hq)
    scale = np.sqrt(d)
    s = q @ np.swapaxes(ke, -1, -2) / scale
    bias = cs[..., :, None] - cs[..., None, :]
    eye = np.eye(L, dtype=bool)
    s = s + np.where(eye, 0.0, bias)
    s = np.where(np.tri(L, dtype=bool), s, -np.inf)
    w = np.exp(s - s.max(-1, keepdims=True))
    w /= w.sum(-1, keepdims=True)
    return q, ke, ve, w, scale, eye


def fox_fwd(q, k, v, cs):
    q, ke, ve, w, _, _ = _fox_parts(q, k, v, cs)
    return (w @ ve).astype(np.float32)


def fox_bwd(q, k, v, cs, dO):
    q, ke, ve, w, scale, eye = _fox_parts(q, k, v, cs)
    dO = np.asarray(dO, np.float64)
    Hkv = np.asarray(k).shape[1]
    g = q.shape[1] // Hkv
    gv = np.swapaxes(w, -1, -2) @ dO
    dw = dO @ np.swapaxes(ve, -1, -2)
    ds = w * (dw - (dw * w).sum(-1, keepdims=True))
    ds_nd = np.where(eye, 0.0, ds)
    gcs = ds_nd.sum(-1) - ds_nd.sum(-2)
    ds = ds / scale
    gq = ds @ ke
    gk = np.swapaxes(ds, -1, -2) @ q

    def fold(x):  # [B, Hq, ...] -> [B, Hkv, ...], summed over each group
        return x.reshape(x.shape[0], Hkv, g, *x.shape[2:]).sum(2)
    return tuple(x.astype(np.float32) for x in (gq, fold(gk), fold(gv), gcs))


# ---------------------------------------------- the reference's own C refs
def ref_linear_scan_cpu(a, b, h0):
    r = ref_cpu_lib()
    a, b, h0 = map(_f32, (a, b, h0))
    B, L, H = a.shape
    out = np.empty_like(a)
    r.ref_linear_scan_cpu(_p(a), _p(b), _p(h0), _p(out), _I(B), _I(L), _I(H))
    return out


def ref_mingru_scan_cpu(z, c, h0):
    r = ref_cpu_lib()
    z, c, h0 = map(_f32, (z, c, h0))
    B, L, H = z.shape
    out = np.empty_like(z)
    r.ref_mingru_scan_cpu(_p(z), _p(c), _p(h0), _p(out), _I(B), _I(L), _I(H))
    return out


def ref_delta_net_scan_cpu(q, k, v, beta):
    r = ref_cpu_lib()
    q, k, v, beta = map(_f32, (q, k, v, beta))
    B, L, H, d = q.shape
    out = np.empty_like(q)
    r.ref_delta_net_scan_cpu(_p(q), _p(k), _p(v), _p(beta), _p(out), _I(B), _I(L), _I(H), _I(d))
    return out


def norm_rel(x, ref):
    """||x - ref||_2 / ||ref||_2 computed in f64 (the parity metric)."""
    x = np.asarray(x, np.float64)
    ref = np.asarray(ref, np.float64)
    den = np.linalg.norm(ref.ravel())
    num = np.linalg.norm((x - ref).ravel())
    return float(num / den) if den > 0 else float(num)
