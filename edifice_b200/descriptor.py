"""ctypes mirror of the descriptor form of the C ABI (``edb_<op>_{fwd,bwd}_desc``).

The argument structs match ``include/edifice_b200.h``; :func:`run` fills one
from torch tensors of any strides (transposed or sliced views included) and
calls the entry point with a workspace from torch's caching allocator on the
current stream.  The library does the gathering and scattering of non-dense
tensors itself; nothing is made contiguous here.
"""
import ctypes

import torch

from . import _lib

MAX_DIMS = 4
SSM_KERNEL, SSM_MODEL = 0, 1
BETA_PER_TOKEN, BETA_PER_ELEMENT = 0, 1


class Tensor(ctypes.Structure):
    _fields_ = [("data", ctypes.c_void_p), ("dtype", ctypes.c_int), ("ndim", ctypes.c_int),
                ("shape", ctypes.c_longlong * MAX_DIMS),
                ("strides", ctypes.c_longlong * MAX_DIMS)]


def _t(*names):
    return [(n, Tensor) for n in names]


class LinearScanArgs(ctypes.Structure):
    _fields_ = [("dtype", ctypes.c_int)] + _t("a", "b", "h0", "h", "dy", "ga", "gb", "gh0")


class MinGRUArgs(ctypes.Structure):
    _fields_ = [("dtype", ctypes.c_int)] + _t("z", "c", "h0", "h", "dy", "gz", "gc", "gh0")


class SelectiveScanArgs(ctypes.Structure):
    _fields_ = ([("dtype", ctypes.c_int), ("semantics", ctypes.c_int),
                 ("dt_min", ctypes.c_float), ("dt_max", ctypes.c_float)]
                + _t("x", "dt", "A", "B", "C", "y")
                + [("dt_mean", ctypes.c_void_p), ("h_ckpt", ctypes.c_void_p)]
                + _t("dy", "gx", "gdt", "gB", "gC"))


class DeltaRuleArgs(ctypes.Structure):
    _fields_ = ([("dtype", ctypes.c_int), ("beta_mode", ctypes.c_int)]
                + _t("q", "k", "v", "beta", "alpha", "o")
                + [("s_ckpt", ctypes.c_void_p)]
                + _t("dO", "gq", "gk", "gv", "gbeta", "galpha"))


class FlashAttentionArgs(ctypes.Structure):
    _fields_ = ([("dtype", ctypes.c_int), ("causal", ctypes.c_int),
                 ("num_kv_heads", ctypes.c_int), ("scale", ctypes.c_float)]
                + _t("q", "k", "v", "o")
                + [("lse", ctypes.c_void_p)]
                + _t("dO", "dq", "dk", "dv"))


class NativeRecArgs(ctypes.Structure):
    _fields_ = [("dtype", ctypes.c_int), ("kind", ctypes.c_int)] + _t("x0", "x1", "h0", "h")


class LaserAttentionArgs(ctypes.Structure):
    _fields_ = ([("dtype", ctypes.c_int), ("causal", ctypes.c_int), ("scale", ctypes.c_float)]
                + _t("q", "k", "v", "v_max", "o")
                + [("resid", ctypes.c_void_p)]
                + _t("dO", "dq", "dk", "dv"))


class FoxAttentionArgs(ctypes.Structure):
    _fields_ = ([("dtype", ctypes.c_int), ("scale", ctypes.c_float)]
                + _t("q", "k", "v", "cs", "o")
                + [("lse", ctypes.c_void_p)]
                + _t("dO", "dq", "dk", "dv", "dcs"))


ARGS = {"linear_scan": LinearScanArgs, "mingru": MinGRUArgs,
        "selective_scan": SelectiveScanArgs, "delta_rule": DeltaRuleArgs,
        "flash_attention": FlashAttentionArgs, "native_rec": NativeRecArgs,
        "laser_attention": LaserAttentionArgs, "fox_attention": FoxAttentionArgs}

_DTYPES = {torch.float32: _lib.EDB_F32, torch.bfloat16: _lib.EDB_BF16}


def dense_strides(shape):
    """Element strides of a dense row-major array of `shape`."""
    out, acc = [], 1
    for n in reversed(shape):
        out.append(acc)
        acc *= n
    return tuple(reversed(out))


def tensor(data, dtype, shape, strides=None):
    """An edb_tensor from a raw device address (strides in elements; None = the
    dense row-major strides of `shape`).  The library reads strides literally: a
    zero stride on an extent > 1 is a broadcast."""
    t = Tensor()
    t.data = data
    t.dtype = dtype
    t.ndim = len(shape)
    strides = dense_strides(shape) if strides is None else strides
    for i, n in enumerate(shape):
        t.shape[i] = n
        t.strides[i] = strides[i]
    return t


def of(x):
    """An edb_tensor describing torch tensor `x` (its own strides), or an empty one."""
    if x is None:
        return Tensor()
    return tensor(x.data_ptr(), _DTYPES[x.dtype], tuple(x.shape), tuple(x.stride()))


def _ptr(x):
    return None if x is None else x.data_ptr()


def make_args(op, dtype, **fields):
    """Fill the args struct of `op`: torch tensors become edb_tensor fields, the
    residual buffers (dt_mean, h_ckpt, s_ckpt, lse, resid) plain pointers, the rest
    scalars.  The struct keeps a reference to every tensor it points at, so a
    temporary view's storage is not handed back to the allocator (and reused,
    e.g. as the workspace) while the struct is alive."""
    a = ARGS[op]()
    a.dtype = _DTYPES[dtype] if isinstance(dtype, torch.dtype) else dtype
    a.keep = [v for v in fields.values() if isinstance(v, torch.Tensor)]
    for name, val in fields.items():
        kind = dict(a._fields_)[name]
        if kind is Tensor:
            setattr(a, name, of(val))
        elif kind is ctypes.c_void_p:
            setattr(a, name, _ptr(val) if isinstance(val, torch.Tensor) else val)
        else:
            setattr(a, name, val)
    return a


def workspace_bytes(op, direction, args):
    fn = getattr(_lib.load(), "edb_%s_%s_desc_workspace" % (op, direction))
    return int(fn(ctypes.byref(args)))


def run(op, direction, args, device=None):
    """Call edb_<op>_<direction>_desc on the current stream of `device` (default:
    the current CUDA device) with a workspace of the queried size allocated there;
    raises EdbError on a non-zero status."""
    lib = _lib.load()
    if device is None:
        device = torch.device("cuda", torch.cuda.current_device())
    need = workspace_bytes(op, direction, args)
    ws = torch.empty(need, dtype=torch.uint8, device=device) if need else None
    stream = torch.cuda.current_stream(device).cuda_stream
    st = getattr(lib, "edb_%s_%s_desc" % (op, direction))(
        ctypes.byref(args), ctypes.c_void_p(stream), None if ws is None else ws.data_ptr(), need)
    _lib.check(st, "edb_%s_%s_desc" % (op, direction))
    return ws
