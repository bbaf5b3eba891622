"""ctypes binding of libedifice_b200.so (the C ABI in include/edifice_b200.h).

The library is loaded from the package directory (built in-tree by
``python -m edifice_b200.build``).  There is no fallback: if the library is
missing or fails to load, every op raises.
"""
import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libedifice_b200.so")

_vp = ctypes.c_void_p
_i = ctypes.c_int
_f = ctypes.c_float
_sz = ctypes.c_size_t

# name -> (restype, argtypes); every entry point declared in include/edifice_b200.h
SIGNATURES = {
    "edb_version": (ctypes.c_char_p, []),
    "edb_status_string": (ctypes.c_char_p, [_i]),
    "edb_get_device_errors": (_i, [ctypes.POINTER(ctypes.c_uint), _i]),
    "edb_set_wait_limit_ns": (_i, [ctypes.c_longlong]),
    "edb_linear_scan_fwd": (_i, [_i, _vp, _vp, _vp, _vp, _i, _i, _i, _vp]),
    "edb_linear_scan_bwd": (_i, [_i, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _vp]),
    "edb_mingru_fwd": (_i, [_i, _vp, _vp, _vp, _vp, _i, _i, _i, _vp]),
    "edb_mingru_bwd": (_i, [_i, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _vp]),
    "edb_native_rec_fwd": (_i, [_i, _i, _vp, _vp, _vp, _vp, _i, _i, _i, _vp]),
    "edb_scan_train_host_workspace": (_sz, [_i, _i, _i, _i]),
    "edb_linear_scan_train_host": (_i, [_i, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i,
                                        _vp, _sz, _vp]),
    "edb_mingru_train_host": (_i, [_i, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _vp,
                                   _sz, _vp]),
    "edb_selective_scan_train_host_workspace": (_sz, [_i, _i, _i, _i, _i]),
    "edb_selective_scan_train_host": (_i, [_i, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                                           _vp, _i, _i, _i, _i, _f, _f, _vp, _sz, _vp]),
    "edb_selective_scan_model_train_host_workspace": (_sz, [_i, _i, _i, _i, _i]),
    "edb_selective_scan_model_train_host": (_i, [_i, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                                                 _vp, _vp, _vp, _i, _i, _i, _i, _f, _f, _vp,
                                                 _sz, _vp]),
    "edb_selective_scan_ckpt_bytes": (_sz, [_i, _i, _i, _i]),
    "edb_selective_scan_fwd": (_i, [_i, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _f,
                                    _f, _vp]),
    "edb_selective_scan_bwd_workspace": (_sz, [_i, _i, _i, _i, _i]),
    "edb_selective_scan_bwd": (_i, [_i, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                                    _i, _i, _i, _i, _f, _f, _vp, _sz, _vp]),
    "edb_selective_scan_model_fwd": (_i, [_i, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i,
                                          _i, _f, _f, _vp]),
    "edb_selective_scan_model_bwd": (_i, [_i, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                                          _vp, _vp, _i, _i, _i, _i, _f, _f, _vp, _sz, _vp]),
    "edb_selective_scan_bwd_noalloc": (_i, [_i, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                                            _vp, _vp, _i, _i, _i, _i, _f, _f, _vp]),
    "edb_flash_attention_fwd": (_i, [_i, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _f,
                                     _vp]),
    "edb_delta_rule_ckpt_bytes": (_sz, [_i, _i, _i, _i, _i, _i]),
    "edb_delta_rule_fwd_workspace": (_sz, [_i, _i, _i, _i, _i, _i]),
    "edb_delta_rule_fwd": (_i, [_i, _vp, _vp, _vp, _vp, _i, _vp, _vp, _i, _i, _i, _i, _vp, _sz,
                                _vp]),
    "edb_delta_rule_bwd_workspace": (_sz, [_i, _i, _i, _i, _i, _i, _i]),
    "edb_delta_rule_bwd": (_i, [_i, _vp, _vp, _vp, _vp, _i, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i,
                                _i, _i, _vp, _sz, _vp]),
    "edb_gated_delta_net_ckpt_bytes": (_sz, [_i, _i, _i, _i, _i, _i]),
    "edb_gated_delta_net_fwd": (_i, [_i, _vp, _vp, _vp, _vp, _i, _vp, _vp, _vp, _i, _i, _i, _i,
                                     _vp]),
    "edb_gated_delta_net_fwd_workspace": (_sz, [_i, _i, _i, _i, _i, _i]),
    "edb_gated_delta_net_fwd_ws": (_i, [_i, _vp, _vp, _vp, _vp, _i, _vp, _vp, _vp, _i, _i, _i,
                                        _i, _vp, _sz, _vp]),
    "edb_gated_delta_net_bwd_workspace": (_sz, [_i, _i, _i, _i, _i, _i, _i]),
    "edb_gated_delta_net_bwd": (_i, [_i, _vp, _vp, _vp, _vp, _i, _vp, _vp, _vp, _vp, _vp, _vp,
                                     _vp, _vp, _i, _i, _i, _i, _vp, _sz, _vp]),
    "edb_flash_attention_train_host_workspace": (_sz, [_i, _i, _i, _i, _i, _i]),
    "edb_flash_attention_train_host": (_i, [_i, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i,
                                            _i, _i, _i, _i, _f, _vp, _sz, _vp]),
    "edb_laser_attention_train_host_workspace": (_sz, [_i, _i, _i, _i, _i, _i]),
    "edb_laser_attention_train_host": (_i, [_i, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i,
                                            _i, _i, _i, _i, _f, _vp, _sz, _vp]),
    "edb_fox_attention_train_host_workspace": (_sz, [_i, _i, _i, _i, _i, _i]),
    "edb_fox_attention_train_host": (_i, [_i, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                                          _i, _i, _i, _i, _i, _f, _vp, _sz, _vp]),
    "edb_delta_rule_train_host_workspace": (_sz, [_i, _i, _i, _i, _i, _i]),
    "edb_delta_rule_train_host": (_i, [_i, _vp, _vp, _vp, _vp, _i, _vp, _vp, _vp, _vp, _vp, _vp,
                                       _i, _i, _i, _i, _vp, _sz, _vp]),
    "edb_gated_delta_net_train_host_workspace": (_sz, [_i, _i, _i, _i, _i, _i]),
    "edb_gated_delta_net_train_host": (_i, [_i, _vp, _vp, _vp, _vp, _i, _vp, _vp, _vp, _vp,
                                            _vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp, _sz,
                                            _vp]),
    "edb_laser_attention_resid_bytes": (_sz, [_i, _i, _i, _i, _i, _i]),
    "edb_laser_attention_fwd": (_i, [_i, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i,
                                     _f, _vp]),
    "edb_laser_attention_bwd_workspace": (_sz, [_i, _i, _i, _i, _i, _i]),
    "edb_laser_attention_bwd": (_i, [_i, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i,
                                     _i, _f, _vp, _sz, _vp]),
    "edb_fox_attention_fwd": (_i, [_i, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _f,
                                   _vp]),
    "edb_fox_attention_bwd_workspace": (_sz, [_i, _i, _i, _i, _i, _i]),
    "edb_fox_attention_bwd": (_i, [_i, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i,
                                   _i, _i, _i, _i, _f, _vp, _sz, _vp]),
    "edb_convert": (_i, [_i, _vp, _i, _vp, _sz, _vp]),
    "edb_flash_attention_bwd_workspace": (_sz, [_i, _i, _i, _i, _i, _i, _i]),
    "edb_flash_attention_bwd": (_i, [_i, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i,
                                     _i, _i, _i, _i, _f, _vp, _sz, _vp]),
}
# descriptor form: every op, both directions, takes (const args*, stream, ws, ws_bytes)
for _op in ("linear_scan", "mingru", "selective_scan", "delta_rule", "flash_attention",
            "native_rec", "laser_attention", "fox_attention"):
    for _dir in (("fwd",) if _op == "native_rec" else ("fwd", "bwd")):
        SIGNATURES["edb_%s_%s_desc_workspace" % (_op, _dir)] = (_sz, [_vp])
        SIGNATURES["edb_%s_%s_desc" % (_op, _dir)] = (_i, [_vp, _vp, _vp, _sz])

EDB_F32, EDB_BF16 = 0, 1
EDB_NATIVE_ELU_GRU, EDB_NATIVE_REAL_GRU, EDB_NATIVE_DIAG_LINEAR = 0, 1, 2

_lib = None


class EdbError(RuntimeError):
    pass


def load():
    """Load the native library (once) and attach prototypes.  Raises if absent."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise EdbError("libedifice_b200.so not built (run `python -m edifice_b200.build`); "
                       "there is no CPU fallback")
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def status_string(st):
    return load().edb_status_string(int(st)).decode()


def check(st, what):
    if st != 0:
        raise EdbError("%s failed: %s (status %d)" % (what, status_string(st), st))


def device_errors(clear=True):
    flags = ctypes.c_uint(0)
    check(load().edb_get_device_errors(ctypes.byref(flags), int(bool(clear))), "edb_get_device_errors")
    return int(flags.value)
