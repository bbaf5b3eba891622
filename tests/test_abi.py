"""CPU checks of the C ABI: the libraries load, export every symbol the headers
declare, and reject bad arguments on the host (no GPU call is made)."""
import ctypes
import os
import re
import subprocess

import pytest

import edifice_b200
from edifice_b200 import _lib, build

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared(header):
    txt = open(os.path.join(ROOT, "include", header)).read()
    txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\*?\s+\*?(\w+)\s*\(", txt, flags=re.M)))


def _exported(path):
    out = subprocess.run(["nm", "-D", "--defined-only", path], capture_output=True, text=True,
                         check=True).stdout
    return {ln.split()[-1] for ln in out.splitlines() if " T " in ln}


@pytest.fixture(scope="module", autouse=True)
def built():
    build.build()


def test_library_loads_and_reports_version():
    lib = edifice_b200.load()
    assert lib.edb_version().decode().startswith("edifice_b200")


def test_every_declared_symbol_is_exported():
    names = _declared("edifice_b200.h")
    assert "edb_linear_scan_fwd" in names and len(names) >= 7
    exp = _exported(_lib.LIB_PATH)
    missing = [n for n in names if n not in exp]
    assert not missing, missing
    # every declared entry point also has a ctypes prototype
    assert set(names) <= set(_lib.SIGNATURES)


@pytest.mark.parametrize("prec", ["f32", "bf16"])
def test_shims_export_reference_names(prec):
    names = _declared("edifice_cuda_kernels.h")
    assert "fused_linear_scan_launch" in names
    exp = _exported(build.SHIMS[prec])
    missing = [n for n in names if n not in exp]
    assert not missing, missing
    ctypes.CDLL(build.SHIMS[prec])  # resolves against libedifice_b200.so


def test_status_strings():
    assert _lib.status_string(0) == "ok"
    assert "shape" in _lib.status_string(1001)
    assert "dtype" in _lib.status_string(1002)


def test_host_validation_rejects_bad_arguments():
    lib = edifice_b200.load()
    dummy = ctypes.c_void_p(16)
    # bad dtype, bad shape, null pointers: all rejected before any CUDA call
    assert lib.edb_linear_scan_fwd(7, dummy, dummy, None, dummy, 1, 1, 1, None) == 1002
    assert lib.edb_linear_scan_fwd(1, dummy, dummy, None, dummy, 0, 4, 4, None) == 1001
    assert lib.edb_linear_scan_fwd(1, None, dummy, None, dummy, 1, 4, 4, None) == 1000
    assert lib.edb_mingru_bwd(0, dummy, dummy, None, dummy, None, dummy, dummy, None, 1, 4, 4,
                              None) == 1000
    assert lib.edb_mingru_fwd(0, dummy, dummy, None, dummy, 2, -1, 4, None) == 1001
    # GatedDeltaNet: alpha is required; a too-small workspace is refused
    assert lib.edb_gated_delta_net_fwd(0, dummy, dummy, dummy, dummy, 1, None, dummy, None, 1,
                                       4, 2, 8, None) == 1000
    assert lib.edb_gated_delta_net_fwd(0, dummy, dummy, dummy, dummy, 1, dummy, dummy, None, 1,
                                       4, 2, 256, None) != 0
    need = lib.edb_gated_delta_net_bwd_workspace(0, 1, 1, 4, 2, 8, 0)
    assert need > 0
    assert lib.edb_gated_delta_net_bwd(0, dummy, dummy, dummy, dummy, 1, dummy, dummy, None,
                                       dummy, dummy, dummy, dummy, dummy, 1, 4, 2, 8, dummy,
                                       need - 1, None) == 1004


# ---------------------------------------------------------------- descriptor form
def test_descriptor_workspace_counts_copies_of_non_dense_tensors():
    from edifice_b200 import descriptor as D
    base, B, L, H = 1 << 24, 2, 8, 64
    dense = lambda off=0: D.tensor(base + off, _lib.EDB_BF16, (B, L, H))
    a = D.make_args("linear_scan", _lib.EDB_BF16)
    a.a, a.b, a.h = dense(), dense(4096), dense(8192)
    assert D.workspace_bytes("linear_scan", "fwd", a) == 0
    # a transposed view of a [B, H, L] buffer needs one dense copy (2 * 8 * 64 bf16 -> 2 KB)
    a.b = D.tensor(base, _lib.EDB_BF16, (B, L, H), (L * H, 1, L))
    assert D.workspace_bytes("linear_scan", "fwd", a) == 2048
    # an unaligned dense pointer is copied too; a broadcast h0 (stride 0) as well
    a.b = dense(2)
    a.h0 = D.tensor(base, _lib.EDB_BF16, (B, H), (0, 1))
    assert D.workspace_bytes("linear_scan", "fwd", a) == 2048 + 256
    # the backward adds the positional entry point's own scratch on top of the copies
    f = D.make_args("flash_attention", _lib.EDB_BF16, causal=1)
    q = D.tensor(base, _lib.EDB_BF16, (1, 4, 256, 128))
    kv = D.tensor(base, _lib.EDB_BF16, (1, 2, 256, 128))
    f.q = f.o = f.dO = f.dq = q
    f.k = f.v = f.dk = f.dv = kv
    lib = edifice_b200.load()
    inner = lib.edb_flash_attention_bwd_workspace(1, 1, 4, 2, 256, 128, 0)
    assert D.workspace_bytes("flash_attention", "bwd", f) == inner
    f.q = D.tensor(base, _lib.EDB_BF16, (1, 4, 256, 128), (256 * 4 * 128, 128, 4 * 128, 1))
    assert D.workspace_bytes("flash_attention", "bwd", f) == inner + 4 * 256 * 128 * 2


def test_descriptor_validation_before_any_gpu_work():
    from edifice_b200 import descriptor as D
    lib = edifice_b200.load()
    base, B, L, H = 1 << 24, 2, 8, 64
    dense = lambda dt=_lib.EDB_BF16, shape=(B, L, H): D.tensor(base, dt, shape)

    def st(op, direction, args, ws=None, nbytes=0):
        fn = getattr(lib, "edb_%s_%s_desc" % (op, direction))
        return fn(ctypes.byref(args), None, ws, nbytes)

    a = D.make_args("linear_scan", _lib.EDB_BF16)
    a.a, a.b = dense(), dense()
    assert st("linear_scan", "fwd", a) == 1000                    # h missing
    a.h = dense(_lib.EDB_F32)
    assert st("linear_scan", "fwd", a) == 1002                    # dtype mismatch
    a.h = dense(shape=(B, L, H + 1))
    assert st("linear_scan", "fwd", a) == 1001                    # shape mismatch
    a.h = D.tensor(base, _lib.EDB_BF16, (B, L, H), (L * H, 0, 1))
    assert st("linear_scan", "fwd", a) == 1001                    # output with a zero stride
    a.h = D.tensor(base, _lib.EDB_BF16, (B, L, H), (0, 0, 0))
    assert st("linear_scan", "fwd", a) == 1001                    # ... and all strides zero
    a.h = dense()
    # an input whose strides are all zero is a broadcast of one element, gathered
    # into a dense copy (so it needs a workspace), never read as a dense array
    a.a = D.tensor(base, _lib.EDB_BF16, (B, L, H), (0, 0, 0))
    assert D.workspace_bytes("linear_scan", "fwd", a) == B * L * H * 2
    assert st("linear_scan", "fwd", a) == 1004
    a.a = dense()
    a.h = D.tensor(base, _lib.EDB_BF16, (B, L, H), (L * H, 1, L))
    assert st("linear_scan", "fwd", a) == 1004                    # needs a workspace
    assert st("linear_scan", "fwd", a, base + 16, 1 << 20) == 1003  # not 256-aligned
    a.dtype = 5
    assert st("linear_scan", "fwd", a) == 1002
    # selective scan: A is required in kernel semantics, dt_mean in model semantics
    s = D.make_args("selective_scan", _lib.EDB_F32, semantics=D.SSM_KERNEL, dt_min=1e-3,
                    dt_max=0.1)
    s.x, s.dt, s.y = (dense(_lib.EDB_F32),) * 3
    s.B = s.C = dense(_lib.EDB_F32, (B, L, 16))
    assert st("selective_scan", "fwd", s) == 1000
    s.semantics = D.SSM_MODEL
    assert st("selective_scan", "fwd", s) == 1000
    s.semantics = 7
    assert st("selective_scan", "fwd", s) == 1005
    # delta rule: beta's rank follows beta_mode; a decay gradient needs a decay
    d = D.make_args("delta_rule", _lib.EDB_BF16, beta_mode=D.BETA_PER_ELEMENT)
    d.q = d.k = d.v = d.o = d.dO = d.gq = d.gk = d.gv = dense(shape=(B, L, 2, 32))
    d.beta = d.gbeta = dense(shape=(B, L, 2))
    assert st("delta_rule", "fwd", d) == 1001
    d.beta_mode = D.BETA_PER_TOKEN
    d.galpha = dense(shape=(B, L, 2))
    assert st("delta_rule", "bwd", d) == 1005
    # flash attention: num_kv_heads must agree with k
    f = D.make_args("flash_attention", _lib.EDB_BF16, num_kv_heads=3)
    f.q = f.o = dense(shape=(1, 4, 64, 64))
    f.k = f.v = dense(shape=(1, 2, 64, 64))
    assert st("flash_attention", "fwd", f) == 1001


def test_descriptor_attention_variants_need_their_residuals():
    from edifice_b200 import descriptor as D
    lib = edifice_b200.load()
    base = 1 << 24
    q = D.tensor(base, _lib.EDB_BF16, (1, 4, 64, 64))
    kv = D.tensor(base, _lib.EDB_BF16, (1, 2, 64, 64))
    la = D.make_args("laser_attention", _lib.EDB_BF16, causal=1)
    la.q = la.o = q
    la.k = la.v = kv
    assert lib.edb_laser_attention_fwd_desc(ctypes.byref(la), None, None, 0) == 1000  # resid
    la.resid = base
    la.v_max = D.tensor(base, _lib.EDB_BF16, (1, 2, 65))
    assert lib.edb_laser_attention_fwd_desc(ctypes.byref(la), None, None, 0) == 1001
    fx = D.make_args("fox_attention", _lib.EDB_BF16)
    fx.q = fx.o = q
    fx.k = fx.v = kv
    fx.cs = D.tensor(base, _lib.EDB_F32, (1, 4, 64))
    assert lib.edb_fox_attention_fwd_desc(ctypes.byref(fx), None, None, 0) == 1000   # lse
    fx.lse = base
    fx.cs = D.tensor(base, _lib.EDB_BF16, (1, 4, 64))
    assert lib.edb_fox_attention_fwd_desc(ctypes.byref(fx), None, None, 0) == 1002   # cs is f32
    nr = D.make_args("native_rec", _lib.EDB_F32, kind=0)
    nr.x0 = nr.x1 = D.tensor(base, _lib.EDB_F32, (2, 8, 16))
    nr.h = D.tensor(base, _lib.EDB_F32, (2, 8, 16), (128, 1, 8))
    assert lib.edb_native_rec_fwd_desc_workspace(ctypes.byref(nr)) == 1024


def test_gated_chunked_form_sizes():
    """bf16 with one beta per token and head_dim 128 takes the chunked form: a
    forward workspace and the chunked residual layout (S^T per chunk start and the
    final one, then the chunk errors U~); the token recurrence needs none."""
    lib = edifice_b200.load()
    B, L, H, d, C = 2, 130, 3, 128, 64
    nc = (L + C - 1) // C
    assert lib.edb_gated_delta_net_fwd_workspace(1, 0, B, L, H, d) > 0
    assert lib.edb_gated_delta_net_ckpt_bytes(1, 0, B, L, H, d) == \
        4 * B * H * ((nc + 1) * d * d + nc * C * d)
    assert lib.edb_gated_delta_net_ckpt_bytes(1, 0, B, L, H, d) == \
        lib.edb_delta_rule_ckpt_bytes(1, 0, B, L, H, d)
    for dt, per_el, dd in ((0, 0, 128), (1, 1, 128), (1, 0, 64)):
        assert lib.edb_gated_delta_net_fwd_workspace(dt, per_el, B, L, H, dd) == 0
        # token recurrence: S every 16 tokens and the final S
        assert lib.edb_gated_delta_net_ckpt_bytes(dt, per_el, B, L, H, dd) == \
            4 * B * H * ((L + 15) // 16 + 1) * dd * dd
    dummy = ctypes.c_void_p(16)
    # a chunked-form call with a null alpha is refused before any allocation
    assert lib.edb_gated_delta_net_fwd(1, dummy, dummy, dummy, dummy, 0, None, dummy, None, B,
                                       L, H, d, None) == 1000
    assert lib.edb_gated_delta_net_fwd_ws(1, dummy, dummy, dummy, dummy, 0, dummy, dummy, None,
                                          B, L, H, d, None, 0, None) == 1004


def test_host_tensor_entry_points_validate_on_host():
    """The host-tensor pipelines reject bad arguments before any CUDA call: null
    pointers, bad shapes (query heads not a multiple of kv heads), a workspace that
    is too small or not 256-byte aligned."""
    lib = edifice_b200.load()
    d = ctypes.c_void_p(256)
    odd = ctypes.c_void_p(272)
    B, Hq, Hkv, L, hd = 2, 4, 2, 128, 64
    for kind in ("flash", "laser"):
        fn = getattr(lib, "edb_%s_attention_train_host" % kind)
        need = getattr(lib, "edb_%s_attention_train_host_workspace" % kind)(1, B, Hq, Hkv, L, hd)
        assert need > 0
        assert getattr(lib, "edb_%s_attention_train_host_workspace" % kind)(1, B, 3, 2, L, hd) == 0
        assert fn(1, None, d, d, d, d, d, d, d, B, Hq, Hkv, L, hd, 1, 0.0, d, need, None) == 1000
        assert fn(1, d, d, d, d, d, d, d, d, B, 3, 2, L, hd, 1, 0.0, d, need, None) == 1001
        assert fn(1, d, d, d, d, d, d, d, d, B, Hq, Hkv, L, hd, 1, 0.0, d, need - 1, None) == 1004
        assert fn(1, d, d, d, d, d, d, d, d, B, Hq, Hkv, L, hd, 1, 0.0, odd, need, None) == 1003
    need = lib.edb_fox_attention_train_host_workspace(1, B, Hq, Hkv, L, hd)
    assert need > 0
    # FoX: cs and dcs are required
    assert lib.edb_fox_attention_train_host(1, d, d, d, None, d, d, d, d, d, d, B, Hq, Hkv, L,
                                            hd, 0.0, d, need, None) == 1000
    for gated in (False, True):
        name = "gated_delta_net" if gated else "delta_rule"
        need = getattr(lib, "edb_%s_train_host_workspace" % name)(1, 0, 4, 130, 2, 128)
        assert need > 0
        args = [1, d, d, d, d, 0] + ([d] if gated else []) + [d, d, d, d, d, d] + \
            ([d] if gated else [])
        fn = getattr(lib, "edb_%s_train_host" % name)
        assert fn(*args, 4, 130, 2, 128, d, need - 1, None) == 1004
        assert fn(*args, 4, 130, 2, 128, odd, need, None) == 1003
        bad = list(args)
        bad[1] = None
        assert fn(*bad, 4, 130, 2, 128, d, need, None) == 1000
    assert lib.edb_gated_delta_net_train_host(1, d, d, d, d, 0, None, d, d, d, d, d, d, d, 4,
                                              130, 2, 128, d, 1 << 30, None) == 1000
    need = lib.edb_selective_scan_model_train_host_workspace(1, 4, 64, 256, 16)
    assert need > 0
    # model semantics: A may be NULL (the fixed diagonal); a null x is refused
    assert lib.edb_selective_scan_model_train_host(1, None, d, None, d, d, d, d, d, d, d, d, 4,
                                                   64, 256, 16, 1e-3, 0.1, d, need,
                                                   None) == 1000
