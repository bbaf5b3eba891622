"""Build recipe for the parity checker -- TEST INFRASTRUCTURE ONLY.

Outputs (all git-ignored, all carried to the GPU box with the tree):

  oracle/liboracle.so
      gcc -O2 -fopenmp build of oracle.c (the CPU restatement of Edifice's Nx
      fallbacks, f64 parity oracle + f32 timed baseline).

  oracle/_ref/libref_cpu.so
      The reference's own C CPU references (native/cuda/test_kernels.cu:
      mingru_scan_cpu :68, linear_scan_cpu :166, delta_net_scan_cpu :205),
      compiled from the reference sources where they lie, plus ref_shim.cpp
      which re-exports those C++ functions under C names.  test_kernels.cu
      also references the reference's forward launch wrappers, so the same
      link includes those kernel files.

  oracle/_ref/libref_kernels_{f32,bf16}.so
      The reference's CUDA kernels for the hot path (native/cuda/fused_*.cu,
      forward and backward of linear/MinGRU/selective scan, delta rule and
      flash attention) built from source for sm_100a.  Used only by GPU tests
      as a second, independent oracle for the paths that have no golden
      vectors (kernel-semantics selective scan, flash attention).

The reference's own Makefile is not run; nvcc is invoked directly on the
listed files.  The _ref outputs are only built where the reference tree
exists (the build container); the GPU box uses the prebuilt files.
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
def reference_root():
    """The reference checkout to compile from: $EDIFICE_REFERENCE_ROOT, else the
    `reference_path` that the build's BASELINE.json records; None when neither is
    set.  Nothing at run time needs it (the GPU box uses the prebuilt files)."""
    env = os.environ.get("EDIFICE_REFERENCE_ROOT")
    if env:
        return env
    try:
        import json
        with open(os.path.join(os.path.dirname(HERE), "BASELINE.json")) as f:
            return json.load(f).get("reference_path") or None
    except (OSError, ValueError):
        return None


REF_ROOT = reference_root()
REF_CUDA = os.path.join(REF_ROOT, "native", "cuda") if REF_ROOT else None
REF_OUT = os.path.join(HERE, "_ref")

ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_CPU_SO = os.path.join(REF_OUT, "libref_cpu.so")
REF_KERNELS_SO = {
    "f32": os.path.join(REF_OUT, "libref_kernels_f32.so"),
    "bf16": os.path.join(REF_OUT, "libref_kernels_bf16.so"),
}

# forward launch wrappers test_kernels.cu declares (it links against all of them)
_REF_TEST_DEPS = [
    "fused_mingru_scan.cu", "fused_minlstm_scan.cu", "fused_native_rec_scan.cu",
    "fused_liquid_scan.cu", "fused_linear_scan.cu", "fused_delta_rule_scan.cu",
]
# hot-path kernels, forward + backward
_REF_HOT = [
    "fused_linear_scan.cu", "fused_linear_scan_backward.cu",
    "fused_mingru_scan.cu", "fused_mingru_scan_backward.cu",
    "fused_selective_scan.cu", "fused_selective_scan_backward.cu",
    "fused_delta_rule_scan.cu", "fused_delta_rule_scan_backward.cu",
    "fused_flash_attention.cu", "fused_flash_attention_backward.cu",
    "fused_native_rec_scan.cu", "fused_elu_gru_scan_backward.cu",
    "fused_real_gru_scan_backward.cu", "fused_diag_linear_scan_backward.cu",
]

NVCC = os.environ.get("NVCC", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _newer(out, srcs):
    if not os.path.exists(out):
        return False
    t = os.path.getmtime(out)
    return all(os.path.getmtime(s) <= t for s in srcs if os.path.exists(s))


def _run(cmd):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("build failed: %s\n%s\n%s" % (" ".join(cmd), r.stdout, r.stderr))


def build_oracle(force=False):
    srcs = [os.path.join(HERE, "oracle.c"), os.path.join(HERE, "oracle_body.h")]
    if not force and _newer(ORACLE_SO, srcs):
        return ORACLE_SO
    _run(["gcc", "-O2", "-march=x86-64-v2", "-fopenmp", "-fPIC", "-shared", "-std=c11",
          srcs[0], "-o", ORACLE_SO, "-lm"])
    return ORACLE_SO


def reference_present():
    return REF_CUDA is not None and os.path.isdir(REF_CUDA)


def build_ref(force=False):
    """Build oracle/_ref from the reference sources.  Returns the list of
    libraries built (empty when the reference tree is absent)."""
    if not reference_present():
        return []
    os.makedirs(REF_OUT, exist_ok=True)
    built = []
    shim = os.path.join(HERE, "ref_shim.cpp")
    cpu_srcs = [os.path.join(REF_CUDA, "test_kernels.cu")] + [
        os.path.join(REF_CUDA, f) for f in _REF_TEST_DEPS]
    if force or not _newer(REF_CPU_SO, cpu_srcs + [shim]):
        _run([NVCC, *ARCH, "-O2", "-std=c++17", "-shared", "-Xcompiler", "-fPIC",
              "-I", REF_CUDA, "-x", "cu", *cpu_srcs, shim, "-o", REF_CPU_SO])
    built.append(REF_CPU_SO)
    hot = [os.path.join(REF_CUDA, f) for f in _REF_HOT]
    for prec, out in REF_KERNELS_SO.items():
        # this file lists the sources, so a change here rebuilds too
        if force or not _newer(out, hot + [os.path.abspath(__file__)]):
            extra = ["-DUSE_BF16"] if prec == "bf16" else []
            _run([NVCC, *ARCH, "-O3", "-std=c++17", "-shared", "-Xcompiler", "-fPIC",
                  "-I", REF_CUDA, *extra, *hot, "-o", out])
        built.append(out)
    return built


def build_all(force=False):
    out = [build_oracle(force)]
    out += build_ref(force)
    return out


if __name__ == "__main__":
    for p in build_all(force="--force" in sys.argv):
        print(p)
