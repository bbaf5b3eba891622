"""Build libedifice_b200.so (sm_100a) and the two reference-named shim libraries.

    python -m edifice_b200.build [--force] [-j N]

Outputs (in-tree, git-ignored, carried to the GPU box with the tree):
  edifice_b200/libedifice_b200.so               all kernels + the edb_* C ABI
  edifice_b200/shim/libedifice_cuda_kernels.so      fused_<op>_launch, f32 names
  edifice_b200/shim/libedifice_cuda_kernels_bf16.so fused_<op>_launch, bf16 names

Each .cu under csrc/ is compiled separately (parallel), then linked by nvcc.
Flags: -gencode arch=compute_100a,code=sm_100a -O3 -lineinfo, C++17.
"""
import argparse
import concurrent.futures as cf
import glob
import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
OBJ = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libedifice_b200.so")
SHIM_DIR = os.path.join(PKG, "shim")
SHIMS = {
    "f32": os.path.join(SHIM_DIR, "libedifice_cuda_kernels.so"),
    "bf16": os.path.join(SHIM_DIR, "libedifice_cuda_kernels_bf16.so"),
}
NVCC = os.environ.get("NVCC", "nvcc")
GENCODE = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = GENCODE + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
                   "-I", os.path.join(ROOT, "include"), "--expt-relaxed-constexpr",
                   "-Xptxas", "-warn-spills"]


def _sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _headers():
    return sorted(glob.glob(os.path.join(CSRC, "*.cuh")) +
                  glob.glob(os.path.join(ROOT, "include", "*.h")))


def _mtime(p):
    return os.path.getmtime(p) if os.path.exists(p) else -1.0


def _compile(src, force, verbose_ptxas=False):
    """Compile one source unless its object is newer than it and every header.
    Returns (object, ptxas log, whether nvcc ran)."""
    obj = os.path.join(OBJ, os.path.basename(src)[:-3] + ".o")
    newest_dep = max([_mtime(src)] + [_mtime(h) for h in _headers()])
    if not force and _mtime(obj) >= newest_dep:
        return obj, "", False
    cmd = [NVCC, *FLAGS, "-c", src, "-o", obj]
    if verbose_ptxas:
        cmd += ["-Xptxas", "-v"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("nvcc failed for %s:\n%s\n%s" % (src, r.stdout, r.stderr))
    return obj, r.stderr, True


def build(force=False, jobs=None, verbose_ptxas=False, report=None):
    """Compile what changed, link, build the shims.  `report` (a callable taking
    one line) receives what was compiled and linked, and what was reused."""
    os.makedirs(OBJ, exist_ok=True)
    os.makedirs(SHIM_DIR, exist_ok=True)
    srcs = _sources()
    jobs = jobs or min(8, os.cpu_count() or 4)
    logs, compiled, reused = [], [], []
    with cf.ThreadPoolExecutor(jobs) as ex:
        futs = [ex.submit(_compile, s, force, verbose_ptxas) for s in srcs]
        objs = []
        for f in futs:
            o, log, ran = f.result()
            objs.append(o)
            (compiled if ran else reused).append(os.path.basename(o))
            if log:
                logs.append(log)
    linked = False
    if force or _mtime(LIB) < max(_mtime(o) for o in objs):
        r = subprocess.run([NVCC, *GENCODE, "-shared", "-o", LIB, *objs, "-lcudart"],
                           capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("link failed:\n%s\n%s" % (r.stdout, r.stderr))
        linked = True
    shim_src = os.path.join(PKG, "shim", "legacy_shim.cpp")
    shims_built = []
    for prec, out in SHIMS.items():
        if force or _mtime(out) < max(_mtime(shim_src), _mtime(LIB)):
            define = ["-DEDB_SHIM_BF16"] if prec == "bf16" else []
            r = subprocess.run(
                ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", *define,
                 "-I", os.path.join(ROOT, "include"), "-I", "/usr/local/cuda/include",
                 shim_src, "-o", out, "-L", PKG, "-ledifice_b200",
                 "-Wl,-rpath,$ORIGIN/..:$ORIGIN", "-L/usr/local/cuda/lib64", "-lcudart"],
                capture_output=True, text=True)
            if r.returncode != 0:
                raise RuntimeError("shim build failed:\n%s\n%s" % (r.stdout, r.stderr))
            shims_built.append(os.path.basename(out))
    if report is not None:
        report("edifice_b200 build: nvcc compiled %d of %d sources for sm_100a%s" % (
            len(compiled), len(srcs), (": " + ", ".join(compiled)) if compiled else ""))
        if reused:
            report("edifice_b200 build: objects newer than their sources, reused: " +
                   ", ".join(reused))
        report("edifice_b200 build: %s %s" % ("linked" if linked else "up to date:",
                                              os.path.relpath(LIB, ROOT)))
        report("edifice_b200 build: shims %s" % (", ".join(shims_built) if shims_built
                                                 else "up to date"))
    return LIB, logs


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", type=int, default=None)
    ap.add_argument("--ptxas-v", action="store_true", help="print register/smem usage")
    a = ap.parse_args()
    lib, logs = build(a.force, a.j, a.ptxas_v, report=print)
    for l in logs:
        sys.stderr.write(l)
    print(lib)


if __name__ == "__main__":
    main()
