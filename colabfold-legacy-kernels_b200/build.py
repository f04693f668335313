"""Builds the sm_100a kernel library in-tree.

    python colabfold-legacy-kernels_b200/build.py [--force] [--jobs N]

Output: src/colabfold_legacy_kernels/kernels/sm100/libcfk_sm100.so (the C ABI of include/cfk.h)
and, when $FFI_INCLUDE points at a jax >= 0.6.2 include directory (xla/ffi/api/ffi.h), also
libcfk_xla_sm100.so with the XLA FFI handlers VoltaMma, VoltaLayerNorm, VoltaGdp and the
backward handlers.

The replacement for scripts/build_kernels.sh of the reference: one nvcc per translation unit,
-gencode arch=compute_100a,code=sm_100a only, libstdc++/libgcc/cudart linked statically so the
library depends on the C library alone.  nvcc cross-compiles, so no GPU is needed.
"""

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
REPO = HERE.parent
CSRC = HERE / "csrc"
INCLUDE = REPO / "include"
BUILD = HERE / "_build"
OUT_DIR = HERE / "src" / "colabfold_legacy_kernels" / "kernels" / "sm100"
LIB = OUT_DIR / "libcfk_sm100.so"
XLA_LIB = OUT_DIR / "libcfk_xla_sm100.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
# No relocatable device code: ptxas ignores setmaxnreg in relocatable code, so the kernels are
# compiled as one translation unit (csrc/all_kernels.cu includes every kernel source).
NVCC_FLAGS = [
    "-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC",
    "-Xcompiler", "-fvisibility=hidden", "--expt-relaxed-constexpr",
    "-diag-suppress", "177,550",
] + ARCH

# The kernels (one unit including status.cu, layer_norm.cu, attention_fwd.cu, attention_bwd.cu,
# gdp.cu and gate.cu) and the host helpers.  ffi_handlers.cc is built separately (needs the XLA
# headers).
SOURCES = ["host.cpp", "all_kernels.cu"]


def nvcc():
    path = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(path).exists():
        raise SystemExit("build.py: nvcc not found (set $NVCC)")
    return path


def headers():
    # every kernel source is an include of all_kernels.cu, so each is a dependency of it
    return (list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h")) +
            [p for p in CSRC.glob("*.cu") if p.name != "all_kernels.cu"])


def stale(target, deps):
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def compile_one(src, extra, force):
    obj = BUILD / (src.name + ".o")
    deps = [src] + headers() + [Path(__file__)]
    if not force and not stale(obj, deps):
        return obj, None
    cmd = [nvcc()] + NVCC_FLAGS + extra + ["-I", str(INCLUDE), "-I", str(CSRC), "-c", str(src),
                                             "-o", str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        return obj, "nvcc failed for %s\n%s\n%s" % (src.name, " ".join(cmd), r.stderr)
    return obj, None


def link(objs, out, extra_libs=()):
    cmd = [nvcc()] + ARCH + ["-shared", "-cudart", "static",
                             "-Xcompiler", "-static-libstdc++", "-Xcompiler", "-static-libgcc",
                             "-Xlinker", "--exclude-libs,ALL", "-o", str(out)] + [str(o) for o in objs] + list(extra_libs)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise SystemExit("link failed:\n%s\n%s" % (" ".join(cmd), r.stderr))


def build(force=False, jobs=None, verbose=True):
    """Compiles what changed and (re)links the library.  Returns the library path."""
    BUILD.mkdir(parents=True, exist_ok=True)
    OUT_DIR.mkdir(parents=True, exist_ok=True)
    srcs = [CSRC / s for s in SOURCES if (CSRC / s).exists()]
    jobs = jobs or min(len(srcs), os.cpu_count() or 4)
    objs, errors = [], []
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        futs = [ex.submit(compile_one, s, [], force) for s in srcs]
        for f in futs:
            obj, err = f.result()
            objs.append(obj)
            if err:
                errors.append(err)
    if errors:
        raise SystemExit("\n".join(errors))
    if force or stale(LIB, objs):
        link(objs, LIB)
        if verbose:
            print("built", LIB)
    ffi_inc = os.environ.get("FFI_INCLUDE")
    if ffi_inc and (Path(ffi_inc) / "xla" / "ffi" / "api" / "ffi.h").is_file():
        obj, err = compile_one(CSRC / "ffi_handlers.cc", ["-x", "cu", "-I", ffi_inc], force)
        if err:
            raise SystemExit(err)
        link(objs + [obj], XLA_LIB)
        if verbose:
            print("built", XLA_LIB)
    return LIB


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--force", action="store_true", help="rebuild everything")
    ap.add_argument("--jobs", type=int, default=None)
    args = ap.parse_args(argv)
    build(force=args.force, jobs=args.jobs)


if __name__ == "__main__":
    sys.exit(main())
