"""Builds the legacy comparator -- TEST INFRASTRUCTURE, not part of the product.

    python oracle/legacy_ref/build.py [--force]

Compiles the reference's kernel sources (cuda/*.cu of sokrypton/colabfold-legacy-kernels) where
they lie under the reference checkout, for sm_100a, into oracle/_ref/liblegacy_*.so.  Each
library wraps one reference file: a wrapper in this directory #includes the source file and
exports a C function that calls the reference's own handler body (VoltaMmaImpl, VoltaWmmaImpl,
LayerNormImpl, GdpImpl, GdpWmmaImpl) on raw device pointers.  The XLA FFI header the sources
include is absent here, so xla/ffi/api/ffi.h in this directory stands in for it at compile time
(it declares only the few types the handler bodies use).  The reference's CUTLASS dependency
(pinned v3.5.1, header-only, not vendored by the reference) is taken from the CUTLASS headers
that ship inside the installed flashinfer package; the reference uses only its
cutlass::arch::Mma<16,8,8> wrapper around mma.sync, which that version provides unchanged.

The libraries are fp16 forward kernels with mma.sync / wmma tensor-core code; they run on a
B200 like any sm_75+ code.  tests/golden/make_golden.py runs them on a GPU to produce the
golden vectors that pin the CPU oracle.  Nothing in the product links or loads them.
"""

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
OUT = REPO / "oracle" / "_ref"


def reference_dir():
    """The reference checkout: $CFK_REFERENCE, else the `reference_path` that BASELINE.json at
    the repository root names; None when neither is set or the directory is absent."""
    path = os.environ.get("CFK_REFERENCE")
    if not path:
        try:
            import json
            path = json.loads((REPO / "BASELINE.json").read_text()).get("reference_path")
        except (OSError, ValueError):
            path = None
    if path and Path(path).is_dir():
        return Path(path)
    return None


REFERENCE = reference_dir()

# wrapper -> reference source it includes
UNITS = {
    "legacy_mma_attn.cu": "volta_mma_attn.cu",
    "legacy_wmma_attn.cu": "volta_wmma_attn.cu",
    "legacy_ops.cu": "volta_ops.cu",
    "legacy_gdp_wmma.cu": "volta_gdp_wmma.cu",
}


def cutlass_include():
    env = os.environ.get("CUTLASS_INCLUDE")
    if env and (Path(env) / "cutlass" / "cutlass.h").is_file():
        return Path(env)
    try:
        import flashinfer  # noqa: F401  (only to locate its data directory)
        base = Path(flashinfer.__file__).resolve().parent
    except Exception:  # flashinfer missing or failing to import: search site-packages
        base = None
        for p in sys.path:
            cand = Path(p) / "flashinfer"
            if (cand / "data" / "cutlass" / "include").is_dir():
                base = cand
                break
    if base is not None:
        inc = base / "data" / "cutlass" / "include"
        if (inc / "cutlass" / "cutlass.h").is_file():
            return inc
    raise SystemExit("legacy_ref: CUTLASS headers not found (set $CUTLASS_INCLUDE)")


def nvcc():
    return os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"


def build(force=False, verbose=True):
    """Builds the libraries when the reference checkout is present; returns their paths."""
    cuda_dir = REFERENCE / "cuda" if REFERENCE is not None else None
    if cuda_dir is None or not cuda_dir.is_dir():
        if verbose:
            print("legacy_ref: no reference checkout ($CFK_REFERENCE or BASELINE.json "
                  "reference_path); skipped")
        return []
    OUT.mkdir(parents=True, exist_ok=True)
    inc = cutlass_include()
    built = []
    for wrapper, src in UNITS.items():
        lib = OUT / ("lib" + wrapper.replace(".cu", ".so"))
        deps = [HERE / wrapper, HERE / "legacy_common.h", HERE / "xla" / "ffi" / "api" / "ffi.h",
                cuda_dir / src, Path(__file__)]
        if not force and lib.exists() and all(d.stat().st_mtime <= lib.stat().st_mtime
                                              for d in deps):
            built.append(lib)
            continue
        cmd = [nvcc(), "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17",
               "-shared", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
               "-cudart", "static", "-diag-suppress", "177,550,20012,20013,20014,20015",
               "-I", str(HERE), "-I", str(cuda_dir), "-I", str(inc),
               str(HERE / wrapper), "-o", str(lib)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise SystemExit("legacy_ref: nvcc failed for %s\n%s\n%s" % (wrapper, " ".join(cmd),
                                                                       r.stderr[-4000:]))
        if verbose:
            print("built", lib)
        built.append(lib)
    return built


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--force", action="store_true")
    args = ap.parse_args(argv)
    build(force=args.force)


if __name__ == "__main__":
    main()
