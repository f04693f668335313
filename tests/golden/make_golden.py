"""Generates the golden vectors that pin the CPU oracle to the reference's own kernels.

    python tests/golden/make_golden.py [--out DIR]      (needs a GPU and oracle/_ref/)

The reference (sokrypton/colabfold-legacy-kernels) ships no tests or fixtures.  Its kernel
sources are compiled as they lie for sm_100a by oracle/legacy_ref/build.py into
oracle/_ref/liblegacy_*.so; this script runs those kernels through the reference's own handler
bodies (VoltaMmaImpl, VoltaWmmaImpl, LayerNormImpl, GdpImpl, GdpWmmaImpl) on small seeded fp16
inputs and stores inputs and outputs as .npz files, one per case.  tests/test_golden.py then
checks the CPU oracle against them on any machine.  The reference kernels are fp16-only and
forward-only; the backward restatements are pinned through torch.autograd of the pinned
forward (tests/test_oracle.py).

Cases cover the reference's dispatch table (D in {8, 16, 32, 64} with several block shapes),
ragged query tiles, masked keys, a batch row with every key masked, a key count that is not a
multiple of block_k (where the reference pads its last tile; see oracle/attention.py), LayerNorm
with a ragged channel count and the gated dual projection with biases and a 0/1 row mask.
"""

import argparse
import ctypes
import json
import sys
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parents[2]
REF = REPO / "oracle" / "_ref"

# name, kernel, N, H, Sq, Sk, D, block_q, block_k, fully-masked batch row (or -1)
ATTN_CASES = [
    ("attn_mma_d32", "mma", 2, 2, 64, 64, 32, 64, 64, -1),
    ("attn_mma_d16_ragged_q", "mma", 2, 2, 96, 64, 16, 64, 32, 1),
    ("attn_mma_d8", "mma", 2, 1, 64, 64, 8, 32, 32, -1),
    ("attn_mma_d64", "mma", 1, 2, 64, 64, 64, 64, 64, -1),
    ("attn_mma_d32_ragged_k", "mma", 2, 2, 64, 80, 32, 64, 32, -1),
    ("attn_mma_d32_ragged_k_fully_masked", "mma", 2, 1, 32, 80, 32, 32, 32, 0),
    ("attn_wmma_d32", "wmma", 2, 2, 64, 64, 32, 64, 64, -1),
    ("attn_wmma_d8", "wmma", 2, 1, 64, 64, 8, 32, 32, -1),
]
LN_CASES = [("ln_c128", 48, 128), ("ln_c100_ragged", 33, 100)]
GDP_CASES = [("gdp_k128_n64", "mma", 200, 128, 64), ("gdp_k64_n40", "mma", 64, 64, 40),
             ("gdp_wmma_k128_n64", "wmma", 200, 128, 64)]


def _lib(name):
    path = REF / ("liblegacy_%s.so" % name)
    if not path.is_file():
        raise SystemExit("missing %s: run python oracle/legacy_ref/build.py first" % path)
    return ctypes.CDLL(str(path))


def _call(fn, *args):
    msg = ctypes.create_string_buffer(512)
    rc = fn(*args, msg, 512)
    if rc != 0:
        raise RuntimeError("%s failed (%d): %s" % (fn.__name__, rc, msg.value.decode()))


def attention_case(torch, name, kind, N, H, Sq, Sk, D, bq, bk, dead, seed):
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((N, H, Sq, D)).astype(np.float16)
    k = rng.standard_normal((N, H, Sk, D)).astype(np.float16)
    v = rng.standard_normal((N, H, Sk, D)).astype(np.float16)
    bias = rng.standard_normal((H, Sq, Sk)).astype(np.float16)
    kmask = (rng.random((N, Sk)) > 0.2).astype(np.uint8)
    if dead >= 0:
        kmask[dead, :] = 0
    scale = np.float32(1.0 / np.sqrt(D))
    dev = torch.device("cuda:0")
    t = {n: torch.from_numpy(a).to(dev) for n, a in
         (("q", q), ("k", k), ("v", v), ("bias", bias), ("kmask", kmask))}
    out = torch.zeros((N, H, Sq, D), dtype=torch.float16, device=dev)
    lib = _lib("mma_attn" if kind == "mma" else "wmma_attn")
    fn = lib.legacy_volta_mma if kind == "mma" else lib.legacy_volta_wmma
    i64, vp = ctypes.c_int64, ctypes.c_void_p
    fn.argtypes = [vp] * 7 + [i64] * 5 + [ctypes.c_float, i64, i64, ctypes.c_char_p, ctypes.c_int]
    _call(fn, torch.cuda.current_stream().cuda_stream, t["q"].data_ptr(), t["k"].data_ptr(),
          t["v"].data_ptr(), t["bias"].data_ptr(), t["kmask"].data_ptr(), out.data_ptr(),
          N, H, Sq, Sk, D, float(scale), bq, bk)
    torch.cuda.synchronize()
    return dict(q=q, k=k, v=v, bias=bias, kmask=kmask, scale=scale,
                block_k=np.int64(bk), out=out.cpu().numpy())


def ln_case(torch, name, M, C, seed):
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal((M, C)) * 2.0 + 0.5).astype(np.float16)
    gamma = (1.0 + 0.1 * rng.standard_normal(C)).astype(np.float32)
    beta = (0.1 * rng.standard_normal(C)).astype(np.float32)
    eps = np.float32(1e-5)
    dev = torch.device("cuda:0")
    xt, gt, bt = (torch.from_numpy(a).to(dev) for a in (x, gamma, beta))
    out = torch.zeros((M, C), dtype=torch.float16, device=dev)
    fn = _lib("ops").legacy_layer_norm
    i64, vp = ctypes.c_int64, ctypes.c_void_p
    fn.argtypes = [vp] * 5 + [i64, i64, ctypes.c_float, ctypes.c_char_p, ctypes.c_int]
    _call(fn, torch.cuda.current_stream().cuda_stream, xt.data_ptr(), gt.data_ptr(),
          bt.data_ptr(), out.data_ptr(), M, C, float(eps))
    torch.cuda.synchronize()
    return dict(x=x, gamma=gamma, beta=beta, eps=eps, out=out.cpu().numpy())


def gdp_case(torch, name, kind, M, K, N, seed):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((M, K)).astype(np.float16)
    wp = (rng.standard_normal((K, N)) / np.sqrt(K)).astype(np.float16)
    wg = (rng.standard_normal((K, N)) / np.sqrt(K)).astype(np.float16)
    bp = (0.1 * rng.standard_normal(N)).astype(np.float16)
    bg = (0.1 * rng.standard_normal(N)).astype(np.float16)
    mask = (rng.random(M) > 0.25).astype(np.float16)
    dev = torch.device("cuda:0")
    ts = [torch.from_numpy(a).to(dev) for a in (x, wp, bp, wg, bg, mask)]
    out = torch.zeros((M, N), dtype=torch.float16, device=dev)
    lib = _lib("ops" if kind == "mma" else "gdp_wmma")
    fn = lib.legacy_gdp if kind == "mma" else lib.legacy_gdp_wmma
    i64, vp = ctypes.c_int64, ctypes.c_void_p
    fn.argtypes = [vp] * 8 + [i64] * 3 + [ctypes.c_char_p, ctypes.c_int]
    _call(fn, torch.cuda.current_stream().cuda_stream, *[t_.data_ptr() for t_ in ts],
          out.data_ptr(), M, K, N)
    torch.cuda.synchronize()
    return dict(x=x, wp=wp, bp=bp, wg=wg, bg=bg, mask=mask, out=out.cpu().numpy())


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--out", default=str(Path(__file__).resolve().parent))
    args = ap.parse_args(argv)
    import torch
    if not torch.cuda.is_available():
        raise SystemExit("make_golden.py needs a GPU")
    out_dir = Path(args.out)
    out_dir.mkdir(parents=True, exist_ok=True)
    index = {}
    for seed, c in enumerate(ATTN_CASES):
        arrays = attention_case(torch, *c, seed=100 + seed)
        np.savez_compressed(out_dir / (c[0] + ".npz"), **arrays)
        index[c[0]] = {"op": "attention", "kernel": c[1], "block_q": c[7], "block_k": c[8]}
    for seed, c in enumerate(LN_CASES):
        np.savez_compressed(out_dir / (c[0] + ".npz"), **ln_case(torch, *c, seed=200 + seed))
        index[c[0]] = {"op": "layer_norm"}
    for seed, c in enumerate(GDP_CASES):
        np.savez_compressed(out_dir / (c[0] + ".npz"), **gdp_case(torch, *c, seed=300 + seed))
        index[c[0]] = {"op": "gdp", "kernel": c[1]}
    (out_dir / "index.json").write_text(json.dumps(index, indent=1, sort_keys=True) + "\n")
    print("wrote %d cases to %s" % (len(index), out_dir))
    # deviation of the CPU oracle from each case, for choosing the test tolerances
    sys.path.insert(0, str(REPO))
    import compare  # noqa: E402  (tests/golden/compare.py)
    for name in sorted(index):
        print(name, json.dumps(compare.deviation(out_dir / (name + ".npz"),
                                                           index[name])))


if __name__ == "__main__":
    sys.path.insert(0, str(Path(__file__).resolve().parent))
    main()
