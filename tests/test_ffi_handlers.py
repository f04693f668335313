"""The XLA FFI handlers (csrc/ffi_handlers.cc) compiled against a stand-in header (CPU test).

jax is not installed here, so the real XLA FFI header is absent.  tests/ffi_shim/ provides a
stand-in whose handler-definition macro checks at compile time that every binding matches its
handler's parameter list, and a driver that runs scenarios through the handler bodies with
null-data buffers: the handler's own validation answers InvalidArgument (rank, shape, mixed
dtypes, N % 8, the reference's (D, block_q, block_k) table), and a valid call reaches the C ABI,
whose null-buffer check answers -- no device is touched.
"""

import ctypes
import shutil
import subprocess
from pathlib import Path

import pytest

from conftest import REPO

SHIM = REPO / "tests" / "ffi_shim"
CSRC = REPO / "colabfold-legacy-kernels_b200" / "csrc"
LIB = REPO / "colabfold-legacy-kernels_b200" / "src" / "colabfold_legacy_kernels" / "kernels" / \
    "sm100" / "libcfk_sm100.so"

HANDLERS = ["VoltaMma", "VoltaWmma", "VoltaLayerNorm", "VoltaGdp", "VoltaGdpWmma",
            "CfkAttentionFwdRes", "CfkAttentionBwd", "CfkLayerNormBwd", "CfkGdpBwd"]


@pytest.fixture(scope="module")
def driver(tmp_path_factory):
    if not LIB.is_file():
        pytest.fail("build the library first (colabfold-legacy-kernels_b200/build.py)")
    cxx = shutil.which("g++")
    out = tmp_path_factory.mktemp("ffi") / "libffi_check.so"
    cmd = [cxx, "-std=c++17", "-O1", "-shared", "-fPIC", "-fvisibility=hidden",
           "-I", str(SHIM), "-I", str(CSRC), "-I", str(REPO / "include"),
           "-I", "/usr/local/cuda/include", str(SHIM / "ffi_check.cc"), "-o", str(out),
           str(LIB), "-Wl,-rpath," + str(LIB.parent)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-3000:]
    lib = ctypes.CDLL(str(out))
    lib.ffi_check.argtypes = [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_int]
    return lib


def run(lib, name):
    msg = ctypes.create_string_buffer(512)
    code = lib.ffi_check(name.encode(), msg, 512)
    return code, msg.value.decode()


def test_every_handler_symbol_is_bound(driver):
    for h in HANDLERS:
        fn = getattr(driver, h + "_bound")
        assert fn() == 1, h


@pytest.mark.parametrize("name,needle", [
    ("mma_ok", "cfk_attn_fwd: null buffer"),
    ("mma_f16_ok", "cfk_attn_fwd: null buffer"),
    ("wmma_tuple_ok", "cfk_attn_fwd: null buffer"),
    ("fwdres_any_tuple", "cfk_attn_fwd: null buffer"),
    ("attn_bwd_ok", "cfk_attn_bwd: null buffer"),
    ("ln_ok", "cfk_ln_fwd: null buffer"),
    ("ln_bwd_ok", "null"),
    ("gdp_ok", "cfk_gdp_fwd: null buffer"),
    ("gdp_wmma_ok", "cfk_gdp_fwd: null buffer"),
    ("gdp_bwd_ok", "null"),
])
def test_valid_calls_reach_the_c_abi(driver, name, needle):
    code, msg = run(driver, name)
    assert code == 1 and needle in msg, (code, msg)


@pytest.mark.parametrize("name,needle", [
    ("mma_mixed", "F16 or all BF16"),
    ("mma_f32", "F16 or all BF16"),
    ("mma_tuple", "unsupported (D, bq, bk)"),
    ("mma_tuple_wmma_only", "unsupported (D, bq, bk)"),
    ("mma_bias_shape", "bias [H,Sq,Sk]"),
    ("attn_bwd_dbias_shape", "dbias [H,Sq,Sk]"),
    ("ln_rank", "x must be [M,C]"),
    ("ln_mixed", "F16 or BF16"),
    ("gdp_n8", "N must be a multiple of 8"),
    ("gdp_mixed", "F16 or all BF16"),
])
def test_handler_validation(driver, name, needle):
    code, msg = run(driver, name)
    assert code == 1 and needle in msg and "cfk_" not in msg.split(":")[0], (code, msg)
