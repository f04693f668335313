"""The C ABI library, without a GPU: it loads, exports exactly the functions include/cfk.h
declares, depends on the C library only (the reference's ldd audit,
.github/workflows/build-and-publish.yml:53-64), and rejects bad arguments before it touches a
device.
"""

import ctypes
import re
import subprocess
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent


def _declared():
    text = (REPO / "include" / "cfk.h").read_text()
    return sorted(set(re.findall(r"CFK_API\s+[\w\s\*]+?\b(cfk_\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def libpath():
    import colabfold_legacy_kernels as clk
    try:
        return clk.c_library_path(100)
    except FileNotFoundError:
        pytest.fail("libcfk_sm100.so is not built; run colabfold-legacy-kernels_b200/build.py")


def test_header_declares_the_c_abi():
    names = _declared()
    for n in ("cfk_attn_fwd", "cfk_attn_bwd", "cfk_attn_bwd_workspace_size", "cfk_ln_fwd",
              "cfk_ln_bwd", "cfk_ln_bwd_workspace_size", "cfk_gdp_fwd", "cfk_gdp_bwd",
              "cfk_gdp_bwd_workspace_size", "cfk_last_error", "cfk_version",
              "cfk_device_status", "cfk_clear_device_status"):
        assert n in names


def test_library_exports_every_declared_symbol(libpath):
    lib = ctypes.CDLL(libpath)
    missing = [n for n in _declared() if not hasattr(lib, n)]
    assert not missing, "not exported: %s" % missing
    out = subprocess.run(["nm", "-D", "--defined-only", libpath], capture_output=True,
                         text=True).stdout
    exported = {l.split()[-1] for l in out.splitlines() if " T " in l}
    extra = {s for s in exported if not s.startswith("__cudaRegisterLinkedBinary")} - set(_declared())
    assert not extra, "unexpected exports: %s" % sorted(extra)


def test_library_links_libc_only(libpath):
    out = subprocess.run(["ldd", libpath], capture_output=True, text=True).stdout
    assert not re.search(r"libcudart|libstdc\+\+|libgcc_s|libcuda\.so", out), out


def test_signatures_match_binding():
    from colabfold_legacy_kernels import cabi
    assert set(cabi.SIGNATURES) | {"cfk_last_error", "cfk_version"} == set(_declared())


def test_bad_arguments_rejected_without_device(libpath):
    from colabfold_legacy_kernels import cabi
    with pytest.raises(cabi.CfkError) as e:
        cabi.call("cfk_attn_fwd", None, 7, None, None, None, None, None, None, None,
                  1, 1, 1, 1, 32, 1.0)
    assert e.value.code == cabi.CFK_ERR_INVALID_ARGUMENT and "dtype" in e.value.message
    with pytest.raises(cabi.CfkError) as e:
        cabi.call("cfk_attn_fwd", None, cabi.CFK_BF16, None, None, None, None, None, None, None,
                  1, 1, 1, 1, 48, 1.0)
    assert "head dim" in e.value.message
    with pytest.raises(cabi.CfkError) as e:
        cabi.call("cfk_ln_fwd", None, cabi.CFK_BF16, None, None, None, None, None, None,
                  4, 0, 1e-5)
    assert e.value.code == cabi.CFK_ERR_INVALID_ARGUMENT
    assert "sm_100a" in cabi.version()


def test_workspace_queries_need_no_device(libpath):
    from colabfold_legacy_kernels import cabi
    assert cabi.workspace_size("cfk_ln_bwd_workspace_size", 1 << 20, 128) > 0


def test_ln_gdp_fwd_arguments_without_device(libpath):
    """cfk_ln_gdp_fwd: the tcgen05 shapes need no workspace, others stage LayerNorm(z) there;
    bad dtype / eps / null buffers are rejected before any device call."""
    from colabfold_legacy_kernels import cabi
    assert cabi.workspace_size("cfk_ln_gdp_fwd_workspace_size", 1 << 20, 128, 256) == 0
    assert cabi.workspace_size("cfk_ln_gdp_fwd_workspace_size", 1000, 40, 24) == 1000 * 40 * 2
    args = [None] * 12  # z .. rstd, workspace pointers
    with pytest.raises(cabi.CfkError) as e:
        cabi.call("cfk_ln_gdp_fwd", None, 9, None, None, None, 1e-5, *args[:8], None, 0,
                  16, 128, 256)
    assert e.value.code == cabi.CFK_ERR_INVALID_ARGUMENT and "dtype" in e.value.message
    with pytest.raises(cabi.CfkError) as e:
        cabi.call("cfk_ln_gdp_fwd", None, cabi.CFK_BF16, None, None, None, -1.0, *args[:8], None,
                  0, 16, 128, 256)
    assert "eps" in e.value.message
    with pytest.raises(cabi.CfkError) as e:
        cabi.call("cfk_ln_gdp_fwd", None, cabi.CFK_BF16, None, None, None, 1e-5, *args[:8], None,
                  0, 16, 128, 256)
    assert "null buffer" in e.value.message


def test_strided_views_checked_without_device(libpath):
    """cfk_attn_*_strided: strides of axes longer than 1 must be positive multiples of 8
    elements (16-byte row starts for TMA and vector access); axes of extent 1 take any stride.
    The checks run before any device call."""
    from colabfold_legacy_kernels import cabi
    N, H, S, D = 3, 2, 40, 32
    packed = (H * S * D, S * D, D)
    bad = cabi.views(packed, packed, (H * D, D, N * H * D + 4), packed)
    with pytest.raises(cabi.CfkError) as e:
        cabi.call("cfk_attn_fwd_strided", None, cabi.CFK_BF16, None, None, None, None, None,
                  None, None, N, H, S, S, D, 1.0, bad)
    assert e.value.code == cabi.CFK_ERR_INVALID_ARGUMENT
    assert "v sequence stride" in e.value.message
    neg = cabi.views(packed, packed, packed, (0, S * D, D))
    with pytest.raises(cabi.CfkError) as e:
        cabi.call("cfk_attn_fwd_strided", None, cabi.CFK_BF16, None, None, None, None, None,
                  None, None, N, H, S, S, D, 1.0, neg)
    assert "out batch stride" in e.value.message
    # extent-1 axes: any stride passes the view checks (the call then fails on null buffers)
    one = cabi.views(*[(5, 3, D)] * 4)
    with pytest.raises(cabi.CfkError) as e:
        cabi.call("cfk_attn_fwd_strided", None, cabi.CFK_BF16, None, None, None, None, None,
                  None, None, 1, 1, S, S, D, 1.0, one)
    assert "null buffer" in e.value.message
    far = cabi.views(packed, packed, packed, ((1 << 38) - 8, S * D, D))
    with pytest.raises(cabi.CfkError) as e:
        cabi.call("cfk_attn_fwd_strided", None, cabi.CFK_BF16, None, None, None, None, None,
                  None, None, 16, H, S, S, D, 1.0, far)
    assert "past 2^40" in e.value.message
    bwd = cabi.views(*([packed] * 7 + [(H * S * D, S * D, 12)]))
    with pytest.raises(cabi.CfkError) as e:
        cabi.call("cfk_attn_bwd_strided", None, cabi.CFK_BF16, *([None] * 13), 0, N, H, S, S, D,
                  1.0, bwd)
    assert "dv sequence stride" in e.value.message
    with pytest.raises(cabi.CfkError) as e:
        cabi.call("cfk_attn_bwd_phase_strided", 3, None, cabi.CFK_BF16, *([None] * 13), 0, N, H,
                  S, S, D, 1.0, None)
    assert "phase 3" in e.value.message


def test_torch_views_choose_the_strided_entry():
    """torch_ops passes packed tensors to the packed entry points and [N,H,S,D] views (D
    contiguous) as cfk_view strides; the check needs no device."""
    import torch
    from colabfold_legacy_kernels import torch_ops
    x = torch.empty(7, 3, 2, 8)            # stored [S, N, H, D]
    packed = torch.empty(3, 2, 7, 8)
    assert torch_ops._strided([packed, packed]) is None
    v = torch_ops._strided([packed, x.permute(1, 2, 0, 3)])
    assert [(e.b, e.h, e.s) for e in v] == [(112, 56, 8), (16, 8, 48)]


def test_gate_arguments_without_device(libpath):
    """cfk_gate_fwd / cfk_gate_bwd reject a bad dtype, a negative count and unaligned or null
    buffers before any device call; n = 0 is a no-op."""
    from colabfold_legacy_kernels import cabi
    with pytest.raises(cabi.CfkError) as e:
        cabi.call("cfk_gate_fwd", None, 5, None, None, None, 8)
    assert "dtype" in e.value.message
    with pytest.raises(cabi.CfkError) as e:
        cabi.call("cfk_gate_fwd", None, cabi.CFK_BF16, 16, 32, 48, -1)
    assert "negative" in e.value.message
    with pytest.raises(cabi.CfkError) as e:
        cabi.call("cfk_gate_bwd", None, cabi.CFK_BF16, 16, 32, 48, 64, 72 + 2, 8)
    assert "aligned" in e.value.message
    assert cabi.call("cfk_gate_fwd", None, cabi.CFK_BF16, None, None, None, 0) == 0


def test_wait_limit_and_selftest_arguments_without_device(libpath):
    """cfk_set_wait_limit_ns and cfk_test_wait_timeout check their arguments before they touch
    a device."""
    from colabfold_legacy_kernels import cabi
    for bad in (0, 10, 99_999, 600_000_000_001):
        with pytest.raises(cabi.CfkError) as e:
            cabi.set_wait_limit_ns(bad)
        assert e.value.code == cabi.CFK_ERR_INVALID_ARGUMENT and "outside" in e.value.message
    with pytest.raises(cabi.CfkError) as e:
        cabi.call("cfk_test_wait_timeout", None, 5_000_000, None)
    assert e.value.code == cabi.CFK_ERR_INVALID_ARGUMENT and "null" in e.value.message
    with pytest.raises(cabi.CfkError) as e:
        cabi.call("cfk_test_wait_timeout", None, 10 ** 9, ctypes.c_void_p(16))
    assert e.value.code == cabi.CFK_ERR_INVALID_ARGUMENT


def test_noalloc_checks_its_width_before_the_device(libpath):
    from colabfold_legacy_kernels import cabi
    with pytest.raises(cabi.CfkError) as e:
        cabi.call("cfk_ln_bwd_noalloc", None, cabi.CFK_BF16, None, None, None, None, None, None,
                  None, None, 4, 2048, 1e-5)
    assert e.value.code == cabi.CFK_ERR_INVALID_ARGUMENT and "1024" in e.value.message


def test_linear_arguments_without_device(libpath):
    """cfk_linear_fwd / cfk_linear_bwd_dx / cfk_linear_bwd_dw(+_workspace_size) reject bad
    shapes, split points, row strides, segment counts and null buffers before any device
    call; zero rows of the forward and the dx pass are no-ops."""
    from colabfold_legacy_kernels import cabi
    bf = cabi.CFK_BF16
    with pytest.raises(cabi.CfkError) as e:   # N % 8 != 0
        cabi.call("cfk_linear_fwd", None, bf, 16, 32, None, 48, 12, None, 0, 12, 4, 64, 12)
    assert e.value.code == cabi.CFK_ERR_INVALID_ARGUMENT and "N % 8" in e.value.message
    with pytest.raises(cabi.CfkError) as e:   # split not at a multiple of 128
        cabi.call("cfk_linear_fwd", None, bf, 16, 32, None, 48, 100, 64, 156, 100, 4, 64, 256)
    assert "n_split" in e.value.message
    with pytest.raises(cabi.CfkError) as e:   # row stride below the row width
        cabi.call("cfk_linear_fwd", None, bf, 16, 32, None, 48, 8, None, 0, 16, 4, 64, 16)
    assert "row stride" in e.value.message
    with pytest.raises(cabi.CfkError) as e:
        cabi.call("cfk_linear_fwd", None, 7, 16, 32, None, 48, 16, None, 0, 16, 4, 64, 16)
    assert "dtype" in e.value.message
    assert cabi.call("cfk_linear_fwd", None, bf, None, None, None, None, 16, None, 0, 16,
                     0, 64, 16) == 0
    segs = cabi.linear_segs((16, 128, 128, 32, None, None))
    with pytest.raises(cabi.CfkError) as e:   # no segments
        cabi.call("cfk_linear_bwd_dx", None, bf, segs, 0, 48, 4, 64)
    assert "segments" in e.value.message
    with pytest.raises(cabi.CfkError) as e:   # five segments
        cabi.call("cfk_linear_bwd_dx", None, bf, cabi.linear_segs(*[(16, 8, 8, 32, None, None)] * 5),
                  5, 48, 4, 64)
    assert "segments" in e.value.message
    with pytest.raises(cabi.CfkError) as e:   # ld < n
        cabi.call("cfk_linear_bwd_dx", None, bf, cabi.linear_segs((16, 64, 128, 32, None, None)),
                  1, 48, 4, 64)
    assert "ld >= n" in e.value.message
    with pytest.raises(cabi.CfkError) as e:   # no weight for the dx pass
        cabi.call("cfk_linear_bwd_dx", None, bf, cabi.linear_segs((16, 128, 128, None, None, None)),
                  1, 48, 4, 64)
    assert "null" in e.value.message
    assert cabi.call("cfk_linear_bwd_dx", None, bf, segs, 1, None, 0, 64) == 0
    with pytest.raises(cabi.CfkError) as e:   # no dw output for the dw pass
        cabi.call("cfk_linear_bwd_dw", None, bf, 16, segs, 1, 4, 64, None, 0)
    assert "null" in e.value.message
    with pytest.raises(cabi.CfkError) as e:
        cabi.call("cfk_linear_bwd_dw_workspace_size", segs, 1, 4, 64, None)
    assert "null" in e.value.message


def test_dbias_exchange_arguments_without_device(libpath):
    """The peer-memory dbias reduce-scatter and its IPC helpers check their arguments before
    they touch a device; the exchange size is dbias rounded up to 256 bytes plus the 128-byte
    sync block."""
    from colabfold_legacy_kernels import cabi
    size = cabi.function("cfk_dbias_exchange_bytes")
    assert size(4, 768, 768) == 4 * 768 * 768 * 4 + 128
    assert size(1, 3, 4) == 256 + 128
    assert size(0, 8, 8) == 0 and size(4, 1 << 21, 8) == 0
    bufs = (ctypes.c_void_p * 2)(256, 512)
    out = ctypes.c_void_p(4096)
    bad = [
        (None, 2, 0, 4, 8, 8, out),            # no buffers
        (bufs, 2, 0, 4, 8, 8, None),           # no output
        (bufs, 1, 0, 4, 8, 8, out),            # one rank
        (bufs, 9, 0, 4, 8, 8, out),            # more than eight
        (bufs, 2, 2, 4, 8, 8, out),            # rank outside the world
        (bufs, 2, 0, 4, 7, 8, out),            # Sq not a multiple of the world size
        (bufs, 2, 0, 4, 8, 6, out),            # Sk not a multiple of 4
        (bufs, 2, 0, 4, 8, 8, ctypes.c_void_p(4100)),             # out misaligned
        ((ctypes.c_void_p * 2)(256, 300), 2, 0, 4, 8, 8, out),    # buffer misaligned
        ((ctypes.c_void_p * 2)(256, None), 2, 0, 4, 8, 8, out),   # a null buffer
    ]
    for b, world, rank, h, sq, sk, o in bad:
        with pytest.raises(cabi.CfkError) as e:
            cabi.call("cfk_dbias_reduce_scatter", None, b, world, rank, h, sq, sk, o)
        assert e.value.code == cabi.CFK_ERR_INVALID_ARGUMENT, (world, rank, sq, sk)
    for name, args in (("cfk_ipc_alloc", (16, None, None)), ("cfk_ipc_open", (None, None)),
                       ("cfk_ipc_close", (None,)), ("cfk_ipc_free", (None,))):
        with pytest.raises(cabi.CfkError) as e:
            cabi.call(name, *args)
        assert e.value.code == cabi.CFK_ERR_INVALID_ARGUMENT
