"""The Python locator keeps the reference's semantics (src/colabfold_legacy_kernels/__init__.py:
5-92 and the CI smoke test .github/workflows/build-and-publish.yml:72-90), extended with cc 100.
"""

import ctypes
from pathlib import Path

import pytest

import colabfold_legacy_kernels as clk


@pytest.fixture
def fake_kernels(tmp_path, monkeypatch):
    """A kernel directory with empty files standing in for the libraries."""
    for cc, libs in {70: ["libvolta_wmma.so", "libvolta_ops.so", "libvolta_gdp_wmma.so"],
                     75: ["libvolta_mma.so", "libvolta_ops.so"],
                     100: ["libcfk_xla_sm100.so"]}.items():
        d = tmp_path / ("sm%d" % cc)
        d.mkdir()
        for lib in libs:
            (d / lib).write_bytes(b"")
    monkeypatch.setattr(clk, "_KERNEL_DIR", tmp_path)
    return tmp_path


def test_public_names():
    assert set(clk.__all__) >= {"KERNELS", "available", "kernel_dir", "library_path",
                                "supported_capabilities", "symbol"}
    assert clk.KERNELS[:3] == ("attention", "layer_norm", "gated_dual_proj")
    assert clk.supported_capabilities() == (70, 75, 100)


def test_unknown_kernel_is_keyerror():
    with pytest.raises(KeyError):
        clk.symbol("softmax", 75)
    with pytest.raises(KeyError):
        clk.library_path("softmax", 100)


def test_symbols_per_capability():
    assert clk.symbol("attention", 75) == "VoltaMma"
    assert clk.symbol("attention", 70) == "VoltaWmma"
    assert clk.symbol("gated_dual_proj", 70) == "VoltaGdpWmma"
    assert clk.symbol("gated_dual_proj", 75) == "VoltaGdp"
    assert clk.symbol("layer_norm", 75) == "VoltaLayerNorm"
    # sm_100: the same handler names as the reference, so registration is unchanged
    assert clk.symbol("attention", 100) == "VoltaMma"
    assert clk.symbol("layer_norm", 100) == "VoltaLayerNorm"
    assert clk.symbol("gated_dual_proj", 100) == "VoltaGdp"
    assert clk.symbol("attention_bwd", 100) == "CfkAttentionBwd"


def test_unsupported_capabilities():
    for cc in (80, 86, 90, 103, 120):
        with pytest.raises(FileNotFoundError):
            clk.symbol("attention", cc)
        assert not clk.available(cc)
    # the new kernels exist for cc 100 only
    with pytest.raises(FileNotFoundError):
        clk.symbol("attention_bwd", 75)


def test_missing_library_is_filenotfound(tmp_path, monkeypatch):
    monkeypatch.setattr(clk, "_KERNEL_DIR", tmp_path)
    with pytest.raises(FileNotFoundError):
        clk.library_path("attention", 100)
    assert not clk.available(100)
    assert not clk.available(75, "attention")


def test_available_and_paths(fake_kernels):
    assert clk.available(70) and clk.available(75) and clk.available(100)
    assert not clk.available(80), "sm_80 must fall back to Pallas"
    assert clk.library_path("attention", 100) == str(fake_kernels / "sm100" / "libcfk_xla_sm100.so")
    assert clk.library_path("layer_norm", 75) == str(fake_kernels / "sm75" / "libvolta_ops.so")
    assert clk.kernel_dir(100) == str(fake_kernels / "sm100")
    # the CI smoke-test loop: skip what a capability does not have
    for cc in (70, 75, 100):
        for kernel in clk.KERNELS:
            if not clk.available(cc, kernel):
                continue
            assert Path(clk.library_path(kernel, cc)).is_file()
            assert isinstance(clk.symbol(kernel, cc), str)


def test_kernel_dir_unknown_capability_like_reference():
    # The reference returns a path for any integer cc without checking it exists.
    assert clk.kernel_dir(80).endswith("sm80")
