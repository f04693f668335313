"""ColabFold Evoformer CUDA kernels: sm_70 and sm_75 (legacy) and sm_100a (B200).

Drop-in for sokrypton/colabfold-legacy-kernels' locator module
(src/colabfold_legacy_kernels/__init__.py:1-92): the same names, arguments, return values and
exceptions, extended with compute capability 100.

    import colabfold_legacy_kernels as clk
    clk.available(cc=100)                  # True if the sm_100 libraries are present
    clk.library_path("attention", cc=100)  # shared library to load
    clk.symbol("attention", cc=100)        # XLA FFI target name to register ("VoltaMma")

For cc=100 the FFI handlers live in libcfk_xla_sm100.so, which is built when the XLA FFI
headers of a jax >= 0.6.2 wheel are available ($FFI_INCLUDE).  The kernels themselves, behind
the C ABI of include/cfk.h, are in libcfk_sm100.so (c_library_path(100)).
"""

from pathlib import Path

__all__ = [
    "KERNELS",
    "available",
    "c_library_path",
    "kernel_dir",
    "library_path",
    "supported_capabilities",
    "symbol",
]

__version__ = "0.3.0"

_KERNEL_DIR = Path(__file__).resolve().parent / "kernels"

_CAPABILITIES = (70, 75, 100)

# Each kernel lists its libraries from the highest compute capability first.  sm_100a code runs
# on compute capability 10.0 only, so cc 100 is an exact match, never a lower bound for newer
# parts (cc 103, 120 stay unavailable).
_TABLE = {
    "attention": (
        (100, "libcfk_xla_sm100.so", "VoltaMma"),
        (75, "libvolta_mma.so", "VoltaMma"),
        (70, "libvolta_wmma.so", "VoltaWmma"),
    ),
    "layer_norm": (
        (100, "libcfk_xla_sm100.so", "VoltaLayerNorm"),
        (70, "libvolta_ops.so", "VoltaLayerNorm"),
    ),
    "gated_dual_proj": (
        (100, "libcfk_xla_sm100.so", "VoltaGdp"),
        (75, "libvolta_ops.so", "VoltaGdp"),
        (70, "libvolta_gdp_wmma.so", "VoltaGdpWmma"),
    ),
    # New capability of the sm_100 build: forward with residuals (out, lse) and the backwards.
    "attention_fwd_res": (
        (100, "libcfk_xla_sm100.so", "CfkAttentionFwdRes"),
    ),
    "attention_bwd": (
        (100, "libcfk_xla_sm100.so", "CfkAttentionBwd"),
    ),
    "layer_norm_bwd": (
        (100, "libcfk_xla_sm100.so", "CfkLayerNormBwd"),
    ),
    "gated_dual_proj_bwd": (
        (100, "libcfk_xla_sm100.so", "CfkGdpBwd"),
    ),
}

# Kernels whose libraries every capability must have for available(cc) to hold.
_CORE = ("attention", "layer_norm", "gated_dual_proj")

KERNELS = tuple(_TABLE)


def supported_capabilities():
    """Give the compute capabilities that this package contains."""
    return _CAPABILITIES


def _resolve(kernel, cc):
    """Find the library and the FFI symbol for one kernel and one capability."""
    if kernel not in _TABLE:
        raise KeyError(
            "unknown kernel %r, expected one of %s" % (kernel, ", ".join(KERNELS)))
    cc = int(cc)
    if cc not in _CAPABILITIES:
        return cc, None, None
    for min_cc, lib, sym in _TABLE[kernel]:
        if min_cc == 100:
            if cc == 100:
                return cc, lib, sym
            continue
        if cc >= min_cc and cc < 100:
            return cc, lib, sym
    return cc, None, None


def kernel_dir(cc):
    """Give the directory of the libraries for one capability."""
    cc, _, _ = _resolve("attention", cc)
    return str(_KERNEL_DIR / ("sm%d" % cc))


def library_path(kernel, cc):
    """Give the path of the library that supplies one kernel."""
    cc, lib, _ = _resolve(kernel, cc)
    if lib is None:
        raise FileNotFoundError(
            "no %s kernel for compute capability %d" % (kernel, cc))
    path = _KERNEL_DIR / ("sm%d" % cc) / lib
    if not path.is_file():
        raise FileNotFoundError("%s is not in this package" % path)
    return str(path)


def symbol(kernel, cc):
    """Give the XLA FFI target name that the library exports."""
    cc, lib, sym = _resolve(kernel, cc)
    if sym is None:
        raise FileNotFoundError(
            "no %s kernel for compute capability %d" % (kernel, cc))
    return sym


def available(cc, kernel=None):
    """Tell if the kernels are present. With kernel=None, test all of them."""
    names = _CORE if kernel is None else (kernel,)
    for name in names:
        try:
            library_path(name, cc)
        except (FileNotFoundError, KeyError):
            return False
    return True


def c_library_path(cc=100):
    """Give the path of the library with the C ABI of include/cfk.h (cc 100 only)."""
    if int(cc) != 100:
        raise FileNotFoundError("the C ABI library exists for compute capability 100 only")
    path = _KERNEL_DIR / "sm100" / "libcfk_sm100.so"
    if not path.is_file():
        raise FileNotFoundError("%s is not in this package (run build.py)" % path)
    return str(path)
