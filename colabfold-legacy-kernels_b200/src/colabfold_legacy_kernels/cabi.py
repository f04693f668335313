"""ctypes binding of the C ABI in include/cfk.h (libcfk_sm100.so).

This is the binding a maintainer would add on the Python side of the reference to call the
kernels without XLA; the torch helpers in `torch_ops` and the tests go through it.  Every
function raises CfkError with the library's message when the call fails.
"""

import ctypes
import threading

from . import c_library_path

CFK_F16 = 0
CFK_BF16 = 1

CFK_OK = 0
CFK_ERR_INVALID_ARGUMENT = 1
CFK_ERR_UNSUPPORTED_DEVICE = 2
CFK_ERR_LAUNCH = 3

_STATUS_NAMES = {
    CFK_ERR_INVALID_ARGUMENT: "invalid argument",
    CFK_ERR_UNSUPPORTED_DEVICE: "unsupported device",
    CFK_ERR_LAUNCH: "launch failure",
}


class CfkError(RuntimeError):
    """A C ABI call returned a nonzero cfk_status."""

    def __init__(self, fn, code, message):
        super().__init__("%s: %s (%d): %s" % (fn, _STATUS_NAMES.get(code, "error"), code, message))
        self.code = code
        self.message = message


_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_f32 = ctypes.c_float
_int = ctypes.c_int
_sz = ctypes.c_size_t



class View(ctypes.Structure):
    """cfk_view: element strides of the batch, head and sequence axes of a [N,H,S,D] tensor."""
    _fields_ = [("b", _i64), ("h", _i64), ("s", _i64)]


def views(*strides):
    """A cfk_view array from (b, h, s) stride triples, for the *_strided entry points."""
    return (View * len(strides))(*[View(*map(int, st)) for st in strides])


_views = ctypes.POINTER(View)


class LinearSeg(ctypes.Structure):
    """cfk_linear_seg: one column block of a projection's output gradient."""
    _fields_ = [("dy", _vp), ("ld", _i64), ("n", _i64), ("w", _vp), ("dw", _vp), ("db", _vp)]


def linear_segs(*segs):
    """A cfk_linear_seg array from (dy, ld, n, w, dw, db) tuples of pointers and sizes."""
    return (LinearSeg * len(segs))(*[LinearSeg(*s) for s in segs])


_segs = ctypes.POINTER(LinearSeg)

# name -> argtypes (restype is int for all but the two string getters and the entries of
# _RESTYPES)
SIGNATURES = {
    "cfk_attn_fwd": [_vp, _int, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                     _i64, _i64, _i64, _i64, _i64, _f32],
    "cfk_attn_bwd_workspace_size": [_i64, _i64, _i64, _i64, _i64, ctypes.POINTER(_sz)],
    "cfk_attn_bwd": [_vp, _int, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                     _vp, _sz, _i64, _i64, _i64, _i64, _i64, _f32],
    "cfk_attn_bwd_phase": [_int, _vp, _int, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                           _vp, _vp, _vp, _sz, _i64, _i64, _i64, _i64, _i64, _f32],
    "cfk_attn_fwd_strided": [_vp, _int, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                             _i64, _i64, _i64, _i64, _i64, _f32, _views],
    "cfk_attn_bwd_strided": [_vp, _int, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                             _vp, _vp, _sz, _i64, _i64, _i64, _i64, _i64, _f32, _views],
    "cfk_attn_bwd_phase_strided": [_int, _vp, _int, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                                   _vp, _vp, _vp, _vp, _vp, _sz, _i64, _i64, _i64, _i64, _i64,
                                   _f32, _views],
    "cfk_gate_fwd": [_vp, _int, _vp, _vp, _vp, _i64],
    "cfk_gate_bwd": [_vp, _int, _vp, _vp, _vp, _vp, _vp, _i64],
    "cfk_ln_fwd": [_vp, _int, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _f32],
    "cfk_ln_bwd_workspace_size": [_i64, _i64, ctypes.POINTER(_sz)],
    "cfk_ln_bwd": [_vp, _int, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _sz, _i64, _i64,
                   _f32],
    "cfk_ln_bwd_noalloc": [_vp, _int, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64,
                           _f32],
    "cfk_gdp_fwd": [_vp, _int, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64],
    "cfk_ln_gdp_fwd_workspace_size": [_i64, _i64, _i64, ctypes.POINTER(_sz)],
    "cfk_ln_gdp_fwd": [_vp, _int, _vp, _vp, _vp, _f32, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                       _vp, _sz, _i64, _i64, _i64],
    "cfk_gdp_bwd_workspace_size": [_i64, _i64, _i64, ctypes.POINTER(_sz)],
    "cfk_gdp_bwd": [_vp, _int, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                    _vp, _sz, _i64, _i64, _i64],
    "cfk_linear_fwd": [_vp, _int, _vp, _vp, _vp, _vp, _i64, _vp, _i64, _i64, _i64, _i64, _i64],
    "cfk_linear_bwd_dx": [_vp, _int, _segs, _int, _vp, _i64, _i64],
    "cfk_linear_bwd_dw_workspace_size": [_segs, _int, _i64, _i64, ctypes.POINTER(_sz)],
    "cfk_linear_bwd_dw": [_vp, _int, _vp, _segs, _int, _i64, _i64, _vp, _sz],
    "cfk_device_status": [ctypes.POINTER(ctypes.c_uint32)],
    "cfk_clear_device_status": [],
    "cfk_set_wait_limit_ns": [ctypes.c_uint64],
    "cfk_get_wait_limit_ns": [ctypes.POINTER(ctypes.c_uint64)],
    "cfk_test_wait_timeout": [_vp, ctypes.c_uint64, _vp],
    "cfk_dbias_exchange_bytes": [_i64, _i64, _i64],
    "cfk_ipc_alloc": [_sz, ctypes.POINTER(_vp), _vp],
    "cfk_ipc_open": [_vp, ctypes.POINTER(_vp)],
    "cfk_ipc_close": [_vp],
    "cfk_ipc_free": [_vp],
    "cfk_dbias_reduce_scatter": [_vp, ctypes.POINTER(_vp), _int, _int, _i64, _i64, _i64, _vp],
}

_RESTYPES = {"cfk_dbias_exchange_bytes": _sz}

CFK_IPC_HANDLE_BYTES = 64  # include/cfk.h

_lib = None
_lock = threading.Lock()


def lib():
    """The loaded library (loaded once)."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                handle = ctypes.CDLL(c_library_path(100))
                handle.cfk_last_error.restype = ctypes.c_char_p
                handle.cfk_last_error.argtypes = []
                handle.cfk_version.restype = ctypes.c_char_p
                handle.cfk_version.argtypes = []
                _lib = handle
    return _lib


_bound = {}


def function(name):
    """The ctypes function `name` of the library with its declared signature."""
    fn = _bound.get(name)
    if fn is None:
        fn = getattr(lib(), name)
        fn.argtypes = SIGNATURES[name]
        fn.restype = _RESTYPES.get(name, ctypes.c_int)
        _bound[name] = fn
    return fn


def call(name, *args):
    """Calls one C ABI function; raises CfkError on a nonzero status."""
    rc = function(name)(*args)
    if rc != CFK_OK:
        msg = lib().cfk_last_error().decode(errors="replace")
        raise CfkError(name, rc, msg)
    return rc


def version():
    return lib().cfk_version().decode()


def workspace_size(name, *dims):
    out = _sz(0)
    call(name, *dims, ctypes.byref(out))
    return int(out.value)


def device_status():
    code = ctypes.c_uint32(0)
    call("cfk_device_status", ctypes.byref(code))
    return int(code.value)


def clear_device_status():
    call("cfk_clear_device_status")


def set_wait_limit_ns(ns):
    """Wait limit of the current device's kernels (cfk_set_wait_limit_ns)."""
    call("cfk_set_wait_limit_ns", int(ns))


def get_wait_limit_ns():
    out = ctypes.c_uint64(0)
    call("cfk_get_wait_limit_ns", ctypes.byref(out))
    return int(out.value)
