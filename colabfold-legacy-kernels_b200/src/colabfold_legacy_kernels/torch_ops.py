"""PyTorch helpers over the C ABI: allocate outputs, pass device pointers and the current
stream, and call the sm_100a kernels.  There is no fallback: a missing library or a non-B200
device raises.

These exist for tests, benchmarks and PyTorch users; XLA users go through the FFI handlers.
"""

import os

import ctypes

import torch

from . import cabi

# Opt-in checking of the device status word after every call (CFK_CHECK_STATUS=1): each call
# then synchronises its device and raises CfkError if a kernel wait gave up, whose outputs are
# undefined.  Off by default, since the synchronisation serialises the host with the GPU.
CHECK_STATUS = os.environ.get("CFK_CHECK_STATUS", "") not in ("", "0")


def check_status(device=None):
    """Synchronises `device` and raises CfkError if a kernel wait on it gave up since the
    status word was last cleared (cabi.clear_device_status)."""
    with torch.cuda.device(device):
        torch.cuda.synchronize()
        code = cabi.device_status()
    if code:
        raise cabi.CfkError("cfk_device_status", cabi.CFK_ERR_LAUNCH,
                            "a kernel wait gave up (status word %d); outputs since then are "
                            "undefined" % code)


def _done(device):
    if CHECK_STATUS:
        check_status(device)

_DTYPES = {torch.float16: cabi.CFK_F16, torch.bfloat16: cabi.CFK_BF16}


def _dtype_code(t):
    try:
        return _DTYPES[t.dtype]
    except KeyError:
        raise TypeError("expected a float16 or bfloat16 tensor, got %s" % t.dtype) from None


def _ptr(t):
    return None if t is None else t.data_ptr()


def _stream(device):
    return torch.cuda.current_stream(device).cuda_stream


def _check(*ts):
    for t in ts:
        if t is not None:
            if not t.is_cuda:
                raise ValueError("tensors must be on a CUDA device")
            if not t.is_contiguous():
                raise ValueError("tensors must be contiguous")


def _check_rows(*ts):
    """[N,H,S,D] tensors may be views (any strides with a contiguous D axis): a transposed
    residue axis or a [N,S,H,D] layout is passed to the kernels as strides, not copied."""
    for t in ts:
        if not t.is_cuda:
            raise ValueError("tensors must be on a CUDA device")
        if t.dim() != 4 or (t.stride(3) != 1 and t.shape[3] > 1):
            raise ValueError("q/k/v/out/dout and their gradients must be [N,H,S,D] with a "
                             "contiguous D axis")


def _strided(ts):
    """None if every tensor is packed, else the cfk_view array of their strides."""
    if all(t.is_contiguous() for t in ts):
        return None
    return cabi.views(*[t.stride()[:3] for t in ts])


def attention_fwd(q, k, v, bias, kmask, scale, return_lse=True, out=None, lse=None):
    """out [N,H,Sq,D] (and lse f32 [N,H,Sq]) of attention with pair bias and key mask.

    q, k, v and `out` may be strided views (cfk_attn_fwd_strided), e.g. x.permute(1, 2, 0, 3)
    of a [S, N, H, D] tensor for attention over its first axis."""
    _check(bias, kmask)
    n, h, sq, d = q.shape
    sk = k.shape[2]
    if out is None:
        out = torch.empty((n, h, sq, d), dtype=q.dtype, device=q.device)
    _check_rows(q, k, v, out)
    if return_lse and lse is None:
        lse = torch.empty((n, h, sq), dtype=torch.float32, device=q.device)
    args = (_stream(q.device), _dtype_code(q), _ptr(q), _ptr(k), _ptr(v), _ptr(bias),
            _ptr(kmask), _ptr(out), _ptr(lse) if return_lse else None, n, h, sq, sk, d,
            float(scale))
    views = _strided((q, k, v, out))
    with torch.cuda.device(q.device):
        if views is None:
            cabi.call("cfk_attn_fwd", *args)
        else:
            cabi.call("cfk_attn_fwd_strided", *args, views)
    _done(q.device)
    return (out, lse) if return_lse else out


def attention_bwd_workspace(n, h, sq, sk, d, device):
    nbytes = cabi.workspace_size("cfk_attn_bwd_workspace_size", n, h, sq, sk, d)
    return torch.empty(max(nbytes, 16), dtype=torch.uint8, device=device)


def attention_bwd(q, k, v, bias, kmask, out, lse, dout, scale, workspace=None, grads=None,
                  phase=None):
    """(dq, dk, dv, dbias) of attention_fwd; dbias is f32 [H,Sq,Sk].

    phase=None runs the whole backward; phase 0, 1 or 2 runs one of its launches
    (cfk_attn_bwd_phase), in which case `workspace` and `grads` must be passed to every phase.
    q, k, v, out, dout and dq, dk, dv may be strided [N,H,S,D] views (cfk_attn_bwd_strided).
    """
    _check(bias, kmask, lse)
    n, h, sq, d = q.shape
    sk = k.shape[2]
    if grads is None:
        grads = tuple(torch.empty((n, h, s, d), dtype=q.dtype, device=q.device)
                      for s in (sq, sk, sk)) + (
                          torch.empty((h, sq, sk), dtype=torch.float32, device=q.device),)
    dq, dk, dv, dbias = grads
    _check_rows(q, k, v, out, dout, dq, dk, dv)
    _check(dbias)
    if workspace is None:
        workspace = attention_bwd_workspace(n, h, sq, sk, d, q.device)
    args = (_stream(q.device), _dtype_code(q), _ptr(q), _ptr(k), _ptr(v), _ptr(bias),
            _ptr(kmask), _ptr(out), _ptr(lse), _ptr(dout), _ptr(dq), _ptr(dk), _ptr(dv),
            _ptr(dbias), _ptr(workspace), workspace.numel(), n, h, sq, sk, d, float(scale))
    views = _strided((q, k, v, out, dout, dq, dk, dv))
    with torch.cuda.device(q.device):
        if views is None:
            if phase is None:
                cabi.call("cfk_attn_bwd", *args)
            else:
                cabi.call("cfk_attn_bwd_phase", int(phase), *args)
        elif phase is None:
            cabi.call("cfk_attn_bwd_strided", *args, views)
        else:
            cabi.call("cfk_attn_bwd_phase_strided", int(phase), *args, views)
    _done(q.device)
    return dq, dk, dv, dbias


def layer_norm_fwd(x, gamma, beta, eps, return_stats=False, out=None):
    _check(x, gamma, beta)
    m, c = x.shape
    y = torch.empty_like(x) if out is None else out
    mean = rstd = None
    if return_stats:
        mean = torch.empty(m, dtype=torch.float32, device=x.device)
        rstd = torch.empty(m, dtype=torch.float32, device=x.device)
    with torch.cuda.device(x.device):
        cabi.call("cfk_ln_fwd", _stream(x.device), _dtype_code(x), _ptr(x), _ptr(gamma),
                  _ptr(beta), _ptr(y), _ptr(mean), _ptr(rstd), m, c, float(eps))
    _done(x.device)
    return (y, mean, rstd) if return_stats else y


def layer_norm_bwd(x, gamma, dy, eps, mean=None, rstd=None, workspace=None, grads=None):
    """(dx, dgamma, dbeta); mean/rstd from layer_norm_fwd(return_stats=True) or recomputed.
    `grads` = (dx, dgamma, dbeta) preallocated (contiguous; dgamma, dbeta f32 [C]) or None."""
    _check(x, gamma, dy, mean, rstd)
    m, c = x.shape
    if grads is None:
        dx = torch.empty_like(x)
        dgamma = torch.empty(c, dtype=torch.float32, device=x.device)
        dbeta = torch.empty(c, dtype=torch.float32, device=x.device)
    else:
        dx, dgamma, dbeta = grads
        _check(dx, dgamma, dbeta)
        if dx.shape != x.shape or dgamma.shape != (c,) or dbeta.shape != (c,) or \
                dgamma.dtype != torch.float32 or dbeta.dtype != torch.float32:
            raise ValueError("grads must be dx like x and f32 dgamma, dbeta of shape [C]")
    if workspace is None:
        nbytes = cabi.workspace_size("cfk_ln_bwd_workspace_size", m, c)
        workspace = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=x.device)
    with torch.cuda.device(x.device):
        cabi.call("cfk_ln_bwd", _stream(x.device), _dtype_code(x), _ptr(x), _ptr(gamma),
                  _ptr(mean), _ptr(rstd), _ptr(dy), _ptr(dx), _ptr(dgamma), _ptr(dbeta),
                  _ptr(workspace), workspace.numel(), m, c, float(eps))
    _done(x.device)
    return dx, dgamma, dbeta


def gdp_fwd(x, wp, bp, wg, bg, mask, out=None):
    """mask[:,None] * (x@wp + bp) * sigmoid(x@wg + bg)."""
    _check(x, wp, bp, wg, bg, mask)
    m, k = x.shape
    n = wp.shape[1]
    if out is None:
        out = torch.empty((m, n), dtype=x.dtype, device=x.device)
    with torch.cuda.device(x.device):
        cabi.call("cfk_gdp_fwd", _stream(x.device), _dtype_code(x), _ptr(x), _ptr(wp), _ptr(bp),
                  _ptr(wg), _ptr(bg), _ptr(mask), _ptr(out), m, k, n)
    _done(x.device)
    return out


def ln_gdp_fwd(z, gamma, beta, eps, wp, bp, wg, bg, mask, out=None, return_stats=False,
               workspace=None):
    """gdp_fwd(layer_norm_fwd(z, gamma, beta, eps), wp, bp, wg, bg, mask) in one kernel where the
    shape allows (cfk_ln_gdp_fwd); with return_stats also the LayerNorm mean and rstd."""
    _check(z, gamma, beta, wp, bp, wg, bg, mask)
    m, k = z.shape
    n = wp.shape[1]
    if out is None:
        out = torch.empty((m, n), dtype=z.dtype, device=z.device)
    mean = rstd = None
    if return_stats:
        mean = torch.empty(m, dtype=torch.float32, device=z.device)
        rstd = torch.empty(m, dtype=torch.float32, device=z.device)
    if workspace is None:
        nbytes = cabi.workspace_size("cfk_ln_gdp_fwd_workspace_size", m, k, n)
        workspace = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=z.device)
    with torch.cuda.device(z.device):
        cabi.call("cfk_ln_gdp_fwd", _stream(z.device), _dtype_code(z), _ptr(z), _ptr(gamma),
                  _ptr(beta), float(eps), _ptr(wp), _ptr(bp), _ptr(wg), _ptr(bg), _ptr(mask),
                  _ptr(out), _ptr(mean), _ptr(rstd), _ptr(workspace), workspace.numel(), m, k, n)
    _done(z.device)
    return (out, mean, rstd) if return_stats else out


def gdp_bwd(x, wp, bp, wg, bg, mask, dout, workspace=None, grads=None):
    """(dx, dwp, dbp, dwg, dbg); weight and bias gradients in f32.  `grads` = those five
    preallocated (contiguous; f32 [K,N], [N], [K,N], [N] for the parameter gradients) or None."""
    _check(x, wp, bp, wg, bg, mask, dout)
    m, k = x.shape
    n = wp.shape[1]
    if grads is None:
        dx = torch.empty_like(x)
        dwp = torch.empty((k, n), dtype=torch.float32, device=x.device)
        dwg = torch.empty((k, n), dtype=torch.float32, device=x.device)
        dbp = torch.empty(n, dtype=torch.float32, device=x.device)
        dbg = torch.empty(n, dtype=torch.float32, device=x.device)
    else:
        dx, dwp, dbp, dwg, dbg = grads
        _check(dx, dwp, dbp, dwg, dbg)
        if dx.shape != x.shape or dwp.shape != (k, n) or dwg.shape != (k, n) or \
                dbp.shape != (n,) or dbg.shape != (n,) or \
                any(t.dtype != torch.float32 for t in (dwp, dbp, dwg, dbg)):
            raise ValueError("grads must be dx like x and f32 dwp, dbp, dwg, dbg")
    if workspace is None:
        nbytes = cabi.workspace_size("cfk_gdp_bwd_workspace_size", m, k, n)
        workspace = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=x.device)
    with torch.cuda.device(x.device):
        cabi.call("cfk_gdp_bwd", _stream(x.device), _dtype_code(x), _ptr(x), _ptr(wp), _ptr(bp),
                  _ptr(wg), _ptr(bg), _ptr(mask), _ptr(dout), _ptr(dx), _ptr(dwp), _ptr(dbp),
                  _ptr(dwg), _ptr(dbg), _ptr(workspace), workspace.numel(), m, k, n)
    _done(x.device)
    return dx, dwp, dbp, dwg, dbg


def _row_stride(t):
    """Row stride of a 2-D tensor whose rows may be strided (a column block of a wider buffer,
    e.g. q of a [M, 3*H*D] projection): the last axis must be contiguous."""
    if not t.is_cuda:
        raise ValueError("tensors must be on a CUDA device")
    if t.dim() != 2 or (t.stride(1) != 1 and t.shape[1] > 1):
        raise ValueError("expected a 2-D tensor with a contiguous last axis")
    return t.stride(0) if t.shape[0] > 1 else t.shape[1]


def linear_fwd(x, w, b=None, out=None):
    """y = x w + b (cfk_linear_fwd): x [M,K], w [K,N] contiguous, b [N] or None, 16-bit.
    out: None (a new [M,N] tensor), one [M,N] tensor whose rows may be strided, or a pair
    (y0 [M, n0], y1 [M, N - n0]) of such tensors (n0 a multiple of 128) that receive columns
    [0, n0) and [n0, N).  Returns out (the pair when a pair was given)."""
    _check(x, w, b)
    m, k = x.shape
    n = w.shape[1]
    if w.shape[0] != k or (b is not None and b.shape != (n,)):
        raise ValueError("x [M,K], w [K,N], b [N]")
    if out is None:
        out = torch.empty((m, n), dtype=x.dtype, device=x.device)
    pair = isinstance(out, (tuple, list))
    y0, y1 = (out[0], out[1]) if pair else (out, None)
    n0 = y0.shape[1]
    if y0.shape[0] != m or (y1 is None and n0 != n) or \
            (y1 is not None and (y1.shape != (m, n - n0))):
        raise ValueError("out must cover [M, N]")
    ld0 = _row_stride(y0)
    ld1 = _row_stride(y1) if y1 is not None else 0
    with torch.cuda.device(x.device):
        cabi.call("cfk_linear_fwd", _stream(x.device), _dtype_code(x), _ptr(x), _ptr(w), _ptr(b),
                  _ptr(y0), ld0, _ptr(y1), ld1, n0, m, k, n)
    _done(x.device)
    return out


def linear_bwd_dx(dys, ws, out=None):
    """dx = sum_s dys[s] ws[s]^T (cfk_linear_bwd_dx): dys [M, n_s] (rows may be strided),
    ws [K, n_s] contiguous; dx [M, K] in their dtype."""
    if not 1 <= len(dys) == len(ws) <= 4:
        raise ValueError("1 to 4 (dy, w) blocks")
    _check(*ws)
    m = dys[0].shape[0]
    k = ws[0].shape[0]
    segs = []
    for dy, w in zip(dys, ws):
        if dy.shape[0] != m or w.shape != (k, dy.shape[1]) or dy.dtype != ws[0].dtype:
            raise ValueError("dy_s [M, n_s] and w_s [K, n_s] of one dtype")
        segs.append((_ptr(dy), _row_stride(dy), dy.shape[1], _ptr(w), None, None))
    dx = torch.empty((m, k), dtype=dys[0].dtype, device=dys[0].device) if out is None else out
    _check(dx)
    with torch.cuda.device(dx.device):
        cabi.call("cfk_linear_bwd_dx", _stream(dx.device), _dtype_code(dx),
                  cabi.linear_segs(*segs), len(segs), _ptr(dx), m, k)
    _done(dx.device)
    return dx


def linear_bwd_dw(x, dys, with_bias, grads=None, workspace=None):
    """[(dw_s, db_s)] with dw_s = x^T dys[s] and db_s = the column sums of dys[s] (None where
    with_bias[s] is false), f32 (cfk_linear_bwd_dw); x [M,K] contiguous is read once.  grads:
    preallocated [(dw_s, db_s)] or None."""
    _check(x)
    m, k = x.shape
    if not 1 <= len(dys) == len(with_bias) <= 4:
        raise ValueError("1 to 4 dy blocks")
    if grads is None:
        grads = [(torch.empty((k, dy.shape[1]), dtype=torch.float32, device=x.device),
                  torch.empty(dy.shape[1], dtype=torch.float32, device=x.device) if wb else None)
                 for dy, wb in zip(dys, with_bias)]
    segs = []
    for dy, (dw, db) in zip(dys, grads):
        _check(dw, db)
        if dy.shape[0] != m or dw.shape != (k, dy.shape[1]) or dw.dtype != torch.float32:
            raise ValueError("dy_s [M, n_s], dw_s f32 [K, n_s]")
        segs.append((_ptr(dy), _row_stride(dy), dy.shape[1], None, _ptr(dw), _ptr(db)))
    arr = cabi.linear_segs(*segs)
    with torch.cuda.device(x.device):
        if workspace is None:
            nbytes = ctypes.c_size_t(0)
            cabi.call("cfk_linear_bwd_dw_workspace_size", arr, len(segs), m, k,
                      ctypes.byref(nbytes))
            workspace = torch.empty(max(int(nbytes.value), 16), dtype=torch.uint8,
                                    device=x.device)
        cabi.call("cfk_linear_bwd_dw", _stream(x.device), _dtype_code(x), _ptr(x), arr,
                  len(segs), m, k, _ptr(workspace), workspace.numel())
    _done(x.device)
    return grads


def gate_fwd(g, o, out=None):
    """sigmoid(g) * o in one pass (cfk_gate_fwd); g, o contiguous 16-bit tensors of one shape."""
    _check(g, o)
    if g.shape != o.shape or g.dtype != o.dtype:
        raise ValueError("g and o must have the same shape and dtype")
    y = torch.empty_like(o) if out is None else out
    with torch.cuda.device(g.device):
        cabi.call("cfk_gate_fwd", _stream(g.device), _dtype_code(g), _ptr(g), _ptr(o), _ptr(y),
                  g.numel())
    _done(g.device)
    return y


def gate_bwd(g, o, dy):
    """(d_o, dg) of gate_fwd in one pass (cfk_gate_bwd)."""
    _check(g, o, dy)
    if not (g.shape == o.shape == dy.shape) or not (g.dtype == o.dtype == dy.dtype):
        raise ValueError("g, o and dy must have the same shape and dtype")
    d_o, dg = torch.empty_like(o), torch.empty_like(g)
    with torch.cuda.device(g.device):
        cabi.call("cfk_gate_bwd", _stream(g.device), _dtype_code(g), _ptr(g), _ptr(o), _ptr(dy),
                  _ptr(d_o), _ptr(dg), g.numel())
    _done(g.device)
    return d_o, dg
