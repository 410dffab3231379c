"""Tensor-level wrappers over libcfgpu's block kernels (cf_ew_binary, cf_ew_unary,
cf_ew_where, cf_ew_clamp, cf_ew_any, cf_bmm, cf_conv_*), used by the gbcsr mirror
(constraintflow.gbcsr) and by the general traversal (cfgpu.general).

Operands are CUDA tensors, possibly broadcast views (zero strides); results are new
contiguous tensors.  PyTorch only allocates the memory and supplies the stream.
"""
import ctypes
import operator

import torch

from cfgpu import _lib

_OPS = {operator.add: "add", operator.sub: "sub", operator.mul: "mul", operator.truediv: "truediv",
        operator.ge: "ge", operator.gt: "gt", operator.le: "le", operator.lt: "lt", operator.eq: "eq",
        operator.ne: "ne", operator.and_: "and_", operator.or_: "or_"}
COMPARISONS = (operator.lt, operator.le, operator.eq, operator.ne, operator.gt, operator.ge, operator.and_,
               operator.or_)


# libcfgpu launches made through these wrappers (each wrapper launches one kernel); the
# engine uses it to count the launches a captured CUDA graph replays
LAUNCHES = [0]


def device():
    if not torch.cuda.is_available():
        raise RuntimeError("the gbcsr ops run on a CUDA device only (libcfgpu); no CPU fallback")
    return torch.device("cuda", torch.cuda.current_device())


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _dt(t):
    return _lib.CF_BOOL if t.dtype == torch.bool else _lib.CF_F32


def _geo(t):
    return _lib.i64_array(list(t.shape)), _lib.i64_array(list(t.stride()))


def as_block_tensor(x, dtype=None):
    """A block payload on the device: bool stays bool, every other dtype becomes float32."""
    t = torch.as_tensor(x)
    if dtype is None:
        dtype = torch.bool if t.dtype == torch.bool else torch.float32
    return t.to(device=device(), dtype=dtype)


def scalar_view(value, shape, dtype):
    """A fill value broadcast to `shape` without materialising it (all strides zero)."""
    t = torch.full((), value, dtype=dtype, device=device())   # a fill kernel: no host copy
    return t.expand(*shape) if len(shape) else t


def binary(op, a, b, out_dtype):
    assert a.shape == b.shape, (a.shape, b.shape)
    out = torch.empty(a.shape, dtype=out_dtype, device=a.device)
    if out.numel() == 0:
        return out
    shp, sa = _geo(a)
    _, sb = _geo(b)
    LAUNCHES[0] += 1
    st = _lib.lib.cf_ew_binary(_lib.OPS[_OPS[op]], a.dim(), shp, a.data_ptr(), _dt(a), sa, b.data_ptr(), _dt(b), sb,
                               out.data_ptr(), _dt(out), _stream())
    _lib.check(st, "cf_ew_binary")
    return out


def unary(name, a, out_dtype):
    out = torch.empty(a.shape, dtype=out_dtype, device=a.device)
    if out.numel() == 0:
        return out
    shp, sa = _geo(a)
    LAUNCHES[0] += 1
    st = _lib.lib.cf_ew_unary(_lib.UOPS[name], a.dim(), shp, a.data_ptr(), _dt(a), sa, out.data_ptr(), _dt(out),
                              _stream())
    _lib.check(st, "cf_ew_unary")
    return out


def where(c, y, z):
    out = torch.empty(c.shape, dtype=torch.float32, device=c.device)
    if out.numel() == 0:
        return out
    shp, sc = _geo(c)
    _, sy = _geo(y)
    _, sz = _geo(z)
    LAUNCHES[0] += 1
    st = _lib.lib.cf_ew_where(c.dim(), shp, c.data_ptr(), sc, y.data_ptr(), sy, z.data_ptr(), sz, out.data_ptr(),
                              _lib.CF_F32, _stream())
    _lib.check(st, "cf_ew_where")
    return out


def clamp(a, const, min_true):
    out = torch.empty(a.shape, dtype=torch.float32, device=a.device)
    if out.numel() == 0:
        return out
    shp, sa = _geo(a)
    LAUNCHES[0] += 1
    st = _lib.lib.cf_ew_clamp(a.dim(), shp, a.data_ptr(), sa, float(const), 1 if min_true else 0, out.data_ptr(),
                              _stream())
    _lib.check(st, "cf_ew_clamp")
    return out


def any_nonzero(a):
    if a.numel() == 0:
        return False
    flag = torch.zeros(1, dtype=torch.int32, device=a.device)
    shp, sa = _geo(a)
    LAUNCHES[0] += 1
    st = _lib.lib.cf_ew_any(a.dim(), shp, a.data_ptr(), _dt(a), sa, flag.data_ptr(), _stream())
    _lib.check(st, "cf_ew_any")
    return bool(flag.item())


def signscale(A, p, q, pc, qc):
    """out = A * (A >= 0 ? p : q) column-wise per batch, dc = sum_n A * (A >= 0 ? pc : qc).

    A [nb, M, N] with unit column stride; p, q, pc, qc [nb, N] contiguous (pc / qc may be
    None: 0).  Returns (out [nb, M, N], dc [nb, M])."""
    nb, M, N = A.shape
    if A.stride(2) != 1:
        A = A.contiguous()
    out = torch.empty(nb, M, N, dtype=torch.float32, device=A.device)
    dc = torch.empty(nb, M, dtype=torch.float32, device=A.device)
    vs = [v.contiguous() if v is not None else None for v in (p, q, pc, qc)]
    LAUNCHES[0] += 1
    st = _lib.lib.cf_signscale(nb, M, N, A.data_ptr(), A.stride(0), A.stride(1), vs[0].data_ptr(), vs[1].data_ptr(),
                               vs[2].data_ptr() if vs[2] is not None else None,
                               vs[3].data_ptr() if vs[3] is not None else None, N, out.data_ptr(), dc.data_ptr(),
                               _stream())
    _lib.check(st, "cf_signscale")
    return out, dc


def bmm(A, B, C=None, accumulate=False):
    """C[b] (+)= A[b] @ B[b]; A [nb, M, K], B [nb, K, N] strided views."""
    nb, M, K = A.shape
    N = B.shape[2]
    if C is None:
        C = torch.empty(nb, M, N, dtype=torch.float32, device=A.device)
    LAUNCHES[0] += 1
    st = _lib.lib.cf_bmm(nb, M, N, K, A.data_ptr(), A.stride(0), A.stride(1), A.stride(2), B.data_ptr(),
                         B.stride(0), B.stride(1), B.stride(2), C.data_ptr(), 1 if accumulate else 0, _stream())
    _lib.check(st, "cf_bmm")
    return C


# ---------------------------------------------------------------- gbcsr conv blocks
def conv_geom(K, C, ox, oy, ix, iy, kx, ky, sx, sy, px, py):
    """The geometry of a conv block (cf_conv_geom)."""
    return _lib.CfConvGeom(*[int(v) for v in (K, C, ox, oy, ix, iy, kx, ky, sx, sy, px, py)])


def conv_densify(g, nb, P, p_bs, p_ks, p_ps):
    """[nb, K*ox*oy, C*ix*iy]: the matrix a conv block stands for (cf_conv_densify)."""
    out = torch.empty(nb, g.K * g.ox * g.oy, g.C * g.ix * g.iy, dtype=torch.float32, device=P.device)
    LAUNCHES[0] += 1
    _lib.check(_lib.lib.cf_conv_densify(ctypes.byref(g), nb, P.data_ptr(), p_bs, p_ks, p_ps, out.data_ptr(),
                                        _stream()), "cf_conv_densify")
    return out


def conv_apply(g, nb, per_b, P, pstr, X, xstr, out, ostr):
    """out = M x for nb*per_b images (cf_conv_apply); pstr = (p_bs, p_ks, p_ps),
    xstr = (x_bs, x_ss, x_es), ostr = (o_bs, o_ss, o_rs) in elements."""
    LAUNCHES[0] += 1
    _lib.check(_lib.lib.cf_conv_apply(ctypes.byref(g), nb, per_b, P.data_ptr(), *pstr, X.data_ptr(), *xstr,
                                      out.data_ptr(), *ostr, _stream()), "cf_conv_apply")
    return out


def conv_scale(g, nb, P, pstr, X, x_bs, x_es):
    """[nb, K*ox*oy, C*kx*ky]: patch values times the input values under them (cf_conv_scale)."""
    out = torch.empty(nb, g.K * g.ox * g.oy, g.C * g.kx * g.ky, dtype=torch.float32, device=P.device)
    LAUNCHES[0] += 1
    _lib.check(_lib.lib.cf_conv_scale(ctypes.byref(g), nb, P.data_ptr(), *pstr, X.data_ptr(), x_bs, x_es,
                                      out.data_ptr(), _stream()), "cf_conv_scale")
    return out


def conv_transpose(g, nb, per_b, Y, ystr, W, OH, OW, out, ostr):
    """Transposed convolution of nb*per_b rows (cf_conv_transpose)."""
    LAUNCHES[0] += 1
    _lib.check(_lib.lib.cf_conv_transpose(ctypes.byref(g), nb, per_b, Y.data_ptr(), *ystr, W.data_ptr(), OH, OW,
                                          out.data_ptr(), *ostr, _stream()), "cf_conv_transpose")
    return out
