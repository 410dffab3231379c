"""CPU oracle for the DeepPoly certification hot path (numpy, float32).

TEST INFRASTRUCTURE ONLY.  Only tests/, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of bench.py may import this module,
and only as the checker or as the timed CPU restatement.  The product path
(cfgpu) never imports it and has no CPU fallback.

What it restates.  The reference compiles examples/compiler_examples/deeppoly.cf
into per-layer transformer code (constraintflow/compiler/codeGen.py) that the layer
loop constraintflow/lib/flow_sparse.py:27-228 calls.  On a chain network
(Input, [Linear|Conv, ReLU]*, Linear, property layer) the arithmetic that code
performs is:

* Affine (deeppoly.cf:14-15, 39): the coefficient matrix of layer m starts as
  W_m (per-region property matrix for the appended spec layer) with constant
  b_m.  A backward traversal (priority2 = -layer, deeppoly.cf:10) substitutes one
  earlier layer per while-iteration.  Each substitution is the sign split
  ``clamp(A,0,True)@L + clamp(A,0,False)@U`` (replace_lower/replace_upper,
  deeppoly.cf:6-7, turned into clamps by constraintflow/compiler/optimizations/
  rewrite.py:116) with inner_prod (constraintflow/gbcsr/tensor_ops.py:370) and
  clamp (tensor_ops.py:765); the constant accumulates
  ``((A+@Lc + A-@Uc) + 0) + c`` (tensor_ops.py:616-687 split the stop / not-stop
  parts).  The input layer's L/U are (empty matrix, constant l0 / u0)
  (constraintflow/lib/spec.py:86-104), so the final substitution folds the
  input box into the constant and the bound is that constant.
* Relu (deeppoly.cf:20-24, 41): l' = relu(l), u' = relu(u);
  L' = 1[l+u>=0] x;  U' = x if l>=0, 0 if u<=0, else lam x + mu with
  lam = u/(u-l), mu = -(u*l)/(u-l) (all float32, same operation order).
* Affine substitution of a conv layer is the transposed convolution of the
  coefficient rows (constraintflow/gbcsr/sparse_block.py:839-928, 1364-1730).
* Input box: clip(X -/+ eps, 0, 1) then dataset normalisation (spec.py:21-47).
* Output: Flow.flow returns the property layer's l/u via get_dense, float64
  (constraintflow/gbcsr/sparse_tensor.py:627-654).

Pinned against: the reference's own outputs on the same seeded networks, stored
by tests/golden/gen_golden.py in tests/golden/*.npz.
"""
import numpy as np

F32 = np.float32


# ---------------------------------------------------------------- relaxation
def relu_relax(l, u, force=None, strict=False):
    """DeepPoly ReLU transformer (deeppoly.cf:20-24,41; generated Relu body).

    Returns (l', u', alpha, lam, mu): L' = alpha*x, U' = lam*x + mu.

    ``strict``: the lower slope is 1 where l + u > 0 (relu_n of zid.cf:22 and of the
    custom-stop programs, deeppoly_custom_stop.cf:25) instead of l + u >= 0; the two differ
    only where l + u == 0 exactly.  Their other strict comparisons (compute_upper: l > 0,
    u < 0) give DeepPoly's values: at l == 0 the slope u / (u - l) is 1 and the offset 0,
    at u == 0 both are 0.

    ``force`` = (l_dec, u_dec) optionally supplies the bounds from which the three
    discrete decisions (l>=0, u<=0, l+u>=0) are taken, while the continuous values
    (lam, mu, relu) still come from (l, u).  A test uses it to replay another
    implementation's decisions: those comparisons are discontinuous, so a bound a
    few ulps from a threshold can flip them and every later layer then differs.
    """
    l = l.astype(F32, copy=False)
    u = u.astype(F32, copy=False)
    ld, ud = (l, u) if force is None else (force[0].astype(F32), force[1].astype(F32))
    zero = F32(0.0)
    l_new = np.where(ld >= zero, l, zero).astype(F32)
    u_new = np.where(ud >= zero, u, zero).astype(F32)
    alpha = (((ld + ud) > zero) if strict else ((ld + ud) >= zero)).astype(F32)
    with np.errstate(divide='ignore', invalid='ignore'):
        den = (u - l).astype(F32)
        lam_unst = (u / den).astype(F32)
        mu_unst = (zero - (u * l).astype(F32) / den).astype(F32)
    pos = ld >= zero
    dead = (~pos) & (ud <= zero)
    lam = np.where(pos, F32(1.0), np.where(dead, zero, lam_unst)).astype(F32)
    mu = np.where(pos | dead, zero, mu_unst).astype(F32)
    return l_new, u_new, alpha, lam, mu


# ---------------------------------------------------------------- substitutions
def _split(A):
    zero = F32(0.0)
    return np.maximum(A, zero), np.minimum(A, zero)


def subst_relu(A, c, alpha, lam, mu, lower):
    """Substitute a ReLU layer: A [B,R,n], c [B,R]; per-region vectors [B,n].

    Lower bound: coeff>=0 -> coeff*L (alpha x), else coeff*U (lam x + mu).
    Upper bound: coeff>=0 -> coeff*U, else coeff*L (deeppoly.cf:6-7).
    """
    Ap, An = _split(A)
    if lower:
        A_new = Ap * alpha[:, None, :] + An * lam[:, None, :]
        dc = np.einsum('brn,bn->br', An, mu, dtype=F32)
    else:
        A_new = Ap * lam[:, None, :] + An * alpha[:, None, :]
        dc = np.einsum('brn,bn->br', Ap, mu, dtype=F32)
    return A_new.astype(F32), ((dc + F32(0.0)) + c).astype(F32)


def _conv_T(A, layer):
    """Rows of A over the conv output [.., Cout*OH*OW] -> rows over its input.

    Transposed convolution (the adjoint of the conv forward) computed as a
    col2im scatter: out[:, ci, s*oy+i-p, s*ox+j-p] += sum_co A[:, co, oy, ox] W[co, ci, i, j].
    """
    Cout, Cin, kh, kw = layer.W.shape
    _, OH, OW = layer.out_shape
    _, IH, IW = layer.in_shape
    s, p = layer.stride, layer.pad
    R = A.shape[0]
    Ahw = A.reshape(R, Cout, OH, OW).transpose(0, 2, 3, 1).reshape(R * OH * OW, Cout)
    Hp, Wp = (OH - 1) * s + kh, (OW - 1) * s + kw
    outp = np.zeros((R, max(Hp, IH + p), max(Wp, IW + p), Cin), F32)
    for i in range(kh):
        for j in range(kw):
            contrib = (Ahw @ layer.W[:, :, i, j]).reshape(R, OH, OW, Cin)
            outp[:, i:i + s * (OH - 1) + 1:s, j:j + s * (OW - 1) + 1:s, :] += contrib
    out = outp[:, p:p + IH, p:p + IW, :]
    return np.ascontiguousarray(out.transpose(0, 3, 1, 2)).reshape(R, Cin * IH * IW)


def _conv_bias(layer):
    _, OH, OW = layer.out_shape
    return np.repeat(layer.b.astype(F32), OH * OW)


def layer_bias(layer):
    return _conv_bias(layer) if layer.kind == 'conv' else layer.b.astype(F32)


def apply_affine_T(A2d, layer):
    """A2d [R, n_out] @ W (Linear) or transposed conv (Conv) -> [R, n_in]."""
    if layer.kind == 'conv':
        return _conv_T(A2d, layer)
    return (A2d @ layer.W.astype(F32)).astype(F32)


def subst_affine(A, c, layer):
    """Substitute an affine layer whose L = U = W x + b: A+@W + A-@W, c + A+@b + A-@b."""
    B, R, n = A.shape
    Ap, An = _split(A)
    W2 = lambda M: apply_affine_T(M.reshape(B * R, n), layer).reshape(B, R, -1)
    A_new = (W2(Ap) + W2(An)).astype(F32)
    b = layer_bias(layer)
    dc = (Ap @ b + An @ b).astype(F32)
    return A_new, ((dc + F32(0.0)) + c).astype(F32)


def concretize(A, c, l0, u0, lower):
    """Fold the input box into the constant (input layer L/U = const l0/u0)."""
    Ap, An = _split(A)
    if lower:
        dc = np.einsum('brn,bn->br', Ap, l0, dtype=F32) + np.einsum('brn,bn->br', An, u0, dtype=F32)
    else:
        dc = np.einsum('brn,bn->br', Ap, u0, dtype=F32) + np.einsum('brn,bn->br', An, l0, dtype=F32)
    return ((dc.astype(F32) + F32(0.0)) + c).astype(F32)


# ---------------------------------------------------------------- network
def _affine_rows(layer, row_lo, row_hi, B):
    """Initial coefficient rows [B, r, n_in] of an affine layer: rows of W (or of the conv Toeplitz)."""
    if layer.kind == 'linear':
        W = layer.W.astype(F32)[row_lo:row_hi]
        return np.broadcast_to(W, (B,) + W.shape)
    n_out = layer.n_out
    E = np.zeros((row_hi - row_lo, n_out), F32)
    E[np.arange(row_hi - row_lo), np.arange(row_lo, row_hi)] = 1.0
    rows = _conv_T(E, layer)
    return np.broadcast_to(rows, (B,) + rows.shape)


def deeppoly(layers, l0, u0, spec_W, row_chunk=4096, force=None):
    """Run DeepPoly over a chain network.

    layers : list of cfgpu.nets.Layer (linear / conv / relu), property layer excluded.
    l0, u0 : [B, n0] float32 normalised input box.
    spec_W : [B, 9, 10] per-region property matrix (bias 0).
    force  : optional (l_all, u_all) [B, N-n0] in the same per-layer order as the
             returned bounds; the ReLU decisions are then taken from them (see relu_relax).
    Returns (bounds, lb, ub): bounds is a list, per layer (excluding input,
    including the property layer), of (l [B,n], u [B,n]); lb/ub float64 [B, 9].
    """
    l0 = np.asarray(l0, F32)
    u0 = np.asarray(u0, F32)
    B = l0.shape[0]
    affine = []       # (layer, relu-after (alpha, lam, mu) or None)
    bounds = []
    relax = {}
    pos = 0
    for idx, L in enumerate(layers + ['spec']):
        if L == 'spec':
            kind = 'spec'
        else:
            kind = L.kind
        if kind == 'relu':
            l_prev, u_prev = bounds[-1]
            n = l_prev.shape[1]
            fz = None if force is None else (force[0][:, pos - n:pos], force[1][:, pos - n:pos])
            ln, un, alpha, lam, mu = relu_relax(l_prev, u_prev, fz)
            pos += n
            relax[len(affine) - 1] = (alpha, lam, mu)
            bounds.append((ln, un))
            continue
        # affine-type layer: backsubstitute to the input, chunked over rows
        n_rows = 9 if kind == 'spec' else L.n_out
        lo_all = np.empty((B, n_rows), F32)
        up_all = np.empty((B, n_rows), F32)
        for r0 in range(0, n_rows, row_chunk):
            r1 = min(n_rows, r0 + row_chunk)
            if kind == 'spec':
                A0 = spec_W[:, r0:r1, :].astype(F32)
                c0 = np.zeros((B, r1 - r0), F32)
            else:
                A0 = _affine_rows(L, r0, r1, B)
                c0 = np.broadcast_to(layer_bias(L)[r0:r1], (B, r1 - r0)).astype(F32)
            for lower in (True, False):
                A, c = np.array(A0, F32), np.array(c0, F32)
                for j in range(len(affine) - 1, -1, -1):
                    if j in relax:
                        alpha, lam, mu = relax[j]
                        A, c = subst_relu(A, c, alpha, lam, mu, lower)
                    A, c = subst_affine(A, c, affine[j])
                    if not np.any(A):
                        A = None
                        break
                if A is None:
                    res = c
                else:
                    res = concretize(A, c, l0, u0, lower)
                (lo_all if lower else up_all)[:, r0:r1] = res
        bounds.append((lo_all, up_all))
        pos += n_rows
        if kind != 'spec':
            affine.append(L)
    lb, ub = bounds[-1]
    return bounds, lb.astype(np.float64), ub.astype(np.float64)


def flatten_bounds(wl_input_size, bounds, B):
    """Concatenate per-layer bounds into the reference's [B, N] neuron order (input excluded)."""
    ls = [b[0] for b in bounds]
    us = [b[1] for b in bounds]
    return np.concatenate(ls, axis=1), np.concatenate(us, axis=1)


# ---------------------------------------------------------------- receptive-field windows
# The same DeepPoly arithmetic for conv networks without dense rows.  A coefficient row of
# a conv neuron (co, oy, ox) is nonzero at every level j below it only inside its
# receptive field: C_j x Ph x Pw positions of level j's image whose origin is
# (oy*sig - pi, ox*sig - pi) (the reference keeps the same information in PatchesBlock,
# constraintflow/gbcsr/sparse_block.py:2576-3100, and its Dense@Kernel products run
# conv_transpose2d, :839-928).  Rows of a linear or property layer use the whole image
# (sig = 0).  Entries at positions outside the level image are exact zeros, so every sum
# below equals the dense one up to float32 summation order.

class _Win:
    """Window geometry at one level: image (C, H, W), window Ph x Pw, origin step sig and
    offset pi (origin of row position (oy, ox) = (oy*sig - pi, ox*sig - pi))."""

    def __init__(self, C, H, W, Ph, Pw, sig, pi):
        self.C, self.H, self.W, self.Ph, self.Pw, self.sig, self.pi = C, H, W, Ph, Pw, sig, pi

    @property
    def size(self):
        return self.C * self.Ph * self.Pw


def _img(layer, side):
    shp = layer.in_shape if side == 'in' else layer.out_shape
    if shp is None or len(shp) == 1:
        n = layer.n_in if side == 'in' else layer.n_out
        return (n, 1, 1)
    return tuple(int(x) for x in shp)


def _window_chain(affine, m):
    """Windows of the rows of affine layer m (m == len(affine): the property layer) at the
    input of affine layers m-1 .. 0 ... (list index k: the window over affine[m-1-k]'s
    output, i.e. before substituting it), then over the network input."""
    spec = m == len(affine)

    def level(j):   # the image at the input of affine layer j: the output image of affine j-1
        return _img(affine[j - 1], 'out') if j > 0 else _img(affine[0], 'in')
    lvl = level(m)
    if not spec and affine[m].kind == 'conv':
        L = affine[m]
        g = _Win(lvl[0], lvl[1], lvl[2], L.W.shape[2], L.W.shape[3], L.stride, L.pad)
    else:
        g = _Win(lvl[0], lvl[1], lvl[2], lvl[1], lvl[2], 0, 0)
    out = [g]
    for j in range(m - 1, -1, -1):
        Lj = affine[j]
        C, H, W = level(j)
        if Lj.kind == 'conv' and g.sig > 0:
            kh, kw = Lj.W.shape[2], Lj.W.shape[3]
            h = _Win(C, H, W, (g.Ph - 1) * Lj.stride + kh, (g.Pw - 1) * Lj.stride + kw,
                     g.sig * Lj.stride, g.pi * Lj.stride + Lj.pad)
        else:
            h = _Win(C, H, W, H, W, 0, 0)
        out.append(h)
        g = h
    return out


def _win_view(img, g, Hm, Wm):
    """[B, C, H, W] -> view [B, Hm, Wm, C, Ph, Pw] of every row position's window (zeros
    outside the image)."""
    B = img.shape[0]
    top = g.pi
    bot = max(0, (Hm - 1) * g.sig - g.pi + g.Ph - g.H)
    left = g.pi
    right = max(0, (Wm - 1) * g.sig - g.pi + g.Pw - g.W)
    pad = np.zeros((B, g.C, g.H + top + bot, g.W + left + right), img.dtype)
    pad[:, :, top:top + g.H, left:left + g.W] = img
    sb, sc, sh, sw = pad.strides
    return np.lib.stride_tricks.as_strided(
        pad, shape=(B, Hm, Wm, g.C, g.Ph, g.Pw),
        strides=(sb, g.sig * sh, g.sig * sw, sc, sh, sw), writeable=False)


def _in_image(g, Hm, Wm):
    """[Hm, Wm, 1, Ph, Pw] mask of window positions inside the level image."""
    oy = np.arange(Hm)[:, None, None, None, None]
    ox = np.arange(Wm)[None, :, None, None, None]
    u = np.arange(g.Ph)[None, None, None, :, None]
    v = np.arange(g.Pw)[None, None, None, None, :]
    Y = oy * g.sig - g.pi + u
    X = ox * g.sig - g.pi + v
    return ((Y >= 0) & (Y < g.H) & (X >= 0) & (X < g.W)).astype(F32)


def _win_conv_T(X, layer, g, h):
    """Transposed convolution of window rows X [M, Cout, g.Ph, g.Pw] (over the conv's output)
    into windows [M, Cin, h.Ph, h.Pw] over its input: out[u*s + ky - D, v*s + kx - D] +=
    X[u, v] W[:, :, ky, kx], D = g.pi*s + pad - h.pi (0 for receptive-field windows, pad for
    whole-image ones); the caller zeroes positions outside the image."""
    Cout, Cin, kh, kw = layer.W.shape
    s = layer.stride
    D = g.pi * s + layer.pad - h.pi
    M = X.shape[0]
    Xhw = np.ascontiguousarray(X.transpose(0, 2, 3, 1)).reshape(M * g.Ph * g.Pw, Cout)
    Hp = max((g.Ph - 1) * s + kh, D + h.Ph)
    Wp = max((g.Pw - 1) * s + kw, D + h.Pw)
    outp = np.zeros((M, Hp, Wp, Cin), F32)
    for i in range(kh):
        for j in range(kw):
            contrib = (Xhw @ layer.W[:, :, i, j].astype(F32)).reshape(M, g.Ph, g.Pw, Cin)
            outp[:, i:i + s * (g.Ph - 1) + 1:s, j:j + s * (g.Pw - 1) + 1:s, :] += contrib
    out = outp[:, D:D + h.Ph, D:D + h.Pw, :]
    return np.ascontiguousarray(out.transpose(0, 3, 1, 2))


def _win_bound(affine, relax, m, A0, c0, Hm, Wm, l0img, u0img, lower):
    """Bound of rows A0 [B, r, C, Ph, Pw] (windows over layer m's input, row i at position
    (oy, ox) = divmod(i % (Hm*Wm), Wm)), constants c0 [B, r].  Rows are all of layer m's
    rows for the given positions (r = Cm * Hm * Wm, or the linear rows with Hm = Wm = 1).

    An affine layer's L and U are the same expression W x + b, so the two products of the
    sign split (clamp(A,0,True) @ W + clamp(A,0,False) @ W) are one product A @ W here: the
    same sum, with float32 rounding of a different order."""
    gs = _window_chain(affine, m)
    B, r = A0.shape[:2]
    k_ = r // (Hm * Wm)
    A, c = A0, c0
    zero = F32(0.0)
    for k, j in enumerate(range(m - 1, -1, -1)):
        g, h = gs[k], gs[k + 1]
        Lj = affine[j]
        A6 = A.reshape(B, k_, Hm, Wm, g.C, g.Ph, g.Pw)
        if j in relax:   # substitute ReLU_j with the region's relaxation at absolute positions
            alpha, lam, mu = (_win_view(v.reshape(B, g.C, g.H, g.W), g, Hm, Wm) for v in relax[j])
            neg = A6 < zero
            # lower bound: a >= 0 -> a*alpha (L), a < 0 -> a*lam + a*mu (U); upper the other way
            fac = np.where(neg, lam[:, None], alpha[:, None]) if lower else np.where(neg, alpha[:, None], lam[:, None])
            side = np.where(neg, A6, zero) if lower else np.where(neg, zero, A6)
            dc = np.einsum('bkhwcuv,bhwcuv->bkhw', side, mu, dtype=F32, optimize=True).reshape(B, r)
            A6 = np.multiply(A6, fac, dtype=F32)
            c = ((dc + zero) + c).astype(F32)
        # substitute affine j: A W, c + A b
        if Lj.kind == 'conv':
            dc = np.einsum('bkhwcuv,c->bkhw', A6, Lj.b.astype(F32), dtype=F32, optimize=True).reshape(B, r)
        else:
            dc = (A6.reshape(B, r, -1) @ Lj.b.astype(F32)).astype(F32)
        c = ((dc + zero) + c).astype(F32)
        Mr = B * r
        if Lj.kind == 'conv':
            A = _win_conv_T(A6.reshape(Mr, g.C, g.Ph, g.Pw), Lj, g, h).reshape(B, k_, Hm, Wm, h.C, h.Ph, h.Pw)
            if h.sig > 0 or h.Ph != h.H or h.Pw != h.W:
                A *= _in_image(h, Hm, Wm)[None, None]
        else:
            A = (A6.reshape(Mr, -1) @ Lj.W.astype(F32)).reshape(B, k_, Hm, Wm, h.C, h.Ph, h.Pw)
    # fold the input box in (input layer L / U = constant l0 / u0)
    g = gs[-1]
    A6 = A.reshape(B, k_, Hm, Wm, g.C, g.Ph, g.Pw)
    lw = _win_view(l0img, g, Hm, Wm)
    uw = _win_view(u0img, g, Hm, Wm)
    neg = A6 < zero
    box = np.where(neg, uw[:, None], lw[:, None]) if lower else np.where(neg, lw[:, None], uw[:, None])
    dc = np.einsum('bkhwcuv,bkhwcuv->bkhw', A6, box, dtype=F32, optimize=True).reshape(B, r)
    return ((dc.astype(F32) + zero) + c).astype(F32)


def _win_rows(layer, g, Hm, Wm, rows_c, B):
    """Initial windows [B, r, C, Ph, Pw] of the rows of output channels rows_c (conv) or of
    rows rows_c (linear): the conv kernel placed at each position's origin, zero outside
    the image; a linear row over the whole image."""
    if layer.kind == 'conv':
        K = layer.W.astype(F32)[rows_c]                              # [rc, Cin, kh, kw]
        mask = _in_image(g, Hm, Wm)                                  # [Hm, Wm, 1, Ph, Pw]
        A = K[:, None, None] * mask[None]                            # [rc, Hm, Wm, Cin, kh, kw]
        A = A.reshape((-1,) + A.shape[3:])
    else:
        A = layer.W.astype(F32)[rows_c].reshape(-1, g.C, g.Ph, g.Pw)
    return np.broadcast_to(A, (B,) + A.shape)


def deeppoly_windows(layers, l0, u0, spec_W, force=None, chunk_floats=1 << 22, threads=None):
    """DeepPoly over a chain network with conv layers on receptive-field windows.

    Same contract as deeppoly(): layers (property layer excluded), l0 / u0 [B, n0], spec_W
    [B, 9, 10], optional force = (l_all, u_all) replaying ReLU decisions; returns (bounds, lb,
    ub).  Rows are processed in chunks of whole output channels (conv) or rows (linear)
    holding about chunk_floats window entries, on `threads` host threads (default: all;
    numpy releases the interpreter lock inside its array loops and BLAS calls)."""
    import concurrent.futures
    import os
    pool = concurrent.futures.ThreadPoolExecutor(threads or os.cpu_count() or 1)
    l0 = np.asarray(l0, F32)
    u0 = np.asarray(u0, F32)
    B = l0.shape[0]
    first = next(L for L in layers if L.kind != 'relu')
    C0, H0, W0 = _img(first, 'in')
    l0img, u0img = l0.reshape(B, C0, H0, W0), u0.reshape(B, C0, H0, W0)
    affine, bounds, relax = [], [], {}
    pos = 0
    for L in layers + ['spec']:
        kind = 'spec' if L == 'spec' else L.kind
        if kind == 'relu':
            l_prev, u_prev = bounds[-1]
            n = l_prev.shape[1]
            fz = None if force is None else (force[0][:, pos - n:pos], force[1][:, pos - n:pos])
            ln, un, alpha, lam, mu = relu_relax(l_prev, u_prev, fz)
            pos += n
            relax[len(affine) - 1] = (alpha, lam, mu)
            bounds.append((ln, un))
            continue
        m = len(affine)
        aff = affine + ([] if kind == 'spec' else [L])
        gs = _window_chain(aff, m)
        if kind == 'conv':
            _, Hm, Wm = L.out_shape
            groups = L.W.shape[0]
            per = Hm * Wm
        else:
            Hm = Wm = 1
            groups = 9 if kind == 'spec' else L.n_out
            per = 1
        n_rows = groups * per
        lo_all = np.empty((B, n_rows), F32)
        up_all = np.empty((B, n_rows), F32)
        wsize = max(g.size for g in gs)
        step = max(1, int(chunk_floats // max(1, B * per * wsize)))

        def work(g0, lower, L=L, kind=kind, gs=gs, aff=aff, m=m, Hm=Hm, Wm=Wm, per=per, step=step,
                 groups=groups, lo_all=lo_all, up_all=up_all):
            g1 = min(groups, g0 + step)
            rr = slice(g0 * per, g1 * per)
            if kind == 'spec':
                g = gs[0]
                A0 = spec_W[:, g0:g1, :].astype(F32).reshape(B, g1 - g0, g.C, g.Ph, g.Pw)
                c0 = np.zeros((B, g1 - g0), F32)
            else:
                A0 = _win_rows(L, gs[0], Hm, Wm, slice(g0, g1), B)
                c0 = np.broadcast_to(layer_bias(L)[rr], (B, (g1 - g0) * per)).astype(F32)
            res = _win_bound(aff, relax, m, np.array(A0, F32), np.array(c0, F32), Hm, Wm, l0img, u0img, lower)
            (lo_all if lower else up_all)[:, rr] = res

        futs = [pool.submit(work, g0, lower) for g0 in range(0, groups, step) for lower in (True, False)]
        for f in futs:
            f.result()
        bounds.append((lo_all, up_all))
        pos += n_rows
        if kind != 'spec':
            affine.append(L)
    pool.shutdown()
    lb, ub = bounds[-1]
    return bounds, lb.astype(np.float64), ub.astype(np.float64)
