"""The general backward traversal on the GPU: DeepPoly and CROWN over networks whose
layers form a DAG (residual Add, Concat) and CROWN's all-crossing branch.

The fused network driver (cf_deeppoly_run) covers chains whose polyexps refer to one
layer each.  Two cases give polyexps that mix layers and are run here instead:
  * Add / Concat layers (constraintflow/lib/flow_sparse.py:67-178): an Add layer's
    l / u are the parents' l / u summed and its L / U the parents' polyexps summed block
    by block; a Concat stacks the parents' bounds and polyexp rows.
  * CROWN's all-crossing ReLU branch (crown.cf:25 as the reference compiles it): with
    c = 1[-l > u], L' = (1 - c) x (the neuron itself) and U' = lam (prev[U] with each
    referenced neuron replaced by its U (coefficient >= 0) or L (< 0)) + (u*(0-1))*l/(u-l),
    lam = u/(u-l), so U' refers one layer deeper than L'.  The other branches are
    whole-layer: any(l >= 0) passes prev[L] / prev[U] through, else any(u <= 0) zeroes.
The bounds of an affine-type layer come from the backward traversal (deeppoly.cf:10 /
crown.cf:10, priority2 = -layer; get_max_priority, constraintflow/gbcsr/tensor_ops.py:557):
every iteration substitutes the LOWEST layer with a non-zero coefficient anywhere in the
batch, the input layer included (it is live from the start, constraintflow/lib/spec.py:134,
and get_default_stop stops only non-live layers), by L (coefficient >= 0) or U (< 0) for
the lower bound and U / L for the upper (replace_lower / replace_upper, clamp sign split,
inner_prod, tensor_ops.py:370,765); the stopped part is added after the substituted one.

Representation: a polyexp is ({layer t: block}, const [B, r]) on the device; layer 0 is
the input, then one neuron layer per network layer, in list order.  A block is either
dense, [1 or B, r, n_t] float32 (a batch-shared layer weight has batch 1), diagonal,
[B, n_t] (a ReLU's per-neuron relaxation over its own input layer, r = n_t), so a ReLU
substitution is a column scaling instead of a product with an n x n matrix, or a conv
layer's weights (_Conv, the KernelBlock of constraintflow/gbcsr/sparse_block.py:1158),
substituted by the transposed convolution of every coefficient row (cf_conv_transpose,
as DenseBlock @ KernelBlock, :839-911) and densified (cf_conv_densify) only where it
starts a traversal or meets another block over the same layer.  Every
arithmetic operation is a libcfgpu kernel (cfgpu.ops: cf_bmm, cf_signscale, cf_ew_binary,
cf_ew_clamp, cf_ew_any; cf_relu_relax for DeepPoly's relaxation); torch provides memory,
views and copies.
"""
import operator

import torch

from . import _lib, ops

BRANCH_PASS, BRANCH_ZERO, BRANCH_CROSS = 0, 1, 2
F32 = torch.float32


class _Conv:
    """A conv layer's weights W [cout, cin, kh, kw] standing for its matrix
    [cout*oh*ow, cin*ih*iw] (square stride and padding, as the reference's reader gives)."""

    def __init__(self, W, geom):
        cin, ih, iw, cout, oh, ow, stride, pad = geom
        kh, kw = int(W.shape[2]), int(W.shape[3])
        self.W = W
        self.g = ops.conv_geom(cout, cin, oh, ow, ih, iw, kh, kw, stride, stride, pad, pad)
        self.ih, self.iw = ih, iw
        self.shape = (1, cout * oh * ow, cin * ih * iw)
        self.ckk = cin * kh * kw

    def dim(self):
        return 4

    def dense(self):
        return ops.conv_densify(self.g, 1, self.W, 0, self.ckk, 0)


def _full(B, t):
    """[1 or B, r, n] -> a [B, r, n] view (batch stride 0 when shared)."""
    if isinstance(t, _Conv):
        t = t.dense()
    return t.expand(B, t.shape[1], t.shape[2]) if t.shape[0] == 1 else t


def _dense(B, M):
    """A block as a dense [B, r, n] (a diagonal block or conv weights materialised)."""
    if M.dim() != 2:
        return _full(B, M)
    n = M.shape[1]
    eye = torch.eye(n, dtype=F32, device=M.device).unsqueeze(0).expand(B, n, n)
    return ops.binary(operator.mul, M.unsqueeze(2).expand(B, n, n), eye, F32)


def _add(a, b):
    return ops.binary(operator.add, a, b, F32)


def _add_block(B, blocks, t, M):
    if t not in blocks:
        blocks[t] = M
    elif blocks[t].dim() == 2 and M.dim() == 2:
        blocks[t] = _add(blocks[t], M)
    else:
        blocks[t] = _add(_dense(B, blocks[t]), _dense(B, M))


def _apply(B, A, M):
    """A [B, r, n_t] times block M over layer s: bmm for dense, column scaling for diagonal,
    the transposed convolution of every row for conv weights."""
    if isinstance(M, _Conv):
        r, cols = A.shape[1], M.shape[2]
        out = torch.empty(B, r, cols, dtype=F32, device=A.device)
        ops.conv_transpose(M.g, B, r, A, (A.stride(0), A.stride(1), A.stride(2)), M.W, M.ih, M.iw, out,
                           (r * cols, cols, 1))
        return out
    if M.dim() == 3:
        return ops.bmm(A, _full(B, M))
    return ops.binary(operator.mul, A, M.unsqueeze(1).expand(A.shape), F32)


def _vec(B, v):
    """[1 or B, n] -> [B, n] (materialised when shared)."""
    return v.expand(B, v.shape[1]).contiguous() if v.shape[0] != B else v


def _rowdot(A, c):
    """A [B, r, n] . c [B, n] -> [B, r]."""
    return ops.bmm(A, c.unsqueeze(2))[:, :, 0]


def _substitute(B, blocks, c, t, P, Q):
    """Replace layer t's neurons: coefficient >= 0 -> P, < 0 -> Q (each (blocks, const)).

    When P and Q are the same polyexp (an affine layer, whose L and U are both W x + b, or
    an Add / Concat of such layers) the sign split A+ P + A- Q is A P: one product instead
    of two (as the tensor-core chain substitutes affine layers)."""
    A = _full(B, blocks.pop(t))
    new = {}
    (ps, pm), = P[0].items() if len(P[0]) == 1 else ((None, None),)
    (qs, qm), = Q[0].items() if len(Q[0]) == 1 else ((None, None),)
    if P is not Q and ps is not None and ps == qs and pm.dim() == 2 and qm.dim() == 2:
        # a ReLU layer's per-neuron relaxations (diagonal blocks over one layer): one fused
        # sign-selected column scaling, the constant terms in the same pass
        out, dc = ops.signscale(A, _vec(B, pm), _vec(B, qm), _vec(B, P[1]), _vec(B, Q[1]))
        new[ps] = out
    elif P is Q:
        for s, M in P[0].items():
            _add_block(B, new, s, _apply(B, A, M))
        dc = _rowdot(A, P[1])
    else:
        Ap = ops.clamp(A, 0.0, True)
        An = ops.clamp(A, 0.0, False)
        for s, M in P[0].items():
            _add_block(B, new, s, _apply(B, Ap, M))
        for s, M in Q[0].items():
            _add_block(B, new, s, _apply(B, An, M))
        dc = _add(_rowdot(Ap, P[1]), _rowdot(An, Q[1]))
    for s, M in blocks.items():     # the stopped part (the other layers) is added after
        _add_block(B, new, s, _full(B, M))
    zero = ops.scalar_view(0.0, tuple(dc.shape), F32)
    return new, _add(_add(dc, zero), c)


def _traverse(B, blocks, c, polys, lower):
    """Backward traversal, lowest layer first, until no coefficient block is left.

    The reference substitutes only live layers (a block with a non-zero coefficient
    somewhere in the batch) and leaves all-zero blocks stopped, where they concretise to 0.
    Substituting an all-zero block instead adds exact zeros to the constant and to the
    blocks of the layers below it, and does not change which other layer comes next, so
    the bounds are the same while the traversal needs no device-to-host liveness test:
    the whole pass is stream-ordered (and can be captured in a CUDA graph)."""
    while blocks:
        t = min(blocks)
        L, U = polys[t]
        blocks, c = _substitute(B, blocks, c, t, L, U) if lower else _substitute(B, blocks, c, t, U, L)
    return c


def _scal(v, like):
    return ops.scalar_view(v, tuple(like.shape), F32)


def _deeppoly_relu(B, k_in, l, u):
    """Generated deeppoly.Relu (deeppoly.cf:20-24,41): L' = alpha x, U' = lam x + mu."""
    n = l.shape[1]
    l_new, u_new, alpha, lam, mu = (torch.empty(B, n, dtype=F32, device=l.device) for _ in range(5))
    lc, uc = l.contiguous(), u.contiguous()
    ops.LAUNCHES[0] += 1
    st = _lib.lib.cf_relu_relax(B, n, lc.data_ptr(), uc.data_ptr(), n, l_new.data_ptr(), u_new.data_ptr(), n,
                                alpha.data_ptr(), lam.data_ptr(), mu.data_ptr(), _lib.CF_RELAX_DEEPPOLY,
                                torch.cuda.current_stream().cuda_stream)
    _lib.check(st, "cf_relu_relax")
    return (({k_in: alpha}, torch.zeros_like(l)), ({k_in: lam}, mu)), (l_new, u_new)


def _crown_relu(B, k_in, l, u, polys):
    """Generated crown Relu (crown.cf:25): one whole-layer branch over the [B, n] bounds."""
    if ops.any_nonzero(ops.binary(operator.ge, l, _scal(0.0, l), torch.bool)):
        return BRANCH_PASS, polys[k_in], (l, u)
    if ops.any_nonzero(ops.binary(operator.le, u, _scal(0.0, u), torch.bool)):
        z = torch.zeros_like(l)
        return BRANCH_ZERO, (({}, z), ({}, z)), (torch.zeros_like(l), torch.zeros_like(u))
    (Lb, Lc), (Ub, Uc) = polys[k_in]
    zero, one = _scal(0.0, l), _scal(1.0, l)
    cflag = ops.unary("to_f32", ops.binary(operator.gt, ops.binary(operator.sub, zero, l, F32), u, torch.bool), F32)
    keep = ops.binary(operator.sub, one, cflag, F32)
    l_new = _add(ops.binary(operator.mul, cflag, zero, F32), ops.binary(operator.mul, keep, l, F32))
    Lpoly = ({k_in: keep}, torch.zeros_like(l))
    # U' = lam * (prev[U] with its neurons replaced by U (coeff >= 0) / L (< 0)) + mu
    sub_b, sub_c = {}, None
    for t, M in Ub.items():
        Mb = _dense(B, M)
        Mp, Mn = ops.clamp(Mb, 0.0, True), ops.clamp(Mb, 0.0, False)
        (tLb, tLc), (tUb, tUc) = polys[t]
        for s, X in tUb.items():
            _add_block(B, sub_b, s, _apply(B, Mp, X))
        for s, X in tLb.items():
            _add_block(B, sub_b, s, _apply(B, Mn, X))
        dcc = _add(_rowdot(Mp, tUc), _rowdot(Mn, tLc))
        sub_c = dcc if sub_c is None else _add(sub_c, dcc)
    if sub_c is None:
        sub_c = torch.zeros_like(l)
    den = ops.binary(operator.sub, u, l, F32)
    lam = ops.binary(operator.truediv, u, den, F32)
    mu = ops.binary(operator.truediv, ops.binary(operator.mul, ops.binary(operator.mul, u, l, F32),
                                                 _scal(-1.0, l), F32), den, F32)
    Uconst = _add(ops.binary(operator.mul, lam, _add(sub_c, Uc), F32), mu)
    Upoly = ({}, Uconst)
    for s, X in sub_b.items():
        Xd = _dense(B, X)
        Upoly[0][s] = ops.binary(operator.mul, lam.unsqueeze(2).expand(Xd.shape), Xd, F32)
    return BRANCH_CROSS, (Lpoly, Upoly), (l_new, u)


def _sum_poly(B, P, Q):
    """An Add layer's polyexp: the parents' polyexps summed block by block."""
    blocks = dict(P[0])
    for t, M in Q[0].items():
        _add_block(B, blocks, t, M)
    return blocks, _add(P[1], Q[1])


def _stack_poly(B, P, Q):
    """A Concat layer's polyexp: the parents' rows stacked (zero rows where a parent has
    no block over a layer)."""
    n1, n2 = P[1].shape[1], Q[1].shape[1]
    blocks = {}
    for t in sorted(set(P[0]) | set(Q[0])):
        parts = []
        for poly, rows in ((P, n1), (Q, n2)):
            if t in poly[0]:
                parts.append(_dense(B, poly[0][t]))
            else:
                width = (P[0][t] if t in P[0] else Q[0][t]).shape[-1]
                parts.append(torch.zeros(B, rows, width, dtype=F32, device=P[1].device))
        blocks[t] = torch.cat(parts, dim=1)
    return blocks, torch.cat([P[1], Q[1]], dim=1)


def run(layers, l0, u0, spec_W, relaxation="deeppoly"):
    """DeepPoly or CROWN bounds of a network of linear / conv / relu / add / concat layers.

    layers: list of (kind, W [n_out, n_in] (conv: [cout, cin, kh, kw]) device float32 or
    None, b [n_out] (conv: [cout]) or None, parents tuple of layer-list indices, -1 = the
    network input[, conv geometry (cin, ih, iw, cout, oh, ow, stride, pad)]), in the order of the
    reference's ONNX reader (breadth first from the input; every parent listed before
    its children).  l0, u0 [B, n0], spec_W [B, n_spec, n_last] device float32; the
    property layer reads the last layer of the list.
    Returns (bounds, branches): bounds per layer (excluding input, including the property
    layer) of (l [B, n], u [B, n]) device float32; branches: BRANCH_* per ReLU layer (CROWN).
    """
    if relaxation not in ("deeppoly", "crown"):
        raise NotImplementedError(f"relaxation {relaxation!r}")
    B = l0.shape[0]
    polys = {0: (({}, l0), ({}, u0))}
    bnd = {0: (l0, u0)}
    branches = []
    nl = len(layers)
    for idx, layer in enumerate(list(layers) + [("spec", spec_W, None, (nl - 1,))]):
        k = idx + 1
        kind, W, bias, parents = layer[:4]
        ks = [p + 1 for p in parents]
        if any(not 0 <= p < k for p in ks):
            raise ValueError(f"layer {idx}: parents {parents} must precede it in the list")
        if kind == "relu":
            l, u = bnd[ks[0]]
            if relaxation == "crown":
                br, polys[k], bnd[k] = _crown_relu(B, ks[0], l, u, polys)
                branches.append(br)
            else:
                polys[k], bnd[k] = _deeppoly_relu(B, ks[0], l, u)
            continue
        if kind in ("add", "concat"):
            if len(ks) != 2:
                raise ValueError(f"layer {idx}: {kind} takes two parents, got {parents}")
            (l1, u1), (l2, u2) = bnd[ks[0]], bnd[ks[1]]
            (L1, U1), (L2, U2) = polys[ks[0]], polys[ks[1]]
            same = L1 is U1 and L2 is U2    # parents whose L and U are one polyexp
            if kind == "add":
                if l1.shape != l2.shape:
                    raise ValueError(f"layer {idx}: add of {tuple(l1.shape)} and {tuple(l2.shape)}")
                bnd[k] = (_add(l1, l2), _add(u1, u2))
                lo = _sum_poly(B, L1, L2)
                polys[k] = (lo, lo if same else _sum_poly(B, U1, U2))
            else:
                bnd[k] = (torch.cat([l1, l2], dim=1), torch.cat([u1, u2], dim=1))
                lo = _stack_poly(B, L1, L2)
                polys[k] = (lo, lo if same else _stack_poly(B, U1, U2))
            continue
        if kind == "spec":
            A0 = W
            c0 = torch.zeros(B, W.shape[1], dtype=F32, device=l0.device)
        elif kind == "linear":
            A0 = W.unsqueeze(0)
            c0 = bias.unsqueeze(0).expand(B, -1).contiguous()
        elif kind == "conv":
            A0 = _Conv(W, layer[4])
            per = A0.shape[1] // int(W.shape[0])      # output positions per channel
            c0 = bias.reshape(1, -1, 1).expand(B, int(W.shape[0]), per).reshape(B, A0.shape[1])
        else:
            raise NotImplementedError(f"a {kind} layer in the general traversal (it runs linear, conv, relu, add "
                                      "and concat layers)")
        res = [_traverse(B, {ks[0]: A0}, c0, polys, lower) for lower in (True, False)]
        bnd[k] = (res[0], res[1])
        poly = ({ks[0]: A0}, c0)
        polys[k] = (poly, poly)
    return [bnd[k] for k in range(1, nl + 2)], branches


def state(l0, u0, bounds):
    """Every neuron's bounds in the reference's neuron order: [B, n0 + sum n_k] each."""
    return (torch.cat([l0] + [b[0] for b in bounds], dim=1), torch.cat([u0] + [b[1] for b in bounds], dim=1))

