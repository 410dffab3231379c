"""The general CROWN traversal on the GPU, for networks where a ReLU layer takes the
all-crossing branch.

The reference compiles examples/compiler_examples/crown.cf:25 (a ternary of tuples) into
whole-layer branches over the layer's [B, n] bounds.  When no neuron of any region has
l >= 0 and none has u <= 0, every neuron crosses zero and the ReLU's polyexps are
  L' = (1 - c) x with c = 1[-l > u]              (the neuron itself, convert_to_poly)
  U' = lam (prev[U] with each referenced neuron replaced by its U (coefficient >= 0) or
       L (< 0)) + (u*(0-1))*l/(u-l),  lam = u/(u-l)
so U' refers one layer deeper than L' and the coefficient expressions of later layers mix
layers.  The backward traversal (crown.cf:10, priority2 = -layer; get_max_priority,
constraintflow/gbcsr/tensor_ops.py:557) then substitutes the LOWEST live layer first,
the input layer included (it is live from the start, constraintflow/lib/spec.py:134, and
get_default_stop stops only non-live layers), so partial coefficients of the input
columns are concretised mid-traversal.  The fused network driver (cf_deeppoly_run) cannot
express this; DeepPolyEngine runs this module instead when the driver reports the branch.

Representation: a polyexp is ({layer t: [1 or B, r, n_t] float32}, const [B, r]) on the
device; layer 0 is the input, then one neuron layer per network layer.  Every arithmetic
operation is a libcfgpu kernel (cfgpu.ops: cf_bmm, cf_ew_clamp, cf_ew_binary, cf_ew_any);
torch provides memory, views and copies.
"""
import operator

import torch

from . import ops

BRANCH_PASS, BRANCH_ZERO, BRANCH_CROSS = 0, 1, 2


def _full(B, t):
    """[1 or B, r, n] -> a [B, r, n] view (batch stride 0 when shared)."""
    return t.expand(B, t.shape[1], t.shape[2]) if t.shape[0] == 1 else t


def _add_block(blocks, t, M):
    blocks[t] = ops.binary(operator.add, blocks[t], M, torch.float32) if t in blocks else M


def _colvec(c):
    return c.unsqueeze(2)           # [B, n] -> [B, n, 1]


def _substitute(B, blocks, c, t, P, Q):
    """Replace layer t's neurons: coefficient >= 0 -> P, < 0 -> Q (each (blocks, const))."""
    A = _full(B, blocks.pop(t))
    Ap = ops.clamp(A, 0.0, True)
    An = ops.clamp(A, 0.0, False)
    new = {}
    for s, M in P[0].items():
        _add_block(new, s, ops.bmm(Ap, _full(B, M)))
    for s, M in Q[0].items():
        _add_block(new, s, ops.bmm(An, _full(B, M)))
    dc = ops.binary(operator.add, ops.bmm(Ap, _colvec(P[1]))[:, :, 0], ops.bmm(An, _colvec(Q[1]))[:, :, 0],
                    torch.float32)
    for s, M in blocks.items():     # the stopped part (the other layers) is added after
        _add_block(new, s, _full(B, M))
    zero = ops.scalar_view(0.0, tuple(dc.shape), torch.float32)
    return new, ops.binary(operator.add, ops.binary(operator.add, dc, zero, torch.float32), c, torch.float32)


def _traverse(B, blocks, c, polys, lower):
    """Backward traversal, lowest live layer first, until no coefficient is left."""
    while True:
        live = [t for t, M in blocks.items() if ops.any_nonzero(M)]
        if not live:
            return c
        t = min(live)
        L, U = polys[t]
        blocks, c = _substitute(B, blocks, c, t, L, U) if lower else _substitute(B, blocks, c, t, U, L)


def _scal(v, like):
    return ops.scalar_view(v, tuple(like.shape), torch.float32)


def run(layers, l0, u0, spec_W):
    """CROWN over a chain network of linear / relu layers on the GPU.

    layers: list of (kind, W [n_out, n_in] device float32 or None, b [n_out] or None).
    l0, u0 [B, n0], spec_W [B, n_spec, n_last] device float32.
    Returns (bounds, branches): bounds per layer (excluding input, including the property
    layer) of (l [B, n], u [B, n]) device float32; branches: BRANCH_* per ReLU layer.
    """
    B = l0.shape[0]
    f32 = torch.float32
    polys = {0: (({}, l0), ({}, u0))}
    bounds = []
    branches = []
    for idx, layer in enumerate(list(layers) + [("spec", None, None)]):
        k = idx + 1
        kind, W, bias = layer
        if kind == "relu":
            l, u = bounds[-1]
            if ops.any_nonzero(ops.binary(operator.ge, l, _scal(0.0, l), torch.bool)):
                branches.append(BRANCH_PASS)
                polys[k] = polys[k - 1]
                bounds.append((l, u))
            elif ops.any_nonzero(ops.binary(operator.le, u, _scal(0.0, u), torch.bool)):
                branches.append(BRANCH_ZERO)
                z = torch.zeros_like(l)
                polys[k] = (({}, z), ({}, z))
                bounds.append((torch.zeros_like(l), torch.zeros_like(u)))
            else:
                branches.append(BRANCH_CROSS)
                polys[k], bounds_k = _crossing(B, k, l, u, polys)
                bounds.append(bounds_k)
            continue
        if kind == "spec":
            A0 = spec_W
            c0 = torch.zeros(B, spec_W.shape[1], dtype=f32, device=l0.device)
        elif kind == "linear":
            A0 = W.unsqueeze(0)
            c0 = bias.unsqueeze(0).expand(B, -1).contiguous()
        else:
            raise NotImplementedError(f"CROWN's all-crossing branch on a {kind} layer (the general traversal "
                                      "runs linear layers only)")
        res = []
        for lower in (True, False):
            res.append(_traverse(B, {k - 1: A0}, c0, polys, lower))
        bounds.append((res[0], res[1]))
        poly = ({k - 1: A0}, c0)
        polys[k] = (poly, poly)
    return bounds, branches


def _crossing(B, k, l, u, polys):
    """Polyexps and bounds of ReLU layer k in the all-crossing branch (generated crown Relu)."""
    f32 = torch.float32
    (Lb, Lc), (Ub, Uc) = polys[k - 1]
    zero, one = _scal(0.0, l), _scal(1.0, l)
    cflag = ops.unary("to_f32", ops.binary(operator.gt, ops.binary(operator.sub, zero, l, f32), u, torch.bool), f32)
    keep = ops.binary(operator.sub, one, cflag, f32)
    l_new = ops.binary(operator.add, ops.binary(operator.mul, cflag, zero, f32),
                       ops.binary(operator.mul, keep, l, f32), f32)
    n = l.shape[1]
    eye = torch.eye(n, dtype=f32, device=l.device).unsqueeze(0).expand(B, n, n)
    Lpoly = ({k - 1: ops.binary(operator.mul, keep.unsqueeze(2).expand(B, n, n), eye, f32)}, torch.zeros_like(l))
    # U' = lam * (prev[U] with its neurons replaced by U (coeff >= 0) / L (< 0)) + mu
    sub_b, sub_c = {}, None
    for t, M in Ub.items():
        Mb = _full(B, M)
        Mp, Mn = ops.clamp(Mb, 0.0, True), ops.clamp(Mb, 0.0, False)
        (tLb, tLc), (tUb, tUc) = polys[t]
        for s, X in tUb.items():
            _add_block(sub_b, s, ops.bmm(Mp, _full(B, X)))
        for s, X in tLb.items():
            _add_block(sub_b, s, ops.bmm(Mn, _full(B, X)))
        dcc = ops.binary(operator.add, ops.bmm(Mp, _colvec(tUc))[:, :, 0], ops.bmm(Mn, _colvec(tLc))[:, :, 0], f32)
        sub_c = dcc if sub_c is None else ops.binary(operator.add, sub_c, dcc, f32)
    if sub_c is None:
        sub_c = torch.zeros_like(l)
    den = ops.binary(operator.sub, u, l, f32)
    lam = ops.binary(operator.truediv, u, den, f32)
    mu = ops.binary(operator.truediv, ops.binary(operator.mul, ops.binary(operator.mul, u, l, f32),
                                                 _scal(-1.0, l), f32), den, f32)
    Uconst = ops.binary(operator.add, ops.binary(operator.mul, lam, ops.binary(operator.add, sub_c, Uc, f32), f32),
                        mu, f32)
    Upoly = ({s: ops.binary(operator.mul, lam.unsqueeze(2).expand(X.shape), X, f32) for s, X in sub_b.items()},
             Uconst)
    return (Lpoly, Upoly), (l_new, u)
