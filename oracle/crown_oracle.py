"""CPU oracle for the reference's DeepPoly and CROWN programs on general networks
(residual Add and Concat layers included) and for CROWN on chains (numpy, float32).

TEST INFRASTRUCTURE ONLY.  Only tests/, ``__graft_entry__.smoke()`` and bench.py's
CPU legs may import this module, as the checker; the product path (cfgpu) never
imports it and has no CPU fallback.

What it restates: examples/compiler_examples/crown.cf as the reference compiler
emits it (tests/golden/generated/crown/transformers.py, the reference's own
output kept as a fixture), run by constraintflow/lib/flow_sparse.py:27-228.

* Relu (crown.cf:25, generated ``Relu``): the ternary of TUPLES is lowered to
  whole-layer ``if any(...)`` branches over the [B, n] bounds of the layer:
    - ``any(l >= 0)``  -> pass-through: l' = l, u' = u, L' = prev[L], U' = prev[U];
    - else ``any(u <= 0)`` -> zero: l' = u' = 0, L' = U' = 0;
    - else (every neuron of every region crosses 0): with c = 1[-l > u],
      l' = c*0 + (1-c)*l, u' = u, L' = (1-c)*x (the neuron itself,
      Llist.convert_to_poly), U' = lam*(U_prev.map(replace_upper)) + (u*(0-1))*l/(u-l)
      with lam = u/(u-l): the affine's U polyexp with every neuron it references
      replaced by that neuron's U (coefficient >= 0) or L (< 0), i.e. one layer deeper.
  The branch is decided over the whole batch, so a region's bounds depend on the
  other regions of the batch (as in the reference).
* Affine (crown.cf:24, deeppoly.cf:39, generated ``Affine``): start from W x + b
  and traverse backwards with priority2 = -layer (crown.cf:10): every while-iteration
  takes the LOWEST layer that has a non-zero coefficient anywhere in the batch
  (get_max_priority, constraintflow/gbcsr/tensor_ops.py:557) and replaces its neurons
  by L (coefficient >= 0) or U (< 0) for the lower bound, U / L for the upper
  (replace_lower/replace_upper, crown.cf:6-7); inner_prod / clamp as in
  tensor_ops.py:370,765.  The input layer is live too (_traverse).  With polyexps that
  mix layers (after a CROWN crossing branch, or any Add / Concat) the substitution
  order matters: a neuron can be substituted several times with partial coefficients.
* DeepPoly Relu (deeppoly.cf:20-24,41): L' = alpha x, U' = lam x + mu
  (deeppoly_oracle.relu_relax), as diagonal blocks over the ReLU's input layer.
* Add (constraintflow/lib/flow_sparse.py:67-88): l = l1 + l2, u = u1 + u2, and the
  layer's L / U are the sums of the parents' polyexps (parents' blocks summed per layer).
* Concat (flow_sparse.py:89-178): bounds and polyexp rows of the two parents stacked.
* Layers are listed in the order of the reference's ONNX reader
  (constraintflow/lib/parse.py:60-300: breadth first from the input);
  each layer names its parents (cfgpu.nets.Layer.parents).

Representation: a polyexp is ({layer t: [B, r, n_t] float32}, const [B, r]);
layer 0 is the input, then one neuron layer per network layer, in order.

Pinned against: the reference's own DeepPoly and CROWN outputs (tests/golden/dp_*.npz,
crown_*.npz, made by tests/golden/gen_golden.py), residual and concat networks included.
"""
import numpy as np

from .deeppoly_oracle import F32, _affine_rows, layer_bias, relu_relax

BRANCH_PASS, BRANCH_ZERO, BRANCH_CROSS = 0, 1, 2


def _split(A):
    return np.maximum(A, F32(0.0)), np.minimum(A, F32(0.0))


def _add_block(blocks, t, M):
    blocks[t] = (blocks[t] + M).astype(F32) if t in blocks else M.astype(F32)


def _substitute(blocks, c, t, P, N_poly, lower):
    """Replace layer t's neurons in (blocks, c): coefficient >= 0 -> P (lower) else N_poly.

    P / N_poly are the (blocks, const) polyexps of layer t's neurons, [B, n_t, .] each.
    Returns the new (blocks, const) = substituted part + the untouched blocks.
    """
    A = blocks.pop(t)
    Ap, An = _split(A)
    first, second = (P, N_poly) if lower else (N_poly, P)
    new = {}
    for s, M in first[0].items():
        _add_block(new, s, np.matmul(Ap, M))
    for s, M in second[0].items():
        _add_block(new, s, np.matmul(An, M))
    dc = (np.einsum('brn,bn->br', Ap, first[1], dtype=F32) +
          np.einsum('brn,bn->br', An, second[1], dtype=F32)).astype(F32)
    for s, M in blocks.items():   # the stopped part (other layers) is added after
        _add_block(new, s, M)
    return new, ((dc + F32(0.0)) + c).astype(F32)


def _traverse(blocks, c, polys, lower, order=min, stop_below=None, bnd=None):
    """Backward traversal, lowest live layer first, until no coefficient is left.

    The input layer is live from the start (constraintflow/lib/spec.py:134-135) and
    get_default_stop (tensor_ops.py:497) stops only non-live layers, so input neurons
    are substituted in the loop like any other layer, by their constant L/U (l0/u0):
    whenever input columns are the lowest live layer, their current coefficients are
    concretised there and then.  The final concretisation (generated ``l_new``) then
    sees an empty matrix and returns the constant.

    stop_below (the custom-stop programs, deeppoly_custom_stop.cf:12-17): neurons of
    layers below it are not substituted; what remains on them is concretised at the end
    with their own bounds bnd[t] (map(simplify_lower / simplify_upper)).
    """
    while True:
        live = [t for t, M in blocks.items() if np.any(M) and (stop_below is None or t >= stop_below)]
        if not live:
            break
        t = order(live)
        L, U = polys[t]
        blocks, c = _substitute(blocks, c, t, L, U, lower)
    if stop_below is not None:
        for t, M in blocks.items():
            if t >= stop_below or not np.any(M):
                continue
            lo, hi = bnd[t]
            pos, neg = (lo, hi) if lower else (hi, lo)
            c = (c + np.einsum('brn,bn->br', np.maximum(M, F32(0)), pos, dtype=F32)
                 + np.einsum('brn,bn->br', np.minimum(M, F32(0)), neg, dtype=F32)).astype(F32)
    return c


def _parents(layers, i):
    p = layers[i].parents
    return tuple(p) if p is not None else (i - 1,)


def _deeppoly_relu(l, u, k_in, B, strict=False):
    """Generated deeppoly.Relu (deeppoly.cf:20-24,41) over its input layer k_in:
    L' = alpha x, U' = lam x + mu as diagonal blocks.  ``strict``: relu_n's l + u > 0
    (deeppoly_custom_stop.cf:25, zid.cf:22)."""
    l_new, u_new, alpha, lam, mu = relu_relax(l, u, strict=strict)
    n = l.shape[1]
    eye = np.eye(n, dtype=F32)[None]
    Lp = ({k_in: (alpha[:, :, None] * eye).astype(F32)}, np.zeros_like(l))
    Up = ({k_in: (lam[:, :, None] * eye).astype(F32)}, mu.astype(F32))
    return (Lp, Up), (l_new, u_new)


def _crown_relu(l, u, k_in, polys, B):
    """Generated crown Relu (crown.cf:25): one whole-layer branch over the [B, n] bounds."""
    zero = F32(0.0)
    (Lb, Lc), (Ub, Uc) = polys[k_in]
    if np.any(l >= zero):
        return BRANCH_PASS, polys[k_in], (l.copy(), u.copy())
    if np.any(u <= zero):
        zc = np.zeros_like(l)
        return BRANCH_ZERO, (({}, zc), ({}, zc)), (np.zeros_like(l), np.zeros_like(u))
    cflag = ((zero - l) > u).astype(F32)
    keep = (F32(1.0) - cflag).astype(F32)
    l_new = ((cflag * zero) + (keep * l)).astype(F32)
    n = l.shape[1]
    eye = np.eye(n, dtype=F32)
    Lpoly = ({k_in: (keep[:, :, None] * eye[None]).astype(F32)}, np.zeros_like(l))
    # U' = lam * (prev[U] with its neurons replaced by U (coeff >= 0) / L (< 0)) + mu
    sub_b, sub_c = {}, None
    for t, M in Ub.items():
        Mb = np.broadcast_to(M, (B,) + M.shape[-2:])
        Mp, Mn = _split(Mb)
        (tLb, tLc), (tUb, tUc) = polys[t]
        for s, X in tUb.items():
            _add_block(sub_b, s, np.matmul(Mp, X))
        for s, X in tLb.items():
            _add_block(sub_b, s, np.matmul(Mn, X))
        dcc = (np.einsum('bnm,bm->bn', Mp, tUc, dtype=F32) +
               np.einsum('bnm,bm->bn', Mn, tLc, dtype=F32)).astype(F32)
        sub_c = dcc if sub_c is None else (sub_c + dcc).astype(F32)
    if sub_c is None:
        sub_c = np.zeros_like(l)
    with np.errstate(divide='ignore', invalid='ignore'):
        den = (u - l).astype(F32)
        lam = (u / den).astype(F32)
        mu = (((u * l).astype(F32) * F32(-1.0)).astype(F32) / den).astype(F32)
    Uconst = ((lam * (sub_c + Uc).astype(F32)).astype(F32) + mu).astype(F32)
    Upoly = ({s: (lam[:, :, None] * X).astype(F32) for s, X in sub_b.items()}, Uconst)
    return BRANCH_CROSS, (Lpoly, Upoly), (l_new, u.copy())


def _sum_poly(P, Q):
    """Polyexp of an Add layer: the two parents' polyexps summed (flow_sparse.py:67-88)."""
    blocks = {}
    for t, M in P[0].items():
        _add_block(blocks, t, M)
    for t, M in Q[0].items():
        _add_block(blocks, t, M)
    return blocks, (P[1] + Q[1]).astype(F32)


def _stack_poly(P, Q, B):
    """Polyexp of a Concat layer: the parents' rows stacked (flow_sparse.py:89-178)."""
    n1, n2 = P[1].shape[1], Q[1].shape[1]
    blocks = {}
    for t in sorted(set(P[0]) | set(Q[0])):
        width = (P[0].get(t) if t in P[0] else Q[0][t]).shape[-1]
        M = np.zeros((B, n1 + n2, width), F32)
        if t in P[0]:
            M[:, :n1] = np.broadcast_to(P[0][t], (B, n1, width))
        if t in Q[0]:
            M[:, n1:] = np.broadcast_to(Q[0][t], (B, n2, width))
        blocks[t] = M
    return blocks, np.concatenate([P[1], Q[1]], axis=1).astype(F32)


def certify(layers, l0, u0, spec_W, relaxation="deeppoly", order=min, interval=False, stop_depth=None,
            strict=False):
    """Run the reference's DeepPoly or CROWN program over a network of linear / conv / relu /
    add / concat layers listed in the reference reader's breadth-first order.

    layers : list of cfgpu.nets.Layer (``parents`` per layer), property layer excluded.
    l0, u0 : [B, n0] float32 normalised input box.
    spec_W : [B, 9, 10] per-region property matrix (bias 0).
    relaxation : 'deeppoly' (deeppoly.cf) or 'crown' (crown.cf).
    order  : which live layer the traversal substitutes next (``min`` = the reference's
             priority2 = -layer; tests plant ``max`` to show the golden vectors pin it).
    interval : crownibp.cf -- every affine layer below the property gets the interval
             bound of its polyexp over the previous layer's l / u (``map(simplify_lower)``
             without a traversal); only the property layer is backsubstituted.
    stop_depth : the custom-stop programs' get_start: the traversal bounding layer k stops at
             neurons of layers below k - stop_depth and concretises there with their l / u.
    strict : DeepPoly's lower slope is 1 where l + u > 0 (the custom-stop programs' relu_n,
             deeppoly_custom_stop.cf:25) instead of l + u >= 0.
    Returns (bounds, lb, ub, branches): bounds per layer (excluding input, including
    the property layer) of (l [B,n], u [B,n]); lb/ub float64 [B, 9]; branches the
    BRANCH_* code of every ReLU layer (CROWN).
    """
    l0 = np.asarray(l0, F32)
    u0 = np.asarray(u0, F32)
    B, n0 = l0.shape
    # polys[k] = (L, U) of neuron layer k; layer 0 = input: (empty, const l0 / u0);
    # neuron layer k = layer k-1 of the list
    polys = {0: (({}, l0), ({}, u0))}
    bnd = {0: (l0, u0)}
    branches = []
    for idx, Lyr in enumerate(layers + ['spec']):
        k = idx + 1
        ks = [k - 1] if Lyr == 'spec' else [p + 1 for p in _parents(layers, idx)]
        kind = 'spec' if Lyr == 'spec' else Lyr.kind
        if kind == 'relu':
            l, u = bnd[ks[0]]
            if relaxation == "crown":
                br, polys[k], bnd[k] = _crown_relu(l, u, ks[0], polys, B)
                branches.append(br)
            else:
                polys[k], bnd[k] = _deeppoly_relu(l, u, ks[0], B, strict)
            continue
        if kind == 'add':
            (l1, u1), (l2, u2) = bnd[ks[0]], bnd[ks[1]]
            bnd[k] = ((l1 + l2).astype(F32), (u1 + u2).astype(F32))
            (L1, U1), (L2, U2) = polys[ks[0]], polys[ks[1]]
            polys[k] = (_sum_poly(L1, L2), _sum_poly(U1, U2))
            continue
        if kind == 'concat':
            (l1, u1), (l2, u2) = bnd[ks[0]], bnd[ks[1]]
            bnd[k] = (np.concatenate([l1, l2], axis=1), np.concatenate([u1, u2], axis=1))
            (L1, U1), (L2, U2) = polys[ks[0]], polys[ks[1]]
            polys[k] = (_stack_poly(L1, L2, B), _stack_poly(U1, U2, B))
            continue
        # affine-type layer (or the appended property layer)
        if kind == 'spec':
            A0 = np.asarray(spec_W, F32)
            c0 = np.zeros((B, A0.shape[1]), F32)
            W_prev = {ks[0]: A0}
        else:
            A0 = np.ascontiguousarray(_affine_rows(Lyr, 0, Lyr.n_out, B)[0])
            c0 = np.broadcast_to(layer_bias(Lyr), (B, Lyr.n_out)).astype(F32)
            W_prev = {ks[0]: A0[None]}
        if interval and kind != 'spec':
            pl, pu = bnd[ks[0]]
            Wp, Wn = np.maximum(A0, F32(0)), np.minimum(A0, F32(0))
            bnd[k] = ((pl @ Wp.T + pu @ Wn.T + c0).astype(F32), (pu @ Wp.T + pl @ Wn.T + c0).astype(F32))
        else:
            res = []
            for lower in (True, False):
                res.append(_traverse({t: np.array(np.broadcast_to(M, (B,) + M.shape[-2:]), F32)
                                      for t, M in W_prev.items()}, c0.copy(), polys, lower, order,
                                     None if stop_depth is None else k - stop_depth, bnd))
            bnd[k] = (res[0], res[1])
        poly = (W_prev, c0)
        polys[k] = (poly, poly)
    bounds = [bnd[k] for k in range(1, len(layers) + 2)]
    lb, ub = bounds[-1]
    return bounds, lb.astype(np.float64), ub.astype(np.float64), branches


def custom_stop(layers, l0, u0, spec_W, depth):
    """The reference's deeppoly_custom_stop.cf / custom_stops/deeppoly_custom_stopNN.cf:
    DeepPoly whose traversal for a neuron of layer k stops at layers below k - depth
    (get_start = depth) and concretises there with those neurons' own bounds.  Their relu_n
    is strict (l + u > 0, deeppoly_custom_stop.cf:25)."""
    return certify(layers, l0, u0, spec_W, "deeppoly", min, stop_depth=depth, strict=True)


def crownibp(layers, l0, u0, spec_W, order=max):
    """The reference's crownibp.cf: interval bounds for every layer below the property,
    DeepPoly's ReLU relaxation from them (relu_n, compute_upper: crownibp.cf:19-21), and
    one backward traversal of the property rows (priority2 = +layer: the highest live layer
    first, crownibp.cf:10,24)."""
    return certify(layers, l0, u0, spec_W, "deeppoly", order, interval=True)


def crown(layers, l0, u0, spec_W, order=min):
    """The reference's CROWN program (certify with relaxation='crown')."""
    return certify(layers, l0, u0, spec_W, "crown", order)
