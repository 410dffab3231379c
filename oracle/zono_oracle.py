"""CPU oracle for the reference's zonotope (DeepZ), interval and polyzono programs (numpy,
float32).

TEST INFRASTRUCTURE ONLY.  Only tests/, ``__graft_entry__.smoke()`` and bench.py's
CPU legs may import this module, as the checker; the product path (cfgpu) never
imports it and has no CPU fallback.

What it restates: the reference compiler's output for
examples/compiler_examples/zono.cf, zono2.cf, ibp.cf and polyzono.cf (kept as fixtures in
tests/golden/generated/<program>/transformers.py), run forward by
constraintflow/lib/flow_sparse.py:27-228.

* Zonotope state (create_Z, constraintflow/lib/spec.py:106-132): every neuron is
  c + sum_e M[., e] eps_e with eps_e in [-1, 1].  The input layer has one noise symbol
  per input neuron: c0 = (l0 + u0) / 2, M0 = diag((u0 - l0) / 2).  Representation here:
  M [B, n, E] (the layer's rows of the reference's [B, N, E] SymExp matrix), c [B, n].
* zono.Affine (zono.cf Affine; generated ``Affine``): c' = W c + b (inner_prod, then
  the bias), M' = W M, and the bounds are the zonotope's concretisation
  l = (sum_e M'+ * (-1) + sum_e M'- * 1) + c', u = (sum_e M'+ * 1 + sum_e M'- * (-1)) + c'
  (the ``map(deepz_lower / deepz_upper)`` over the noise terms).  Conv layers apply the
  convolution to every noise column.
* zono.Relu: get_new_eps (constraintflow/lib/symexp.py:14) opens one fresh noise symbol
  per neuron of the layer (columns E .. E+n-1, a diagonal of ones).  With the previous
  layer's l, u, (M, c):
    x = (u * z) / (u - l) + ((u * l) * (eps - 1)) / (2 * (u - l)),
  i.e. const (u*c)/(u-l) + ((u*l)*(-1))/(2*(u-l)), old columns (u*M)/(u-l), the neuron's
  fresh column (u*l)/(2*(u-l)); Z' = where(l >= 0, Z, where(u <= 0, 0, x)).  The ReLU
  layer's own l, u are set to 0 (the program's tuple is (0, 0, Z')).
* zono2.Relu: the ternary of tuples is lowered to whole-layer branches over the batch
  (as with crown.cf): any(l >= 0) -> (l, u, Z) unchanged; else any(u <= 0) -> zeros;
  else l' = (u*l)/(u-l), u' = u, Z' = (u*Z)/(u-l) - ((u*l)/(2*(u-l))) * (1 + eps).
* ibp (ibp.cf): Affine l' = (W+ l + W- u) + b, u' = (W+ u + W- l) + b;
  Relu l' = 1[l>=0] l + (1 - 1[l>=0]) 0 (same for u).
* polyzono (polyzono.cf:30-46): DeepPoly's state and the zonotope side by side; an
  affine layer's bounds are max / min of the two (cf_max / cf_min,
  constraintflow/gbcsr/tensor_ops.py:226, :245), and both ReLU relaxations use the met
  bounds (``polyzono`` below).

Pinned against: the reference's own outputs (tests/golden/zono_*.npz, zono2_*.npz,
ibp_*.npz, pz_*.npz, made by tests/golden/gen_golden.py).
"""
import numpy as np

from .deeppoly_oracle import F32, _conv_T, layer_bias

BRANCH_PASS, BRANCH_ZERO, BRANCH_CROSS = 0, 1, 2


def _parents(layers, i):
    p = layers[i].parents
    return tuple(p) if p is not None else (i - 1,)


def weight_matrix(layer):
    """Dense [n_out, n_in] matrix of an affine layer (the conv's Toeplitz matrix)."""
    if layer.kind == 'linear':
        return layer.W.astype(F32)
    n_out = layer.n_out
    return _conv_T(np.eye(n_out, dtype=F32), layer)


def create_z(l0, u0):
    """spec.py:106-132: c0 = (l+u)/2, M0 = diag((u-l)/2) over one symbol per input neuron."""
    mid = ((l0 + u0) / F32(2)).astype(F32)
    dist = ((u0 - l0) / F32(2)).astype(F32)
    B, n = l0.shape
    M = np.zeros((B, n, n), F32)
    M[:, np.arange(n), np.arange(n)] = dist
    return M, mid


def zono_affine(M, c, W, b):
    """Generated zono.Affine: (l, u, M', c').  W [n_out, n_in] or per-region [B, n_out, n_in]."""
    if W.ndim == 2:
        Mn = np.matmul(W[None], M).astype(F32)
        cn = np.einsum('oi,bi->bo', W, c, dtype=F32).astype(F32)
    else:
        Mn = np.matmul(W, M).astype(F32)
        cn = np.einsum('boi,bi->bo', W, c, dtype=F32).astype(F32)
    cn = (cn + b).astype(F32)
    pos = np.maximum(Mn, F32(0)).sum(axis=2, dtype=F32)
    neg = np.minimum(Mn, F32(0)).sum(axis=2, dtype=F32)
    l = ((pos * F32(-1)) + neg + cn).astype(F32)
    u = (pos + (neg * F32(-1)) + cn).astype(F32)
    return l, u, Mn, cn


def zono_relu(l, u, M, c):
    """Generated zono.Relu: (M', c') with n fresh noise columns appended."""
    B, n, E = M.shape
    with np.errstate(divide='ignore', invalid='ignore', over='ignore'):
        den = (u - l).astype(F32)
        den2 = (F32(2) * den).astype(F32)
        ul = (u * l).astype(F32)
        cx = (((u * c).astype(F32) / den).astype(F32) + ((ul * F32(-1)).astype(F32) / den2).astype(F32)).astype(F32)
        Mx_old = ((u[:, :, None] * M).astype(F32) / den[:, :, None]).astype(F32)
        new_coef = (ul / den2).astype(F32)
    pos = l >= F32(0)
    dead = (~pos) & (u <= F32(0))
    Mn = np.zeros((B, n, E + n), F32)
    Mn[:, :, :E] = np.where(pos[:, :, None], M, np.where(dead[:, :, None], F32(0), Mx_old))
    diag = np.where(pos | dead, F32(0), new_coef).astype(F32)
    Mn[:, np.arange(n), E + np.arange(n)] = diag
    cn = np.where(pos, c, np.where(dead, F32(0), cx)).astype(F32)
    return Mn, cn


def zono2_relu(l, u, M, c):
    """Generated zono2.Relu: one whole-layer branch.  Returns (branch, l', u', M', c')."""
    B, n, E = M.shape
    if np.any(l >= F32(0)):
        return BRANCH_PASS, l, u, M, c
    if np.any(u <= F32(0)):
        z = np.zeros_like(l)
        return BRANCH_ZERO, z, z.copy(), np.zeros((B, n, E), F32), z.copy()
    with np.errstate(divide='ignore', invalid='ignore'):
        ul = (u * l).astype(F32)
        den = (u - l).astype(F32)
        l_new = (ul / den).astype(F32)
        c17 = ((u * c).astype(F32) / den).astype(F32)
        M19 = ((u[:, :, None] * M).astype(F32) / den[:, :, None]).astype(F32)
        k1 = (ul / (F32(2) * den).astype(F32)).astype(F32)
    c16 = (k1 * F32(1)).astype(F32)                       # k1 * (1 + eps): const part 1 + 0
    Mn = np.zeros((B, n, E + n), F32)
    Mn[:, :, :E] = M19
    Mn[:, np.arange(n), E + np.arange(n)] = (F32(0) - k1).astype(F32)
    return BRANCH_CROSS, l_new, u.copy(), Mn, (c17 - c16).astype(F32)


def _bias(layer):
    return layer_bias(layer)


def zono(layers, l0, u0, spec_W, program="zono"):
    """Run zono.cf (DeepZ) or zono2.cf over a network (chain or Add / Concat DAG).

    Returns (bounds, lb, ub, branches): bounds per layer (excluding input, including the
    property layer) of (l [B,n], u [B,n]); lb/ub float64 [B, 9]; branches per ReLU (zono2).
    """
    l0 = np.asarray(l0, F32)
    u0 = np.asarray(u0, F32)
    M0, c0 = create_z(l0, u0)
    E = M0.shape[2]
    state = {0: (l0, u0, M0, c0)}
    branches = []
    for idx, L in enumerate(list(layers) + ['spec']):
        k = idx + 1
        ks = [k - 1] if L == 'spec' else [p + 1 for p in _parents(layers, idx)]
        kind = 'spec' if L == 'spec' else L.kind
        pl, pu, pM, pc = state[ks[0]]
        pM = _widen(pM, E)
        if kind == 'relu':
            if program == "zono2":
                br, ln, un, Mn, cn = zono2_relu(pl, pu, pM, pc)
                branches.append(br)
                if Mn.shape[2] > E:
                    E = Mn.shape[2]
            else:
                Mn, cn = zono_relu(pl, pu, pM, pc)
                E = Mn.shape[2]
                ln, un = np.zeros_like(pl), np.zeros_like(pu)
            state[k] = (ln, un, Mn, cn)
            continue
        if kind in ('add', 'concat'):
            ql, qu, qM, qc = state[ks[1]]
            qM = _widen(qM, E)
            if kind == 'add':
                Mn = (pM + qM).astype(F32)
                cn = (pc + qc).astype(F32)
                state[k] = ((pl + ql).astype(F32), (pu + qu).astype(F32), Mn, cn)
            else:
                state[k] = (np.concatenate([pl, ql], 1), np.concatenate([pu, qu], 1),
                            np.concatenate([pM, qM], 1), np.concatenate([pc, qc], 1))
            continue
        if kind == 'spec':
            W, b = np.asarray(spec_W, F32), np.zeros(spec_W.shape[1], F32)
        else:
            W, b = weight_matrix(L), _bias(L)
        ln, un, Mn, cn = zono_affine(pM, pc, W, b)
        state[k] = (ln, un, Mn, cn)
    bounds = [state[k][:2] for k in range(1, len(layers) + 2)]
    lb, ub = bounds[-1]
    return bounds, lb.astype(np.float64), ub.astype(np.float64), branches


def _widen(M, E):
    """A symbol matrix with zero columns for symbols opened after it was formed
    (SymExpSparse.expand_mat, symexp.py:200)."""
    if M.shape[2] == E:
        return M
    out = np.zeros(M.shape[:2] + (E,), F32)
    out[:, :, :M.shape[2]] = M
    return out


def ibp(layers, l0, u0, spec_W):
    """Run ibp.cf: interval bounds layer by layer.  Returns (bounds, lb, ub)."""
    l0 = np.asarray(l0, F32)
    u0 = np.asarray(u0, F32)
    state = {0: (l0, u0)}
    zero = F32(0)
    for idx, L in enumerate(list(layers) + ['spec']):
        k = idx + 1
        ks = [k - 1] if L == 'spec' else [p + 1 for p in _parents(layers, idx)]
        kind = 'spec' if L == 'spec' else L.kind
        pl, pu = state[ks[0]]
        if kind == 'relu':
            fl = (pl >= zero).astype(F32)
            fu = (pu >= zero).astype(F32)
            state[k] = (((fl * pl) + ((F32(1) - fl) * zero)).astype(F32),
                        ((fu * pu) + ((F32(1) - fu) * zero)).astype(F32))
            continue
        if kind in ('add', 'concat'):
            ql, qu = state[ks[1]]
            state[k] = (((pl + ql), (pu + qu)) if kind == 'add' else
                        (np.concatenate([pl, ql], 1), np.concatenate([pu, qu], 1)))
            continue
        if kind == 'spec':
            W = np.asarray(spec_W, F32)
            b = np.zeros(W.shape[1], F32)
            Wp, Wn = np.maximum(W, zero), np.minimum(W, zero)
            l = (np.einsum('boi,bi->bo', Wp, pl, dtype=F32) + np.einsum('boi,bi->bo', Wn, pu, dtype=F32)).astype(F32)
            u = (np.einsum('boi,bi->bo', Wp, pu, dtype=F32) + np.einsum('boi,bi->bo', Wn, pl, dtype=F32)).astype(F32)
        else:
            W, b = weight_matrix(L), _bias(L)
            Wp, Wn = np.maximum(W, zero), np.minimum(W, zero)
            l = (pl @ Wp.T + pu @ Wn.T).astype(F32)
            u = (pu @ Wp.T + pl @ Wn.T).astype(F32)
        state[k] = ((l + b).astype(F32), (u + b).astype(F32))
    bounds = [state[k] for k in range(1, len(layers) + 2)]
    lb, ub = bounds[-1]
    return bounds, lb.astype(np.float64), ub.astype(np.float64)


def polyzono(layers, l0, u0, spec_W):
    """Run polyzono.cf over a chain network: the DeepPoly state (L, U polyexps, backward
    traversal lowest layer first) and the zonotope Z carried side by side.

    Affine (generated polyzono.Affine): l = max(Z's concretisation, the DeepPoly backward
    bound), u = min(...); L = U = W x + b; Z' = W Z + b.  Relu: l' = relu(l), u' = relu(u) and
    DeepPoly's L', U' from the combined bounds (its strict comparisons in relu and
    compute_upper give the same values as deeppoly.cf's at l = 0 or u = 0); Z' as in zono.cf,
    also from the combined bounds.  Returns (bounds, lb, ub).
    """
    from .crown_oracle import _deeppoly_relu, _traverse
    from .deeppoly_oracle import _affine_rows
    l0 = np.asarray(l0, F32)
    u0 = np.asarray(u0, F32)
    B = l0.shape[0]
    polys = {0: (({}, l0), ({}, u0))}
    bnd = {0: (l0, u0)}
    M, c = create_z(l0, u0)
    E = M.shape[2]
    for idx, L in enumerate(list(layers) + ['spec']):
        k = idx + 1
        kind = 'spec' if L == 'spec' else L.kind
        pl, pu = bnd[k - 1]
        M = _widen(M, E)
        if kind == 'relu':
            polys[k], bnd[k] = _deeppoly_relu(pl, pu, k - 1, B)
            M, c = zono_relu(pl, pu, M, c)
            E = M.shape[2]
            continue
        if kind == 'spec':
            A0 = np.asarray(spec_W, F32)
            c0 = np.zeros((B, A0.shape[1]), F32)
            W_prev = {k - 1: A0}
            Wm, b = A0, np.zeros(A0.shape[1], F32)
        else:
            A0 = np.ascontiguousarray(_affine_rows(L, 0, L.n_out, B)[0])
            c0 = np.broadcast_to(layer_bias(L), (B, L.n_out)).astype(F32)
            W_prev = {k - 1: A0[None]}
            Wm, b = weight_matrix(L), _bias(L)
        res = [_traverse({t: np.array(np.broadcast_to(X, (B,) + X.shape[-2:]), F32) for t, X in W_prev.items()},
                         c0.copy(), polys, lower) for lower in (True, False)]
        lz, uz, M, c = zono_affine(M, c, Wm, b)
        bnd[k] = (np.maximum(lz, res[0]).astype(F32), np.minimum(uz, res[1]).astype(F32))
        poly = (W_prev, c0)
        polys[k] = (poly, poly)
    bounds = [bnd[k] for k in range(1, len(layers) + 2)]
    lb, ub = bounds[-1]
    return bounds, lb.astype(np.float64), ub.astype(np.float64)


def zid(layers, l0, u0, spec_W, zono_upto=4, strict=True):
    """Run zid.cf over a chain network (examples/compiler_examples/zid.cf:30-78): list layers
    with reference index <= 4 (the input is 0) bound their neurons by the zonotope (the
    affine's concretisation; the ReLU carries Z as zono.cf does), layers above by the
    interval over the previous layer's l / u (map(simplify_lower)), and the property rows
    by the DeepPoly traversal (priority2 = -layer) through the polyexps of every layer.
    Every ReLU layer takes DeepPoly's relaxation from its input's bounds with relu_n's
    strict test l + u > 0 (zid.cf:22; ``strict=False`` plants the non-strict test).
    Returns (bounds, lb, ub)."""
    from .crown_oracle import _deeppoly_relu, _traverse
    from .deeppoly_oracle import _affine_rows
    l0 = np.asarray(l0, F32)
    u0 = np.asarray(u0, F32)
    B = l0.shape[0]
    polys = {0: (({}, l0), ({}, u0))}
    bnd = {0: (l0, u0)}
    M, c = create_z(l0, u0)
    E = M.shape[2]
    for idx, L in enumerate(list(layers) + ['spec']):
        k = idx + 1
        kind = 'spec' if L == 'spec' else L.kind
        pl, pu = bnd[k - 1]
        if kind == 'relu':
            polys[k], bnd[k] = _deeppoly_relu(pl, pu, k - 1, B, strict=strict)
            if k <= zono_upto:
                M, c = zono_relu(pl, pu, _widen(M, E), c)
                E = M.shape[2]
            continue
        if kind == 'spec':
            A0 = np.asarray(spec_W, F32)
            c0 = np.zeros((B, A0.shape[1]), F32)
            W_prev = {k - 1: A0}
            res = [_traverse({t: np.array(np.broadcast_to(X, (B,) + X.shape[-2:]), F32) for t, X in W_prev.items()},
                             c0.copy(), polys, lower) for lower in (True, False)]
            bnd[k] = (res[0], res[1])
            continue
        A0 = np.ascontiguousarray(_affine_rows(L, 0, L.n_out, B)[0])
        c0 = np.broadcast_to(layer_bias(L), (B, L.n_out)).astype(F32)
        if k <= zono_upto:
            lz, uz, M, c = zono_affine(_widen(M, E), c, weight_matrix(L), _bias(L))
            E = M.shape[2]
            bnd[k] = (lz, uz)
        else:
            Wp, Wn = np.maximum(A0, F32(0)), np.minimum(A0, F32(0))
            bnd[k] = ((pl @ Wp.T + pu @ Wn.T + c0).astype(F32), (pu @ Wp.T + pl @ Wn.T + c0).astype(F32))
        poly = ({k - 1: A0[None]}, c0)
        polys[k] = (poly, poly)
    bounds = [bnd[k] for k in range(1, len(layers) + 2)]
    lb, ub = bounds[-1]
    return bounds, lb.astype(np.float64), ub.astype(np.float64)
