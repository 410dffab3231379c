"""GPU tests of the individual C-ABI kernels (relaxation, step, concretisation, gbcsr
elementwise ops) against the oracle / numpy on seeded inputs, including ragged and
empty shapes."""
import ctypes

import numpy as np
import pytest
import torch

from oracle import deeppoly_oracle as O

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def _lib():
    from cfgpu import _lib
    return _lib


def _stream():
    return torch.cuda.current_stream(DEV).cuda_stream


def _t(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def _relu_inputs(rng, B, n):
    l = rng.standard_normal((B, n)).astype(np.float32)
    u = l + np.abs(rng.standard_normal((B, n))).astype(np.float32)
    l[:, :3] = [-1.0, 0.0, 2.0]
    u[:, :3] = [1.0, 0.0, 2.0]          # symmetric tie (l+u == 0), zero box, stable
    return l, u


@pytest.mark.parametrize("B,n", [(1, 1), (3, 17), (7, 200), (64, 100)])
def test_relu_relax_bit_exact(B, n):
    L = _lib()
    rng = np.random.default_rng(B * 1000 + n)
    l, u = _relu_inputs(rng, B, max(n, 3))
    n = l.shape[1]
    lt, ut = _t(l), _t(u)
    lo, uo, a, lam, mu = (torch.empty(B, n, device=DEV) for _ in range(5))
    st = L.lib.cf_relu_relax(B, n, lt.data_ptr(), ut.data_ptr(), n, lo.data_ptr(), uo.data_ptr(), n,
                             a.data_ptr(), lam.data_ptr(), mu.data_ptr(), 0, _stream())
    L.check(st)
    ref = O.relu_relax(l, u)
    for got, want in zip((lo, uo, a, lam, mu), ref):
        np.testing.assert_array_equal(got.cpu().numpy(), want)


@pytest.mark.parametrize("B,R,K,N,relu,lower_only", [(1, 1, 1, 1, True, False), (2, 5, 33, 17, True, False),
                                                     (3, 50, 200, 784, True, False), (4, 9, 10, 200, False, False),
                                                     (2, 64, 64, 64, True, False), (1, 130, 70, 129, True, True)])
def test_backsub_step_against_float64(B, R, K, N, relu, lower_only):
    L = _lib()
    rng = np.random.default_rng(B + R + K + N)
    A = rng.standard_normal((2, B, R, K)).astype(np.float32)
    c = rng.standard_normal((2, B, R)).astype(np.float32)
    W = rng.standard_normal((K, N)).astype(np.float32)
    bias = rng.standard_normal(K).astype(np.float32)
    if relu:
        l, u = _relu_inputs(rng, B, max(K, 3))
        l, u = l[:, :K], u[:, :K]
        _, _, al, lam, mu = O.relu_relax(l, u)
    Aout = torch.empty(2, B, R, N, device=DEV)
    cout = torch.empty(2, B, R, device=DEV)
    At, ct, Wt, bt = _t(A), _t(c), _t(W), _t(bias)
    rel = [None, None, None]
    if relu:
        alt, lamt, mut = _t(al), _t(lam), _t(mu)
        rel = [alt.data_ptr(), lamt.data_ptr(), mut.data_ptr()]
    st = L.lib.cf_backsub_step(B, R, K, N, At.data_ptr(), B * R * K, R * K, K, ct.data_ptr(), B * R, R,
                               *rel, Wt.data_ptr(), bt.data_ptr(), Aout.data_ptr(), cout.data_ptr(), _stream())
    L.check(st)
    torch.cuda.synchronize()
    # float64 reference of the same step
    A64 = A.astype(np.float64)
    res_A = np.empty((2, B, R, N))
    res_c = np.empty((2, B, R))
    for s in range(2):
        a = A64[s]
        if relu:
            pf, nf = (al, lam) if s == 0 else (lam, al)
            T = np.where(a >= 0, a * pf[:, None, :], a * nf[:, None, :])
            mterm = np.where(a < 0, a, 0) if s == 0 else np.where(a > 0, a, 0)
            cm = np.einsum('brk,bk->br', mterm, mu.astype(np.float64))
        else:
            T, cm = a, 0.0
        res_A[s] = T @ W.astype(np.float64)
        res_c[s] = c[s] + cm + T @ bias.astype(np.float64)
    scale = np.abs(res_A).max() + 1e-30
    np.testing.assert_allclose(Aout.cpu().numpy(), res_A, rtol=1e-5, atol=1e-5 * scale)
    np.testing.assert_allclose(cout.cpu().numpy(), res_c, rtol=1e-5, atol=1e-5 * (np.abs(res_c).max() + 1))


def test_backsub_step_broadcast_rows():
    """Zero region/bound strides: the first step reads one shared weight matrix."""
    L = _lib()
    rng = np.random.default_rng(7)
    B, R, K, N = 3, 20, 40, 30
    Wm = rng.standard_normal((R, K)).astype(np.float32)
    bm = rng.standard_normal(R).astype(np.float32)
    W = rng.standard_normal((K, N)).astype(np.float32)
    bias = rng.standard_normal(K).astype(np.float32)
    l, u = _relu_inputs(rng, B, K)
    _, _, al, lam, mu = O.relu_relax(l, u)
    Aout = torch.empty(2, B, R, N, device=DEV)
    cout = torch.empty(2, B, R, device=DEV)
    ts = [_t(x) for x in (Wm, bm, W, bias, al, lam, mu)]
    st = L.lib.cf_backsub_step(B, R, K, N, ts[0].data_ptr(), 0, 0, K, ts[1].data_ptr(), 0, 0, ts[4].data_ptr(),
                               ts[5].data_ptr(), ts[6].data_ptr(), ts[2].data_ptr(), ts[3].data_ptr(),
                               Aout.data_ptr(), cout.data_ptr(), _stream())
    L.check(st)
    A = np.broadcast_to(Wm, (B, R, K)).astype(np.float32)
    for s, lower in ((0, True), (1, False)):
        An, cn = O.subst_relu(A, np.broadcast_to(bm, (B, R)).astype(np.float32), al, lam, mu, lower)
        want = An.astype(np.float64) @ W
        np.testing.assert_allclose(Aout[s].cpu().numpy(), want, rtol=1e-5, atol=1e-5 * np.abs(want).max())


@pytest.mark.parametrize("B,R,n0", [(1, 1, 1), (2, 9, 784), (5, 33, 3072)])
def test_concretize(B, R, n0):
    L = _lib()
    rng = np.random.default_rng(n0)
    A = rng.standard_normal((2, B, R, n0)).astype(np.float32)
    c = rng.standard_normal((2, B, R)).astype(np.float32)
    l0 = rng.standard_normal((B, n0)).astype(np.float32)
    u0 = l0 + np.abs(rng.standard_normal((B, n0))).astype(np.float32)
    out_l = torch.full((B, R + 3), float("nan"), device=DEV)
    out_u = torch.full((B, R + 3), float("nan"), device=DEV)
    At, ct, lt, ut = _t(A), _t(c), _t(l0), _t(u0)
    st = L.lib.cf_concretize(B, R, n0, At.data_ptr(), B * R * n0, R * n0, n0, ct.data_ptr(), B * R, R,
                             lt.data_ptr(), ut.data_ptr(), out_l.data_ptr(), out_u.data_ptr(), R + 3, _stream())
    L.check(st)
    wl = O.concretize(A[0], c[0], l0, u0, True)
    wu = O.concretize(A[1], c[1], l0, u0, False)
    gl, gu = out_l.cpu().numpy(), out_u.cpu().numpy()
    sc = np.abs(A).sum(-1).max() * np.abs(np.concatenate([l0, u0])).max()
    np.testing.assert_allclose(gl[:, :R], wl, rtol=1e-5, atol=1e-6 * sc)
    np.testing.assert_allclose(gu[:, :R], wu, rtol=1e-5, atol=1e-6 * sc)
    assert np.isnan(gl[:, R:]).all() and np.isnan(gu[:, R:]).all()  # untouched padding


OPS = ["add", "sub", "mul", "truediv", "ge", "gt", "le", "lt", "eq", "ne", "and_", "or_", "max", "min"]


@pytest.mark.parametrize("op", OPS)
def test_ew_binary_broadcast(op):
    L = _lib()
    rng = np.random.default_rng(len(op))
    shape = (3, 5, 7)
    x = rng.standard_normal(shape).astype(np.float32)
    y = rng.standard_normal((1, 5, 1)).astype(np.float32)
    x[0, 0, :2] = 0.0
    y[0, 0, 0] = 0.0
    xt, yt = _t(x), _t(y)
    is_bool = op in ("ge", "gt", "le", "lt", "eq", "ne", "and_", "or_")
    out = torch.empty(shape, device=DEV, dtype=torch.uint8 if is_bool else torch.float32)
    shp = L.i64_array(shape)
    xs = L.i64_array([35, 7, 1])
    ys = L.i64_array([0, 1, 0])
    st = L.lib.cf_ew_binary(L.OPS[op], 3, shp, xt.data_ptr(), 0, xs, yt.data_ptr(), 0, ys, out.data_ptr(),
                            1 if is_bool else 0, _stream())
    L.check(st)
    yb = np.broadcast_to(y, shape)
    f = {"add": np.add, "sub": np.subtract, "mul": np.multiply, "truediv": np.divide, "ge": np.greater_equal,
         "gt": np.greater, "le": np.less_equal, "lt": np.less, "eq": np.equal, "ne": np.not_equal,
         "and_": lambda a, b: (a != 0) & (b != 0), "or_": lambda a, b: (a != 0) | (b != 0),
         "max": np.maximum, "min": np.minimum}[op]
    with np.errstate(divide="ignore", invalid="ignore"):
        want = f(x, yb)
    got = out.cpu().numpy()
    if is_bool:
        np.testing.assert_array_equal(got.astype(bool), want)
    else:
        np.testing.assert_array_equal(got, want.astype(np.float32))


def test_ew_unary_where_clamp_any():
    L = _lib()
    rng = np.random.default_rng(3)
    shape = (4, 6)
    x = rng.standard_normal(shape).astype(np.float32)
    x[0, 0] = 0.0
    xt = _t(x)
    shp = L.i64_array(shape)
    cs = L.i64_array([6, 1])
    s = _stream()
    neg = torch.empty(shape, device=DEV)
    L.check(L.lib.cf_ew_unary(L.UOPS["neg"], 2, shp, xt.data_ptr(), 0, cs, neg.data_ptr(), 0, s))
    np.testing.assert_array_equal(neg.cpu().numpy(), -x)
    notx = torch.empty(shape, device=DEV, dtype=torch.uint8)
    L.check(L.lib.cf_ew_unary(L.UOPS["not_"], 2, shp, xt.data_ptr(), 0, cs, notx.data_ptr(), 1, s))
    np.testing.assert_array_equal(notx.cpu().numpy().astype(bool), x == 0)
    cond = _t((x > 0).astype(np.uint8))
    y = _t(np.full(shape, 5.0, np.float32))
    z = _t(np.array([[-1.0]], np.float32))
    out = torch.empty(shape, device=DEV)
    L.check(L.lib.cf_ew_where(2, shp, cond.data_ptr(), cs, y.data_ptr(), cs, z.data_ptr(), L.i64_array([0, 0]),
                              out.data_ptr(), 0, s))
    np.testing.assert_array_equal(out.cpu().numpy(), np.where(x > 0, 5.0, -1.0).astype(np.float32))
    for mt in (1, 0):
        L.check(L.lib.cf_ew_clamp(2, shp, xt.data_ptr(), cs, 0.0, mt, out.data_ptr(), s))
        want = np.maximum(x, 0) if mt else np.minimum(x, 0)
        np.testing.assert_array_equal(out.cpu().numpy(), want)
    flag = torch.zeros(1, dtype=torch.int32, device=DEV)
    zeros = _t(np.zeros(shape, np.float32))
    L.check(L.lib.cf_ew_any(2, shp, zeros.data_ptr(), 0, cs, flag.data_ptr(), s))
    assert int(flag.item()) == 0
    L.check(L.lib.cf_ew_any(2, shp, xt.data_ptr(), 0, cs, flag.data_ptr(), s))
    assert int(flag.item()) == 1


def test_signscale_matches_torch():
    """cf_signscale: sign-selected column scaling and the constant row sums, against a
    float64 torch restatement."""
    import torch
    from cfgpu import ops
    g = torch.Generator().manual_seed(7)
    dev = torch.device("cuda:0")
    nb, M, N = 3, 37, 203
    A = torch.randn(nb, M, N, generator=g)
    A[0, 0, :5] = 0.0
    p, q, pc, qc = (torch.randn(nb, N, generator=g) for _ in range(4))
    out, dc = ops.signscale(A.to(dev), p.to(dev), q.to(dev), pc.to(dev), qc.to(dev))
    pos = A >= 0
    ref = torch.where(pos, A * p[:, None, :], A * q[:, None, :])
    rdc = torch.where(pos, A.double() * pc[:, None, :].double(), A.double() * qc[:, None, :].double()).sum(-1)
    assert torch.equal(out.cpu(), ref)
    assert torch.allclose(dc.cpu().double(), rdc, rtol=1e-5, atol=1e-5)
    out2, dc2 = ops.signscale(A.to(dev), p.to(dev), q.to(dev), None, qc.to(dev))
    rdc2 = torch.where(pos, torch.zeros_like(A).double(), A.double() * qc[:, None, :].double()).sum(-1)
    assert torch.equal(out2.cpu(), ref) and torch.allclose(dc2.cpu().double(), rdc2, rtol=1e-5, atol=1e-5)
