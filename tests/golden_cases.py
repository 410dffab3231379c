"""Loader for the reference-generated golden vectors (tests/golden/*.npz)."""
import glob
import os

import numpy as np

from cfgpu import nets

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def names(program="deeppoly", max_wid=4):
    out = []
    for f in sorted(glob.glob(os.path.join(GOLDEN, "*.npz"))):
        z = np.load(f)
        if str(z["program"]) == program and int(z["wid"]) <= max_wid:
            out.append(os.path.basename(f)[:-4])
    return out


def chain_names(program="deeppoly"):
    """Cases of `program` on chain networks (linear / conv / relu only), every workload."""
    return [n for n in names(program, max_wid=99) if nets.is_chain(nets.workload(_wid(n)).layers)]


def has_conv(name):
    return any(L.kind == "conv" for L in nets.workload(_wid(name)).layers)


def _wid(name):
    return int(np.load(os.path.join(GOLDEN, name + ".npz"))["wid"])


def _expand_compact(wl, z, l0, u0):
    """Full [B, N - n0] per-neuron l/u of a compactly stored case (gen_golden.COMPACT): the
    affine and property columns as stored, each ReLU layer's columns where(x >= 0, x, 0) of
    the affine layer below it (deeppoly.cf:20-24), and the input box recomputed (the stored
    rows of the reference's own input box are l_in / u_in)."""
    B = int(z["B"])
    la, ua = z["l_aff"], z["u_aff"]
    ls, us = [], []
    pos = 0
    for L in wl.layers:
        if L.kind == "relu":
            for dst in (ls, us):
                x = dst[-1]
                dst.append(np.where(x >= 0, x, np.float32(0)).astype(np.float32))
        else:
            ls.append(la[:, pos:pos + L.n_out])
            us.append(ua[:, pos:pos + L.n_out])
            pos += L.n_out
    ls.append(la[:, pos:])
    us.append(ua[:, pos:])
    assert ls[-1].shape == (B, 9)
    return np.concatenate(ls, axis=1), np.concatenate(us, axis=1)


class Case:
    def __init__(self, name):
        z = np.load(os.path.join(GOLDEN, name + ".npz"))
        self.name = name
        self.program = str(z["program"])
        self.wid = int(z["wid"])
        self.B = int(z["B"])
        self.eps = float(z["eps"])
        self.wl = nets.workload(self.wid)
        assert abs(nets.weights_digest(self.wl.layers) - float(z["weights_digest"])) < 1e-6 * max(
            1.0, abs(float(z["weights_digest"]))), "synthetic network drifted from the golden vectors"
        self.X = z["X"]
        self.y = z["y"]
        self.lb, self.ub = z["lb"], z["ub"]
        n0 = self.wl.input_size
        l0, u0 = nets.input_box(self.X, self.eps, self.wl.dataset)
        self.l0, self.u0 = l0.numpy(), u0.numpy()
        self.compact = "compact" in z.files
        if self.compact:
            self.l_all, self.u_all = _expand_compact(self.wl, z, self.l0, self.u0)
            # the reference's own input box is kept for the first regions only
            self.l0_ref, self.u0_ref = z["l_in"], z["u_in"]
        else:
            self.l_all, self.u_all = z["l_all"][:, n0:], z["u_all"][:, n0:]
            self.l0_ref, self.u0_ref = z["l_all"][:, :n0], z["u_all"][:, :n0]
        self.spec_W = nets.spec_weight(self.y).numpy()
        self.sizes = [L.n_out for L in self.wl.layers] + [9]
        kinds = [L.kind for L in self.wl.layers]
        self.relu_layers = [i for i in range(len(kinds) - 1) if kinds[i + 1] == "relu"]
