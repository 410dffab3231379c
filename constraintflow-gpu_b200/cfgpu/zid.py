"""zid.cf: zonotope bounds for the first layers, interval bounds above them, DeepPoly for the
property rows (examples/compiler_examples/zid.cf:30-78).

Per list layer k (the reference's layer index; the input is 0):

  k <= 4    Affine: l, u = the zonotope's concretisation (map(deepz_lower / deepz_upper));
            Relu:   DeepPoly's relaxation from those bounds, Z carried as zono.cf does.
  k > 4     Affine: the interval over the previous layer's l / u (map(simplify_lower)).
            Relu:   DeepPoly's relaxation.
  property  the DeepPoly traversal (priority2 = -layer) through every layer's polyexps.

Both halves are libcfgpu's own per-layer drivers: a zonotope pass (CF_RELAX_ZONO) for the
layers up to 4 and a crownibp.cf pass with zid.cf's strict lower-slope test
(CF_RELAX_CROWNIBP_STRICT: interval layers, DeepPoly relaxation with relu_n's l + u > 0,
zid.cf:22, one backsubstitution of the property rows) for all layers, whose affine bounds
up to layer 4 are replaced by the zonotope's before the ReLU above them is relaxed.
"""
import torch

from . import _lib
from .engine import DeepPolyEngine
from .layerwise import LayerRun

ZONO_UPTO = 4   # zid.cf:38, 62: curr[layer] <= 4


class ZidEngine:
    """A chain network resident on one GPU for zid.cf (same interface as DeepPolyEngine)."""

    certifier = "zid"

    def __init__(self, layers, input_size, device="cuda", n_spec=9, zono_upto=ZONO_UPTO):
        layers = list(layers)
        self.zono_upto = int(zono_upto)
        self.cb = DeepPolyEngine(layers, input_size, device, n_spec=n_spec, certifier="crownibp", relu_strict=True)
        if self.cb.net is None:
            raise NotImplementedError("zid on a network with Add / Concat layers (the zonotope driver runs "
                                      "chain networks)")
        self.zn = DeepPolyEngine(layers, input_size, device, n_spec=n_spec, certifier="zono")
        self.device = self.cb.device
        self.input_size, self.n_spec, self.n_last = self.cb.input_size, self.cb.n_spec, self.cb.n_last
        self.N, self.kinds, self.chain, self.net = self.cb.N, self.cb.kinds, True, self.cb.net
        self.replayed_launches = 0
        self.col, c = [], self.input_size
        for k in range(self.cb.net.n_layers):
            self.col.append(c)
            c += int(self.cb._layers[k].n_out)
        self.width = [int(self.cb._layers[k].n_out) for k in range(self.cb.net.n_layers)]

    def input_spec(self, X, y, eps, dataset):
        return self.cb.input_spec(X, y, eps, dataset)

    def run(self, l0, u0, spec_W, want_state=False, out=None, check_device=False):
        r = ZidRun(self, l0, u0, spec_W)
        for i in range(r.n_layers + 1):
            r.layer(i)
        lb, ub = r.finish() if check_device else (r.lb, r.ub)
        if out is not None:
            out[0].copy_(lb)
            out[1].copy_(ub)
            lb, ub = out
        if want_state:
            return lb, ub, r.state_l, r.state_u
        return lb, ub

    def certify(self, X, y, eps, dataset, out=None):
        l0, u0, W = self.input_spec(X, y, eps, dataset)
        return self.run(l0, u0, W, out=out)


class ZidRun:
    """One pass over a batch, layer by layer (the LayerRun interface)."""

    def __init__(self, engine, l0, u0, spec_W):
        self.engine = engine
        self.cb = LayerRun(engine.cb, l0, u0, spec_W)
        self.zn = LayerRun(engine.zn, l0, u0, spec_W)
        self.n_layers = self.cb.n_layers
        self.state_l, self.state_u = self.cb.state_l, self.cb.state_u
        self.lb, self.ub = self.cb.lb, self.cb.ub
        self.done = -1

    def layer(self, i):
        """Run network layer i (i == n_layers: the property layer); layers run in order."""
        if i != self.done + 1:
            raise ValueError(f"layer {i} after layer {self.done}: layers run in order")
        zono = i < self.n_layers and i + 1 <= self.engine.zono_upto
        if zono:
            self.zn.layer(i)
        self.cb.layer(i)
        if zono and self.engine.kinds[i] in ("linear", "conv"):
            c0, c1 = self.engine.col[i], self.engine.col[i] + self.engine.width[i]
            self.cb.state_l[:, c0:c1].copy_(self.zn.state_l[:, c0:c1])
            self.cb.state_u[:, c0:c1].copy_(self.zn.state_u[:, c0:c1])
        self.done = i
        return self

    def finish(self):
        """Device status of both passes and the float64 property bounds."""
        if self.done != self.n_layers:
            raise ValueError(f"pass stopped after layer {self.done} of {self.n_layers}")
        stream = torch.cuda.current_stream(self.engine.device).cuda_stream
        _lib.check(_lib.lib.cf_deeppoly_check(self.zn.ws.data_ptr(), stream), "device status")
        return self.cb.finish()
