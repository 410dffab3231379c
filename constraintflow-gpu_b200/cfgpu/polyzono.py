"""polyzono.cf: the DeepPoly state (l, u, L, U) and the zonotope Z carried side by side
(examples/compiler_examples/polyzono.cf:30-46).

Per layer the program computes both certifiers' results and meets their bounds:

  Affine: l = max(Z's concretisation, DeepPoly's backward bound), u = min(...)
          (polyzono.cf:32-33; the generated code's cf_max / cf_min,
          constraintflow/gbcsr/tensor_ops.py:226, :245); L = U = W x + b; Z' = W Z + b.
  Relu:   l' = relu(l), u' = relu(u); DeepPoly's relaxation (relu_n, compute_upper) and the
          zonotope's (fresh noise symbols), both from the met bounds (polyzono.cf:39-45).

Both halves are libcfgpu's own per-layer drivers (cf_deeppoly_layer on a DeepPoly and on a
zonotope network description).  Each reads an affine layer's bounds from its state columns
when it relaxes the ReLU above it, so one cf_bounds_meet per affine layer -- writing the
met bounds into both states -- is all the coupling the program needs.  relu_n keeps
deeppoly.cf's lower-slope choice (l + u >= 0); compute_upper's strict comparisons give the
same values as deeppoly.cf's at l = 0 or u = 0, so DeepPoly's relaxation kernel applies.
"""
import torch

from . import _lib
from .engine import DeepPolyEngine
from .layerwise import LayerRun


class PolyZonoEngine:
    """A chain network resident on one GPU for polyzono.cf; same interface as
    DeepPolyEngine (run / certify / input_spec / kinds / N)."""

    certifier = "polyzono"

    def __init__(self, layers, input_size, device="cuda", n_spec=9):
        layers = list(layers)
        self.dp = DeepPolyEngine(layers, input_size, device, n_spec=n_spec, certifier="deeppoly")
        if self.dp.net is None:
            raise NotImplementedError("polyzono on a network with Add / Concat layers (the zonotope driver runs "
                                      "chain networks)")
        self.zn = DeepPolyEngine(layers, input_size, device, n_spec=n_spec, certifier="zono")
        self.device = self.dp.device
        self.input_size, self.n_spec, self.n_last = self.dp.input_size, self.dp.n_spec, self.dp.n_last
        self.N, self.kinds, self.chain = self.dp.N, self.dp.kinds, True
        self.net = self.dp.net
        self.replayed_launches = 0
        # first state column of every layer (the input occupies [0, input_size)); the
        # property layer's columns are the last n_spec
        self.col = []
        c = self.input_size
        for k in range(self.dp.net.n_layers):
            self.col.append(c)
            c += int(self.dp._layers[k].n_out)
        self.spec_col = c
        self.width = [int(self.dp._layers[k].n_out) for k in range(self.dp.net.n_layers)]

    def input_spec(self, X, y, eps, dataset):
        return self.dp.input_spec(X, y, eps, dataset)

    def run(self, l0, u0, spec_W, want_state=False, out=None, check_device=False):
        """Bounds for B regions: (lb, ub) float64 [B, n_spec] and, if want_state, the met
        state (state_l, state_u) float32 [B, N]."""
        r = PolyZonoRun(self, l0, u0, spec_W, out=out)
        for i in range(r.n_layers + 1):
            r.layer(i)
        lb, ub = r.finish() if check_device else (r.lb, r.ub)
        if want_state:
            return lb, ub, r.state_l, r.state_u
        return lb, ub

    def certify(self, X, y, eps, dataset, out=None):
        l0, u0, W = self.input_spec(X, y, eps, dataset)
        return self.run(l0, u0, W, out=out)


class PolyZonoRun:
    """One pass over a batch, layer by layer (the LayerRun interface): a DeepPoly and a
    zonotope LayerRun on the same inputs, their bounds met after every affine layer."""

    def __init__(self, engine, l0, u0, spec_W, out=None):
        self.engine = engine
        self.dp = LayerRun(engine.dp, l0, u0, spec_W)
        self.zn = LayerRun(engine.zn, l0, u0, spec_W)
        self.B = self.dp.B
        self.n_layers = self.dp.n_layers
        self.state_l, self.state_u = self.dp.state_l, self.dp.state_u
        if out is None:
            self.lb, self.ub = self.dp.lb, self.dp.ub
        else:
            self.lb, self.ub = out
        self.done = -1

    def _meet(self, col, n, final):
        stream = torch.cuda.current_stream(self.engine.device).cuda_stream
        N = self.engine.N
        st = _lib.lib.cf_bounds_meet(self.B, n, self.dp.state_l.data_ptr() + 4 * col,
                                     self.dp.state_u.data_ptr() + 4 * col, N,
                                     self.zn.state_l.data_ptr() + 4 * col, self.zn.state_u.data_ptr() + 4 * col, N,
                                     self.lb.data_ptr() if final else None, self.ub.data_ptr() if final else None,
                                     stream)
        _lib.check(st, "cf_bounds_meet")

    def layer(self, i):
        """Run network layer i (i == n_layers: the property layer); layers run in order."""
        if i != self.done + 1:
            raise ValueError(f"layer {i} after layer {self.done}: layers run in order")
        self.dp.layer(i)
        self.zn.layer(i)
        if i == self.n_layers:
            self._meet(self.engine.spec_col, self.engine.n_spec, True)
        elif self.engine.kinds[i] in ("linear", "conv"):
            self._meet(self.engine.col[i], self.engine.width[i], False)
        self.done = i
        return self

    def finish(self):
        """Device status of both passes and the float64 property bounds."""
        if self.done != self.n_layers:
            raise ValueError(f"pass stopped after layer {self.done} of {self.n_layers}")
        self.dp.finish()
        self.zn.finish()
        return self.lb, self.ub
