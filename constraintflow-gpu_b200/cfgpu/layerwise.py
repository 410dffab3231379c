"""Per-layer execution of a certifier pass: the layer loop driven from Python, one fused
libcfgpu call per network layer (cf_deeppoly_layer), as the reference's Flow.flow calls the
generated transformer once per layer (constraintflow/lib/flow_sparse.py:27-228).

Programs emitted by cfgpu.codegen call ``LayerRun.layer(i)`` from their per-layer
transformer methods.  The bounds are those of the whole-network driver
(DeepPolyEngine.run / cf_deeppoly_run).
"""
import ctypes

import torch

from . import _lib


class LayerRun:
    """One pass over a batch: device inputs, the abstract state and the workspace that
    carries the layers' intermediate results from one call to the next."""

    def __init__(self, engine, l0, u0, spec_W):
        if engine.net is None:
            raise NotImplementedError("per-layer runs cover chain networks (networks with Add / Concat layers run "
                                      "as a whole: DeepPolyEngine.run)")
        self.engine = engine
        self.B = int(l0.shape[0])
        dev = engine.device
        for t, shp in ((l0, (self.B, engine.input_size)), (u0, (self.B, engine.input_size)),
                       (spec_W, (self.B, engine.n_spec, engine.n_last))):
            if tuple(t.shape) != shp or t.dtype != torch.float32 or not t.is_contiguous() or t.device != dev:
                raise Exception(f"SHAPE MISMATCH: expected contiguous float32 {shp} on {dev}, "
                                f"got {tuple(t.shape)} {t.dtype} on {t.device}")
        self.l0, self.u0, self.spec_W = l0, u0, spec_W
        self.state_l = torch.empty(self.B, engine.N, dtype=torch.float32, device=dev)
        self.state_u = torch.empty_like(self.state_l)
        self.lb = torch.empty(self.B, engine.n_spec, dtype=torch.float64, device=dev)
        self.ub = torch.empty_like(self.lb)
        nbytes = engine.workspace_bytes(self.B)
        self.ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        self.n_layers = int(engine.net.n_layers)
        self.done = -1

    def layer(self, i):
        """Run network layer i (i == n_layers: the property layer); layers run in order."""
        if i != self.done + 1:
            raise ValueError(f"layer {i} after layer {self.done}: layers run in order")
        stream = torch.cuda.current_stream(self.engine.device).cuda_stream
        st = _lib.lib.cf_deeppoly_layer(ctypes.byref(self.engine.net), int(i), self.B, self.l0.data_ptr(),
                                        self.u0.data_ptr(), self.spec_W.data_ptr(), self.state_l.data_ptr(),
                                        self.state_u.data_ptr(), self.lb.data_ptr(), self.ub.data_ptr(),
                                        self.ws.data_ptr(), self.ws.numel(), stream)
        _lib.check(st, "cf_deeppoly_layer")
        self.done = i
        return self

    def finish(self):
        """Device status (bounded waits; CROWN's all-crossing branch) and the float64 bounds."""
        if self.done != self.n_layers:
            raise ValueError(f"pass stopped after layer {self.done} of {self.n_layers}")
        stream = torch.cuda.current_stream(self.engine.device).cuda_stream
        _lib.check(_lib.lib.cf_deeppoly_check(self.ws.data_ptr(), stream), "device status")
        return self.lb, self.ub


_OP_OF_KIND = {"linear": "Affine", "conv": "Affine", "relu": "Relu"}


def run_operation(abs_elem, op, layer_index):
    """The fused call behind one operation of an emitted transformer: runs model layer
    `layer_index` (1 = the first network layer; the property layer last) on the pass that
    Flow.flow attached to the abstract element, after checking that the layer is of the
    operation's kind."""
    run = getattr(abs_elem, "cf_run", None)
    if run is None:
        raise RuntimeError("no per-layer pass is attached to this abstract element (Flow.flow attaches it)")
    li = int(layer_index) - 1
    kinds = run.engine.kinds
    kind = "linear" if li == run.n_layers else kinds[li]
    if _OP_OF_KIND.get(kind) != op:
        raise ValueError(f"layer {layer_index} is a {kind} layer; the transformer called {op}")
    run.layer(li)
