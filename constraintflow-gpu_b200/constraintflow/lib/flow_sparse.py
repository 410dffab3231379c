"""Flow: the layer loop of a certifier over a network (reference:
constraintflow/lib/flow_sparse.py:15-228).

The reference calls the generated transformer's Affine / Relu on every layer and does
the arithmetic op by op.  Here the whole loop of a recognised certifier runs in one call
of the B200 network driver (cf_deeppoly_run through cfgpu.engine), which computes the
same abstract state: every neuron's l/u is written back into abs_elem.d['l'|'u'] and the
property layer's bounds are returned as float64 (lb, ub), as Flow.flow returns them.

Recognition: the compiler emits a class with Affine and Relu methods.  The program is
identified by the semantic fingerprint of those two methods (program_fingerprint.py: a
hash of their syntax trees with the compiler's variable names canonicalised), which must be
the fingerprint of the reference compiler's own output for one of the example programs the
runtime implements: deeppoly.cf, deeppoly_efficient.cf (composes to DeepPoly's bounds),
crown.cf, crownibp.cf, zono.cf, ibp.cf, polyzono.cf, zid.cf and the custom-stop DeepPoly
programs (deeppoly_custom_stop.cf, custom_stops/*.cf).  A program that differs from those
in any threshold, slope, operator or control flow raises NotImplementedError; the two
constants the runtime takes as parameters are read from the source first: the custom-stop
programs' get_start (the generated Affine computes curr[layer] - get_start) and zid.cf's
zonotope layer bound (curr[layer] <= K, in its Affine and its Relu alike).
A transformer object may also declare itself with a ``cf_certifier`` attribute (the code
that cfgpu.codegen emits, after its own semantic checks of the program).
"""
import inspect

import torch

from constraintflow.gbcsr.sparse_block import DenseBlock
from constraintflow.gbcsr.sparse_tensor import SparseTensor

from . import program_fingerprint as PF
from .network import LayerType

def _methods_source(transformer):
    cls = type(transformer)
    try:
        return inspect.getsource(cls.Affine), inspect.getsource(cls.Relu)
    except (AttributeError, OSError, TypeError) as e:
        raise NotImplementedError(f"cannot read the generated transformer: {e}")


def _known(transformer):
    """(certifier, strict ReLU test) of a generated transformer from its fingerprint."""
    _methods_source(transformer)
    fp = PF.fingerprint(type(transformer))
    hit = PF.KNOWN.get(fp)
    if hit is None:
        raise NotImplementedError(
            "this runtime runs the reference compiler's output for deeppoly.cf, deeppoly_efficient.cf, "
            "crown.cf, crownibp.cf, zono.cf, ibp.cf, polyzono.cf, zid.cf and the custom-stop DeepPoly "
            f"programs; the given transformer ({type(transformer).__name__}, fingerprint {fp}) computes "
            "something else")
    return hit


def zid_upto_of(transformer):
    """The layer up to which zid.cf bounds neurons by the zonotope (curr[layer] <= 4,
    zid.cf:38): declared by ``cf_zono_upto`` or read from the generated Affine and Relu, which
    must both test the same bound."""
    declared = getattr(transformer, "cf_zono_upto", None)
    if declared is not None:
        return int(declared)
    affine, relu = _methods_source(transformer)
    found_a, found_r = PF.params(affine, "zono_upto"), PF.params(relu, "zono_upto")
    if len(found_a) != 1 or found_a != found_r:
        raise NotImplementedError(f"zid-style program with layer bounds {sorted(found_a)} (Affine) and "
                                  f"{sorted(found_r)} (Relu)")
    return found_a.pop()


def stop_depth_of(transformer):
    """get_start of a custom-stop DeepPoly program (the traversal bounding a neuron of layer
    k stops below layer k - get_start, deeppoly_custom_stop.cf:12-17), None for a traversal
    to the input.  Declared by a ``cf_stop_depth`` attribute or read from the generated
    Affine, which computes curr[layer] - get_start."""
    declared = getattr(transformer, "cf_stop_depth", None)
    if declared is not None or getattr(transformer, "cf_certifier", None) is not None:
        return declared
    try:
        affine = inspect.getsource(type(transformer).Affine)
    except (AttributeError, OSError, TypeError):
        return None
    found = PF.params(affine, "stop_depth")
    if len(found) > 1:
        raise NotImplementedError(f"traversal stops at several depths {sorted(found)}")
    return found.pop() if found else None


def relu_is_strict(transformer):
    """DeepPoly's Relu with strict comparisons (relu_n: l + u > 0; compute_upper: l > 0,
    u < 0), as the custom-stop programs write it (deeppoly_custom_stop.cf:22-24)."""
    declared = getattr(transformer, "cf_relu_strict", None)
    if declared is not None or getattr(transformer, "cf_certifier", None) is not None:
        return bool(declared)
    try:
        return _known(transformer)[1]
    except NotImplementedError:
        return False


def certifier_of(transformer):
    """'deeppoly', 'crown', 'zono', 'ibp', 'polyzono', 'crownibp' or 'zid' for a recognised
    generated transformer, else raises NotImplementedError."""
    declared = getattr(transformer, "cf_certifier", None)
    if declared is not None:
        return declared
    return _known(transformer)[0]


class _EngineLayer:
    def __init__(self, kind, W=None, b=None, in_shape=None, out_shape=None, stride=1, pad=0, parents=None):
        self.kind, self.W, self.b = kind, W, b
        self.in_shape, self.out_shape, self.stride, self.pad = in_shape, out_shape, stride, pad
        self.parents = parents


def engine_layers(model):
    """The network as the driver's layer list (property layer excluded): linear / conv /
    relu / add / concat, each with its parents as indices into that list (-1 = input)."""
    out = []
    last = len(model) - 1
    if list(model[last].parents) != [last - 1]:
        raise NotImplementedError("the property layer must read the last layer of the network")
    for i, layer in enumerate(model):
        if layer.type == LayerType.Input or i == last:
            continue
        parents = tuple(int(p) - 1 for p in layer.parents)
        if layer.type == LayerType.Linear:
            bias = layer.bias if layer.bias is not None else torch.zeros(layer.weight.shape[0])
            out.append(_EngineLayer("linear", layer.weight.float(), bias.float(), parents=parents))
        elif layer.type == LayerType.Conv2D:
            parent = model[layer.parents[0]]
            bias = getattr(layer, "bias_channel", None)
            if bias is None:
                bias = layer.bias.reshape(layer.weight.shape[0], -1)[:, 0]
            out.append(_EngineLayer("conv", layer.weight.float(), bias.float(), in_shape=tuple(parent.shape[1:]),
                                    out_shape=tuple(layer.shape[1:]), stride=layer.stride[0], pad=layer.padding[0],
                                    parents=parents))
        elif layer.type == LayerType.ReLU:
            out.append(_EngineLayer("relu", parents=parents))
        elif layer.type == LayerType.Add:
            out.append(_EngineLayer("add", parents=parents))
        elif layer.type == LayerType.Concat:
            out.append(_EngineLayer("concat", parents=parents))
        else:
            raise NotImplementedError(f"layer type {layer.type} (the driver runs Linear, Conv2D, ReLU, Add and "
                                      "Concat layers)")
    return out


class Flow:
    def __init__(self, abs_elem, transformer, model, print_intermediate_results=False, no_sparsity=False):
        self.abs_elem = abs_elem
        self.transformer = transformer
        self.model = model
        self.input_size = model.input_size
        self.batch_size = abs_elem.batch_size
        self.print_intermediate_results = print_intermediate_results
        self.no_sparsity = no_sparsity

    def flow(self):
        from cfgpu.engine import DeepPolyEngine
        certifier = certifier_of(self.transformer)
        dev = torch.device("cuda", torch.cuda.current_device())
        n0 = self.input_size
        B = self.batch_size
        l_in = self.abs_elem.d["l"]
        u_in = self.abs_elem.d["u"]
        l0 = l_in.get_dense_device()[:, :n0].contiguous()
        u0 = u_in.get_dense_device()[:, :n0].contiguous()
        spec = self.model[-1]
        W = torch.as_tensor(spec.weight, dtype=torch.float32).to(dev).contiguous()
        if certifier == "polyzono":
            from cfgpu.polyzono import PolyZonoEngine
            eng = PolyZonoEngine(engine_layers(self.model), n0, dev, n_spec=int(W.shape[1]))
        elif certifier == "zid":
            from cfgpu.zid import ZidEngine
            eng = ZidEngine(engine_layers(self.model), n0, dev, n_spec=int(W.shape[1]),
                            zono_upto=zid_upto_of(self.transformer))
        else:
            eng = DeepPolyEngine(engine_layers(self.model), n0, dev, n_spec=int(W.shape[1]), certifier=certifier,
                                 stop_depth=stop_depth_of(self.transformer) if certifier == "deeppoly" else None,
                                 relu_strict=certifier == "deeppoly" and relu_is_strict(self.transformer))
        if getattr(self.transformer, "cf_layerwise", False) and eng.net is not None:
            lb, ub, sl, su = self._layer_by_layer(eng, l0, u0, W)
        else:
            lb, ub, sl, su = eng.run(l0, u0, W, want_state=True)
        total = torch.tensor([B, self.model.size])
        self.abs_elem.d["l"] = SparseTensor([torch.tensor([0, 0])], [DenseBlock(sl)], 2, total,
                                            dense_const=float("-inf"))
        self.abs_elem.d["u"] = SparseTensor([torch.tensor([0, 0])], [DenseBlock(su)], 2, total,
                                            dense_const=float("inf"))
        self.abs_elem.d["llist"][:] = True
        lb, ub = lb.cpu(), ub.cpu()
        if self.print_intermediate_results:
            for i, layer in enumerate(self.model):
                print(i, layer.type, layer.shape)
                print(f"l: {sl[:, layer.start:layer.end].cpu()}")
                print(f"u: {su[:, layer.start:layer.end].cpu()}")
        return lb, ub

    def _layer_by_layer(self, eng, l0, u0, W):
        """Programs emitted by cfgpu.codegen: the transformer's operation is called for every
        layer in order (as flow_sparse.py:27-228 does), each one fused libcfgpu call."""
        from cfgpu.layerwise import LayerRun
        from cfgpu.polyzono import PolyZonoRun
        from cfgpu.zid import ZidRun
        run = {"polyzono": PolyZonoRun, "zid": ZidRun}.get(eng.certifier, LayerRun)(eng, l0, u0, W)
        self.abs_elem.cf_run = run
        B = self.batch_size
        try:
            for tmp, layer in enumerate(self.model):
                if layer.type == LayerType.Input:
                    continue
                op = "Relu" if layer.type == LayerType.ReLU else "Affine"
                getattr(self.transformer, op)(self.abs_elem, None, None, self.model.size, layer.size, None,
                                              self.input_size, B, layer_index=tmp)
            lb, ub = run.finish()
        except NotImplementedError:
            if eng.certifier != "crown":
                raise
            # a CROWN layer took the all-crossing branch: the whole-network driver runs the
            # general traversal for it
            return eng.run(l0, u0, W, want_state=True)
        finally:
            self.abs_elem.cf_run = None
        return lb, ub, run.state_l, run.state_u
