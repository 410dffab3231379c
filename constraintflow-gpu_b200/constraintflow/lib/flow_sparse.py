"""Flow: the layer loop of a certifier over a network (reference:
constraintflow/lib/flow_sparse.py:15-228).

The reference calls the generated transformer's Affine / Relu on every layer and does
the arithmetic op by op.  Here the whole loop of a recognised certifier runs in one call
of the B200 network driver (cf_deeppoly_run through cfgpu.engine), which computes the
same abstract state: every neuron's l/u is written back into abs_elem.d['l'|'u'] and the
property layer's bounds are returned as float64 (lb, ub), as Flow.flow returns them.

Recognition: the compiler emits a class with Affine and Relu methods; the program is
identified from the operations its generated code performs.  Every supported program
has the same Affine (the backward traversal with priority2 = -layer: clamp sign split,
inner_prod, get_max_priority over the negated layer index) and one of three Relu bodies:
  * deeppoly.cf: per-neuron triangle relaxation over the neuron itself (convert_to_poly,
    the u/(u-l) slope, where() on l>=0 / u<=0);
  * deeppoly_efficient.cf: the same relaxation applied to the affine's L/U polyexps
    (get_elem('L'/'U', prev)); it composes to exactly DeepPoly's bounds;
  * crown.cf: whole-layer if(any(...)) branches with the -l > u lower-slope choice.
Two forward programs are recognised by their own Affine / Relu:
  * zono.cf (DeepZ): the Affine maps the previous layer's symbolic expression Z and
    concretises sum |coefficient|; the Relu opens fresh noise symbols (get_new_eps);
  * ibp.cf: interval arithmetic on the previous layer's l / u (clamp sign split, no
    traversal); the Relu clamps l and u.
polyzono.cf carries both states: its Affine is DeepPoly's traversal met (cf_max / cf_min)
with the zonotope's concretisation, its Relu both relaxations (convert_to_poly and
get_new_eps); it runs as cfgpu.polyzono's coupled DeepPoly and zonotope passes.
crownibp.cf branches its Affine on the last_layer metadata: interval bounds below the
property (map(simplify_lower) over the previous layer's l / u), the traversal for the
property rows; its Relu is DeepPoly's.
zid.cf branches on last_layer and on curr[layer] <= 4: zonotope bounds up to layer 4,
interval bounds above, the traversal for the property rows (cfgpu.zid).
The custom-stop DeepPoly programs (deeppoly_custom_stop.cf, custom_stops/) stop their
traversal at layers below curr[layer] - get_start: the generated Affine subtracts the
constant get_start from the layer metadata (stop_depth_of), and the driver runs DeepPoly
with that stop depth.
A transformer object may also declare itself with a ``cf_certifier`` attribute
('deeppoly', 'crown', 'zono', 'ibp', 'polyzono' or 'crownibp').  Other programs (zono2.cf's whole-layer branches
among them) raise NotImplementedError.
"""
import inspect
import re

import torch

from constraintflow.gbcsr.sparse_block import DenseBlock
from constraintflow.gbcsr.sparse_tensor import SparseTensor

from .network import LayerType

_AFFINE = ("clamp(", "inner_prod(", "get_max_priority(", "filter_trav_exp_not_stop(",
           "get_metadata('layer'", "operator.neg")
_DEEPPOLY_RELU = ("convert_to_poly(", "operator.truediv", "operator.le", "operator.ge", "where(")
_EFFICIENT_RELU = ("get_elem('L', prev", "get_elem('U', prev", "operator.truediv", "operator.le", "operator.ge",
                   "where(")
_CROWN_RELU = ("if(", "any(", "operator.gt", "convert_to_poly(", "operator.truediv", "get_elem('U', prev")
# zono.cf: forward symbol algebra (Affine concretises sum |coefficient|, Relu opens fresh symbols)
_ZONO_AFFINE = ("get_elem('Z', prev", "get_mat(SymExpSparse.count", "inner_prod(", "clamp(", ".sum(2")
_ZONO_RELU = ("get_new_eps(", "get_elem('Z', prev", "operator.truediv", "operator.le", "operator.ge", "where(")
# ibp.cf: interval arithmetic over the previous layer's l / u
_IBP_AFFINE = ("inner_prod(", "clamp(", "get_elem('l'", "get_elem('u'")
_IBP_RELU = ("convert_to_float(", "operator.ge", "get_elem('l', prev", "get_elem('u', prev")
# crownibp.cf: interval bounds below the property (a branch on the last_layer metadata), the
# traversal only for the property rows; DeepPoly's Relu
_CROWNIBP_AFFINE = ("get_metadata('last_layer'", "if(", "clamp(", "inner_prod(", "get_max_priority(",
                    "get_metadata('layer'", "get_elem('l'", "get_elem('u'")
# polyzono.cf: DeepPoly's traversal met with the zonotope bound; both relaxations in the Relu
_POLYZONO_AFFINE = _AFFINE + ("get_elem('Z', prev", "cf_max(", "cf_min(")
_POLYZONO_RELU = ("convert_to_poly(", "get_new_eps(", "get_elem('Z', prev", "operator.truediv", "where(")


_STOP_DEPTH = re.compile(r"curr\.get_metadata\('layer'[^)]*\), SparseTensor\(\[\], \[\], 0, torch\.tensor\(\[\]\), "
                         r"dense_const=(\d+), type= type\(\d+\)\)(?:\.\w+\([^()]*(?:\([^()]*\))?[^()]*\))*, "
                         r"operator\.sub")


_ZID_UPTO = re.compile(r"curr\.get_metadata\('layer'[^)]*\), SparseTensor\(\[\], \[\], 0, torch\.tensor\(\[\]\), "
                       r"dense_const=(\d+), type= type\(\d+\)\)(?:\.\w+\([^()]*(?:\([^()]*\))?[^()]*\))*, "
                       r"operator\.le")


def zid_upto_of(transformer):
    """The layer up to which zid.cf bounds neurons by the zonotope (curr[layer] <= 4,
    zid.cf:38): declared by ``cf_zono_upto`` or read from the generated Affine."""
    declared = getattr(transformer, "cf_zono_upto", None)
    if declared is not None:
        return int(declared)
    found = {int(m) for m in _ZID_UPTO.findall(inspect.getsource(type(transformer).Affine))}
    if len(found) != 1:
        raise NotImplementedError(f"zid-style program with layer thresholds {sorted(found)}")
    return found.pop()


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
    found = {int(m) for m in _STOP_DEPTH.findall(affine)}
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
        relu = inspect.getsource(type(transformer).Relu)
    except (AttributeError, OSError, TypeError):
        return False
    return ("if(" not in relu and "any(" not in relu and "operator.ge" not in relu and "operator.le" not in relu
            and all(k in relu for k in ("convert_to_poly(", "operator.truediv", "operator.gt", "operator.lt",
                                        "where(")))


def certifier_of(transformer):
    """'deeppoly', 'crown', 'zono', 'ibp', 'polyzono', 'crownibp' or 'zid' for a recognised
    generated transformer, else raises."""
    declared = getattr(transformer, "cf_certifier", None)
    if declared is not None:
        return declared
    cls = type(transformer)
    try:
        relu = inspect.getsource(cls.Relu)
        affine = inspect.getsource(cls.Affine)
    except (AttributeError, OSError, TypeError) as e:
        raise NotImplementedError(f"cannot read the generated transformer: {e}")
    if (all(k in affine for k in ("get_metadata('last_layer'", "get_metadata('layer'", "get_elem('Z', prev",
                                   "get_max_priority(", "clamp(", "inner_prod("))
            and all(k in relu for k in ("get_metadata('last_layer'", "get_new_eps(", "convert_to_poly(",
                                        "get_elem('Z', prev"))):
        return "zid"
    if all(k in affine for k in _POLYZONO_AFFINE) and all(k in relu for k in _POLYZONO_RELU):
        if "if(" in relu or "any(" in relu:
            raise NotImplementedError("a polyzono-style program with whole-layer branches")
        return "polyzono"
    if all(k in affine for k in _CROWNIBP_AFFINE) and "if(" not in relu and "any(" not in relu and (
            all(k in relu for k in _DEEPPOLY_RELU)):
        return "crownibp"
    if all(k in affine for k in _AFFINE) and relu_is_strict(transformer):
        return "deeppoly"
    if all(k in affine for k in _AFFINE):
        branches = "if(" in relu or "any(" in relu or "operator.gt" in relu
        if not branches and (all(k in relu for k in _DEEPPOLY_RELU) or all(k in relu for k in _EFFICIENT_RELU)):
            return "deeppoly"
        if all(k in relu for k in _CROWN_RELU):
            return "crown"
    branches = "if(" in relu or "any(" in relu
    if all(k in affine for k in _ZONO_AFFINE) and all(k in relu for k in _ZONO_RELU) and not branches:
        return "zono"
    if (all(k in affine for k in _IBP_AFFINE) and all(k in relu for k in _IBP_RELU) and "get_max_priority(" not in affine
            and "get_new_eps(" not in relu and "convert_to_poly(" not in relu and not branches):
        return "ibp"
    raise NotImplementedError("this runtime runs the DeepPoly, CROWN, zonotope (zono.cf), interval (ibp.cf), "
                              "polyzono.cf, crownibp.cf and zid.cf certifier programs; the given "
                              f"transformer ({cls.__name__}) is a different program")


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
