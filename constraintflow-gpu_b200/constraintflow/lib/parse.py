"""ONNX network reader: same layer list, shapes and neuron numbering as the reference's
constraintflow/lib/parse.py:29-301.

Reads Conv (attributes positional as torch exports them: [2] kernel_shape, [3] pads,
[4] strides, parse.py:110-112), Gemm (weight input 1, bias input 2), MatMul (weight
input 0, data input 1), Relu, Sigmoid, Add (of two layers: an Add layer; with a constant:
folded into the previous layer's bias) and Concat of two layers; other nodes (Flatten,
...) are identity.  The robustness property is always appended as a Linear layer with the
per-region weight reading the last layer read (parse.py:230-238).  The list is then put
in breadth-first order from the input, a layer entering the queue once all its parents
have been placed (parse.py:250-300), and the neuron ranges renumbered in that order.
Works with the `onnx` package, or with any module of that name whose ``load(name)``
returns an object with the same ``graph`` fields.
"""
import copy
import math
from collections import deque

import numpy as np
import torch

from .network import Layer, LayerType, Network


def compute_size(shape):
    s = 1
    for v in shape:
        s *= int(v)
    return s


def get_net_format(net_name):
    if "onnx" in net_name:
        return "onnx"
    if "pt" in net_name:
        return "torch"
    return None


def _to_array(init):
    try:
        from onnx import numpy_helper
        return np.asarray(numpy_helper.to_array(init))
    except ImportError:
        return np.asarray(init.array)


def get_net(net_name, spec_weight, spec_bias, no_sparsity=False):
    if get_net_format(net_name) != "onnx":
        raise ValueError("Unsupported net format!")
    import onnx
    net = parse_onnx_layers(onnx.load(net_name), spec_weight, spec_bias, no_sparsity)
    net.net_name = net_name
    return net


def parse_onnx_layers(net, spec_weight, spec_bias, no_sparsity=False):
    g = net.graph
    input_shape = [int(d.dim_value) for d in g.input[0].type.tensor_type.shape.dim]
    input_shape = [1 if i == 0 else v for i, v in enumerate(input_shape)]
    if len(input_shape) == 3:
        input_shape = [1] + input_shape
    input_size = compute_size(input_shape)
    layers = Network(input_name=g.input[0].name, input_shape=input_shape, input_size=input_size, input_start=0,
                     input_end=input_size, net_format="onnx", no_sparsity=no_sparsity)
    layers.num_layers = len(g.node)
    vals = {init.name: torch.tensor(_to_array(init)) for init in g.initializer}
    layers.size = input_size
    layers.append(Layer(type=LayerType.Input, shape=input_shape, size=input_size, start=0, end=input_size))
    ids = {g.input[0].name: 0}
    index = 0
    shape = input_shape
    for node in g.node:
        op = node.op_type
        src = str(node.input[0]) if len(node.input) else None
        if op == "Conv":
            index += 1
            w = vals[node.input[1]]
            b = vals[node.input[2]] if len(node.input) > 2 else torch.zeros(w.shape[0])
            layer = Layer(weight=w, bias=b, type=LayerType.Conv2D, identifier=index, parents=[ids[src]])
            layer.kernel_size = tuple(int(v) for v in node.attribute[2].ints[:2])
            layer.padding = tuple(int(v) for v in node.attribute[3].ints[:2])
            layer.stride = tuple(int(v) for v in node.attribute[4].ints[:2])
            layer.dilation = (1, 1)
            i1, i2, i3, i4 = layers[ids[src]].shape
            k1, k2, k3, k4 = w.shape
            o3 = math.floor((i3 + 2 * layer.padding[0] - k3) / layer.stride[0]) + 1
            o4 = math.floor((i4 + 2 * layer.padding[1] - k4) / layer.stride[1]) + 1
            layer.shape = [i1, k1, o3, o4]
            layer.bias_channel = b
            layer.bias = b.unsqueeze(1).repeat(1, o3 * o4).flatten()  # one bias per neuron (parse.py:126)
        elif op == "Gemm":
            index += 1
            w = vals[node.input[1]]
            layer = Layer(weight=w, bias=vals[node.input[2]], type=LayerType.Linear, identifier=index,
                          parents=[ids[src]])
            layer.shape = [shape[0], int(w.shape[0]), 1, 1]
        elif op in ("Relu", "Sigmoid"):
            index += 1
            layer = Layer(type=LayerType.ReLU if op == "Relu" else LayerType.Sigmoid, identifier=index,
                          parents=[ids[src]])
            layer.shape = list(layers[ids[src]].shape)
        elif op == "MatMul":
            index += 1
            w = vals[node.input[0]]
            layer = Layer(weight=w, bias=None, type=LayerType.Linear, identifier=index,
                          parents=[ids[str(node.input[1])]])
            layer.shape = [1, int(w.shape[0]), 1, 1]
        elif op == "Add" and len(node.input) > 1 and node.input[1] in vals:
            ids[str(node.output[0])] = index
            layers[-1].bias = vals[node.input[1]]
            continue
        elif op == "Add":
            index += 1
            pa = [ids[str(node.input[0])], ids[str(node.input[1])]]
            layer = Layer(type=LayerType.Add, identifier=index, parents=pa)
            layer.shape = copy.deepcopy(list(layers[pa[0]].shape))
        elif op == "Concat":
            if not all(str(i) in ids for i in node.input[:2]):
                raise NotImplementedError("Concat of a tensor that is not a layer output")
            index += 1
            pa = [ids[str(node.input[0])], ids[str(node.input[1])]]
            layer = Layer(type=LayerType.Concat, identifier=index, parents=pa)
            layer.shape = [1, int(layers[pa[0]].shape[1]) + int(layers[pa[1]].shape[1]), 1, 1]
        else:
            if src is not None and src in ids:
                ids[str(node.output[0])] = ids[src]
            continue
        ids[str(node.output[0])] = index
        layer.size = compute_size(layer.shape)
        layer.start = layers.size
        layers.size += layer.size
        layer.end = layers.size
        layers.append(layer)
        shape = layer.shape
    spec = Layer(weight=spec_weight, bias=spec_bias, type=LayerType.Linear, identifier=index + 1,
                 parents=[layers[-1].identifier])
    spec.last_layer = True
    spec.shape = [1, int(spec_weight.shape[-2]), 1, 1]
    spec.size = compute_size(spec.shape)
    spec.start = layers.size
    layers.size += spec.size
    spec.end = layers.size
    layers.append(spec)
    return _breadth_first(layers)


def _breadth_first(layers):
    """The layers in breadth-first order from the input: a layer is queued when the last
    of its parents is placed (children visited in identifier order); identifiers, parents,
    children and neuron ranges are renumbered in the new order (parse.py:250-300)."""
    by_id = {lay.identifier: lay for lay in layers}
    for lay in layers:
        lay.children = []
    for lay in layers:
        for p in lay.parents:
            by_id[p].children.append(lay.identifier)
    placed = {}
    order = []
    queue = deque([by_id[0]])
    while queue:
        lay = queue.popleft()
        if lay.identifier in placed:
            continue
        placed[lay.identifier] = len(order)
        order.append(lay)
        for c in lay.children:
            if c not in placed and all(p in placed for p in by_id[c].parents):
                queue.append(by_id[c])
    if len(order) != len(layers):
        raise ValueError("network graph: some layers are not reachable from the input")
    out = layers.similar()
    start = 0
    for lay in order:
        lay.identifier = placed[lay.identifier]
        lay.parents = [placed[p] for p in lay.parents]
        lay.children = [placed[c] for c in lay.children]
        if lay.type != LayerType.Input:
            lay.start, lay.end = start, start + lay.size
        start += lay.size
        out.append(lay)
    out.size = start
    return out
