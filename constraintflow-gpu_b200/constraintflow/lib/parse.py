"""ONNX network reader: same layer list, shapes and neuron numbering as the reference's
constraintflow/lib/parse.py:29-301.

Reads Conv (attributes positional as torch exports them: [2] kernel_shape, [3] pads,
[4] strides, parse.py:110-112), Gemm (weight input 1, bias input 2), Relu, Sigmoid, and
a constant Add folded into the previous layer's bias; other nodes (Flatten, ...) are
identity.  The robustness property is always appended as a final Linear layer with the
per-region weight (parse.py:230-238).  Works with the `onnx` package, or with any module
of that name whose ``load(name)`` returns an object with the same ``graph`` fields.
"""
import math

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
        elif op == "Add" and len(node.input) > 1 and node.input[1] in vals:
            ids[str(node.output[0])] = index
            layers[-1].bias = vals[node.input[1]]
            continue
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
    for lay in layers:
        for p in lay.parents:
            layers[p].children.append(lay.identifier)
    return layers
