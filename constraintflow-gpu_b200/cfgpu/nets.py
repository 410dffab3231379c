"""Seeded synthetic networks and input regions for the certification workloads.

No public model or dataset is available offline, so every workload is a seeded
network built in memory plus uniformly drawn input centres:

* weights: ``torch.nn.init.kaiming_normal_`` (fan_in, gain sqrt(2)) drawn from one
  ``torch.Generator().manual_seed(seed)`` in layer order (weight, then bias);
* biases: zero, except the 784-(100x6)-10 MLP whose biases are N(0, 0.01);
* centres: ``torch.rand(B, C, H, W, generator=manual_seed(100 + workload id))`` (the tied
  workload copies pixel 2r to pixel 2r+1 for its tied pairs);
* label: argmax of the float32 forward pass at the *normalised* centre.

The layer list mirrors what the reference's ONNX reader produces
(constraintflow/lib/parse.py:60-248): Gemm -> Linear, Conv -> Conv2D, Relu -> ReLU,
with the robustness property appended as a final per-region Linear layer
(constraintflow/lib/parse.py:230-238, constraintflow/lib/spec.py:61-72).
"""
from dataclasses import dataclass, field
import math

import numpy as np
import torch

MNIST_MEAN = (0.1307,)
MNIST_STD = (0.3081,)
CIFAR_MEAN = (0.4914, 0.4822, 0.4465)
CIFAR_STD = (0.2023, 0.1994, 0.2010)


@dataclass
class Layer:
    """One network layer.  ``kind`` is 'linear', 'conv', 'relu', 'add' or 'concat'.

    Linear: W [out, in], b [out].  Conv: W [Cout, Cin, kh, kw], b [Cout], square
    ``stride``/``pad``; ``in_shape``/``out_shape`` are (C, H, W).
    ``parents``: indices of the input layers in the layer list (-1 = the network input);
    None means the previous layer.  'add' sums its two parents elementwise, 'concat'
    stacks them (constraintflow/lib/parse.py:165-200, flow_sparse.py:67-178).
    """
    kind: str
    W: np.ndarray = None
    b: np.ndarray = None
    stride: int = 1
    pad: int = 0
    in_shape: tuple = None
    out_shape: tuple = None
    parents: tuple = None

    @property
    def n_in(self):
        return int(np.prod(self.in_shape))

    @property
    def n_out(self):
        return int(np.prod(self.out_shape))


@dataclass
class Workload:
    wid: int
    name: str
    input_shape: tuple
    layers: list
    B: int
    eps: float
    dataset: str
    seed: int
    description: str = ""
    extra: dict = field(default_factory=dict)

    @property
    def input_size(self):
        return int(np.prod(self.input_shape))


def _kaiming(shape, g):
    w = torch.empty(*shape)
    torch.nn.init.kaiming_normal_(w, generator=g)
    return w


def _mlp(sizes, seed, bias_std):
    g = torch.Generator().manual_seed(seed)
    layers = []
    for i in range(len(sizes) - 1):
        w = _kaiming((sizes[i + 1], sizes[i]), g)
        if bias_std:
            b = torch.randn(sizes[i + 1], generator=g) * bias_std
        else:
            b = torch.zeros(sizes[i + 1])
        layers.append(Layer('linear', w.numpy(), b.numpy(), in_shape=(sizes[i], 1, 1),
                            out_shape=(sizes[i + 1], 1, 1)))
        if i < len(sizes) - 2:
            layers.append(Layer('relu', in_shape=(sizes[i + 1], 1, 1), out_shape=(sizes[i + 1], 1, 1)))
    return layers


def _convnet(in_shape, convs, fcs, seed):
    g = torch.Generator().manual_seed(seed)
    C, H, W = in_shape
    layers = []
    for (oc, k, s, p) in convs:
        w = _kaiming((oc, C, k, k), g)
        b = torch.zeros(oc)
        OH, OW = (H + 2 * p - k) // s + 1, (W + 2 * p - k) // s + 1
        layers.append(Layer('conv', w.numpy(), b.numpy(), stride=s, pad=p, in_shape=(C, H, W),
                            out_shape=(oc, OH, OW)))
        layers.append(Layer('relu', in_shape=(oc, OH, OW), out_shape=(oc, OH, OW)))
        C, H, W = oc, OH, OW
    sizes = [C * H * W] + list(fcs)
    for i in range(len(sizes) - 1):
        w = _kaiming((sizes[i + 1], sizes[i]), g)
        b = torch.zeros(sizes[i + 1])
        layers.append(Layer('linear', w.numpy(), b.numpy(), in_shape=(sizes[i], 1, 1),
                            out_shape=(sizes[i + 1], 1, 1)))
        if i < len(sizes) - 2:
            layers.append(Layer('relu', in_shape=(sizes[i + 1], 1, 1), out_shape=(sizes[i + 1], 1, 1)))
    return layers


def _residual(seed):
    """784 -> 100, then two residual blocks [fc, relu, fc] + skip, relu; -> 10."""
    g = torch.Generator().manual_seed(seed)

    def fc(n_in, n_out, parents=None):
        return Layer('linear', _kaiming((n_out, n_in), g).numpy(), (torch.randn(n_out, generator=g) * 0.01).numpy(),
                     in_shape=(n_in, 1, 1), out_shape=(n_out, 1, 1), parents=parents)

    def relu(n, parents=None):
        return Layer('relu', in_shape=(n, 1, 1), out_shape=(n, 1, 1), parents=parents)

    L = [fc(784, 100), relu(100)]                         # 0, 1
    for _ in range(2):
        skip = len(L) - 1
        L += [fc(100, 100), relu(100), fc(100, 100)]
        L.append(Layer('add', in_shape=(100, 1, 1), out_shape=(100, 1, 1), parents=(len(L) - 1, skip)))
        L.append(relu(100))
    L.append(fc(100, 10))
    return L


def _resconv(seed):
    """1x28x28 -> conv 4x3x3 stride 2 (4x14x14), relu; a residual block [conv 4x3x3, relu,
    conv 4x3x3] (stride 1, padding 1) + skip, relu; -> 10.  Conv layers inside an Add network."""
    g = torch.Generator().manual_seed(seed)

    def conv(cin, cout, h, s, parents=None):
        w = _kaiming((cout, cin, 3, 3), g)
        b = torch.randn(cout, generator=g) * 0.01
        oh = (h + 2 - 3) // s + 1
        return Layer('conv', w.numpy(), b.numpy(), stride=s, pad=1, in_shape=(cin, h, h), out_shape=(cout, oh, oh),
                     parents=parents)

    def relu(shape, parents=None):
        return Layer('relu', in_shape=shape, out_shape=shape, parents=parents)

    sh = (4, 14, 14)
    L = [conv(1, 4, 28, 2), relu(sh)]                                            # 0, 1
    L += [conv(4, 4, 14, 1), relu(sh), conv(4, 4, 14, 1)]                        # 2, 3, 4
    L.append(Layer('add', in_shape=sh, out_shape=sh, parents=(4, 1)))           # 5
    L.append(relu(sh))                                                           # 6
    L.append(Layer('linear', _kaiming((10, 784), g).numpy(), (torch.randn(10, generator=g) * 0.01).numpy(),
                   in_shape=(784, 1, 1), out_shape=(10, 1, 1)))                  # 7
    return L


def _branches(seed):
    """784 -> 60 -> relu, two branches 60 -> 40 -> relu, concatenated (80) -> 10.

    Listed in the reference reader's breadth-first layer order (parse.py:250-300), which
    also numbers the layers: both branch Gemms, then both ReLUs."""
    g = torch.Generator().manual_seed(seed)

    def fc(n_in, n_out, parents=None):
        return Layer('linear', _kaiming((n_out, n_in), g).numpy(), (torch.randn(n_out, generator=g) * 0.01).numpy(),
                     in_shape=(n_in, 1, 1), out_shape=(n_out, 1, 1), parents=parents)

    def relu(n, parents=None):
        return Layer('relu', in_shape=(n, 1, 1), out_shape=(n, 1, 1), parents=parents)

    L = [fc(784, 60), relu(60)]                            # 0, 1
    L += [fc(60, 40, (1,)), fc(60, 40, (1,))]              # 2, 3: the two branches
    L += [relu(40, (2,)), relu(40, (3,))]                  # 4, 5
    L.append(Layer('concat', in_shape=(80, 1, 1), out_shape=(80, 1, 1), parents=(4, 5)))   # 6
    L.append(fc(80, 10))                                   # 7
    return L


def _tied(seed, pairs=32):
    """784-64-50-10 ReLU MLP whose first `pairs` first-layer neurons are x[2r] - x[2r+1]
    (weights exactly +1 and -1, bias 0).  With the two pixels of each pair equal
    (``centres`` ties them), such a neuron's lower and upper bounds are exact negatives
    (l + u == 0) under every certifier: the two products are exact, so the sum is rounded
    once whatever the order.  That is where the strict lower-slope test of zid.cf and the
    custom-stop programs (relu_n: l + u > 0) and DeepPoly's (l + u >= 0) part."""
    layers = _mlp([784, 64, 50, 10], seed, None)
    W = layers[0].W.copy()
    W[:pairs] = 0.0
    for r in range(pairs):
        W[r, 2 * r], W[r, 2 * r + 1] = 1.0, -1.0
    layers[0].W = W
    return layers


def parents_of(layers, i):
    """Parent indices of layer i (-1 = the network input)."""
    p = layers[i].parents
    return tuple(p) if p is not None else (i - 1,)


def is_chain(layers):
    return all(L.kind in ('linear', 'conv', 'relu') and parents_of(layers, i) == (i - 1,)
               for i, L in enumerate(layers))


def workload(wid):
    """The certification workloads: id -> Workload (full batch size).  0-4 and 7 are chains;
    5 (residual blocks), 6 (concatenated branches) and 8 (conv layers in a residual block)
    are DAGs; 7 has exactly tied ReLU inputs (a parity case for the lower-slope tests)."""
    if wid == 0:
        return Workload(0, "mlp_784-50x3-10", (1, 28, 28), _mlp([784, 50, 50, 50, 10], 0, None),
                        1, 0.01, 'mnist', 0, "DeepPoly, ReLU MLP 784-50-50-50-10, 1 region, eps 0.01")
    if wid == 1:
        return Workload(1, "mlp_784-100x6-10", (1, 28, 28), _mlp([784] + [100] * 6 + [10], 1, 0.01),
                        64, 0.005, 'mnist', 1, "DeepPoly, ReLU MLP 784-(100x6)-10, bias N(0,0.01), 64 regions")
    if wid == 2:
        return Workload(2, "mlp_784-200x9-10", (1, 28, 28), _mlp([784] + [200] * 9 + [10], 2, None),
                        256, 0.002, 'mnist', 2, "DeepPoly, ReLU MLP 784-(200x9)-10, 256 regions, eps 0.002")
    if wid == 3:
        return Workload(3, "conv_1x28x28_c16c32_fc100_fc10", (1, 28, 28),
                        _convnet((1, 28, 28), [(16, 4, 2, 0), (32, 4, 2, 0)], [100, 10], 3),
                        128, 0.02, 'mnist', 3, "DeepPoly, conv net 1x28x28, 128 regions, eps 0.02")
    if wid == 4:
        return Workload(4, "conv_3x32x32_c32c32c64c64_fc512x2_fc10", (3, 32, 32),
                        _convnet((3, 32, 32), [(32, 3, 1, 1), (32, 4, 2, 1), (64, 3, 1, 1), (64, 4, 2, 1)],
                                 [512, 512, 10], 4),
                        1024, 2.0 / 255.0, 'cifar', 4, "DeepPoly, conv net 3x32x32, 1024 regions, eps 2/255")
    if wid == 5:
        return Workload(5, "resmlp_784-100-2x(100,100,add)-10", (1, 28, 28), _residual(5),
                        32, 0.002, 'mnist', 5, "DeepPoly, residual MLP (two skip blocks), 32 regions")
    if wid == 6:
        return Workload(6, "branch_784-60-(40|40)-concat-10", (1, 28, 28), _branches(6),
                        32, 0.002, 'mnist', 6, "DeepPoly, two branches concatenated, 32 regions")
    if wid == 8:
        return Workload(8, "resconv_1x28x28_c4s2-(c4,c4,add)-10", (1, 28, 28), _resconv(8), 16, 0.01, 'mnist', 8,
                        "DeepPoly, conv layers inside a residual block, 16 regions")
    if wid == 7:
        return Workload(7, "tied_784-64-50-10", (1, 28, 28), _tied(7), 16, 0.01, 'mnist', 7,
                        "ReLU MLP 784-64-50-10 with 32 exactly tied first-layer neurons (l + u == 0), "
                        "16 regions, eps 0.01", extra={"tied_pairs": 32})
    raise ValueError(f"unknown workload {wid}")


def centres(wl, B=None):
    """Uniform [0,1] input centres [B, C, H, W] float32 (first B of the seeded draw)."""
    Bfull = wl.B if B is None else max(B, wl.B)
    g = torch.Generator().manual_seed(100 + wl.wid)
    X = torch.rand(Bfull, *wl.input_shape, generator=g)
    tp = wl.extra.get("tied_pairs", 0)
    if tp:
        flat = X.view(Bfull, -1)
        flat[:, 1:2 * tp:2] = flat[:, 0:2 * tp:2]
    return X[: (wl.B if B is None else B)].contiguous()


def _norm(x, dataset):
    """Dataset normalisation exactly as constraintflow/lib/spec.py:21-47 (float32)."""
    if dataset == 'mnist':
        mean = torch.tensor(MNIST_MEAN).reshape(-1, 1)
        std = torch.tensor(MNIST_STD).reshape(-1, 1)
        return (x - mean) / std
    mean = torch.tensor(CIFAR_MEAN).reshape(1, -1, 1, 1)
    std = torch.tensor(CIFAR_STD).reshape(1, -1, 1, 1)
    return (x - mean.expand(x.shape)) / std.expand(x.shape)


def input_box(X, eps, dataset):
    """L-inf box clipped to [0,1] then normalised, flattened: (l0, u0) [B, n0] float32.

    Follows constraintflow/lib/spec.py:21-47 (create_l / create_u) op for op.
    """
    X = torch.as_tensor(X, dtype=torch.float32)
    lo = torch.clip(X - eps, min=0., max=1.)
    hi = torch.clip(X + eps, min=0., max=1.)
    lo = _norm(lo, dataset).reshape(X.shape[0], -1)
    hi = _norm(hi, dataset).reshape(X.shape[0], -1)
    return lo.contiguous(), hi.contiguous()


def forward(layers, x):
    """float32 forward pass of the layer list on [B, C, H, W] inputs -> logits [B, 10]."""
    x = torch.as_tensor(x, dtype=torch.float32)
    outs = []
    for i, L in enumerate(layers):
        ps = parents_of(layers, i)
        h = x if ps[0] < 0 else outs[ps[0]]
        if L.kind == 'conv':
            h = torch.nn.functional.conv2d(h, torch.from_numpy(L.W), torch.from_numpy(L.b),
                                           stride=L.stride, padding=L.pad)
        elif L.kind == 'linear':
            h = h.reshape(h.shape[0], -1) @ torch.from_numpy(L.W).T + torch.from_numpy(L.b)
        elif L.kind == 'relu':
            h = torch.relu(h)
        elif L.kind == 'add':
            h = h + outs[ps[1]]
        elif L.kind == 'concat':
            h = torch.cat([h.reshape(h.shape[0], -1), outs[ps[1]].reshape(h.shape[0], -1)], dim=1)
        outs.append(h)
    return outs[-1]


def labels(wl, X):
    """Argmax label at the normalised centre, as the robustness property needs."""
    return forward(wl.layers, _norm(torch.as_tensor(X), wl.dataset)).argmax(-1)


def spec_weight(y, num_classes=10):
    """Per-region property matrix y[label] - y[j], j != label: [B, 9, 10] float32.

    Same construction as constraintflow/lib/spec.py:61-72.
    """
    y = torch.as_tensor(y)
    B = y.shape[0]
    eye = torch.eye(num_classes)
    w = eye[y].unsqueeze(1) - eye.unsqueeze(0)
    keep = ~(y.unsqueeze(1) == torch.arange(num_classes).unsqueeze(0))
    return w[keep].view(B, num_classes - 1, num_classes).contiguous()


def weights_digest(layers):
    """Order-sensitive float64 checksum of all weights (guards fixture/generator drift)."""
    s = 0.0
    for i, L in enumerate(layers):
        if L.W is not None:
            s += (i + 1) * float(np.asarray(L.W, np.float64).sum()) + 0.5 * float(np.abs(L.W).astype(np.float64).sum())
            s += (i + 7) * float(np.asarray(L.b, np.float64).sum())
    return s


def neuron_layout(wl):
    """Neuron numbering of the reference (input, then each layer, then the 9-row spec layer).

    Returns a list of (kind, start, end) per layer including the input and the
    property layer, matching constraintflow/lib/parse.py:243-248 and :284-295.
    """
    out = [('input', 0, wl.input_size)]
    pos = wl.input_size
    for L in wl.layers:
        out.append((L.kind, pos, pos + L.n_out))
        pos += L.n_out
    out.append(('spec', pos, pos + 9))
    return out


def conv_out(h, k, s, p):
    return math.floor((h + 2 * p - k) / s) + 1
