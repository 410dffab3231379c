"""Input specification: the L-inf box around each centre and the robustness property.

Same entry points and arithmetic as the reference's constraintflow/lib/spec.py:
ImageDataset.create_l / create_u (:21-47, clip then dataset normalisation, float32),
get_output_spec_weight_and_bias (:61-72, rows e_label - e_k for k != label),
create_L / create_U (:86-104) and get_network_and_input_spec (:139-152).  l and u are
SparseTensors over all N neurons holding the input box in the input columns (fill
-inf / +inf elsewhere, as create_sparse_init :75-84 builds them).
"""
import copy

import torch

from constraintflow.gbcsr.sparse_block import DenseBlock
from constraintflow.gbcsr.sparse_tensor import SparseTensor

from .parse import get_net
from .polyexp import PolyExpSparse
from .symexp import SymExpSparse


class ImageDataset:
    mnist_mean = torch.tensor([0.1307]).reshape(-1, 1)
    mnist_std = torch.tensor([0.3081]).reshape(-1, 1)
    cifar10_mean = torch.tensor([0.4914, 0.4822, 0.4465]).reshape(1, -1, 1, 1)
    cifar10_std = torch.tensor([0.2023, 0.1994, 0.2010]).reshape(1, -1, 1, 1)
    imagenet_mean = torch.tensor([0.485, 0.456, 0.406]).reshape(1, -1, 1, 1)
    imagenet_std = torch.tensor([0.229, 0.224, 0.225]).reshape(1, -1, 1, 1)

    @staticmethod
    def _normalise(x, dataset):
        if dataset == "mnist":
            return (x - ImageDataset.mnist_mean) / ImageDataset.mnist_std
        if dataset in ("cifar10", "cifar"):
            return (x - ImageDataset.cifar10_mean.expand(x.shape)) / ImageDataset.cifar10_std.expand(x.shape)
        if dataset in ("tinyimagenet", "imagenet"):
            return (x - ImageDataset.imagenet_mean.expand(x.shape)) / ImageDataset.imagenet_std.expand(x.shape)
        return x

    @staticmethod
    def create_l(image, network_size, batch_size, eps=0.01, dataset="mnist", no_sparsity=False):
        l = ImageDataset._normalise(torch.clip(image - eps, min=0., max=1.), dataset).reshape(batch_size, -1)
        return create_sparse_init(l, float("-inf"), batch_size, network_size, no_sparsity)

    @staticmethod
    def create_u(image, network_size, batch_size, eps=0.01, dataset="mnist", no_sparsity=False):
        u = ImageDataset._normalise(torch.clip(image + eps, min=0., max=1.), dataset).reshape(batch_size, -1)
        return create_sparse_init(u, float("inf"), batch_size, network_size, no_sparsity)

    @staticmethod
    def get_output_spec_weight_and_bias(X, y, dataset="mnist"):
        num_classes = 200 if dataset in ("tinyimagenet", "imagenet") else 10
        eye = torch.eye(num_classes).type_as(X)
        weight = eye[y].unsqueeze(1) - eye.unsqueeze(0)
        keep = ~(y.unsqueeze(1) == torch.arange(num_classes).type_as(y).unsqueeze(0))
        weight = weight[keep].view(X.size(0), num_classes - 1, num_classes)
        return weight, torch.zeros(num_classes - 1, dtype=torch.float32)


def create_sparse_init(x, dense_const, batch_size, network_size, no_sparsity=False):
    return SparseTensor([torch.tensor([0, 0])], [DenseBlock(x)], 2, torch.tensor([batch_size, network_size]),
                        dense_const=dense_const)


def create_L(l, network, batch_size, no_sparsity=False):
    L = PolyExpSparse(network, SparseTensor([], [], 3, torch.tensor([batch_size, network.size, network.size])), 0)
    L.const = copy.copy(l)
    return L


def create_U(u, network, batch_size, no_sparsity=False):
    U = PolyExpSparse(network, SparseTensor([], [], 3, torch.tensor([batch_size, network.size, network.size])), 0)
    U.const = copy.copy(u)
    return U


def create_Z(l, u, network, no_sparsity=False):
    """Zonotope start state of zono.cf-style programs (reference spec.py:106-132).  The
    network driver builds it on the device from the input box (c0 = (l+u)/2, one symbol
    per input neuron with coefficient (u-l)/2); this object only carries the network."""
    return SymExpSparse(network, None, None)


def create_llist(network):
    return torch.tensor([True] + [False] * (len(network) - 1))


def get_network_and_input_spec(network_file, batch_size, X, y, dataset, eps, train=False, no_sparsity=False):
    if dataset == "tinyimagenet":
        X = X.to(torch.float32) / 255.0
    spec_weight, spec_bias = ImageDataset.get_output_spec_weight_and_bias(X, y, dataset)
    network = get_net(network_file, spec_weight, spec_bias, no_sparsity)
    l = ImageDataset.create_l(X, network.size, batch_size, eps, dataset, no_sparsity)
    u = ImageDataset.create_u(X, network.size, batch_size, eps, dataset, no_sparsity)
    L = create_L(l, network, batch_size, no_sparsity)
    U = create_U(u, network, batch_size, no_sparsity)
    Z = create_Z(l, u, network, no_sparsity)
    return network, l, u, L, U, Z, create_llist(network)
