"""Network and layer descriptions (same names and fields as the reference's
constraintflow/lib/network.py:8-87: Network is a list of Layer; every neuron of the
network has an index, each layer owning the range [start, end))."""
from enum import Enum


class Network(list):
    def __init__(self, net_name=None, input_name=None, input_shape=None, input_size=0, input_start=0, input_end=0,
                 num_layers=0, torch_net=None, net_format="torch", no_sparsity=False):
        super().__init__()
        self.net_name = net_name
        self.input_name = input_name
        self.input_shape = input_shape
        self.input_size = input_size
        self.size = 0
        self.input_start = input_start
        self.input_end = input_end
        self.num_layers = num_layers
        self.torch_net = torch_net
        self.net_format = net_format
        self.no_sparsity = no_sparsity

    def similar(self):
        res = Network(self.net_name, self.input_name, self.input_shape, self.input_size, self.input_start,
                      self.input_end, self.num_layers, self.torch_net, self.net_format, self.no_sparsity)
        res.size = self.size
        return res


class LayerType(Enum):
    Conv2D = 1
    Linear = 2
    ReLU = 3
    Flatten = 4
    MaxPool1D = 5
    Normalization = 6
    NoOp = 7
    Tanh = 8
    Input = 9
    Concat = 10
    Sigmoid = 11
    Add = 12


class Layer:
    def __init__(self, weight=None, bias=None, type=None, shape=None, start=None, end=None, size=0, prev=None,
                 prev_weight=None, mean=0, sigma=1, identifier=0, parents=None):
        self.weight = weight
        self.bias = bias
        self.type = type
        self.shape = shape
        self.size = size
        self.start = start
        self.end = end
        self.prev = prev if prev is not None else {}
        self.prev_weight = prev_weight if prev_weight is not None else {}
        self.index_hash = dict()
        self.mean = mean
        self.sigma = sigma
        self.identifier = identifier
        self.parents = list(parents) if parents is not None else []
        self.children = list()
        self.last_layer = False
