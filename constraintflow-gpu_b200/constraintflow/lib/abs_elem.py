"""The abstract element: per-neuron state of the certifier (reference:
constraintflow/lib/abs_elem.py:10-963).  d['l'], d['u'] are SparseTensors over all N
neurons, d['L'], d['U'] linear expressions, d['llist'] the processed-layer mask."""
import torch


class Abs_elem_sparse:
    def __init__(self, d, types, network, batch_size=1, no_sparsity=False):
        if d.keys() != types.keys():
            raise TypeError("abs elem inconsistent")
        self.d = d
        self.types = types
        self.network = network
        self.batch_size = batch_size
        self.no_sparsity = no_sparsity

    def get_poly_size(self):
        last = int(torch.nonzero(self.d["llist"]).flatten()[-1].item())
        return self.network[last].end
