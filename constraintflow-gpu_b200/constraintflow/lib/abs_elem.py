"""The abstract element: per-neuron state of the certifier (reference:
constraintflow/lib/abs_elem.py:10-963).  d['l'], d['u'] are SparseTensors over all N
neurons, d['L'], d['U'] linear expressions, d['llist'] the processed-layer mask.

Flow (flow_sparse.py) reads the input box from d['l'] / d['u'], runs the recognised program
as one fused pass on the GPU and writes every neuron's bounds back into d['l'] / d['u'] with
d['llist'] all set, as the reference's final state has them.  The per-layer gather and
scatter that generated transformer bodies call (get_elem, update) belong to the op-by-op
interpretation of a program, which this runtime does not provide: they raise
NotImplementedError, as Flow does for a program it does not recognise.
"""
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
        """End of the last live layer's neuron columns (reference abs_elem.py:50)."""
        last = int(torch.nonzero(torch.as_tensor(self.d["llist"])).flatten()[-1].item())
        return self.network[last].end

    def live_layers(self):
        return torch.nonzero(torch.as_tensor(self.d["llist"])).flatten().tolist()

    def get_elem(self, key, llist, *args, **kwargs):
        raise NotImplementedError("Abs_elem_sparse.get_elem: generated transformer bodies are not interpreted op "
                                  "by op; Flow runs recognised programs as fused GPU passes")

    def update(self, llist, abs_shape, *args, **kwargs):
        raise NotImplementedError("Abs_elem_sparse.update: generated transformer bodies are not interpreted op "
                                  "by op; Flow runs recognised programs as fused GPU passes")
