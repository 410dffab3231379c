"""Lists of layers referenced by the generated transformers
(reference: constraintflow/lib/llist.py:12-778): a list of layer indices, or the range
[start, end), with the leading shape the generated code broadcasts over.

The network driver takes whole networks (weights, strides, paddings from the layer list),
so the per-layer metadata blocks (get_metadata), the weight products (dot) and the ReLU
polyexps (convert_to_poly) of the op-by-op interpretation are not provided: they raise
NotImplementedError.
"""


class Llist:
    def __init__(self, network, initial_shape=None, start=None, end=None, llist=None):
        self.network = network
        self.initial_shape = list(initial_shape) if initial_shape is not None else [1]
        self.start = start
        self.end = end
        self.llist = list(llist) if llist is not None else []
        self.llist_flag = llist is not None

    def layers(self):
        """The layer indices this list stands for."""
        return list(self.llist) if self.llist_flag else list(range(self.start, self.end))

    def coalesce(self):
        return self

    def decoalesce(self):
        return self

    def get_metadata(self, elem, batch_size, *args, **kwargs):
        raise NotImplementedError(f"Llist.get_metadata({elem!r}): the op-by-op interpretation of generated "
                                  "transformers is not provided (Flow runs recognised programs fused)")

    def dot(self, mats, total_size, *args, **kwargs):
        raise NotImplementedError("Llist.dot: the op-by-op interpretation of generated transformers is not "
                                  "provided (Flow runs recognised programs fused)")

    def convert_to_poly(self, abs_elem, *args, **kwargs):
        raise NotImplementedError("Llist.convert_to_poly: the op-by-op interpretation of generated transformers "
                                  "is not provided (Flow runs recognised programs fused)")
