"""Lists of layers referenced by the generated transformers
(reference: constraintflow/lib/llist.py:12-778).  The network driver consumes whole
networks, so only the constructor and the layer bookkeeping are needed here."""


class Llist:
    def __init__(self, network, initial_shape=None, start=None, end=None, llist=None):
        self.network = network
        self.initial_shape = list(initial_shape) if initial_shape is not None else [1]
        self.start = start
        self.end = end
        self.llist = list(llist) if llist is not None else []
        self.llist_flag = llist is not None

    def coalesce(self):
        return self

    def decoalesce(self):
        return self
