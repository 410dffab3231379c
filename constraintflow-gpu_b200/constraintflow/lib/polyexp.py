"""Linear expressions over neurons: mat [.., n, N] plus const [.., n]
(reference: constraintflow/lib/polyexp.py:6-182)."""


class PolyExpSparse:
    def __init__(self, network, mat, const):
        self.network = network
        self.mat = mat
        self.const = const

    def get_mat(self, abs_elem=None, *args, **kwargs):
        return self.mat

    def get_const(self, *args, **kwargs):
        return self.const

    def create_similar(self, network=None, mat=None, const=None):
        return PolyExpSparse(network if network is not None else self.network,
                             mat if mat is not None else self.mat,
                             const if const is not None else self.const)

    def __repr__(self):
        return f"PolyExpSparse(mat={self.mat}, const={self.const})"
