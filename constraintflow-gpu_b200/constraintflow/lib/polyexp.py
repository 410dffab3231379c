"""Linear expressions over neurons: mat [.., n, N] plus const [.., n]
(reference: constraintflow/lib/polyexp.py:6-182).

The drop-in Flow runs the programs it recognises as fused passes (cf_deeppoly_run), so
generated code never drives these objects there; they keep the reference's constructor
and accessors for code that builds or reads them directly.
"""
import torch


class PolyExpSparse:
    def __init__(self, network, mat, const):
        self.network = network
        self.mat = mat
        self.const = const

    def get_mat(self, abs_elem=None, *args, **kwargs):
        """mat's blocks over the columns of the live layers (the first live layer's start to
        the last one's end, reference polyexp.py:131-137, SparseTensor.get_sparse_custom_range);
        the whole mat without an abstract element or when mat is a number."""
        if abs_elem is None or isinstance(self.mat, (int, float)):
            return self.mat
        live = torch.nonzero(torch.as_tensor(abs_elem.d["llist"])).flatten().tolist()
        start, end = self.network[live[0]].start, self.network[live[-1]].end
        lo = [0] * self.mat.dims
        hi = [int(v) for v in self.mat.total_size]
        lo[-1], hi[-1] = int(start), int(end)
        return self.mat.get_sparse_custom_range(torch.tensor(lo), torch.tensor(hi))

    def get_const(self, *args, **kwargs):
        return self.const

    def copy(self):
        return PolyExpSparse(self.network, self.mat, self.const)

    def create_similar(self, network=None, mat=None, const=None):
        return PolyExpSparse(network if network is not None else self.network,
                             mat if mat is not None else self.mat,
                             const if const is not None else self.const)

    def __repr__(self):
        return f"PolyExpSparse(mat={self.mat}, const={self.const})"
