"""Typed blocks of the gbcsr block-sparse tensor, held on the GPU.

Same class names and constructor arguments as the reference
(constraintflow/gbcsr/sparse_block.py:120-147, 628, 1158, 1832, 2576, 3404, 3797), so code
that builds blocks directly keeps working.  Each block exposes ``view()``: a CUDA tensor
of the block's full shape, possibly a broadcast view (ConstBlock and RepeatBlock
materialise nothing).  Arithmetic on blocks is done by SparseTensor through libcfgpu.
"""
import operator

import torch

from . import _dev


def _shape(total_shape):
    return [int(x) for x in torch.as_tensor(total_shape).reshape(-1).tolist()]


class SparseBlock:
    def __init__(self, block, total_shape, block_type="D"):
        self.total_shape = torch.as_tensor(_shape(total_shape), dtype=torch.int64)
        self.block_type = block_type
        if isinstance(block, torch.Tensor):
            self.block = _dev.as_block_tensor(block)
        elif isinstance(block, bool):
            self.block = block
        else:
            self.block = float(block)

    @property
    def shape(self):
        return _shape(self.total_shape)

    @property
    def is_const(self):
        return False

    def view(self):
        raise NotImplementedError(type(self).__name__)


class DenseBlock(SparseBlock):
    def __init__(self, block):
        super().__init__(block, torch.tensor(list(block.shape)), "D")
        self.batch_size = self.shape[0] if self.shape else 1

    def view(self):
        return self.block


class ConstBlock(SparseBlock):
    """A block whose every element is one value (reference: sparse_block.py:3404)."""

    def __init__(self, block, total_shape):
        if isinstance(block, torch.Tensor):
            block = block.item()
        super().__init__(block, total_shape, "C")

    @property
    def is_const(self):
        return True

    @property
    def value(self):
        return self.block

    def view(self):
        dtype = torch.bool if isinstance(self.block, bool) else torch.float32
        return _dev.scalar_view(self.block, self.shape, dtype)


class RepeatBlock(SparseBlock):
    """A block broadcast along its size-1 dims (reference: sparse_block.py:3797)."""

    def __init__(self, block, total_shape):
        super().__init__(block, total_shape, "R")

    def view(self):
        return self.block.expand(*self.shape)


class DiagonalBlock(SparseBlock):
    """Diagonal between dims (diag_index-1, diag_index); the payload omits dim diag_index
    (reference: sparse_block.py:1832-1905, diag_embed)."""

    def __init__(self, block, total_shape, diag_index):
        super().__init__(block, total_shape, "Diag")
        self.diag_index = int(diag_index)
        self.batch_size = self.shape[0]
        self._dense = None

    def view(self):
        if self._dense is None:
            shp = self.shape
            d = self.diag_index
            n = shp[d]
            dev = self.block.device
            idx = torch.arange(n, device=dev)
            eye_shape = [1] * len(shp)
            eye_shape[d - 1] = n
            eye_shape[d] = n
            # cond = (i == j) laid out over dims (d-1, d); value = payload broadcast over dim d
            row = idx.reshape([n if k == d - 1 else 1 for k in range(len(shp))]).to(torch.float32)
            col = idx.reshape([n if k == d else 1 for k in range(len(shp))]).to(torch.float32)
            cond = _dev.binary(operator.eq, row.expand(*shp), col.expand(*shp), torch.bool)
            val = self.block.unsqueeze(d).expand(*shp)
            zero = _dev.scalar_view(0.0, shp, torch.float32)
            self._dense = _dev.where(cond, val, zero)
        return self._dense


class KernelBlock(SparseBlock):
    """Convolution weights standing for their Toeplitz matrix (reference: sparse_block.py:1158).

    Constructible for compatibility; conv backsubstitution runs in the network driver
    (cf_deeppoly_run's receptive-field windows), not through block algebra."""

    def __init__(self, block, total_shape, ix, iy, ox, oy, sx, sy, px, py):
        super().__init__(block, total_shape, "K")
        self.ix, self.iy, self.ox, self.oy = ix, iy, ox, oy
        self.sx, self.sy, self.px, self.py = sx, sy, px, py

    def view(self):
        raise NotImplementedError("KernelBlock densification: conv layers run in cf_deeppoly_run")


class PatchesBlock(SparseBlock):
    """Per-position conv patches (reference: sparse_block.py:2576); see KernelBlock."""

    def __init__(self, block, total_shape, ix, iy, ox, oy, sx, sy, px, py, kx, ky, num_channels, num_kernels):
        super().__init__(block, total_shape, "P")
        self.geometry = (ix, iy, ox, oy, sx, sy, px, py, kx, ky, num_channels, num_kernels)

    def view(self):
        raise NotImplementedError("PatchesBlock densification: conv layers run in cf_deeppoly_run")
