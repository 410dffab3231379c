"""Typed blocks of the gbcsr block-sparse tensor, held on the GPU.

Same class names and constructor arguments as the reference
(constraintflow/gbcsr/sparse_block.py:120-147, 628, 1158, 1832, 2576, 3404, 3797), so code
that builds blocks directly keeps working.  Each block exposes ``view()``: a CUDA tensor
of the block's full shape, possibly a broadcast view (ConstBlock and RepeatBlock
materialise nothing).  Arithmetic on blocks is done by SparseTensor through libcfgpu.

The conv blocks (KernelBlock, PatchesBlock) also carry the reference's block algebra --
densification, the products with dense, diagonal, constant and other conv blocks, the
conversion of weights to per-position patches, sums and elementwise ops -- computed by
libcfgpu's conv-block kernels (cf_conv_densify, cf_conv_apply, cf_conv_scale,
cf_conv_transpose) and block kernels; their matmul methods return (block, -1) where the
reference returns (block, trace index).
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

    def matmul_equal_dims(self, sp_block, json_list=None, lhs_index=-1, rhs_index=-1):
        """[B, R, K] @ block (reference: DenseBlock.matmul_equal_dims sparse_block.py:748-962):
        a dense or densified block by cf_bmm, a diagonal as a column scaling, a KernelBlock as
        the transposed convolution of every row (F.conv_transpose2d, :839-911), a zero
        constant stays zero."""
        a = self.block
        if isinstance(sp_block, DiagonalBlock):
            d = sp_block.block.unsqueeze(sp_block.diag_index - 1)
            return DenseBlock(_dev.binary(operator.mul, a, d.expand(*a.shape), torch.float32)), -1
        if isinstance(sp_block, KernelBlock):
            B, R, Kd = a.shape
            if Kd != sp_block.rows:
                raise Exception("SHAPE MISMATCH")
            cols = sp_block.num_channels * sp_block.ix * sp_block.iy
            out = torch.empty(B, R, cols, dtype=torch.float32, device=a.device)
            _dev.conv_transpose(sp_block._geom(), B, R, a, (a.stride(0), a.stride(1), a.stride(2)), sp_block.block,
                                sp_block.ix, sp_block.iy, out, (R * cols, cols, 1))
            return DenseBlock(out), -1
        if isinstance(sp_block, ConstBlock):
            if sp_block.block == 0:
                tot = self.shape
                tot[-1] = sp_block.shape[-1]
                return ConstBlock(0, torch.tensor(tot)), -1
            raise NotImplementedError("DenseBlock @ a nonzero ConstBlock")
        b = sp_block.view()
        if b.shape[0] != a.shape[0]:
            b = b.expand(a.shape[0], *b.shape[1:])
        return DenseBlock(_dev.bmm(a, b if b.dtype == torch.float32 else b.float())), -1

    def matmul_unequal_dims(self, sp_block, json_list=None, lhs_index=-1, rhs_index=-1):
        """[B, R, K] @ [B, K] (:964)."""
        b = sp_block.view()
        return DenseBlock(_dev.bmm(self.block, (b if b.dtype == torch.float32 else b.float()).unsqueeze(-1))
                          .squeeze(-1)), -1


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

    def matmul_equal_dims(self, sp_block, json_list=None, lhs_index=-1, rhs_index=-1):
        """diag(d) @ block (reference: DiagonalBlock.matmul_equal_dims sparse_block.py:2211-2348):
        rows scaled by d; a KernelBlock becomes patches scaled row by row (:2265-2330)."""
        d = self.block.unsqueeze(self.diag_index)
        if isinstance(sp_block, KernelBlock):
            p = sp_block.convert_to_patches().block
            B = int(d.shape[0])
            out = _dev.binary(operator.mul, d.expand(B, *p.shape[1:]), p.expand(B, *p.shape[1:]), torch.float32)
            return PatchesBlock(out, sp_block.total_shape, sp_block.ix, sp_block.iy, sp_block.ox, sp_block.oy,
                                sp_block.sx, sp_block.sy, sp_block.px, sp_block.py, sp_block.kx, sp_block.ky,
                                sp_block.num_channels, sp_block.num_kernels), -1
        if isinstance(sp_block, DiagonalBlock):
            raise NotImplementedError("DiagonalBlock @ DiagonalBlock")
        if isinstance(sp_block, (DenseBlock, RepeatBlock)):
            b = sp_block.view()
            return DenseBlock(_dev.binary(operator.mul, d.expand(*b.shape), b if b.dtype == torch.float32 else b.float(),
                                          torch.float32)), -1
        raise Exception(f"Unrecognized sparse block type: {type(sp_block)}")


def _fit_total(A, total):
    """A dense [nb, rows, cols] matrix laid out over the block's total shape (the reference's
    PatchesBlock.get_dense, sparse_block.py:3218-3231: a missing dim is inserted where the
    shapes first differ and broadcast)."""
    total = [int(v) for v in total]
    if list(A.shape) == total:
        return A
    if len(A.shape) == len(total):
        return A.expand(*total)
    if list(A.shape) == total[:-1]:
        return A.unsqueeze(-1).expand(*total)
    diff = -1
    for i in range(len(A.shape)):
        if diff == -1 and total[i] != A.shape[i]:
            diff = i
        if diff != -1 and total[i + 1] != A.shape[i]:
            raise NotImplementedError(f"conv block densification: {list(A.shape)} over {total}")
    if diff == -1:
        diff = len(A.shape)
    return A.unsqueeze(diff).expand(*total)


def _identity(op):
    return {operator.add: 0, operator.mul: 1, operator.truediv: 1, operator.sub: 0, operator.and_: True,
            operator.or_: False}.get(op)


def _annihilator(op):
    return {operator.mul: 0, operator.and_: False, operator.or_: True}.get(op)


def _payload_op(a, b, op):
    """op on block payloads (a tensor, b a tensor broadcastable to it or a number)."""
    dt = torch.bool if op in _dev.COMPARISONS else torch.float32
    if not isinstance(b, torch.Tensor):
        b = _dev.scalar_view(float(b), list(a.shape), torch.float32)
    else:
        b = b.expand(*a.shape)
    return _dev.binary(op, a, b, dt)


class _ConvBlock(SparseBlock):
    """What KernelBlock and PatchesBlock share: the geometry, elementwise ops, shape edits."""

    def parameters(self):
        return [self.ix, self.iy, self.ox, self.oy, self.sx, self.sy, self.px, self.py, self.kx, self.ky,
                self.num_channels, self.num_kernels]

    def _geom(self, sx=None, sy=None):
        return _dev.conv_geom(self.num_kernels, self.num_channels, self.ox, self.oy, self.ix, self.iy, self.kx,
                              self.ky, self.sx if sx is None else sx, self.sy if sy is None else sy, self.px, self.py)

    @property
    def rows(self):
        return self.num_kernels * self.ox * self.oy

    def view(self):
        cache = getattr(self, "_view", None)
        if cache is None or cache[0] is not self.block:
            self._view = (self.block, _fit_total(self.get_dense(), self.shape))
        return self._view[1]

    def _with_total(self, total):
        return self.create_similar(self.block, total_shape=total)

    def repeat(self, repeat_dims, json_list=None, template_index=-1, simulacrum=False):
        res = self._with_total(self.total_shape * torch.as_tensor(repeat_dims, dtype=torch.int64))
        return (res, -1) if simulacrum else res

    def unsqueeze(self, index, json_list=None, template_index=-1, simulacrum=False):
        t = self.total_shape
        res = self._with_total(torch.cat([t[:index], torch.ones(1, dtype=torch.int64), t[index:]]))
        return (res, -1) if simulacrum else res

    def squeeze(self, index, json_list=None, template_index=-1, simulacrum=False):
        t = self.total_shape
        res = self._with_total(torch.cat([t[:index], t[index + 1:]]))
        return (res, -1) if simulacrum else res

    def binary(self, sp_block, op, json_list=None, lhs_index=-1, rhs_index=-1):
        """x op y with the reference's block rules (SparseBlock.binary sparse_block.py:181-420,
        PatchesBlock.binary :3327): a constant that is op's identity or annihilator, or one
        that keeps 0 at 0, acts on the payload; two conv blocks of the same kind and
        geometry combine payloads; a KernelBlock meets other kinds as patches; everything
        else is densified."""
        if isinstance(sp_block, ConstBlock):
            c = sp_block.block
            if _identity(op) is not None and c == _identity(op):
                return self, -1
            if _annihilator(op) is not None and c == _annihilator(op):
                return sp_block, -1
            if op(0, c) in (0, False):
                return self.create_similar(_payload_op(self.block, c, op)), -1
        if type(sp_block) is type(self) and self.parameters() == sp_block.parameters():
            a, b = self.block, sp_block.block
            if a.shape[0] < b.shape[0]:
                a = a.expand(b.shape[0], *a.shape[1:])
            return self.create_similar(_payload_op(a, b, op)), -1
        if isinstance(self, PatchesBlock) and isinstance(sp_block, RepeatBlock):
            reps = [int(t) // int(b) for t, b in zip(sp_block.shape, sp_block.block.shape)]
            if sum(r != 1 for r in reps) == 1 and reps[-1] > 1:
                return self.create_similar(_payload_op(self.block, sp_block.block.expand(*self.block.shape), op)), -1
        if isinstance(self, KernelBlock):
            return self.convert_to_patches().binary(sp_block, op)
        if isinstance(sp_block, KernelBlock):
            return self.binary(sp_block.convert_to_patches(), op)
        a, b = self.view(), sp_block.view()
        dt = torch.bool if op in _dev.COMPARISONS else torch.float32
        return DenseBlock(_dev.binary(op, a.float() if a.dtype != torch.float32 else a,
                                      b.float() if b.dtype != torch.float32 else b, dt)), -1


class KernelBlock(_ConvBlock):
    """Convolution weights W [K, C, kx, ky] standing for the conv's matrix
    [K*ox*oy, C*ix*iy] (reference: sparse_block.py:1158-1830)."""

    def __init__(self, block, total_shape, ix, iy, ox, oy, sx, sy, px, py):
        super().__init__(block, total_shape, "K")
        self.block = self.block.contiguous()
        self.ix, self.iy, self.ox, self.oy = int(ix), int(iy), int(ox), int(oy)
        self.sx, self.sy, self.px, self.py = int(sx), int(sy), int(px), int(py)
        self.kx, self.ky = int(self.block.shape[-2]), int(self.block.shape[-1])
        self.num_channels, self.num_kernels = int(self.block.shape[1]), int(self.block.shape[0])

    def _pstr(self):
        return 0, self.num_channels * self.kx * self.ky, 0

    def create_similar(self, block, json_list=None, template_index=-1, simulacrum=False, total_shape=None):
        res = KernelBlock(block, self.total_shape if total_shape is None else total_shape, self.ix, self.iy,
                          self.ox, self.oy, self.sx, self.sy, self.px, self.py)
        return (res, -1) if simulacrum else res

    def get_dense(self, json_list=None, template_index=-1, simulacrum=False):
        """[1, K*ox*oy, C*ix*iy] (KernelBlock.get_dense :1195)."""
        d = _dev.conv_densify(self._geom(), 1, self.block, *self._pstr())
        return (d, -1) if simulacrum else d

    def convert_to_patches(self, json_list=None, template_index=-1, simulacrum=False):
        """The weights repeated at every output position: PatchesBlock payload
        [1, K*ox*oy, C*kx*ky] (:1730-1806)."""
        K, ckk, pos = self.num_kernels, self.num_channels * self.kx * self.ky, self.ox * self.oy
        src = self.block.reshape(1, K, 1, ckk).expand(1, K, pos, ckk)
        pay = _dev.unary("to_f32", src, torch.float32).reshape(1, K * pos, ckk)
        res = PatchesBlock(pay, self.total_shape, self.ix, self.iy, self.ox, self.oy, self.sx, self.sy, self.px,
                           self.py, self.kx, self.ky, self.num_channels, self.num_kernels)
        return (res, -1) if simulacrum else res

    def matmul_equal_dims(self, sp_block, json_list=None, lhs_index=-1, rhs_index=-1):
        """M @ block (:1364-1607): a diagonal scales the patches (PatchesBlock), a zero constant
        stays zero, a dense [B, C*ix*iy, S] block is convolved column by column (F.conv2d),
        patches are densified first, other kinds go through convert_to_patches."""
        if isinstance(sp_block, DiagonalBlock):
            d = sp_block.block
            B = int(sp_block.batch_size)
            if list(d.shape) != [B, self.num_channels * self.ix * self.iy]:
                raise Exception("SHAPE MISMATCH")
            out = _dev.conv_scale(self._geom(), B, self.block, self._pstr(), d, d.stride(0), d.stride(-1))
            return PatchesBlock(out, self.total_shape, self.ix, self.iy, self.ox, self.oy, self.sx, self.sy, self.px,
                                self.py, self.kx, self.ky, self.num_channels, self.num_kernels), -1
        if isinstance(sp_block, ConstBlock):
            if sp_block.block == 0:
                tot = self.shape
                tot[-1] = sp_block.shape[-1]
                return ConstBlock(0, torch.tensor(tot)), -1
            raise NotImplementedError("KernelBlock @ a nonzero ConstBlock")
        if isinstance(sp_block, DenseBlock):
            b = sp_block.block
            B, prev, S = b.shape
            if prev != self.num_channels * self.ix * self.iy:
                raise Exception("SHAPE MISMATCH")
            out = torch.empty(B, self.rows, S, dtype=torch.float32, device=b.device)
            _dev.conv_apply(self._geom(), B, S, self.block, self._pstr(), b, (b.stride(0), b.stride(2), b.stride(1)),
                            out, (self.rows * S, 1, S))
            return DenseBlock(out), -1
        if isinstance(sp_block, PatchesBlock):
            return self.matmul_equal_dims(DenseBlock(sp_block.get_dense()))
        return self.convert_to_patches().matmul_equal_dims(sp_block)

    def matmul_unequal_dims(self, sp_block, json_list=None, lhs_index=-1, rhs_index=-1):
        """M @ vector (:1631-1728): a dense [B, C*ix*iy] block is convolved (F.conv2d)."""
        if isinstance(sp_block, DenseBlock):
            x = sp_block.block
            B = int(x.shape[0])
            if x.dim() != 2 or x.shape[1] != self.num_channels * self.ix * self.iy:
                raise Exception("SHAPE MISMATCH")
            out = torch.empty(B, self.rows, dtype=torch.float32, device=x.device)
            _dev.conv_apply(self._geom(), B, 1, self.block, self._pstr(), x, (x.stride(0), 0, x.stride(1)), out,
                            (self.rows, 0, 1))
            return DenseBlock(out), -1
        if isinstance(sp_block, (DiagonalBlock, KernelBlock)):
            raise NotImplementedError(f"KernelBlock @ {type(sp_block).__name__} (vector)")
        if isinstance(sp_block, ConstBlock):
            if sp_block.block == 0:
                return ConstBlock(0, torch.tensor(self.shape[:-1])), -1
            raise NotImplementedError("KernelBlock @ a nonzero ConstBlock (vector)")
        raise Exception(f"Unrecognized sparse block type: {type(sp_block)}")


class PatchesBlock(_ConvBlock):
    """Per-row conv patches: payload [B, K*ox*oy, C*kx*ky], row (k, oxi, oyi) holding the
    patch placed at input rows oxi*sx - px .. and columns oyi*sy - py .. (reference:
    sparse_block.py:2576-3402)."""

    def __init__(self, block, total_shape, ix, iy, ox, oy, sx, sy, px, py, kx, ky, num_channels, num_kernels):
        super().__init__(block, total_shape, "P")
        if self.block.dtype != torch.bool and self.block.stride(-1) != 1:
            self.block = _dev.unary("to_f32", self.block, torch.float32)
        self.ix, self.iy, self.ox, self.oy = int(ix), int(iy), int(ox), int(oy)
        self.sx, self.sy, self.px, self.py = int(sx), int(sy), int(px), int(py)
        self.kx, self.ky = int(kx), int(ky)
        self.num_channels, self.num_kernels = int(num_channels), int(num_kernels)
        self.batch_size = int(self.block.shape[0])
        if self.block.dim() != 3 or list(self.block.shape[1:]) != [self.rows, self.num_channels * self.kx * self.ky]:
            raise Exception(f"SHAPE MISMATCH (patches payload {list(self.block.shape)})")

    def _pstr(self, nb=None):
        s1 = self.block.stride(1)
        bs = 0 if self.block.shape[0] == 1 else self.block.stride(0)
        return bs, self.ox * self.oy * s1, s1

    def create_similar(self, block, json_list=None, template_index=-1, simulacrum=False, total_shape=None):
        res = PatchesBlock(block, self.total_shape if total_shape is None else total_shape, self.ix, self.iy,
                           self.ox, self.oy, self.sx, self.sy, self.px, self.py, self.kx, self.ky, self.num_channels,
                           self.num_kernels)
        return (res, -1) if simulacrum else res

    def get_dense(self, json_list=None, template_index=-1, simulacrum=False):
        """[B, K*ox*oy, C*ix*iy] laid out over the total shape (:3089-3248; the reference
        places patches with the x stride in both dims)."""
        B = int(self.total_shape[0])
        if self.block.shape[0] not in (1, B):
            raise NotImplementedError(f"PatchesBlock payload batch {self.block.shape[0]} over {B} regions")
        d = _dev.conv_densify(self._geom(sx=self.sx, sy=self.sx), B, self.block, *self._pstr())
        d = _fit_total(d, self.shape) if d.dim() != len(self.shape) else d
        return (d, -1) if simulacrum else d

    def total_expand(self, json_list=None, template_index=-1, simulacrum=False):
        """The payload broadcast to the block's leading dims (:3373)."""
        self.block = self.block.expand(*(self.shape[:-1] + [int(self.block.shape[-1])]))
        return (self, template_index) if simulacrum else self

    def sum(self, dim, json_list=None, template_index=-1, simulacrum=False):
        """Over the last dim: the payload's row sums (the patch entries, :3279-3306);
        otherwise the dense matrix's."""
        if dim == len(self.shape) - 1 or dim == -1:
            p = self.block
            nb, R, J = p.shape
            out = _dev.bmm(p, _dev.scalar_view(1.0, [nb, J, 1], torch.float32))
            return DenseBlock(out.reshape(nb, R)), -1
        d = self.get_dense()
        nb, R, Cn = d.shape
        if dim == 1:
            out = _dev.bmm(_dev.scalar_view(1.0, [nb, 1, R], torch.float32), d)
            return DenseBlock(out.reshape(nb, Cn)), -1
        if dim == 0:
            out = _dev.bmm(_dev.scalar_view(1.0, [1, 1, nb], torch.float32), d.reshape(1, nb, R * Cn))
            return DenseBlock(out.reshape(R, Cn)), -1
        raise NotImplementedError(f"PatchesBlock.sum over dim {dim}")

    def matmul_equal_dims(self, sp_block, json_list=None, lhs_index=-1, rhs_index=-1):
        """patches @ block (:2737-2940): with a KernelBlock every patch is transposed-convolved
        by the next layer's weights (the patches grow, stride and padding compose); with a
        DiagonalBlock every patch value is scaled by the input value under it."""
        if isinstance(sp_block, KernelBlock):
            if sp_block.num_kernels != self.num_channels:
                raise Exception("SHAPE MISMATCH")
            p = self.block
            nb, R, J = p.shape
            if J != self.num_channels * self.kx * self.ky:
                raise Exception("SHAPE MISMATCH")
            OH = (self.kx - 1) * sp_block.sx + sp_block.kx
            OW = (self.ky - 1) * sp_block.sy + sp_block.ky
            g = _dev.conv_geom(self.num_channels, sp_block.num_channels, self.kx, self.ky, OH, OW, sp_block.kx,
                               sp_block.ky, sp_block.sx, sp_block.sy, 0, 0)
            E = sp_block.num_channels * OH * OW
            out = torch.empty(nb, R, E, dtype=torch.float32, device=p.device)
            _dev.conv_transpose(g, nb, R, p, (p.stride(0), p.stride(1), p.stride(2)), sp_block.block, OH, OW, out,
                                (R * E, E, 1))
            # composed stride and padding as the reference computes them
            # (compute_patches_stride_padding :2712 with 2-tuples: the second dim's values)
            stride = self.sy * sp_block.sy
            pad = self.py * sp_block.sy + sp_block.py
            t0, t1 = self.total_shape, sp_block.total_shape
            total = torch.cat([torch.maximum(t0[:-2], t1[:-2]), t0[-2:-1], t1[-1:]])
            return PatchesBlock(out, total, sp_block.ix, sp_block.iy, self.ox, self.oy, stride, stride, pad, pad, OH,
                                OW, sp_block.num_channels, self.num_kernels), -1
        if isinstance(sp_block, DiagonalBlock):
            d = sp_block.block
            B = int(sp_block.batch_size)
            if self.block.shape[0] not in (1, B) or list(d.shape) != [B, self.num_channels * self.ix * self.iy]:
                raise Exception("SHAPE MISMATCH")
            out = _dev.conv_scale(self._geom(), B, self.block, self._pstr(), d, d.stride(0), d.stride(-1))
            return self.create_similar(out), -1
        raise NotImplementedError(f"PatchesBlock @ {type(sp_block).__name__}")

    def matmul_unequal_dims(self, sp_block, json_list=None, lhs_index=-1, rhs_index=-1):
        """patches @ vector (:2942-3086): every row's patch dotted with the input values under
        it."""
        if isinstance(sp_block, DenseBlock):
            x = sp_block.block
            B = int(x.shape[0])
            if self.block.shape[0] not in (1, B) or x.dim() != 2 or x.shape[1] != self.num_channels * self.ix * self.iy:
                raise Exception("SHAPE MISMATCH")
            out = torch.empty(B, self.rows, dtype=torch.float32, device=x.device)
            _dev.conv_apply(self._geom(), B, 1, self.block, self._pstr(), x, (x.stride(0), 0, x.stride(1)), out,
                            (self.rows, 0, 1))
            return DenseBlock(out), -1
        if isinstance(sp_block, ConstBlock) and sp_block.block == 0:
            return ConstBlock(0, torch.tensor(self.shape[:-1])), -1
        if isinstance(sp_block, RepeatBlock):
            return self.matmul_unequal_dims(DenseBlock(_dev.unary("to_f32", sp_block.view(), torch.float32)))
        raise NotImplementedError(f"PatchesBlock @ {type(sp_block).__name__} (vector)")
