"""The gbcsr block-sparse tensor on the GPU.

A SparseTensor is a total size, a fill value (``dense_const``) and disjoint boxes, each
holding a typed block (reference format: constraintflow/gbcsr/sparse_tensor.py:492-561).
Operations between tensors work on the common refinement of their boxes: along every
dim, the start/end coordinates of all boxes of all operands are merged into breakpoints;
each cell of the resulting grid is covered by at most one block per operand, so the
cell's value is an elementwise (or, for matmul, a per-cell GEMM) function of block
views and fill values.  Cells covered by no block of any operand stay fill.  This gives
the dense result the reference's block-union algorithms produce (union_tensors :1044,
binary :1242, matmul :1671, sp_where :2447) on every layout, including overlaps that
the reference does not split.  All arithmetic runs in libcfgpu kernels (see _dev.py).

Method signatures accept (and ignore) the reference's JIT-capture keyword arguments.
"""
import bisect
import itertools
import operator

import torch

from . import _dev
from .sparse_block import ConstBlock, DenseBlock, SparseBlock

ANNIHILATOR = {operator.mul: 0.0, operator.and_: False}


def _ints(x):
    return [int(v) for v in torch.as_tensor(x).reshape(-1).tolist()]


def _torch_dtype(typ):
    return torch.bool if typ is bool else torch.float32


class SparseTensor:
    def __init__(self, start_indices, blocks, dims, total_size, end_indices=None, type=float, dense_const=0.0):
        self.total_size = torch.as_tensor(_ints(total_size), dtype=torch.int64).int()
        self.dims = int(dims)
        self.type = bool if type is bool else float
        self.blocks = list(blocks)
        self.start_indices = [torch.as_tensor(_ints(s), dtype=torch.int64) for s in start_indices]
        if end_indices is None:
            self.end_indices = [s + b.total_shape for s, b in zip(self.start_indices, self.blocks)]
        else:
            self.end_indices = [torch.as_tensor(_ints(e), dtype=torch.int64) for e in end_indices]
        self.num_blocks = len(self.blocks)
        if isinstance(dense_const, torch.Tensor):
            dense_const = dense_const.item()
        self.dense_const = dense_const
        if self.num_blocks and self.check_dense():
            self.dense_const = False if self.type is bool else 0.0

    # ------------------------------------------------------------------ structure
    @property
    def shape(self):
        return _ints(self.total_size)

    def _boxes(self):
        return [(_ints(s), _ints(e)) for s, e in zip(self.start_indices, self.end_indices)]

    def check_dense(self):
        vol = 1
        for v in self.shape:
            vol *= v
        covered = 0
        for s, e in self._boxes():
            c = 1
            for a, b in zip(s, e):
                c *= max(0, b - a)
            covered += c
        return covered >= vol

    def exists_sub_block(self, start_index, end_index):
        """Some block contains the box [start, end) and is not a zero/False constant
        (reference: sparse_tensor.py:851-858)."""
        st, en = _ints(start_index), _ints(end_index)
        for (s, e), blk in zip(self._boxes(), self.blocks):
            if all(a >= s_ and b <= e_ for a, b, s_, e_ in zip(st, en, s, e)):
                if isinstance(blk, ConstBlock) and blk.block == self.dense_const and not self.dense_const:
                    return False
                return True
        return False

    def get_block_id(self, start_index, end_index):
        st, en = _ints(start_index), _ints(end_index)
        res, rs, re_ = [], [], []
        for i, (s, e) in enumerate(self._boxes()):
            if all(a >= s_ and b <= e_ for a, b, s_, e_ in zip(s, e, st, en)):
                res.append(i)
                rs.append(self.start_indices[i])
                re_.append(self.end_indices[i])
        return res, rs, re_

    # ------------------------------------------------------------------ dense views
    def _fill_view(self, shape):
        return _dev.scalar_view(self.dense_const, shape, _torch_dtype(self.type))

    def _cell_view(self, bid, lo, hi):
        shape = [b - a for a, b in zip(lo, hi)]
        if bid is None:
            return self._fill_view(shape)
        s = _ints(self.start_indices[bid])
        v = self.blocks[bid].view()
        sl = tuple(slice(a - o, b - o) for a, b, o in zip(lo, hi, s))
        return v[sl]

    def _cell_const(self, bid):
        """(True, value) when the cell is constant: fill or a ConstBlock."""
        if bid is None:
            return True, self.dense_const
        blk = self.blocks[bid]
        if isinstance(blk, ConstBlock):
            return True, blk.block
        return False, None

    def get_dense_device(self):
        out = torch.empty(self.shape, dtype=_torch_dtype(self.type), device=_dev.device())
        out.copy_(self._fill_view(self.shape))
        for (s, e), blk in zip(self._boxes(), self.blocks):
            out[tuple(slice(a, b) for a, b in zip(s, e))].copy_(blk.view())
        return out

    def get_dense(self, *args, **kwargs):
        """Dense CPU tensor, float64 for float tensors as the reference returns
        (sparse_tensor.py:627-654: torch.ones(total_size, dtype=float))."""
        d = self.get_dense_device().cpu()
        return d.to(torch.float64) if self.type is float else d

    # ------------------------------------------------------------------ grid refinement
    @staticmethod
    def _breakpoints(shape, tensors, dims_map=None):
        bps = []
        for d, n in enumerate(shape):
            pts = {0, n}
            for t, dm in zip(tensors, dims_map or [None] * len(tensors)):
                if t is None:
                    continue
                td = d if dm is None else dm[d]
                if td is None:
                    continue
                for s, e in t._boxes():
                    pts.add(max(0, min(n, s[td])))
                    pts.add(max(0, min(n, e[td])))
            bps.append(sorted(pts))
        return bps

    @staticmethod
    def _cover(t, bps, dmap=None):
        """cell index tuple -> block id of t (dims of t mapped from grid dims by dmap)."""
        cover = {}
        ndim = len(bps)
        for bid, (s, e) in enumerate(t._boxes()):
            ranges = []
            for d in range(ndim):
                td = d if dmap is None else dmap[d]
                if td is None:
                    ranges.append(range(len(bps[d]) - 1))
                    continue
                i0 = bisect.bisect_left(bps[d], s[td])
                i1 = bisect.bisect_left(bps[d], e[td])
                ranges.append(range(i0, i1))
            for cell in itertools.product(*ranges):
                cover[cell] = bid
        return cover

    # ------------------------------------------------------------------ elementwise
    def _elementwise(self, others, fn, out_type, dense_const, const_fn=None):
        """Apply fn(views...) on every grid cell covered by a block of any operand."""
        tens = [self] + list(others)
        bps = self._breakpoints(self.shape, tens)
        covers = [self._cover(t, bps) for t in tens]
        cells = set()
        for c in covers:
            cells.update(c.keys())
        starts, blocks = [], []
        for cell in sorted(cells):
            lo = [bps[d][i] for d, i in enumerate(cell)]
            hi = [bps[d][i + 1] for d, i in enumerate(cell)]
            if any(b <= a for a, b in zip(lo, hi)):
                continue
            bids = [c.get(cell) for c in covers]
            if const_fn is not None:
                consts = [t._cell_const(b) for t, b in zip(tens, bids)]
                hit, val = const_fn(consts)
                if hit:
                    if val != dense_const:
                        starts.append(torch.tensor(lo))
                        blocks.append(ConstBlock(val, torch.tensor([b - a for a, b in zip(lo, hi)])))
                    continue
            views = [t._cell_view(b, lo, hi) for t, b in zip(tens, bids)]
            starts.append(torch.tensor(lo))
            blocks.append(DenseBlock(fn(*views)))
        return SparseTensor(starts, blocks, self.dims, self.total_size, type=out_type, dense_const=dense_const)

    def _coerce(self, other):
        if isinstance(other, SparseTensor):
            return other
        if isinstance(other, torch.Tensor) and other.numel() == 1:
            other = other.item()
        if isinstance(other, (bool, int, float)):
            typ = bool if isinstance(other, bool) else float
            return SparseTensor([], [], self.dims, self.total_size, type=typ, dense_const=other)
        if isinstance(other, torch.Tensor):
            return convert_dense_to_sparse(other)
        raise TypeError(f"cannot combine SparseTensor with {type(other)}")

    def binary(self, sp_tensor, op, *args, **kwargs):
        other = self._coerce(sp_tensor)
        if _ints(other.total_size) != self.shape:
            raise Exception("SHAPE MISMATCH")
        out_type = bool if op in _dev.COMPARISONS else self.type
        if op == operator.truediv and other.check_dense():
            dc = 0.0
        else:
            dc = op(self.dense_const, other.dense_const)
        if out_type is float:
            dc = float(dc)
        out_dtype = _torch_dtype(out_type)
        ann = ANNIHILATOR.get(op)

        def const_fn(consts):
            # conjunction ops skip work against an absorbing constant: x*0 = 0, x and False
            # = False, and 0/y = 0 for a constant-zero numerator (op_helper.py:6-35), which is
            # also what the reference returns where IEEE arithmetic would give NaN (0*inf, 0/0)
            if op is operator.truediv:
                is_c, v = consts[0]
                return (True, 0.0) if (is_c and v == 0) else (False, None)
            if ann is None:
                return False, None
            for is_c, v in consts:
                if is_c and v == ann:
                    return True, (False if op is operator.and_ else 0.0)
            return False, None

        def fn(a, b):
            if a.dtype != b.dtype and op not in (operator.and_, operator.or_):
                a, b = a.float(), b.float()
            return _dev.binary(op, a, b, out_dtype)
        return self._elementwise([other], fn, out_type, dc, const_fn)

    def unary(self, op, *args, **kwargs):
        if op == operator.not_:
            dc = not self.dense_const
            out_type = bool
            name = "not_"
        elif op == operator.neg:
            dc = -self.dense_const
            out_type = self.type
            name = "neg"
        else:
            raise NotImplementedError(f"unary {op}")
        starts, blocks = [], []
        for (s, e), blk in zip(self._boxes(), self.blocks):
            starts.append(torch.tensor(s))
            if isinstance(blk, ConstBlock):
                blocks.append(ConstBlock(op(blk.block), blk.total_shape))
            else:
                blocks.append(DenseBlock(_dev.unary(name, blk.view(), _torch_dtype(out_type))))
        return SparseTensor(starts, blocks, self.dims, self.total_size, type=out_type, dense_const=dc)

    def float(self, *args, **kwargs):
        if self.type is float:
            return self
        starts, blocks = [], []
        for (s, e), blk in zip(self._boxes(), self.blocks):
            starts.append(torch.tensor(s))
            if isinstance(blk, ConstBlock):
                blocks.append(ConstBlock(float(blk.block), blk.total_shape))
            else:
                blocks.append(DenseBlock(_dev.unary("to_f32", blk.view(), torch.float32)))
        return SparseTensor(starts, blocks, self.dims, self.total_size, type=float, dense_const=float(self.dense_const))

    def clamp(self, const, min_true, *args, **kwargs):
        """min_true: clamp(min=const), else clamp(max=const), applied to the blocks; the fill
        value is kept as it is, as the reference does (sparse_tensor.py:2333-2384)."""
        c = float(const)
        dc = self.dense_const
        starts, blocks = [], []
        for (s, e), blk in zip(self._boxes(), self.blocks):
            starts.append(torch.tensor(s))
            if isinstance(blk, ConstBlock):
                v = blk.block
                blocks.append(ConstBlock(max(v, c) if min_true else min(v, c), blk.total_shape))
            else:
                blocks.append(DenseBlock(_dev.clamp(blk.view(), c, min_true)))
        return SparseTensor(starts, blocks, self.dims, self.total_size, type=float, dense_const=float(dc))

    def any(self, *args, **kwargs):
        if not self.check_dense():
            if self.dense_const:
                return True
        for blk in self.blocks:
            if isinstance(blk, ConstBlock):
                if blk.block:
                    return True
            elif _dev.any_nonzero(blk.view()):
                return True
        return False

    # ------------------------------------------------------------------ shape ops
    def unsqueeze(self, index, *args, **kwargs):
        index = int(index)
        shape = self.shape
        shape.insert(index, 1)
        starts, ends, blocks = [], [], []
        for (s, e), blk in zip(self._boxes(), self.blocks):
            starts.append(torch.tensor(s[:index] + [0] + s[index:]))
            ends.append(torch.tensor(e[:index] + [1] + e[index:]))
            bs = blk.shape
            bs.insert(index, 1)
            if isinstance(blk, ConstBlock):
                blocks.append(ConstBlock(blk.block, torch.tensor(bs)))
            else:
                blocks.append(DenseBlock(blk.view().unsqueeze(index)))
        return SparseTensor(starts, blocks, self.dims + 1, torch.tensor(shape), ends, self.type, self.dense_const)

    def squeeze(self, index, *args, **kwargs):
        index = int(index)
        shape = self.shape
        assert shape[index] == 1, "squeeze of a dim that is not 1"
        shape.pop(index)
        starts, ends, blocks = [], [], []
        for (s, e), blk in zip(self._boxes(), self.blocks):
            starts.append(torch.tensor(s[:index] + s[index + 1:]))
            ends.append(torch.tensor(e[:index] + e[index + 1:]))
            bs = blk.shape
            bs.pop(index)
            if isinstance(blk, ConstBlock):
                blocks.append(ConstBlock(blk.block, torch.tensor(bs)))
            else:
                blocks.append(DenseBlock(blk.view().squeeze(index)))
        return SparseTensor(starts, blocks, self.dims - 1, torch.tensor(shape), ends, self.type, self.dense_const)

    def repeat(self, repeat_dims, *args, **kwargs):
        """Broadcast along size-1 dims (reference: sparse_tensor.py:2273, RepeatBlock)."""
        rd = _ints(repeat_dims)
        shape = self.shape
        for d, r in enumerate(rd):
            if r != 1 and shape[d] != 1:
                raise NotImplementedError("repeat of a dim larger than 1")
        new_shape = [a * r for a, r in zip(shape, rd)]
        starts, ends, blocks = [], [], []
        for (s, e), blk in zip(self._boxes(), self.blocks):
            starts.append(torch.tensor([a * r for a, r in zip(s, rd)]))
            ends.append(torch.tensor([b * r for b, r in zip(e, rd)]))
            bs = [a * r for a, r in zip(blk.shape, rd)]
            if isinstance(blk, ConstBlock):
                blocks.append(ConstBlock(blk.block, torch.tensor(bs)))
            else:
                blocks.append(DenseBlock(blk.view().expand(*bs)))
        return SparseTensor(starts, blocks, self.dims, torch.tensor(new_shape), ends, self.type, self.dense_const)

    # ------------------------------------------------------------------ matmul
    def matmul(self, y, *args, **kwargs):
        """x [B, R, K] @ y [B, K, N] -> [B, R, N]; x [B, R, K] @ y [B, K] -> [B, R]
        (reference: SparseTensor.matmul sparse_tensor.py:1671-2060)."""
        if not isinstance(y, SparseTensor):
            y = convert_dense_to_sparse(y)
        xs, ys = self.shape, y.shape
        if self.dims != 3 or y.dims not in (2, 3):
            raise NotImplementedError(f"matmul of {self.dims}-d by {y.dims}-d tensors")
        unequal = y.dims == 2
        B, R, K = xs
        N = 1 if unequal else ys[2]
        if ys[0] != B or ys[1] != K:
            raise Exception("SHAPE MISMATCH")
        if any(b.block_type in ("K", "P") for b in self.blocks + y.blocks):
            res = self._matmul_blocks(y, unequal)
            if res is not None:
                return res
        # grid dims: (batch, R, K, N); x covers (0,1,2), y covers (0,2,3) (unequal: (0,2))
        x_map = [0, 1, 2, None]
        y_map = [0, None, 1, None] if unequal else [0, None, 1, 2]
        bps = [self._bp_union(B, [(self, 0), (y, 0)]), self._bp_union(R, [(self, 1)]),
               self._bp_union(K, [(self, 2), (y, 1)]),
               [0, 1] if unequal else self._bp_union(N, [(y, 2)])]
        xc = self._cover(self, bps, x_map)
        yc = self._cover(y, bps, y_map)
        starts, blocks = [], []
        for ib, ir, iN in itertools.product(range(len(bps[0]) - 1), range(len(bps[1]) - 1), range(len(bps[3]) - 1)):
            lo = [bps[0][ib], bps[1][ir], bps[3][iN]]
            hi = [bps[0][ib + 1], bps[1][ir + 1], bps[3][iN + 1]]
            out = None
            for ik in range(len(bps[2]) - 1):
                k0, k1 = bps[2][ik], bps[2][ik + 1]
                bx = xc.get((ib, ir, ik, iN))
                by = yc.get((ib, ir, ik, iN))
                cx = self._cell_const(bx)
                cy = y._cell_const(by)
                if (cx[0] and cx[1] == 0) or (cy[0] and cy[1] == 0):
                    continue
                xv = self._cell_view(bx, [lo[0], lo[1], k0], [hi[0], hi[1], k1])
                if unequal:
                    yv = y._cell_view(by, [lo[0], k0], [hi[0], k1]).unsqueeze(2)
                else:
                    yv = y._cell_view(by, [lo[0], k0, lo[2]], [hi[0], k1, hi[2]])
                if xv.dtype != torch.float32:
                    xv = xv.float()
                if yv.dtype != torch.float32:
                    yv = yv.float()
                out = _dev.bmm(xv, yv, out, accumulate=out is not None)
            if out is None:
                continue
            if unequal:
                starts.append(torch.tensor(lo[:2]))
                blocks.append(DenseBlock(out[:, :, 0]))
            else:
                starts.append(torch.tensor(lo))
                blocks.append(DenseBlock(out))
        total = [B, R] if unequal else [B, R, N]
        return SparseTensor(starts, blocks, len(total), torch.tensor(total), type=float, dense_const=0.0)

    def _matmul_blocks(self, y, unequal):
        """The reference's block-pair product (sparse_tensor.py:1780-2050) where every pair of
        blocks that meets does so over the same range of the contracted dim and the products
        land in disjoint boxes: each pair is one block-level product (so a conv block stays a
        KernelBlock / PatchesBlock where the reference keeps it so).  None otherwise: the
        grid refinement then computes the same values on dense cell views."""
        starts, ends, blocks = [], [], []
        xb, yb = self._boxes(), y._boxes()
        for (sx_, ex_), bx in zip(xb, self.blocks):
            for (sy_, ey_), by in zip(yb, y.blocks):
                if max(sx_[0], sy_[0]) >= min(ex_[0], ey_[0]):
                    continue
                ky = (sy_[1], ey_[1])
                if max(sx_[2], ky[0]) >= min(ex_[2], ky[1]):
                    continue
                if (sx_[2], ex_[2]) != ky:
                    return None
                if unequal:
                    blk = bx.matmul_unequal_dims(by)[0]
                    st = [min(sx_[0], sy_[0]), sx_[1]]
                    en = [max(ex_[0], ey_[0]), ex_[1]]
                else:
                    blk = bx.matmul_equal_dims(by)[0]
                    st = [min(sx_[0], sy_[0]), sx_[1], sy_[2]]
                    en = [max(ex_[0], ey_[0]), ex_[1], ey_[2]]
                for s0, e0 in zip(starts, ends):
                    if all(max(a, c) < min(b, d) for a, b, c, d in zip(st, en, s0, e0)):
                        return None
                if isinstance(blk, ConstBlock) and blk.block == 0:
                    continue
                starts.append(st)
                ends.append(en)
                blocks.append(blk)
        total = self.shape[:2] if unequal else self.shape[:2] + [y.shape[2]]
        return SparseTensor(starts, blocks, len(total), torch.tensor(total), ends, type=float, dense_const=0.0)

    def get_sparse_custom_range(self, start_index, end_index, *args, **kwargs):
        """The blocks inside the box [start, end), at their own positions in a tensor of the
        same total size and fill (reference: sparse_tensor.py:873-960): blocks outside the box
        are left out, a block that straddles its border raises NotImplementedError, as there."""
        st, en = _ints(start_index), _ints(end_index)
        starts, ends, blocks = [], [], []
        for (s, e), blk in zip(self._boxes(), self.blocks):
            inside = all(a >= c and b <= d for a, b, c, d in zip(s, e, st, en))
            meets = all(max(a, c) < min(b, d) for a, b, c, d in zip(s, e, st, en))
            if inside:
                starts.append(s)
                ends.append(e)
                blocks.append(blk)
            elif meets:
                raise NotImplementedError("get_sparse_custom_range: a block straddles the range")
        return SparseTensor(starts, blocks, self.dims, self.total_size, ends, self.type, self.dense_const)

    def _bp_union(self, n, pairs):
        pts = {0, n}
        for t, d in pairs:
            for s, e in t._boxes():
                pts.add(max(0, min(n, s[d])))
                pts.add(max(0, min(n, e[d])))
        return sorted(pts)

    # ------------------------------------------------------------------ misc
    def __repr__(self):
        return (f"SparseTensor(total_size={self.shape}, type={self.type.__name__}, dense_const={self.dense_const}, "
                f"blocks={[b.block_type for b in self.blocks]})")


def convert_dense_to_sparse(x, total_size=None, *args, **kwargs):
    """A dense tensor as a one-block SparseTensor (reference: sparse_tensor.py:92)."""
    if isinstance(x, (bool, int, float)):
        typ = bool if isinstance(x, bool) else float
        return SparseTensor([], [], len(_ints(total_size)), total_size, type=typ, dense_const=x)
    t = torch.as_tensor(x)
    typ = bool if t.dtype == torch.bool else float
    return SparseTensor([torch.zeros(t.dim(), dtype=torch.int64)], [DenseBlock(t)], t.dim(),
                        torch.tensor(list(t.shape)), type=typ, dense_const=False if typ is bool else 0.0)


def sp_where(x, y, z, *args, **kwargs):
    """x ? y : z on block-sparse operands (reference: sparse_tensor.py:2447)."""
    dc = y.dense_const if x.dense_const else z.dense_const

    def fn(c, a, b):
        if c.dtype != torch.bool:
            c = _dev.binary(operator.ne, c.float(), _dev.scalar_view(0.0, list(c.shape), torch.float32), torch.bool)
        return _dev.where(c, a.float() if a.dtype != torch.float32 else a, b.float() if b.dtype != torch.float32 else b)
    return x._elementwise([y, z], fn, float, float(dc))


def sparse_max(x, y, *args, **kwargs):
    return x._elementwise([y], lambda a, b: _dev.where(_dev.binary(operator.ge, a, b, torch.bool), a, b), float,
                          float(max(x.dense_const, y.dense_const)))


def sparse_min(x, y, *args, **kwargs):
    return x._elementwise([y], lambda a, b: _dev.where(_dev.binary(operator.le, a, b, torch.bool), a, b), float,
                          float(min(x.dense_const, y.dense_const)))
