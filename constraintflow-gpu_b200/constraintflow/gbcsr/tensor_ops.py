"""The gbcsr free functions that ConstraintFlow's generated code calls, on the GPU.

Same names, arguments and error behaviour as the reference's
constraintflow/gbcsr/tensor_ops.py (type checks raise Exception('TYPE MISMATCH'), shape
checks Exception('SHAPE MISMATCH')); the JIT keyword arguments (layer_index, counter,
inside_while, while_number, while_iteration) are accepted and ignored.  Dispatch: a
SparseTensor operand goes to the block-sparse implementation (sparse_tensor.py, all
arithmetic in libcfgpu); plain Python / torch operands are combined as the reference
does.
"""
import operator

import torch

from .sparse_block import ConstBlock
from .sparse_tensor import SparseTensor, convert_dense_to_sparse, sp_where, sparse_max, sparse_min

_NUM = (float, int, torch.float, torch.int)


def _type_eq(x, y):
    if x == y:
        return True
    return x in _NUM and y in _NUM


_TYPES = {bool: torch.bool, int: torch.int, float: torch.float}


def checkTypes(x, y):
    """tensor_ops.py:18-50."""
    if isinstance(x, SparseTensor):
        if isinstance(y, SparseTensor) and not _type_eq(x.type, y.type):
            raise Exception("TYPE MISMATCH")
        if isinstance(y, (float, int, bool)) and not _type_eq(x.type, type(y)):
            raise Exception("TYPE MISMATCH")
        if isinstance(y, torch.Tensor) and not _type_eq(_TYPES[x.type], y.dtype):
            raise Exception("TYPE MISMATCH")
    elif isinstance(y, SparseTensor):
        if isinstance(x, (float, int, bool)) and not _type_eq(y.type, type(x)):
            raise Exception("TYPE MISMATCH")
    elif not isinstance(x, torch.Tensor) and not isinstance(y, torch.Tensor) and not _type_eq(type(x), type(y)):
        raise Exception("TYPE MISMATCH")


def checkShapes(x, y):
    """tensor_ops.py:52-77."""
    if isinstance(x, SparseTensor):
        if isinstance(y, torch.Tensor) and list(x.shape) != list(y.shape):
            raise Exception("SHAPE MISMATCH")
        if isinstance(y, SparseTensor) and x.shape != y.shape:
            raise Exception("SHAPE MISMATCH")
    elif isinstance(y, SparseTensor):
        if isinstance(x, torch.Tensor) and list(x.shape) != y.shape:
            raise Exception("SHAPE MISMATCH")
    elif isinstance(x, torch.Tensor) and isinstance(y, torch.Tensor) and x.shape != y.shape:
        raise Exception("SHAPE MISMATCH")


def sanityCheck(x, y):
    checkTypes(x, y)
    checkShapes(x, y)


def unary(x, op, layer_index=None, counter=None, inside_while=False, while_number=None, while_iteration=None):
    if isinstance(x, SparseTensor):
        return x.unary(op)
    return op(x)


def any(x, layer_index=None, counter=None, inside_while=False, while_number=None, while_iteration=None):
    if type(x) != torch.Tensor and type(x) != SparseTensor:
        raise Exception("TYPE MISMATCH")
    return x.any()


def all(x, layer_index=None, counter=None, inside_while=False, while_number=None, while_iteration=None):
    if type(x) != torch.Tensor:
        raise Exception("TYPE MISMATCH")
    return x.all()


def binary(x, y, op, layer_index=None, counter=None, inside_while=False, while_number=None, while_iteration=None,
           parent_json_list=None):
    sanityCheck(x, y)
    if isinstance(x, SparseTensor):
        return x.binary(y, op)
    if isinstance(y, SparseTensor):
        return convert_dense_to_sparse(x, y.total_size).binary(y, op)
    return op(x, y)


def cf_max(x, y, layer_index=None, counter=None, inside_while=False, while_number=None, while_iteration=None):
    sanityCheck(x, y)
    if isinstance(x, SparseTensor) and isinstance(y, SparseTensor):
        return sparse_max(x, y)
    return torch.max(x, y)


def cf_min(x, y, layer_index=None, counter=None, inside_while=False, while_number=None, while_iteration=None):
    sanityCheck(x, y)
    if isinstance(x, SparseTensor) and isinstance(y, SparseTensor):
        return sparse_min(x, y)
    return torch.min(x, y)


def _size(v):
    if isinstance(v, SparseTensor):
        return v.shape
    if isinstance(v, torch.Tensor):
        return list(v.shape)
    return None


def where(x, y, z, layer_index=None, counter=None, inside_while=False, while_number=None, while_iteration=None):
    """x ? y : z (tensor_ops.py:278-368)."""
    if isinstance(x, torch.Tensor) and isinstance(y, torch.Tensor) and isinstance(z, torch.Tensor):
        checkShapes(x, y)
        sanityCheck(y, z)
        return torch.where(x, y, z)
    if isinstance(x, bool) and isinstance(y, float) and isinstance(z, float):
        return y if x else z
    total = next((s for s in (_size(x), _size(y), _size(z)) if s is not None), None)

    def sp(v, typ):
        if isinstance(v, SparseTensor):
            return v
        if isinstance(v, torch.Tensor):
            return convert_dense_to_sparse(v)
        return SparseTensor([], [], len(total), torch.tensor(total), type=typ, dense_const=v)
    x1, y1, z1 = sp(x, bool), sp(y, float), sp(z, float)
    checkShapes(x1, y1)
    sanityCheck(y1, z1)
    return sp_where(x1, y1, z1)


def inner_prod(x, y, layer_index=None, counter=None, inside_while=False, while_number=None, while_iteration=None):
    """Batched contraction over the last dim of x (tensor_ops.py:370-481)."""
    checkTypes(x, y)
    xs, ys = _size(x), _size(y)
    if len(xs) == len(ys):
        if xs[-1] != ys[-2] or xs[:-2] != ys[:-2]:
            raise Exception("SHAPE MISMATCH")
    elif len(xs) > len(ys):
        if xs[-1] != ys[-1] or xs[:-2] != ys[:-1]:
            raise Exception("SHAPE MISMATCH")
    else:
        raise Exception("SHAPE MISMATCH")
    if isinstance(x, SparseTensor) or isinstance(y, SparseTensor):
        xx = x if isinstance(x, SparseTensor) else convert_dense_to_sparse(x)
        return xx.matmul(y)
    return x @ y


def convert_to_float(x):
    if isinstance(x, (torch.Tensor, SparseTensor)):
        return x.float()
    return x


def get_default_stop(shape, abs_elem, batch_size, curr_size, poly_size, layer_index=None, counter=None,
                     inside_while=False, while_number=None, while_iteration=None):
    """Stop mask over [B, curr, poly]: False on every live layer's columns, True elsewhere
    (tensor_ops.py:497-546)."""
    starts, ends, blocks = [], [], []
    live = [bool(v) for v in abs_elem.d["llist"]]
    for i, layer in enumerate(abs_elem.network):
        if i < len(live) and live[i]:
            starts.append(torch.tensor([0, 0, layer.start]))
            ends.append(torch.tensor([batch_size, curr_size, layer.end]))
            blocks.append(ConstBlock(False, torch.tensor([batch_size, curr_size, layer.size])))
    return SparseTensor(starts, blocks, len(shape), torch.tensor(shape), ends, type=bool, dense_const=True)


def get_max_priority(sp_tensor, active_vertices, layer_index=None, counter=None, inside_while=False,
                     while_number=None, while_iteration=None):
    """True on the blocks of the highest-priority layer that still has active vertices
    (tensor_ops.py:557-614)."""
    pri = []
    for i in range(sp_tensor.num_blocks):
        assert isinstance(sp_tensor.blocks[i], ConstBlock)
        if active_vertices.exists_sub_block(sp_tensor.start_indices[i], sp_tensor.end_indices[i]):
            pri.append(sp_tensor.blocks[i].block)
        else:
            pri.append(float("-inf"))
    best = max(pri) if pri else float("-inf")
    starts, ends, blocks = [], [], []
    for i in range(sp_tensor.num_blocks):
        if pri[i] == best:
            blocks.append(ConstBlock(True, sp_tensor.blocks[i].total_shape))
            starts.append(sp_tensor.start_indices[i])
            ends.append(sp_tensor.end_indices[i])
    return SparseTensor(starts, blocks, sp_tensor.dims, sp_tensor.total_size, ends, type=bool, dense_const=False)


def filter_trav_exp_stop(trav_exp, stop, layer_index=None, counter=None, inside_while=False, while_number=None,
                         while_iteration=None):
    """The part of the expression whose vertices stop (tensor_ops.py:616-640)."""
    mat = binary(trav_exp.mat, convert_to_float(stop), operator.mul)
    return trav_exp.create_similar(mat=mat)


def filter_trav_exp_not_stop(trav_exp, stop, layer_index=None, counter=None, inside_while=False, while_number=None,
                             while_iteration=None):
    """The part that is substituted, with a zero constant (tensor_ops.py:642-687)."""
    if isinstance(trav_exp.const, SparseTensor):
        const = SparseTensor([], [], trav_exp.const.dims, trav_exp.const.total_size, type=float, dense_const=0)
    else:
        const = 0
    mat = binary(trav_exp.mat, convert_to_float(stop.unary(operator.not_)), operator.mul)
    return trav_exp.create_similar(mat=mat, const=const)


def get_dims(x, layer_index=None, counter=None, inside_while=False, while_number=None, while_iteration=None):
    if isinstance(x, SparseTensor):
        return x.dims
    if isinstance(x, torch.Tensor):
        return x.dim()
    raise AssertionError(f"get_dims type of x: {type(x)}")


def get_shape_1(x):
    if isinstance(x, SparseTensor):
        return x.total_size[1]
    if not isinstance(x, torch.Tensor):
        raise Exception("TYPE MISMATCH")
    return x.shape[1]


def repeat(mat, repeat_dims, layer_index=None, counter=None, inside_while=False, while_number=None,
           while_iteration=None):
    if isinstance(mat, float):
        return mat * torch.ones(*(torch.as_tensor(repeat_dims).tolist()))
    if isinstance(mat, torch.Tensor):
        return mat.repeat(*(torch.as_tensor(repeat_dims).tolist()))
    return mat.repeat(repeat_dims)


def clamp(mat, const, min_true, layer_index=None, counter=None, inside_while=False, while_number=None,
          while_iteration=None):
    """Sign split: clamp(min=const) if min_true else clamp(max=const) (tensor_ops.py:765-836)."""
    if isinstance(mat, float):
        if min_true:
            return mat if mat > const else const
        return mat if mat < const else const
    if isinstance(mat, torch.Tensor):
        return mat.clamp(min=const) if min_true else mat.clamp(max=const)
    return mat.clamp(const, min_true)
