"""The drop-in package imports on a machine without a GPU and its host-side logic
(structure, shape/type checks) works without launching anything."""
import operator

import pytest
import torch


def test_modules_import_with_reference_names():
    from constraintflow.gbcsr import tensor_ops as T
    from constraintflow.gbcsr.sparse_tensor import SparseTensor, convert_dense_to_sparse, sp_where
    from constraintflow.gbcsr.sparse_block import (DenseBlock, ConstBlock, DiagonalBlock, RepeatBlock, KernelBlock,
                                                   PatchesBlock)
    for name in ("unary", "any", "binary", "where", "inner_prod", "clamp", "repeat", "convert_to_float",
                 "get_default_stop", "get_max_priority", "filter_trav_exp_stop", "filter_trav_exp_not_stop",
                 "get_dims", "cf_max", "cf_min"):
        assert callable(getattr(T, name))


def test_structure_without_device():
    from constraintflow.gbcsr.sparse_tensor import SparseTensor
    from constraintflow.gbcsr import tensor_ops as T
    x = SparseTensor([], [], 3, torch.tensor([2, 3, 4]), dense_const=0.0)
    assert x.shape == [2, 3, 4] and not x.check_dense()
    assert T.get_dims(x) == 3
    with pytest.raises(Exception, match="TYPE MISMATCH"):
        T.binary(x, True, operator.and_)
    y = SparseTensor([], [], 3, torch.tensor([2, 3, 5]), dense_const=0.0)
    with pytest.raises(Exception, match="SHAPE MISMATCH"):
        T.binary(x, y, operator.add)
    with pytest.raises(Exception, match="SHAPE MISMATCH"):
        T.inner_prod(x, y)
    assert T.binary(2, 1, operator.sub) == 1
    assert T.clamp(-1.5, 0, True) == 0 and T.clamp(-1.5, 0, False) == -1.5
