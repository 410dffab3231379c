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


def test_generated_programs_are_recognised():
    """The reference compiler's own output for deeppoly.cf, deeppoly_efficient.cf and
    crown.cf (tests/golden/generated/) is recognised by the drop-in Flow without a GPU."""
    import importlib.util
    import os
    import sys
    from constraintflow.lib.flow_sparse import certifier_of
    here = os.path.dirname(os.path.abspath(__file__))
    for program, expect in (("deeppoly", "deeppoly"), ("deeppoly_efficient", "deeppoly"), ("crown", "crown")):
        path = os.path.join(here, "golden", "generated", program, "transformers.py")
        saved = sys.modules.pop("transformers", None)
        try:
            spec = importlib.util.spec_from_file_location("transformers", path)
            mod = importlib.util.module_from_spec(spec)
            sys.modules["transformers"] = mod
            spec.loader.exec_module(mod)
            assert certifier_of(mod.deeppoly()) == expect
        finally:
            sys.modules.pop("transformers", None)
            if saved is not None:
                sys.modules["transformers"] = saved
