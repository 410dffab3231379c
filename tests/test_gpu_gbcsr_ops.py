"""Operator-level parity of the gbcsr mirror (constraintflow.gbcsr, on the GPU) with the
reference's own tensor_ops on seeded block-sparse inputs (tests/golden/gbcsr_ops.pkl,
made by tests/golden/gen_gbcsr_ops.py).  Elementwise ops must match bit for bit;
contractions within float32 reordering tolerance."""
import operator
import os
import pickle

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

CASES = pickle.load(open(os.path.join(os.path.dirname(__file__), "golden", "gbcsr_ops.pkl"), "rb"))


def _build(desc):
    from constraintflow.gbcsr.sparse_tensor import SparseTensor
    from constraintflow.gbcsr.sparse_block import DenseBlock, ConstBlock, DiagonalBlock, RepeatBlock
    starts, blocks = [], []
    for b in desc["blocks"]:
        starts.append(torch.tensor(b["start"]))
        if b["kind"] == "D":
            blocks.append(DenseBlock(torch.from_numpy(np.array(b["data"]))))
        elif b["kind"] == "C":
            blocks.append(ConstBlock(b["value"], torch.tensor(b["shape"])))
        elif b["kind"] == "Diag":
            blocks.append(DiagonalBlock(torch.from_numpy(b["data"]), torch.tensor(b["shape"]), b["diag_index"]))
        elif b["kind"] == "R":
            blocks.append(RepeatBlock(torch.from_numpy(b["data"]), torch.tensor(b["shape"])))
    typ = bool if desc["type"] == "bool" else float
    return SparseTensor(starts, blocks, len(desc["total"]), torch.tensor(desc["total"]), type=typ,
                        dense_const=desc["dc"])


def _run(case):
    from constraintflow.gbcsr import tensor_ops as T
    a = case["args"]
    op = case["op"]
    if op == "binary":
        return T.binary(_build(a["x"]), _build(a["y"]), getattr(operator, a["op"]))
    if op == "binary_scalar_r":
        return T.binary(_build(a["x"]), a["y"], getattr(operator, a["op"]))
    if op == "binary_scalar_l":
        return T.binary(a["x"], _build(a["y"]), getattr(operator, a["op"]))
    if op == "unary":
        return T.unary(_build(a["x"]), getattr(operator, a["op"]))
    if op == "clamp":
        return T.clamp(_build(a["x"]), a["const"], a["min_true"])
    if op == "where":
        return T.where(_build(a["c"]), _build(a["y"]), _build(a["z"]))
    if op == "any":
        return T.any(_build(a["x"]))
    if op == "inner_prod":
        return T.inner_prod(_build(a["x"]), _build(a["y"]))
    if op == "unsqueeze":
        return _build(a["x"]).unsqueeze(a["index"])
    if op == "squeeze":
        return _build(a["x"]).squeeze(a["index"])
    if op == "repeat":
        return T.repeat(_build(a["x"]), torch.tensor(a["dims"]))
    if op == "custom_range":
        return _build(a["x"]).get_sparse_custom_range(torch.tensor(a["start"]), torch.tensor(a["end"]))
    if op == "convert_to_float":
        return T.convert_to_float(_build(a["x"]))
    raise ValueError(op)


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_gbcsr_op_matches_reference(case):
    from constraintflow.gbcsr.sparse_tensor import SparseTensor
    want = case["result"]
    if want["kind"] == "error":
        with pytest.raises(ZeroDivisionError):
            _run(case)
        return
    got = _run(case)
    if want["kind"] == "scalar":
        assert got == want["value"]
        return
    assert isinstance(got, SparseTensor)
    assert got.type.__name__ == want["type"]
    assert got.shape == list(want["total"])
    d = got.get_dense().numpy()
    # where the reference's own result contradicts the elementwise meaning of the op on its
    # dense inputs (its block union mishandles some partially overlapping boxes), the
    # elementwise result is the expectation
    ref = case["semantic"] if case.get("reference_inconsistent") else want["dense"]
    assert d.dtype == ref.dtype
    if case["op"] == "inner_prod":
        np.testing.assert_allclose(d, ref, rtol=1e-5, atol=1e-5 * (np.abs(ref).max() + 1))
    else:
        np.testing.assert_array_equal(d, ref)
    if not got.check_dense():  # the fill value is observable only where no block lies
        if want["type"] == "bool":
            assert bool(got.dense_const) == bool(want["dc"])
        else:
            assert (got.dense_const == want["dc"]) or (np.isnan(got.dense_const) and np.isnan(want["dc"]))
