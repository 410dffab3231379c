"""gbcsr conv blocks (KernelBlock, PatchesBlock) on the GPU against the reference's own block
algebra (tests/golden/gbcsr_conv_blocks.pkl, made by tests/golden/gen_conv_blocks.py from
constraintflow/gbcsr/sparse_block.py and sparse_tensor.py).

Every case rebuilds the reference's operands in the mirror (constraintflow.gbcsr, computing
through libcfgpu's cf_conv_* and block kernels) and checks the kind of the result block,
its conv geometry, its payload and its dense matrix.  The reference's
PatchesBlock.get_dense advances one output row by the padded input HEIGHT times the stride
(sparse_block.py:3162), so on a non-square image it misplaces the patch rows; the mirror
places them by the padded width (the conv's own matrix, as KernelBlock.get_dense gives it),
and those cases, flagged by the generator, are checked against the conv matrix instead.
Densification, the conversion to patches and the diagonal products are single products or
copies: bit-exact.  Products that sum (conv2d / conv_transpose2d / unfold-and-sum in the
reference) agree within 1e-5 of the result's scale.
"""
import operator
import os
import pickle

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
CASES = pickle.load(open(os.path.join(HERE, "golden", "gbcsr_conv_blocks.pkl"), "rb"))
EXACT = {"kernel_get_dense", "kernel_to_patches", "kernel_at_diag", "diag_at_kernel", "tensor_kernel_dense",
         "patches_at_diag", "kernel_at_zero", "patches_add_patches", "patches_mul_const", "kernel_mul_const"}


def _t(a):
    return torch.from_numpy(np.ascontiguousarray(a))


def _run(case):
    from constraintflow.gbcsr.sparse_block import ConstBlock, DenseBlock, DiagonalBlock, KernelBlock
    from constraintflow.gbcsr.sparse_tensor import SparseTensor
    a = case["args"]
    g = a["g"]
    B, rows, cols = g["B"], g["K"] * g["ox"] * g["oy"], g["C"] * g["ix"] * g["iy"]

    def kb():
        return KernelBlock(_t(a["W"]), torch.tensor([B, rows, cols]), g["ix"], g["iy"], g["ox"], g["oy"], g["sx"],
                           g["sy"], g["px"], g["py"])

    def diag(d, n):
        return DiagonalBlock(_t(d), torch.tensor([B, n, n]), 2)

    def pb(d=None):
        return kb().matmul_equal_dims(diag(a["d"] if d is None else d, cols))[0]

    def kb2():
        g2 = a["g2"]
        return KernelBlock(_t(a["W2"]), torch.tensor([B, cols, g2["C"] * g2["ix"] * g2["iy"]]), g2["ix"], g2["iy"],
                           g2["ox"], g2["oy"], g2["sx"], g2["sy"], g2["px"], g2["py"])

    op = case["op"]
    if op == "kernel_get_dense":
        return kb().get_dense()
    if op == "kernel_to_patches":
        return kb().convert_to_patches()
    if op == "kernel_at_diag":
        return kb().matmul_equal_dims(diag(a["d"], cols))
    if op == "kernel_at_dense":
        return kb().matmul_equal_dims(DenseBlock(_t(a["X"])))
    if op == "kernel_at_vec":
        return kb().matmul_unequal_dims(DenseBlock(_t(a["v"])))
    if op == "kernel_at_zero":
        return kb().matmul_equal_dims(ConstBlock(0, torch.tensor([B, cols, a["S"]])))
    if op == "dense_at_kernel":
        return DenseBlock(_t(a["Y"])).matmul_equal_dims(kb())
    if op == "diag_at_kernel":
        return diag(a["e"], rows).matmul_equal_dims(kb())
    if op == "tensor_kernel_dense":
        return SparseTensor([torch.tensor([0, 0, 0])], [kb()], 3, torch.tensor([B, rows, cols]))
    if op == "tensor_kernel_matmul":
        X = a["X"]
        y = SparseTensor([torch.tensor([0, 0, 0])], [DenseBlock(_t(X))], 3, torch.tensor(list(X.shape)))
        return SparseTensor([torch.tensor([0, 0, 0])], [kb()], 3, torch.tensor([B, rows, cols])).matmul(y)
    if op == "patches_at_vec":
        return pb().matmul_unequal_dims(DenseBlock(_t(a["v"])))
    if op == "patches_at_diag":
        return pb().matmul_equal_dims(diag(a["d2"], cols))
    if op == "patches_sum":
        return pb().sum(2)
    if op == "dense_at_patches":
        return DenseBlock(_t(a["Y"])).matmul_equal_dims(pb())
    if op == "kernel_at_patches":
        g3 = a["g3"]
        k3 = KernelBlock(_t(a["W3"]), torch.tensor([B, g3["K"] * g3["ox"] * g3["oy"], rows]), g3["ix"], g3["iy"],
                         g3["ox"], g3["oy"], g3["sx"], g3["sy"], g3["px"], g3["py"])
        return k3.matmul_equal_dims(pb())
    if op == "patches_at_kernel":
        return pb().matmul_equal_dims(kb2())
    if op == "kernel_patches_at_kernel":
        return kb().convert_to_patches().matmul_equal_dims(kb2())
    if op == "patches_add_patches":
        return pb().binary(pb(a["d2"]), operator.add)
    if op == "patches_mul_const":
        return pb().binary(ConstBlock(a["c"], torch.tensor([B, rows, cols])), operator.mul)
    if op == "kernel_mul_const":
        return kb().binary(ConstBlock(a["c"], torch.tensor([B, rows, cols])), operator.mul)
    raise AssertionError(op)


def _close(mine, ref, exact, what):
    mine = np.asarray(mine, dtype=np.float32)
    ref = np.asarray(ref, dtype=np.float32)
    assert mine.shape == ref.shape, (what, mine.shape, ref.shape)
    if exact:
        assert np.array_equal(mine, ref), (what, float(np.abs(mine - ref).max()))
    else:
        scale = max(float(np.abs(ref).max()), 1e-30)
        err = float(np.abs(mine - ref).max())
        assert err <= 1e-5 * scale, (what, err, scale)


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_conv_block_op_matches_reference(case):
    from constraintflow.gbcsr.sparse_block import ConstBlock, KernelBlock, PatchesBlock
    from constraintflow.gbcsr.sparse_tensor import SparseTensor
    ref = dict(case["result"])
    ref.update(case.get("semantic", {}))
    exact = case["op"] in EXACT
    res = _run(case)
    if isinstance(res, tuple):
        res = res[0]
    if ref["kind"] == "sparse":
        assert isinstance(res, SparseTensor)
        _close(res.get_dense().float().numpy(), ref["dense"], exact, "dense")
        return
    if ref["kind"] == "tensor":
        _close(res.cpu().numpy(), ref["dense"], exact, "dense")
        return
    assert type(res).__name__ == ref["kind"], (type(res).__name__, ref["kind"])
    assert [int(v) for v in res.total_shape] == ref["total"]
    if isinstance(res, ConstBlock):
        assert float(res.block) == ref["value"]
        return
    if isinstance(res, (KernelBlock, PatchesBlock)):
        assert [int(v) for v in res.parameters()] == ref["params"]
    _close(res.block.cpu().numpy(), ref["payload"], exact, "payload")
    if "dense" in ref:
        _close(res.get_dense().cpu().numpy(), ref["dense"], exact, "dense")


def test_conv_block_cases_present():
    ops = {c["op"] for c in CASES}
    assert len(CASES) >= 90 and len(ops) == 20


def test_reference_inconsistent_cases_are_non_square_patches():
    """The reference's patch placement differs from the conv matrix only where a PatchesBlock
    of a non-square image is densified; on every square case the generator found them equal."""
    bad = [c for c in CASES if c.get("reference_inconsistent")]
    assert bad and all(c["args"]["g"]["ix"] != c["args"]["g"]["iy"] for c in bad)
    square_patch_cases = [c for c in CASES if c["args"]["g"]["ix"] == c["args"]["g"]["iy"] and
                          c["result"].get("kind") == "PatchesBlock"]
    assert square_patch_cases and not any(c.get("reference_inconsistent") for c in square_patch_cases)
