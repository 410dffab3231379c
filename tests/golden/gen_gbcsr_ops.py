"""Generate operator-level golden vectors for the gbcsr tensor ops by running the
REFERENCE's own constraintflow/gbcsr/tensor_ops.py on seeded block-sparse inputs.

Test infrastructure; runs only where the reference checkout is present (REF_ROOT).
    python tests/golden/gen_gbcsr_ops.py      -> tests/golden/gbcsr_ops.pkl

Each case records its inputs as plain data (total size, type, fill value and a list of
blocks: start index, kind D / C / Diag / R and the block payload), the operation and
its arguments, and the reference's result as a dense array (SparseTensor.get_dense),
plus the result's type and fill value.  The mirror under test rebuilds the same inputs
from this description.
"""
import operator
import os
import pickle
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF_ROOT = os.environ.get("CF_REFERENCE_ROOT", "")

BIN_OPS = ["add", "sub", "mul", "truediv", "ge", "gt", "le", "lt", "eq", "ne"]
BOOL_OPS = ["and_", "or_"]


def main():
    if not REF_ROOT or not os.path.isdir(os.path.join(REF_ROOT, "constraintflow")):
        sys.exit("set CF_REFERENCE_ROOT to the reference checkout (the directory holding constraintflow/)")
    sys.argv = ["x"]
    sys.path.insert(0, os.path.join(HERE, "refshim", "stubs"))
    sys.path.insert(0, REF_ROOT)
    import torch
    from constraintflow.gbcsr import tensor_ops as T
    from constraintflow.gbcsr.sparse_tensor import SparseTensor
    from constraintflow.gbcsr.sparse_block import DenseBlock, ConstBlock, DiagonalBlock, RepeatBlock

    rng = np.random.default_rng(2024)

    def rand_layout(total, typ, dc, kinds=("D", "C", "E"), split_rows=False):
        """Disjoint boxes: the last dim cut into segments, each a block kind or empty (E)."""
        total = list(total)
        n = total[-1]
        cuts = sorted(set([0, n] + list(rng.choice(np.arange(1, n), size=min(3, n - 1), replace=False))))
        blocks = []
        for a, b in zip(cuts[:-1], cuts[1:]):
            kind = kinds[rng.integers(len(kinds))]
            if kind == "E":
                continue
            if split_rows and len(total) >= 2 and total[-2] > 1 and rng.random() < 0.5:
                rcut = int(rng.integers(1, total[-2]))
                row_ranges = [(0, rcut), (rcut, total[-2])]
            else:
                row_ranges = [(0, total[-2])] if len(total) >= 2 else [None]
            for rr in row_ranges:
                shape = list(total)
                start = [0] * len(total)
                shape[-1] = b - a
                start[-1] = a
                if rr is not None:
                    shape[-2] = rr[1] - rr[0]
                    start[-2] = rr[0]
                if kind == "D":
                    if typ == "bool":
                        data = rng.random(shape) < 0.5
                    else:
                        data = rng.standard_normal(shape).astype(np.float32)
                        data[rng.random(shape) < 0.2] = 0.0
                    blocks.append(dict(kind="D", start=start, data=data))
                else:
                    if typ == "bool":
                        val = bool(rng.random() < 0.5)
                    else:
                        val = float(rng.choice([0.0, 1.0, -2.5, 0.75]))
                    blocks.append(dict(kind="C", start=start, value=val, shape=shape))
        return dict(total=total, type=typ, dc=dc, blocks=blocks)

    def build(desc):
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

    def dense(x):
        if isinstance(x, str):
            return dict(kind="error", error=x)
        if isinstance(x, SparseTensor):
            d = x.get_dense()
            return dict(kind="sparse", dense=d.numpy(), type=x.type.__name__, dc=x.dense_const,
                        total=x.total_size.tolist())
        if isinstance(x, torch.Tensor):
            return dict(kind="tensor", dense=x.numpy())
        return dict(kind="scalar", value=x)

    cases = []

    def add(name, op, args, res):
        case = dict(name=name, op=op, args=args, result=dense(res))
        # Boolean ops and where are exact: check the reference against its own elementwise
        # meaning on the dense inputs.  Where they disagree (partially overlapping boxes that
        # the reference's block union mishandles) the case records the elementwise result too.
        sem = None
        if op == "binary" and args["op"] in ("and_", "or_"):
            sem = getattr(np, "logical_" + args["op"][:-1])(build(args["x"]).get_dense().numpy(),
                                                            build(args["y"]).get_dense().numpy())
        elif op == "where":
            sem = np.where(build(args["c"]).get_dense().numpy(), build(args["y"]).get_dense().numpy(),
                           build(args["z"]).get_dense().numpy())
        if sem is not None and case["result"]["kind"] == "sparse" and not np.array_equal(sem, case["result"]["dense"]):
            case["reference_inconsistent"] = True
            case["semantic"] = sem
        cases.append(case)

    skipped = []

    def attempt(name, fn):
        """The reference's block union handles a subset of overlaps (split_blocks raises
        NotImplementedError otherwise); only layouts it supports become cases."""
        try:
            return fn()
        except NotImplementedError:
            skipped.append(name)
            return None
        except ZeroDivisionError:
            return "ZeroDivisionError"
        except Exception as e:  # a failure inside the reference's own block code
            skipped.append(f"{name} ({type(e).__name__})")
            return None

    # binary: sparse x sparse (float), all arithmetic/comparison ops, mixed layouts and fills
    for k in range(24):
        total = [int(rng.integers(1, 4)), int(rng.integers(1, 6)), int(rng.integers(3, 12))]
        dcx, dcy = float(rng.choice([0.0, 0.0, 1.0, -1.5])), float(rng.choice([0.0, 0.0, 2.0]))
        dx = rand_layout(total, "float", dcx, split_rows=True)
        dy = rand_layout(total, "float", dcy, split_rows=True)
        op = BIN_OPS[k % len(BIN_OPS)]
        res = attempt(f"binary_{op}_{k}", lambda: T.binary(build(dx), build(dy), getattr(operator, op)))
        if res is not None:
            add(f"binary_{op}_{k}", "binary", dict(x=dx, y=dy, op=op), res)
    # binary with a python scalar on either side
    for k, op in enumerate(["add", "mul", "sub", "ge", "le", "ne"]):
        total = [2, 3, 7]
        dx = rand_layout(total, "float", 0.0)
        res = attempt("c", lambda: T.binary(build(dx), 0.5 * (k - 2), getattr(operator, op)))
        if res is not None:
            add(f"binary_scalar_r_{op}", "binary_scalar_r", dict(x=dx, y=0.5 * (k - 2), op=op), res)
    for k, op in enumerate(["add", "mul", "sub"]):
        total = [2, 3, 7]
        dx = rand_layout(total, "float", 0.0)
        res = attempt("c", lambda: T.binary(1.5, build(dx), getattr(operator, op)))
        if res is not None:
            add(f"binary_scalar_l_{op}", "binary_scalar_l", dict(x=1.5, y=dx, op=op), res)
    # boolean ops
    for k in range(8):
        total = [2, int(rng.integers(1, 5)), int(rng.integers(3, 10))]
        dx = rand_layout(total, "bool", bool(k % 2), split_rows=True)
        dy = rand_layout(total, "bool", bool((k // 2) % 2), split_rows=True)
        op = BOOL_OPS[k % 2]
        res = attempt(f"binary_{op}_{k}", lambda: T.binary(build(dx), build(dy), getattr(operator, op)))
        if res is not None:
            add(f"binary_{op}_{k}", "binary", dict(x=dx, y=dy, op=op), res)
    # unary
    for k in range(6):
        total = [2, 3, int(rng.integers(3, 10))]
        typ = "bool" if k % 2 else "float"
        dx = rand_layout(total, typ, (bool(k % 3 == 0) if typ == "bool" else float(k % 3 == 0)))
        op = "not_" if typ == "bool" else "neg"
        res = attempt("c", lambda: T.unary(build(dx), getattr(operator, op)))
        if res is not None:
            add(f"unary_{op}_{k}", "unary", dict(x=dx, op=op), res)
    # clamp (the sign split)
    for k in range(8):
        total = [int(rng.integers(1, 4)), int(rng.integers(1, 5)), int(rng.integers(3, 10))]
        dx = rand_layout(total, "float", float(rng.choice([0.0, -1.0, 2.0])), split_rows=True)
        min_true = bool(k % 2)
        res = attempt("c", lambda: T.clamp(build(dx), 0, min_true))
        if res is not None:
            add(f"clamp_{int(min_true)}_{k}", "clamp", dict(x=dx, const=0, min_true=min_true), res)
    # where
    for k in range(8):
        total = [2, int(rng.integers(1, 4)), int(rng.integers(3, 9))]
        dc = rand_layout(total, "bool", bool(k % 2), split_rows=True)
        dy = rand_layout(total, "float", 0.0)
        dz = rand_layout(total, "float", float(k % 3))
        res = attempt(f"where_{k}", lambda: T.where(build(dc), build(dy), build(dz)))
        if res is not None:
            add(f"where_{k}", "where", dict(c=dc, y=dy, z=dz), res)
    # any
    for k in range(6):
        total = [2, 3, 5]
        dx = rand_layout(total, "bool", False, kinds=("C", "E") if k < 3 else ("D", "C", "E"))
        res = attempt("c", lambda: T.any(build(dx)))
        if res is not None:
            add(f"any_{k}", "any", dict(x=dx), res)
    # inner_prod: [B,R,K] @ [B,K,N] and [B,R,K] @ [B,K]
    for k in range(10):
        B, R, K, N = 2, int(rng.integers(1, 5)), int(rng.integers(3, 9)), int(rng.integers(2, 8))
        dx = rand_layout([B, R, K], "float", 0.0, kinds=("D", "E", "C"))
        if k % 2 == 0:
            dy = rand_layout([B, K, N], "float", 0.0, kinds=("D", "E"))
        else:
            dy = rand_layout([B, K], "float", 0.0, kinds=("D", "E"))
        res = attempt(f"inner_prod_{k}", lambda: T.inner_prod(build(dx), build(dy)))
        if res is not None:
            add(f"inner_prod_{k}", "inner_prod", dict(x=dx, y=dy), res)
    # diagonal and repeat blocks through binary / inner_prod
    for k in range(4):
        B, n = 2, int(rng.integers(2, 6))
        diag = rng.standard_normal((B, n)).astype(np.float32)
        dd = dict(total=[B, n, n], type="float", dc=0.0,
                  blocks=[dict(kind="Diag", start=[0, 0, 0], data=diag, shape=[B, n, n], diag_index=2)])
        dx = dict(total=[B, 3, n], type="float", dc=0.0,
                  blocks=[dict(kind="D", start=[0, 0, 0], data=rng.standard_normal((B, 3, n)).astype(np.float32))])
        res = attempt(f"inner_prod_diag_{k}", lambda: T.inner_prod(build(dx), build(dd)))
        if res is not None:
            add(f"inner_prod_diag_{k}", "inner_prod", dict(x=dx, y=dd), res)
        rep = rng.standard_normal((1, 3, n)).astype(np.float32)
        dr = dict(total=[B, 3, n], type="float", dc=0.0,
                  blocks=[dict(kind="R", start=[0, 0, 0], data=rep, shape=[B, 3, n])])
        res = T.binary(build(dr), build(dx), operator.mul)
        add(f"binary_repeat_{k}", "binary", dict(x=dr, y=dx, op="mul"), res)
    # shape ops
    for k in range(4):
        dx = rand_layout([2, 3, 6], "float", float(k % 2))
        add(f"unsqueeze_{k}", "unsqueeze", dict(x=dx, index=k % 3), build(dx).unsqueeze(k % 3))
        dq = rand_layout([2, 1, 6], "float", 0.0)
        add(f"squeeze_{k}", "squeeze", dict(x=dq, index=1), build(dq).squeeze(1))
        d1 = rand_layout([1, 4], "float", float(k % 2))
        add(f"repeat_{k}", "repeat", dict(x=d1, dims=[3, 1]), T.repeat(build(d1), torch.tensor([3, 1])))
    for k in range(2):
        dx = rand_layout([2, 3, 5], "bool", bool(k))
        add(f"convert_to_float_{k}", "convert_to_float", dict(x=dx), T.convert_to_float(build(dx)))
    # sub-tensor over a box (SparseTensor.get_sparse_custom_range, sparse_tensor.py:873; what
    # PolyExpSparse.get_mat takes over the live layers' columns, polyexp.py:131-137)
    for k in range(6):
        dx = rand_layout([2, 3, 10], "float", float(k % 2), split_rows=True)
        a = int(rng.integers(0, 5))
        b = int(rng.integers(a + 1, 11))
        st, en = [0, 0, a], [2, 3, b]
        res = attempt(f"custom_range_{k}",
                      lambda: build(dx).get_sparse_custom_range(torch.tensor(st), torch.tensor(en)))
        if res is not None:
            add(f"custom_range_{k}", "custom_range", dict(x=dx, start=st, end=en), res)

    with open(os.path.join(HERE, "gbcsr_ops.pkl"), "wb") as fh:
        pickle.dump(cases, fh, protocol=4)
    print(f"{len(cases)} cases; skipped (unsupported by the reference): {skipped}")


if __name__ == "__main__":
    main()
