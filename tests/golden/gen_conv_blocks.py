"""Generate operator-level golden vectors for the gbcsr conv blocks (KernelBlock,
PatchesBlock) by running the REFERENCE's own constraintflow/gbcsr/sparse_block.py and
sparse_tensor.py on seeded inputs.

Test infrastructure; runs only where the reference checkout is present (REF_ROOT).
    CF_REFERENCE_ROOT=<reference checkout> python tests/golden/gen_conv_blocks.py
        -> tests/golden/gbcsr_conv_blocks.pkl

Each case records the conv geometry, the operands as plain arrays, the operation and the
reference's result: the result block's kind, its payload (for conv blocks also their
geometry) and its dense matrix (get_dense), so the mirror is checked both on the structure
it keeps and on the values.
"""
import os
import pickle
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF_ROOT = os.environ.get("CF_REFERENCE_ROOT", "")

# (name, K, C, ix, iy, kx, ky, sx, sy, px, py)
GEOMS = [
    ("k3s1p1", 2, 3, 5, 5, 3, 3, 1, 1, 1, 1),
    ("k3s2p1", 4, 2, 7, 7, 3, 3, 2, 2, 1, 1),
    ("k4s2p1", 3, 2, 8, 8, 4, 4, 2, 2, 1, 1),
    ("k2s1p0", 2, 1, 4, 6, 2, 2, 1, 1, 0, 0),
    ("rect", 3, 2, 6, 5, 3, 2, 2, 1, 1, 0),
]


def out_size(i, k, s, p):
    return (i + 2 * p - k) // s + 1


def main():
    if not REF_ROOT or not os.path.isdir(os.path.join(REF_ROOT, "constraintflow")):
        sys.exit("set CF_REFERENCE_ROOT to the reference checkout (the directory holding constraintflow/)")
    sys.argv = ["x"]
    sys.path.insert(0, os.path.join(HERE, "refshim", "stubs"))
    sys.path.insert(0, REF_ROOT)
    import torch
    from constraintflow.gbcsr.sparse_block import (ConstBlock, DenseBlock, DiagonalBlock, KernelBlock,
                                                   PatchesBlock, RepeatBlock)
    from constraintflow.gbcsr.sparse_tensor import SparseTensor

    rng = np.random.default_rng(7)
    torch.manual_seed(7)

    def f32(*shape):
        return rng.standard_normal(shape).astype(np.float32)

    def record(res):
        if isinstance(res, tuple):
            res = res[0]
        if isinstance(res, SparseTensor):
            return dict(kind="sparse", dense=res.get_dense().float().numpy(),
                        blocks=[b.block_type for b in res.blocks])
        if isinstance(res, torch.Tensor):
            return dict(kind="tensor", dense=res.float().numpy())
        out = dict(kind=type(res).__name__, total=[int(v) for v in res.total_shape])
        if isinstance(res, ConstBlock):
            out["value"] = float(res.block)
        else:
            out["payload"] = res.block.float().numpy() if res.block.dtype != torch.bool else res.block.numpy()
        if isinstance(res, (KernelBlock, PatchesBlock)):
            out["params"] = [int(v) for v in res.parameters()]
            try:
                out["dense"] = res.get_dense().float().numpy()
            except RuntimeError as e:   # the reference's PatchesBlock.get_dense places patches with
                out["dense_error"] = str(e).splitlines()[0]   # one stride: unequal strides fail there
        return out

    def patches_dense_semantic(res):
        """The conv matrix a PatchesBlock stands for, placed row by row (x pitch = padded
        width).  The reference's get_dense advances one output row by the padded HEIGHT
        times the stride (sparse_block.py:3162), which is the same only for square inputs."""
        P = res.block.float().numpy()
        B = int(res.total_shape[0])
        K, C, ix, iy, ox, oy = res.num_kernels, res.num_channels, res.ix, res.iy, res.ox, res.oy
        kx, ky, s, px, py = res.kx, res.ky, res.sx, res.px, res.py
        out = np.zeros((B, K * ox * oy, C * ix * iy), np.float32)
        for b in range(B):
            pb_ = P[0 if P.shape[0] == 1 else b]
            for k in range(K):
                for oxi in range(ox):
                    for oyi in range(oy):
                        r = (k * ox + oxi) * oy + oyi
                        for c in range(C):
                            for dx in range(kx):
                                for dy in range(ky):
                                    x, y = oxi * s - px + dx, oyi * s - py + dy
                                    if 0 <= x < ix and 0 <= y < iy:
                                        out[b, r, (c * ix + x) * iy + y] = pb_[r, (c * kx + dx) * ky + dy]
        return out

    cases = []
    pb_of = {}

    def add(name, op, args, fn):
        try:
            res = fn()
        except NotImplementedError as e:
            res = None
            cases.append(dict(name=name, op=op, args=args, result=dict(kind="NotImplementedError", msg=str(e))))
            return
        case = dict(name=name, op=op, args=args, result=record(res))
        # where the reference densified a PatchesBlock of a non-square image, record the
        # result of the same operation on the conv matrix placed row by row as well
        r = res[0] if isinstance(res, tuple) else res
        if isinstance(r, PatchesBlock) and "dense" in case["result"]:
            sem = patches_dense_semantic(r)
            if not np.array_equal(sem, case["result"]["dense"]):
                case["reference_inconsistent"] = True
                case["semantic"] = dict(dense=sem)
        if op in ("dense_at_patches", "kernel_at_patches"):
            pbk = pb_of[name]()
            sem_p = torch.from_numpy(patches_dense_semantic(pbk))
            if not np.array_equal(sem_p.numpy(), pbk.get_dense().float().numpy()):
                lhs = (torch.from_numpy(args["Y"]) if op == "dense_at_patches"
                       else KernelBlock(torch.from_numpy(args["W3"]), torch.tensor([1, 1, 1]), args["g3"]["ix"],
                                        args["g3"]["iy"], args["g3"]["ox"], args["g3"]["oy"], 1, 1, 1, 1).get_dense())
                case["reference_inconsistent"] = True
                case["semantic"] = dict(payload=(lhs @ sem_p).numpy())
        cases.append(case)

    for gname, K, C, ix, iy, kx, ky, sx, sy, px, py in GEOMS:
        ox, oy = out_size(ix, kx, sx, px), out_size(iy, ky, sy, py)
        rows, cols = K * ox * oy, C * ix * iy
        B = 2
        geom = dict(K=K, C=C, ix=ix, iy=iy, ox=ox, oy=oy, kx=kx, ky=ky, sx=sx, sy=sy, px=px, py=py, B=B)
        W = f32(K, C, kx, ky)

        def kb(W=W, B=B):
            return KernelBlock(torch.from_numpy(W), torch.tensor([B, rows, cols]), ix, iy, ox, oy, sx, sy, px, py)

        square = sx == sy
        add(f"{gname}_kernel_get_dense", "kernel_get_dense", dict(g=geom, W=W), lambda: kb().get_dense())
        add(f"{gname}_kernel_to_patches", "kernel_to_patches", dict(g=geom, W=W), lambda: kb().convert_to_patches())
        d = f32(B, cols)
        add(f"{gname}_kernel_at_diag", "kernel_at_diag", dict(g=geom, W=W, d=d),
            lambda: kb().matmul_equal_dims(DiagonalBlock(torch.from_numpy(d), torch.tensor([B, cols, cols]), 2)))
        S = 3
        X = f32(B, cols, S)
        add(f"{gname}_kernel_at_dense", "kernel_at_dense", dict(g=geom, W=W, X=X),
            lambda: kb().matmul_equal_dims(DenseBlock(torch.from_numpy(X))))
        v = f32(B, cols)
        add(f"{gname}_kernel_at_vec", "kernel_at_vec", dict(g=geom, W=W, v=v),
            lambda: kb().matmul_unequal_dims(DenseBlock(torch.from_numpy(v))))
        add(f"{gname}_kernel_at_zero", "kernel_at_zero", dict(g=geom, W=W, S=S),
            lambda: kb().matmul_equal_dims(ConstBlock(0, torch.tensor([B, cols, S]))))
        Y = f32(B, 4, rows)
        add(f"{gname}_dense_at_kernel", "dense_at_kernel", dict(g=geom, W=W, Y=Y),
            lambda: DenseBlock(torch.from_numpy(Y)).matmul_equal_dims(kb()))
        e = f32(B, rows)
        add(f"{gname}_diag_at_kernel", "diag_at_kernel", dict(g=geom, W=W, e=e),
            lambda: DiagonalBlock(torch.from_numpy(e), torch.tensor([B, rows, rows]), 2).matmul_equal_dims(kb()))
        # a SparseTensor holding the conv block: its dense form and a product with a dense tensor
        add(f"{gname}_tensor_kernel_dense", "tensor_kernel_dense", dict(g=geom, W=W),
            lambda: SparseTensor([torch.tensor([0, 0, 0])], [kb()], 3, torch.tensor([B, rows, cols])))
        add(f"{gname}_tensor_kernel_matmul", "tensor_kernel_matmul", dict(g=geom, W=W, X=X),
            lambda: SparseTensor([torch.tensor([0, 0, 0])], [kb()], 3, torch.tensor([B, rows, cols])).matmul(
                SparseTensor([torch.tensor([0, 0, 0])], [DenseBlock(torch.from_numpy(X))], 3,
                             torch.tensor([B, cols, S]))))
        if not square:
            continue
        # patches from a diagonal product (one payload per region)
        def pb(d=d):
            return kb().matmul_equal_dims(DiagonalBlock(torch.from_numpy(d), torch.tensor([B, cols, cols]), 2))[0]
        add(f"{gname}_patches_at_vec", "patches_at_vec", dict(g=geom, W=W, d=d, v=v),
            lambda: pb().matmul_unequal_dims(DenseBlock(torch.from_numpy(v))))
        d2 = f32(B, cols)
        add(f"{gname}_patches_at_diag", "patches_at_diag", dict(g=geom, W=W, d=d, d2=d2),
            lambda: pb().matmul_equal_dims(DiagonalBlock(torch.from_numpy(d2), torch.tensor([B, cols, cols]), 2)))
        add(f"{gname}_patches_sum", "patches_sum", dict(g=geom, W=W, d=d), lambda: pb().sum(2))
        pb_of[f"{gname}_dense_at_patches"] = pb
        pb_of[f"{gname}_kernel_at_patches"] = pb
        add(f"{gname}_dense_at_patches", "dense_at_patches", dict(g=geom, W=W, d=d, Y=Y),
            lambda: DenseBlock(torch.from_numpy(Y)).matmul_equal_dims(pb()))
        # the next layer's weights (K -> 2 channels, 3x3, stride 1, padding 1) times the patches
        W3 = f32(2, K, 3, 3)
        g3 = dict(K=2, C=K, ix=ox, iy=oy, ox=ox, oy=oy, kx=3, ky=3, sx=1, sy=1, px=1, py=1)
        add(f"{gname}_kernel_at_patches", "kernel_at_patches", dict(g=geom, W=W, d=d, g3=g3, W3=W3),
            lambda: KernelBlock(torch.from_numpy(W3), torch.tensor([B, 2 * ox * oy, rows]), ox, oy, ox, oy, 1, 1, 1,
                                1).matmul_equal_dims(pb()))
        # patches times the previous layer's weights: a conv C2 -> C whose output is ix x iy
        for s2, k2, p2 in ((1, 3, 1), (2, 3, 1)):
            C2 = 2
            ix2 = (ix - 1) * s2 - 2 * p2 + k2
            if (ix2 + 2 * p2 - k2) // s2 + 1 != ix:
                continue
            W2 = f32(C, C2, k2, k2)
            g2 = dict(K=C, C=C2, ix=ix2, iy=ix2, ox=ix, oy=iy, kx=k2, ky=k2, sx=s2, sy=s2, px=p2, py=p2)
            if iy != ix:
                continue

            def kb2(W2=W2, g2=g2):
                return KernelBlock(torch.from_numpy(W2), torch.tensor([B, C * ix * iy, C2 * g2["ix"] * g2["iy"]]),
                                   g2["ix"], g2["iy"], ix, iy, s2, s2, p2, p2)
            add(f"{gname}_patches_at_kernel_s{s2}", "patches_at_kernel", dict(g=geom, W=W, d=d, g2=g2, W2=W2),
                lambda: pb().matmul_equal_dims(kb2()))
            add(f"{gname}_kernel_patches_at_kernel_s{s2}", "kernel_patches_at_kernel", dict(g=geom, W=W, g2=g2, W2=W2),
                lambda: kb().convert_to_patches().matmul_equal_dims(kb2()))
        # elementwise ops on conv blocks
        add(f"{gname}_patches_add_patches", "patches_add_patches", dict(g=geom, W=W, d=d, d2=d2),
            lambda: pb().binary(pb(d2), __import__("operator").add))
        add(f"{gname}_patches_mul_const", "patches_mul_const", dict(g=geom, W=W, d=d, c=2.5),
            lambda: pb().binary(ConstBlock(2.5, torch.tensor([B, rows, cols])), __import__("operator").mul))
        add(f"{gname}_kernel_mul_const", "kernel_mul_const", dict(g=geom, W=W, c=-0.5),
            lambda: kb().binary(ConstBlock(-0.5, torch.tensor([B, rows, cols])), __import__("operator").mul))
    with open(os.path.join(HERE, "gbcsr_conv_blocks.pkl"), "wb") as f:
        pickle.dump(cases, f)
    kinds = {}
    for c in cases:
        kinds[c["op"]] = kinds.get(c["op"], 0) + 1
    print(len(cases), "cases", kinds)


if __name__ == "__main__":
    main()
