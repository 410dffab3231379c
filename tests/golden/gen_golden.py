"""Generate the golden vectors under tests/golden/ by running the REFERENCE itself.

This script is test infrastructure.  It runs only in a container that has the
reference checkout (ConstraintFlow, pure Python + PyTorch) at REF_ROOT; the GPU
box never runs it.  Usage::

    CF_REFERENCE_ROOT=<reference checkout> python tests/golden/gen_golden.py          # all cases
    CF_REFERENCE_ROOT=<reference checkout> python tests/golden/gen_golden.py dp_w0    # names starting dp_w0

For every case it
  1. compiles the reference's own certifier program
     (examples/compiler_examples/{deeppoly,crown,deeppoly2,deeppoly_efficient}.cf) with the reference
     compiler (constraintflow/compiler/compile.py:66-97) into a scratch dir;
  2. builds the seeded synthetic network in memory (cfgpu/nets.py) and hands it
     to the reference's ONNX reader through the in-memory onnx stand-in
     (refshim/stubs/onnx), exactly the fields constraintflow/lib/parse.py reads;
  3. runs the generated ``main.run`` body (network + spec, Abs_elem_sparse,
     Flow(...).flow(), as emitted by constraintflow/compiler/codeGen.py:26-36)
     on CPU, the way constraintflow/cli.py:344-354 calls it (no dataset download);
  4. stores the inputs, the final bounds (float64, as Flow.flow returns them) and
     the full per-neuron l/u state of the abstract element into ``<case>.npz``.

Shims (refshim/): an ANTLR v3-ATN loader (the generated parser predates the
installed antlr4 runtime) and stub plotting/graphviz modules that the reference
imports but never calls on this path.
"""
import importlib.util
import json
import os
import subprocess
import sys
import tempfile
import time

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
REF_ROOT = os.environ.get("CF_REFERENCE_ROOT", "")
PKG = os.path.join(REPO, "constraintflow-gpu_b200")

# certifier programs of examples/compiler_examples/ whose generated code is kept and run
PROGRAMS = ("deeppoly", "crown", "deeppoly2", "deeppoly_efficient", "zono", "zono2", "ibp", "polyzono", "crownibp")

# name -> (program, workload id, batch, eps)
CASES = {
    "dp_w0_b1_e1e-2": ("deeppoly", 0, 1, 0.01),
    "dp_w0_b4_e1e-3": ("deeppoly", 0, 4, 0.001),
    "dp_w0_b4_e0": ("deeppoly", 0, 4, 0.0),
    "dp_w1_b16_e5e-3": ("deeppoly", 1, 16, 0.005),
    "dp_w1_b16_e5e-4": ("deeppoly", 1, 16, 0.0005),
    "dp_w1_b16_e5e-5": ("deeppoly", 1, 16, 0.00005),
    "dp_w2_b8_e2e-3": ("deeppoly", 2, 8, 0.002),
    "dp_w2_b8_e2e-4": ("deeppoly", 2, 8, 0.0002),
    "dp_w2_b8_e2e-5": ("deeppoly", 2, 8, 0.00002),
    "dp_w3_b4_e2e-2": ("deeppoly", 3, 4, 0.02),
    "dp_w3_b4_e2e-3": ("deeppoly", 3, 4, 0.002),
    "dp_w3_b4_e2e-4": ("deeppoly", 3, 4, 0.0002),
    "dp_w4_b1_e2o255": ("deeppoly", 4, 1, 2.0 / 255.0),
    "dp_w4_b1_e2o2550": ("deeppoly", 4, 1, 2.0 / 2550.0),
    # the benchmark batch of the 9x200 MLP and an 8-region batch of the CIFAR conv net, stored
    # compactly (COMPACT below)
    "dp_w2_b256_e2e-3": ("deeppoly", 2, 256, 0.002),
    "dp_w4_b8_e2o255": ("deeppoly", 4, 8, 2.0 / 255.0),
    "dp_w4_b8_e2o2550": ("deeppoly", 4, 8, 2.0 / 2550.0),
    "crown_w0_b4_e1e-2": ("crown", 0, 4, 0.01),
    "crown_w0_b4_e1e-3": ("crown", 0, 4, 0.001),
    "crown_w2_b4_e2e-3": ("crown", 2, 4, 0.002),
    "crown_w2_b4_e2e-4": ("crown", 2, 4, 0.0002),
    # CROWN's whole-layer ReLU branches: eps 0.05 takes the zero branch at the first ReLU,
    # eps >= 0.1 the all-crossing branch at every ReLU (mixed-layer polyexps)
    "crown_w0_b2_e5e-2": ("crown", 0, 2, 0.05),
    "crown_w0_b2_e1e-1": ("crown", 0, 2, 0.1),
    "crown_w0_b2_e3e-1": ("crown", 0, 2, 0.3),
    "crown_w1_b2_e5e-2": ("crown", 1, 2, 0.05),
    "crown_w1_b2_e1e-1": ("crown", 1, 2, 0.1),
    # deeppoly_efficient.cf: ReLU polyexps over the affine's inputs (prev[L] / prev[U])
    "dpe_w0_b4_e1e-3": ("deeppoly_efficient", 0, 4, 0.001),
    "dpe_w2_b4_e2e-4": ("deeppoly_efficient", 2, 4, 0.0002),
    # DAG networks: residual blocks (Add) and concatenated branches (Concat)
    "dp_w5_b4_e2e-3": ("deeppoly", 5, 4, 0.002),
    "dp_w5_b4_e2e-4": ("deeppoly", 5, 4, 0.0002),
    "dp_w6_b4_e2e-3": ("deeppoly", 6, 4, 0.002),
    "dp_w6_b4_e2e-4": ("deeppoly", 6, 4, 0.0002),
    "crown_w5_b2_e2e-3": ("crown", 5, 2, 0.002),
    "crown_w6_b2_e2e-3": ("crown", 6, 2, 0.002),
    "crown_w6_b2_e1e-1": ("crown", 6, 2, 0.1),
    # zonotope (DeepZ) and interval programs: forward flow
    "zono_w0_b4_e1e-3": ("zono", 0, 4, 0.001),
    "zono_w0_b4_e1e-2": ("zono", 0, 4, 0.01),
    "zono_w1_b8_e5e-4": ("zono", 1, 8, 0.0005),
    "zono_w2_b4_e2e-3": ("zono", 2, 4, 0.002),
    "zono_w2_b4_e2e-4": ("zono", 2, 4, 0.0002),
    "zono_w3_b2_e2e-3": ("zono", 3, 2, 0.002),
    "zono2_w0_b4_e1e-3": ("zono2", 0, 4, 0.001),
    "zono2_w0_b2_e5e-2": ("zono2", 0, 2, 0.05),
    "zono_w5_b4_e2e-3": ("zono", 5, 4, 0.002),
    "ibp_w0_b4_e1e-3": ("ibp", 0, 4, 0.001),
    "ibp_w2_b4_e2e-4": ("ibp", 2, 4, 0.0002),
    "ibp_w3_b2_e2e-3": ("ibp", 3, 2, 0.002),
    "ibp_w5_b4_e2e-4": ("ibp", 5, 4, 0.0002),
    # polyzono.cf: DeepPoly backsubstitution and the zonotope in one state
    "pz_w0_b4_e1e-2": ("polyzono", 0, 4, 0.01),
    "pz_w1_b8_e5e-4": ("polyzono", 1, 8, 0.0005),
    "pz_w2_b4_e2e-3": ("polyzono", 2, 4, 0.002),
    "pz_w2_b4_e2e-4": ("polyzono", 2, 4, 0.0002),
    # crownibp.cf: interval bounds for every layer, backsubstitution for the property only
    "cibp_w0_b4_e1e-3": ("crownibp", 0, 4, 0.001),
    "cibp_w0_b4_e1e-2": ("crownibp", 0, 4, 0.01),
    "cibp_w1_b8_e5e-4": ("crownibp", 1, 8, 0.0005),
    "cibp_w2_b4_e2e-4": ("crownibp", 2, 4, 0.0002),
    "cibp_w3_b2_e2e-3": ("crownibp", 3, 2, 0.002),
    # deeppoly_custom_stop.cf and custom_stops/: the traversal stops get_start layers below the
    # bounded neuron and concretises there with those neurons' l / u
    "cs3_w0_b4_e1e-2": ("deeppoly_custom_stop", 0, 4, 0.01),
    "cs3_w2_b4_e2e-4": ("deeppoly_custom_stop", 2, 4, 0.0002),
    "cs0_w0_b4_e1e-3": ("custom_stops/deeppoly_custom_stop00", 0, 4, 0.001),
    "cs1_w0_b4_e1e-3": ("custom_stops/deeppoly_custom_stop01", 0, 4, 0.001),
    "cs2_w1_b8_e5e-4": ("custom_stops/deeppoly_custom_stop02", 1, 8, 0.0005),
    "cs5_w2_b4_e2e-4": ("custom_stops/deeppoly_custom_stop05", 2, 4, 0.0002),
    "cs8_w2_b4_e2e-4": ("custom_stops/deeppoly_custom_stop08", 2, 4, 0.0002),
    # zid.cf: zonotope bounds for list layers up to 4, interval bounds above, DeepPoly for the
    # property rows
    "zid_w0_b4_e1e-2": ("zid", 0, 4, 0.01),
    "zid_w2_b4_e2e-3": ("zid", 2, 4, 0.002),
    "zid_w1_b8_e5e-4": ("zid", 1, 8, 0.0005),
    "zid_w3_b2_e2e-3": ("zid", 3, 2, 0.002),
    # the tied network (32 first-layer neurons with l + u == 0 exactly): zid.cf and the
    # custom-stop programs test l + u > 0, deeppoly.cf and crownibp.cf l + u >= 0
    "zid_w7_b4_e1e-2": ("zid", 7, 4, 0.01),
    "cs3_w7_b4_e1e-2": ("deeppoly_custom_stop", 7, 4, 0.01),
    "dp_w7_b4_e1e-2": ("deeppoly", 7, 4, 0.01),
    "cibp_w7_b4_e1e-2": ("crownibp", 7, 4, 0.01),
    # conv layers inside a residual block (workload 8).  crown.cf on a conv network stops in
    # the reference itself (KernelBlock.matmul_unequal_dims, sparse_block.py:1726, raises
    # "Unrecognized sparse block type: RepeatBlock"), so it has no golden case.
    "dp_w8_b4_e1e-2": ("deeppoly", 8, 4, 0.01),
    "dp_w8_b4_e1e-3": ("deeppoly", 8, 4, 0.001),
}


# Cases stored compactly: the per-neuron l/u of the affine layers and the property rows only
# (l_aff / u_aff), the input box of the first COMPACT_INPUT_ROWS regions (l_in / u_in); a
# ReLU layer's columns are where(x >= 0, x, 0) of the affine layer below it (deeppoly.cf:20-24:
# l' = l if l >= 0 else 0, u' likewise), which the generator checks before dropping them.
COMPACT = {"dp_w2_b256_e2e-3", "dp_w4_b8_e2o255", "dp_w4_b8_e2o2550"}
COMPACT_INPUT_ROWS = 2


def _load_nets():
    spec = importlib.util.spec_from_file_location("cfgpu_nets", os.path.join(PKG, "cfgpu", "nets.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _onnx_graph(nets, wl):
    """In-memory graph with the fields constraintflow/lib/parse.py:60-200 reads.

    Conv attributes are positional in torch-export order
    (dilations, group, kernel_shape, pads, strides): parse.py:110-112.  A leading
    Flatten (skipped by the reader as identity, parse.py:240-247) keeps the
    4-D input shape for the first Gemm (parse.py:137).  Add / Concat nodes name their two
    parents' outputs (parse.py:165-200).
    """
    import types
    NS = types.SimpleNamespace
    inits, nodes = [], []
    out_name = {-1: "input"}
    flattened = False
    for i, L in enumerate(wl.layers):
        ps = nets.parents_of(wl.layers, i)
        src = out_name[ps[0]]
        name = f"n{i}"
        if L.kind == "conv":
            k = L.W.shape[2]
            inits += [NS(name=f"c{i}.weight", array=L.W), NS(name=f"c{i}.bias", array=L.b)]
            nodes.append(NS(op_type="Conv", input=[src, f"c{i}.weight", f"c{i}.bias"], output=[name],
                            attribute=[NS(ints=[1, 1]), NS(ints=[1]), NS(ints=[k, k]),
                                       NS(ints=[L.pad] * 4), NS(ints=[L.stride] * 2)]))
        elif L.kind == "linear":
            if not flattened:
                nodes.append(NS(op_type="Flatten", input=[src], output=["flat"], attribute=[]))
                out_name[ps[0]] = src = "flat"
                flattened = True
            inits += [NS(name=f"fc{i}.weight", array=L.W), NS(name=f"fc{i}.bias", array=L.b)]
            nodes.append(NS(op_type="Gemm", input=[src, f"fc{i}.weight", f"fc{i}.bias"], output=[name],
                            attribute=[]))
        elif L.kind == "relu":
            nodes.append(NS(op_type="Relu", input=[src], output=[name], attribute=[]))
        elif L.kind in ("add", "concat"):
            nodes.append(NS(op_type="Add" if L.kind == "add" else "Concat", input=[src, out_name[ps[1]]],
                            output=[name], attribute=[]))
        else:
            raise ValueError(L.kind)
        out_name[i] = name
    C, H, W = wl.input_shape
    dims = [NS(dim_value=v) for v in (1, C, H, W)]
    return NS(input=[NS(name="input", type=NS(tensor_type=NS(shape=NS(dim=dims))))],
              node=nodes, initializer=inits)


def _compact(wl, l_all, u_all):
    """Affine-layer and property columns, and the first regions' input box (COMPACT)."""
    import numpy as np
    n0 = wl.input_size
    keep, pos, prev = [], n0, None
    for L in wl.layers:
        sl = slice(pos, pos + L.n_out)
        if L.kind == "relu":
            for a in (l_all, u_all):
                x = a[:, prev]
                assert np.array_equal(a[:, sl], np.where(x >= 0, x, np.float32(0))), "ReLU columns not derivable"
        else:
            keep.append(sl)
        prev = sl
        pos += L.n_out
    keep.append(slice(pos, l_all.shape[1]))  # property rows
    cols = np.concatenate([np.arange(s.start, s.stop) for s in keep])
    r = COMPACT_INPUT_ROWS
    return {"compact": True, "l_aff": l_all[:, cols], "u_aff": u_all[:, cols],
            "l_in": l_all[:r, :n0], "u_in": u_all[:r, :n0]}


def worker(program, outdir, case_names):
    """Runs inside a fresh interpreter: the reference package on sys.path first."""
    sys.argv = ["x"]
    sys.path.insert(0, os.path.join(HERE, "refshim", "stubs"))
    sys.path.insert(0, os.path.join(HERE, "refshim"))
    sys.path.insert(0, REF_ROOT)
    import numpy as np
    import torch
    import antlr_v3_shim  # noqa: F401  (must precede the reference's parser import)
    import onnx
    from constraintflow.compiler import compile as cfcompile
    nets = _load_nets()

    src = os.path.join(REF_ROOT, "examples", "compiler_examples", f"{program}.cf")
    os.makedirs(outdir, exist_ok=True)
    cfcompile.compile(src, outdir)
    # keep the generated program: the drop-in runtime must run it unchanged
    keep = os.path.join(HERE, "generated", program)
    os.makedirs(keep, exist_ok=True)
    for f in ("main.py", "transformers.py"):
        with open(os.path.join(outdir, f)) as fi, open(os.path.join(keep, f), "w") as fo:
            fo.write(fi.read())
    sys.path.insert(0, outdir)
    import constraintflow.lib.flow_sparse as fs
    captured = {}
    orig_flow = fs.Flow.flow

    def flow_and_keep(self):
        res = orig_flow(self)
        captured["abs_elem"] = self.abs_elem
        captured["model"] = self.model
        return res
    fs.Flow.flow = flow_and_keep
    import main as cfmain

    for name in case_names:
        prog, wid, B, eps = CASES[name]
        wl = nets.workload(wid)
        X = nets.centres(wl, B)
        y = nets.labels(wl, X)
        net_name = f"{name}.onnx"
        onnx.register(net_name, _onnx_graph(nets, wl))
        torch.set_num_threads(os.cpu_count())
        t0 = time.perf_counter()
        lb, ub = cfmain.run(net_name, B, eps, X, y, wl.dataset, False, False, False)
        dt = time.perf_counter() - t0
        ae = captured["abs_elem"]
        l_all = ae.d["l"].get_dense().to(torch.float32).numpy()
        u_all = ae.d["u"].get_dense().to(torch.float32).numpy()
        layout = [(str(layer.type).split(".")[-1], int(layer.start), int(layer.end)) for layer in captured["model"]]
        state = {"l_all": l_all, "u_all": u_all}
        if name in COMPACT:
            state = _compact(wl, l_all, u_all)
        np.savez_compressed(
            os.path.join(HERE, f"{name}.npz"),
            program=program, wid=wid, B=B, eps=eps, dataset=wl.dataset,
            X=X.numpy(), y=y.numpy().astype(np.int64),
            weights_digest=nets.weights_digest(wl.layers),
            lb=lb.numpy(), ub=ub.numpy(), **state,
            layout=json.dumps(layout), ref_seconds=dt)
        print(json.dumps({"case": name, "seconds": round(dt, 2), "lb_dtype": str(lb.dtype),
                          "certified": int((lb >= 0).all(dim=1).sum()), "B": B}), flush=True)


def main():
    if not REF_ROOT or not os.path.isdir(os.path.join(REF_ROOT, "constraintflow")):
        sys.exit("set CF_REFERENCE_ROOT to the reference checkout (the directory holding constraintflow/)")
    sel = sys.argv[1:]
    if sel == ["--programs-only"]:
        for prog in PROGRAMS:
            with tempfile.TemporaryDirectory() as tmp:
                code = ("import sys; sys.path.insert(0, %r); import gen_golden as g; g.worker(%r, %r, [])"
                        % (HERE, prog, os.path.join(tmp, "out")))
                subprocess.run([sys.executable, "-c", code], cwd=tmp, check=True)
        return
    names = [n for n in CASES if not sel or any(n.startswith(s) for s in sel)]
    by_prog = {}
    for n in names:
        by_prog.setdefault(CASES[n][0], []).append(n)
    for prog, case_names in by_prog.items():
        with tempfile.TemporaryDirectory() as tmp:
            code = ("import sys; sys.path.insert(0, %r); import gen_golden as g; g.worker(%r, %r, %r)"
                    % (HERE, prog, os.path.join(tmp, "out"), case_names))
            subprocess.run([sys.executable, "-c", code], cwd=tmp, check=True)


if __name__ == "__main__":
    main()
