"""The drop-in package imports on a machine without a GPU and its host-side logic
(structure, shape/type checks) works without launching anything."""
import operator

import numpy as np

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


def test_generic_runtime_refuses_explicitly():
    """The op-by-op interpretation of generated transformer bodies is not provided: its entry
    points raise NotImplementedError (as Flow does for an unrecognised program) instead of
    returning something else; PolyExpSparse.get_mat keeps the live layers' columns only."""
    import types
    from constraintflow.gbcsr.sparse_tensor import SparseTensor
    from constraintflow.lib.abs_elem import Abs_elem_sparse
    from constraintflow.lib.llist import Llist
    from constraintflow.lib.polyexp import PolyExpSparse
    net = [types.SimpleNamespace(start=0, end=4), types.SimpleNamespace(start=4, end=7),
           types.SimpleNamespace(start=7, end=9)]
    d = {"llist": torch.tensor([True, True, False]), "l": None, "u": None}
    ae = Abs_elem_sparse(d, {"llist": "bool", "l": "Float", "u": "Float"}, net, batch_size=2)
    assert ae.get_poly_size() == 7 and ae.live_layers() == [0, 1]
    ll = Llist(net, [1], None, None, [1])
    assert ll.layers() == [1] and Llist(net, [1], 0, 2).layers() == [0, 1]
    for call in (lambda: ae.get_elem("l", ll), lambda: ae.update(ll, []), lambda: ll.get_metadata("weight", 2),
                 lambda: ll.dot(None, 7), lambda: ll.convert_to_poly(ae)):
        with pytest.raises(NotImplementedError):
            call()
    mat = SparseTensor([], [], 3, torch.tensor([2, 3, 9]), dense_const=0.0)
    got = PolyExpSparse(net, mat, 0.0).get_mat(ae)
    assert got.shape == [2, 3, 9] and got.num_blocks == 0


def test_generated_programs_are_recognised():
    """The reference compiler's own output for deeppoly.cf, deeppoly_efficient.cf,
    crown.cf, zono.cf, ibp.cf and polyzono.cf (tests/golden/generated/) is recognised by the drop-in
    Flow without a GPU; zono2.cf (whole-layer branches, not run) is refused."""
    import importlib.util
    import os
    import sys
    from constraintflow.lib.flow_sparse import certifier_of
    here = os.path.dirname(os.path.abspath(__file__))
    for program, expect in (("deeppoly", "deeppoly"), ("deeppoly_efficient", "deeppoly"), ("crown", "crown"),
                            ("zono", "zono"), ("ibp", "ibp"), ("polyzono", "polyzono"), ("crownibp", "crownibp"),
                            ("zid", "zid"), ("zono2", None)):
        path = os.path.join(here, "golden", "generated", program, "transformers.py")
        saved = sys.modules.pop("transformers", None)
        try:
            spec = importlib.util.spec_from_file_location("transformers", path)
            mod = importlib.util.module_from_spec(spec)
            sys.modules["transformers"] = mod
            spec.loader.exec_module(mod)
            cls = getattr(mod, program if program in ("ibp", "polyzono", "crownibp", "zid") else
                          "zono" if program.startswith("zono") else "deeppoly")
            if expect is None:
                with pytest.raises(NotImplementedError):
                    certifier_of(cls())
            else:
                assert certifier_of(cls()) == expect
        finally:
            sys.modules.pop("transformers", None)
            if saved is not None:
                sys.modules["transformers"] = saved


@pytest.mark.parametrize("wid", [0, 3, 5, 6])
def test_onnx_reader_layer_list(wid):
    """The ONNX reader mirror on the synthetic networks: the layer list, parents and
    neuron ranges the driver receives are those of the network (workload 6 lists its
    layers breadth first, as the reference's reader orders them)."""
    import os
    import sys
    from cfgpu import nets
    from constraintflow.lib.parse import parse_onnx_layers
    from constraintflow.lib.network import LayerType
    from constraintflow.lib.flow_sparse import engine_layers
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, os.path.join(here, "golden"))
    import gen_golden
    wl = nets.workload(wid)
    spec = torch.zeros(1, 9, wl.layers[-1].n_out)
    import types
    graph = types.SimpleNamespace(graph=gen_golden._onnx_graph(nets, wl))
    model = parse_onnx_layers(graph, spec, torch.zeros(1, 9))
    assert model[0].type == LayerType.Input and model[-1].last_layer
    start = 0
    for i, lay in enumerate(model):
        assert lay.identifier == i and lay.start == start
        assert all(p < i for p in lay.parents)
        start = lay.end
    assert model.size == start == wl.input_size + sum(L.n_out for L in wl.layers) + 9
    eng = engine_layers(model)
    assert [L.kind for L in eng] == [L.kind for L in wl.layers]
    assert [L.parents for L in eng] == [nets.parents_of(wl.layers, i) for i in range(len(wl.layers))]
    for a, b in zip(eng, wl.layers):
        if b.W is not None:
            np.testing.assert_array_equal(a.W.numpy(), b.W)


def test_onnx_reader_orders_breadth_first():
    """Branches written depth first in the ONNX graph (Linear, ReLU of one branch, then
    the other's) come out breadth first, as the reference's reader lists them."""
    import os
    import sys
    import types
    from cfgpu import nets
    from constraintflow.lib.parse import parse_onnx_layers
    from constraintflow.lib.flow_sparse import engine_layers
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden"))
    import gen_golden
    wl = nets.workload(6)
    bfs = wl.layers
    dfs_order = [0, 1, 2, 4, 3, 5, 6, 7]           # new position -> index in the breadth-first list
    pos = {old: new for new, old in enumerate(dfs_order)}
    dfs = [nets.Layer(**{**bfs[o].__dict__, "parents": tuple(pos[p] if p >= 0 else -1
                                                              for p in nets.parents_of(bfs, o))})
           for o in dfs_order]
    graph = types.SimpleNamespace(graph=gen_golden._onnx_graph(nets, types.SimpleNamespace(**{**wl.__dict__,
                                                                                             "layers": dfs})))
    model = parse_onnx_layers(graph, torch.zeros(1, 9, 10), torch.zeros(1, 9))
    eng = engine_layers(model)
    assert [L.kind for L in eng] == [L.kind for L in bfs]
    assert [L.parents for L in eng] == [nets.parents_of(bfs, i) for i in range(len(bfs))]
    for a, b in zip(eng, bfs):
        if b.W is not None:
            np.testing.assert_array_equal(a.W.numpy(), b.W)


def test_custom_stop_programs_are_recognised():
    """The reference compiler's output for deeppoly_custom_stop.cf and custom_stops/ runs as
    DeepPoly with the program's stop depth (get_start) and its strict lower-slope test."""
    import importlib.util
    import os
    import sys
    from constraintflow.lib.flow_sparse import certifier_of, relu_is_strict, stop_depth_of
    here = os.path.dirname(os.path.abspath(__file__))
    for program, depth in (("deeppoly_custom_stop", 3), ("custom_stops/deeppoly_custom_stop00", 0),
                           ("custom_stops/deeppoly_custom_stop05", 5), ("custom_stops/deeppoly_custom_stop08", 8),
                           ("deeppoly", None), ("crownibp", None)):
        path = os.path.join(here, "golden", "generated", program, "transformers.py")
        saved = sys.modules.pop("transformers", None)
        try:
            spec = importlib.util.spec_from_file_location("transformers", path)
            mod = importlib.util.module_from_spec(spec)
            sys.modules["transformers"] = mod
            spec.loader.exec_module(mod)
            obj = getattr(mod, "crownibp" if program == "crownibp" else "deeppoly")()
            assert stop_depth_of(obj) == depth
            assert relu_is_strict(obj) == (depth is not None)
            if depth is not None:
                assert certifier_of(obj) == "deeppoly"
        finally:
            sys.modules.pop("transformers", None)
            if saved is not None:
                sys.modules["transformers"] = saved


def _load_transformer(src, clsname, tmp_path, tag):
    import importlib.util
    import sys
    path = tmp_path / f"transformers_{tag}.py"
    path.write_text(src)
    saved = sys.modules.pop("transformers", None)
    try:
        spec = importlib.util.spec_from_file_location("transformers", str(path))
        mod = importlib.util.module_from_spec(spec)
        sys.modules["transformers"] = mod
        spec.loader.exec_module(mod)
        return getattr(mod, clsname)()
    finally:
        sys.modules.pop("transformers", None)
        if saved is not None:
            sys.modules["transformers"] = saved


def _generated(program):
    import os
    here = os.path.dirname(os.path.abspath(__file__))
    with open(os.path.join(here, "golden", "generated", program, "transformers.py")) as fh:
        return fh.read()


def _relu_part(src):
    i = src.index("def Relu(")
    return src[:i], src[i:]


def test_fingerprints_of_generated_programs():
    """The table of known fingerprints is what the reference compiler's output hashes to."""
    from constraintflow.lib import program_fingerprint as PF
    import tempfile
    import pathlib
    with tempfile.TemporaryDirectory() as d:
        for program, cls, expect in (("deeppoly", "deeppoly", ("deeppoly", False)),
                                     ("deeppoly_efficient", "deeppoly", ("deeppoly", False)),
                                     ("crown", "deeppoly", ("crown", False)), ("zono", "zono", ("zono", False)),
                                     ("ibp", "ibp", ("ibp", False)), ("polyzono", "polyzono", ("polyzono", False)),
                                     ("crownibp", "crownibp", ("crownibp", False)), ("zid", "zid", ("zid", True)),
                                     ("deeppoly_custom_stop", "deeppoly", ("deeppoly", True)),
                                     ("custom_stops/deeppoly_custom_stop05", "deeppoly", ("deeppoly", True))):
            obj = _load_transformer(_generated(program), cls, pathlib.Path(d), program.replace("/", "_"))
            assert PF.KNOWN.get(PF.fingerprint(type(obj))) == expect, program


def test_dropin_recognition_survives_renaming(tmp_path):
    """The compiler's CSE variable names do not enter the fingerprint."""
    import re
    from constraintflow.lib.flow_sparse import certifier_of
    src = re.sub(r"\bcse_var_(\d+)\b", lambda m: f"tmp_{int(m.group(1)) * 7 + 3}", _generated("deeppoly"))
    assert certifier_of(_load_transformer(src, "deeppoly", tmp_path, "renamed")) == "deeppoly"


@pytest.mark.parametrize("program,cls,mistake", [
    # the lower-slope test l + u >= 0 made strict (one comparison only)
    ("deeppoly", "deeppoly", lambda a, r: (a, r.replace("operator.add, layer_index = layer_index, counter = -1, "
                                                        "inside_while = False, while_number = -1), cse_var_39, "
                                                        "operator.ge", "operator.add, layer_index = layer_index, "
                                                        "counter = -1, inside_while = False, while_number = -1), "
                                                        "cse_var_39, operator.gt", 1))),
    # a threshold: the ReLU's zero constant made 1
    ("deeppoly", "deeppoly", lambda a, r: (a, r.replace("dense_const=0.0", "dense_const=1.0", 1))),
    # a slope: u / (u - l) made u * (u - l)
    ("deeppoly", "deeppoly", lambda a, r: (a, r.replace("operator.truediv", "operator.mul", 1))),
    # the traversal: the negated layer priority made positive
    ("deeppoly", "deeppoly", lambda a, r: (a.replace("operator.neg", "operator.pos", 1), r)),
    # the sign split threshold of the backsubstitution
    ("crown", "deeppoly", lambda a, r: (a.replace("dense_const=0.0", "dense_const=0.5", 1), r)),
    # a zonotope program whose ReLU scales the fresh symbols differently
    ("zono", "zono", lambda a, r: (a, r.replace("operator.truediv", "operator.mul", 1))),
])
def test_dropin_refuses_planted_mistakes(program, cls, mistake, tmp_path):
    """A generated program that differs from a known one in a threshold, a slope, an
    operator or its traversal is refused instead of being run as the known program."""
    from constraintflow.lib.flow_sparse import certifier_of
    affine, relu = _relu_part(_generated(program))
    a2, r2 = mistake(affine, relu)
    assert (a2, r2) != (affine, relu), "the planted mistake did not change the program"
    with pytest.raises(NotImplementedError):
        certifier_of(_load_transformer(a2 + r2, cls, tmp_path, "planted"))


def test_zid_thresholds_must_agree(tmp_path):
    """zid.cf tests curr[layer] <= K in its Affine and in its Relu; a program whose two
    bounds differ is refused (each alone would be a valid parameter)."""
    from constraintflow.lib.flow_sparse import certifier_of, zid_upto_of
    affine, relu = _relu_part(_generated("zid"))
    obj = _load_transformer(affine + relu, "zid", tmp_path, "zid_ok")
    assert certifier_of(obj) == "zid" and zid_upto_of(obj) == 4
    bad = _load_transformer(affine + relu.replace("dense_const=4, type= type(4)", "dense_const=5, type= type(5)"),
                            "zid", tmp_path, "zid_bad")
    assert certifier_of(bad) == "zid"      # the bound itself is a parameter
    with pytest.raises(NotImplementedError):
        zid_upto_of(bad)
