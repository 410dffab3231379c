"""The compiler backend (cfgpu.codegen) on the reference's example programs, without a GPU:
its analysis of the ASTs the reference front end built (tests/golden/ast/, made by
tests/golden/gen_codegen.py), the code it emits, its refusals, and planted mistakes in a
program that it must refuse."""
import copy
import importlib.util
import json
import os
import sys

import pytest

from cfgpu import codegen

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = os.path.join(HERE, "golden")
sys.path.insert(0, GOLDEN)
import ast_json  # noqa: E402

RUNS = {"deeppoly": "deeppoly", "deeppoly_efficient": "deeppoly", "crown": "crown", "zono": "zono", "ibp": "ibp",
        "polyzono": "polyzono", "crownibp": "crownibp", "deeppoly_custom_stop": "deeppoly"}
REFUSED = ("deeppoly_priority", "deeppolyh", "zono2", "ibp2")


def _ast(prog):
    with open(os.path.join(GOLDEN, "ast", f"{prog}.json")) as f:
        return ast_json.from_json(json.load(f))


@pytest.mark.parametrize("prog", sorted(RUNS))
def test_backend_recognises_program(prog):
    a = codegen.analyse(_ast(prog))
    assert a.certifier == RUNS[prog]
    assert a.ops["Affine"] in ("backsub", "zonotope", "interval", "backsub+zonotope", "interval+backsub",
                               "backsub-stop")
    assert a.ops["Relu"] is not None


@pytest.mark.parametrize("prog", sorted(RUNS))
def test_emitted_code_is_committed(prog):
    files = codegen.generate(_ast(prog), f"{prog}.cf")
    for name, text in files.items():
        with open(os.path.join(GOLDEN, "generated_cfgpu", prog, name)) as f:
            assert f.read() == text


@pytest.mark.parametrize("prog", REFUSED)
def test_backend_refuses_other_programs(prog):
    with pytest.raises(codegen.CodegenError):
        codegen.analyse(_ast(prog))
    refused = json.load(open(os.path.join(GOLDEN, "generated_cfgpu", "refused.json")))
    assert prog in refused and "deeppoly2" in refused and "hybrid_zono" in refused


def _funcs(ast):
    out = {}

    def walk(s):
        if type(s).__name__ == "SeqNode":
            walk(s.stmt1)
            walk(s.stmt2)
        elif type(s).__name__ == "FuncNode":
            out[s.decl.name.name] = s
    walk(ast.stmt)
    return out


@pytest.mark.parametrize("mistake", ["replace_sign", "priority_order", "relu_slope", "simplify_choice"])
def test_planted_mistakes_are_refused(mistake):
    """Mistakes planted in deeppoly.cf's AST (each changes the certifier's meaning) make the
    backend refuse the program instead of running the DeepPoly kernels."""
    ast = copy.deepcopy(_ast("deeppoly"))
    f = _funcs(ast)
    if mistake == "replace_sign":          # coefficient >= 0 substitutes U instead of L
        f["replace_lower"].expr.texpr.right.elem.name = "U"
    elif mistake == "priority_order":      # highest layer first
        f["priority2"].expr = f["priority2"].expr.expr
    elif mistake == "relu_slope":          # lower relaxation on l >= 0 instead of l + u >= 0
        f["relu_n"].expr.cond.left = f["relu_n"].expr.cond.left.left
    elif mistake == "simplify_choice":     # concretise a negative coefficient with l
        f["simplify_lower"].expr.fexpr.right.elem.name = "l"
    assert codegen.analyse(copy.deepcopy(_ast("deeppoly"))).certifier == "deeppoly"
    with pytest.raises(codegen.CodegenError) as e:
        codegen.analyse(ast)
    assert ("Relu (unrecognised)" if mistake == "relu_slope" else "Affine (unrecognised)") in str(e.value)


@pytest.mark.parametrize("prog", sorted(RUNS))
def test_emitted_transformer_declares_its_family(prog):
    from constraintflow.lib.flow_sparse import certifier_of
    path = os.path.join(GOLDEN, "generated_cfgpu", prog, "transformers.py")
    spec = importlib.util.spec_from_file_location(f"cfgpu_emitted_{prog}", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    a = codegen.analyse(_ast(prog))
    obj = getattr(mod, a.name)()
    assert obj.cf_layerwise and certifier_of(obj) == RUNS[prog]


def _nodes(n, kind, out=None):
    """Every node of class `kind` under n (depth first)."""
    out = [] if out is None else out
    if type(n).__name__ == kind:
        out.append(n)
    if isinstance(n, (list, tuple)):
        for x in n:
            _nodes(x, kind, out)
    elif hasattr(n, "__dict__"):
        for k, v in vars(n).items():
            if k not in ("left", "right") or not hasattr(n, "texpr"):
                _nodes(v, kind, out)
    return out


@pytest.mark.parametrize("mistake", ["meet_direction", "zono_sign", "zono_relu_scale"])
def test_planted_polyzono_mistakes_are_refused(mistake):
    """Mistakes planted in polyzono.cf's AST make the backend refuse it: the lower bound
    met with min instead of max; the zonotope's lower concretisation with +|c|; the
    fresh-symbol coefficient of the zonotope ReLU halved once more."""
    ast = copy.deepcopy(_ast("polyzono"))
    f = _funcs(ast)
    if mistake == "meet_direction":
        meets = [m for m in _nodes(ast.stmt, "MaxOpNode") if m.op == "max"]
        assert meets
        meets[0].op = "min"
    elif mistake == "zono_sign":           # deepz_lower(c) = c > 0 ? c * 1 : c * 1
        f["deepz_lower"].expr.texpr = f["deepz_lower"].expr.fexpr
    elif mistake == "zono_relu_scale":     # x(l, u, z): (u l (eps - 1)) / (4 (u - l))
        f["x"].expr.right.right.left.value = 4
    assert codegen.analyse(copy.deepcopy(_ast("polyzono"))).certifier == "polyzono"
    with pytest.raises(codegen.CodegenError) as e:
        codegen.analyse(ast)
    assert ("Relu (unrecognised)" if mistake == "zono_relu_scale" else "Affine (unrecognised)") in str(e.value)


@pytest.mark.parametrize("mistake", ["interval_sign", "last_layer_test", "property_replace"])
def test_planted_crownibp_mistakes_are_refused(mistake):
    """Mistakes planted in crownibp.cf's AST make the backend refuse it: the interval lower
    bound concretising a positive coefficient with u; the branch taken for a layer other
    than the last one; the property traversal substituting U for a positive coefficient
    of the lower bound."""
    ast = copy.deepcopy(_ast("crownibp"))
    f = _funcs(ast)
    if mistake == "interval_sign":         # simplify_lower(n, c) = c >= 0 ? n[u] * c : c * n[u]
        f["simplify_lower"].expr.texpr.left.elem.name = "u"
    elif mistake == "last_layer_test":     # curr[last_layer] == 0
        _nodes(ast.stmt, "TransRetIfNode")[0].cond.right.value = 0
    elif mistake == "property_replace":    # replace_lower(n, c) = c >= 0 ? c * n[U] : c * n[U]
        f["replace_lower"].expr.texpr.right.elem.name = "U"
    assert codegen.analyse(copy.deepcopy(_ast("crownibp"))).certifier == "crownibp"
    with pytest.raises(codegen.CodegenError) as e:
        codegen.analyse(ast)
    assert "Affine (unrecognised)" in str(e.value)


def test_custom_stop_depth_and_strict_relu():
    """deeppoly_custom_stop.cf: the traversal stops get_start = 3 layers down and relu_n tests
    l + u > 0; the emitted transformer declares both.  With the stop's comparison planted
    the other way (the top layers stop instead) the backend refuses the program."""
    a = codegen.analyse(_ast("deeppoly_custom_stop"))
    assert (a.certifier, a.stop_depth, a.relu_strict) == ("deeppoly", 3, True)
    text = codegen.generate(_ast("deeppoly_custom_stop"))["transformers.py"]
    assert "cf_stop_depth = 3" in text and "cf_relu_strict = True" in text
    plain = codegen.analyse(_ast("deeppoly"))
    assert (plain.stop_depth, plain.relu_strict) == (None, False)
    ast = copy.deepcopy(_ast("deeppoly_custom_stop"))
    f = _funcs(ast)
    f["stop_traverse"].expr.op = ">"
    with pytest.raises(codegen.CodegenError) as e:
        codegen.analyse(ast)
    assert "Affine (unrecognised)" in str(e.value)
