"""Runs cfgpu.codegen (the compiler backend) on the reference's example certifier programs.

Test infrastructure.  It runs only where the reference checkout (REF_ROOT) is present;
the GPU box never runs it.  For every program of examples/compiler_examples/ listed in
PROGRAMS it
  1. parses and type-checks the .cf file with the REFERENCE front end
     (constraintflow/ast_cflow: lexer, parser, astBuilder, astTC; the ANTLR v3-ATN shim of
     tests/golden/refshim as for gen_golden.py);
  2. stores the AST as JSON under tests/golden/ast/<program>.json (class name and fields of
     every node), so that the backend's analysis is tested without the reference;
  3. hands the AST to cfgpu.codegen: the emitted main.py / transformers.py go to
     tests/golden/generated_cfgpu/<program>/, or the refusal is recorded in
     tests/golden/generated_cfgpu/refused.json.

    python tests/golden/gen_codegen.py
"""
import importlib.util
import json
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
REF_ROOT = os.environ.get("CF_REFERENCE_ROOT", "")
PKG = os.path.join(REPO, "constraintflow-gpu_b200")
# the programs the backend runs, then programs it must refuse (other traversal order,
# ReLU relaxation or domain), then programs the reference front end itself refuses
PROGRAMS = ("deeppoly", "deeppoly_efficient", "crown", "zono", "ibp", "polyzono", "crownibp", "deeppoly_custom_stop",
            "deeppoly_priority", "deeppolyh", "zono2", "ibp2",
            "deeppoly2", "hybrid_zono")


def to_json(n):
    """Generic AST -> JSON: objects become {'_': class name, field: value}."""
    if isinstance(n, (list, tuple)):
        return {"_list": [to_json(x) for x in n], "_tuple": isinstance(n, tuple)}
    if isinstance(n, (str, int, float, bool)) or n is None:
        return n
    if hasattr(n, "__dict__"):
        out = {"_": type(n).__name__}
        for k, v in vars(n).items():
            if k in ("left", "right") and hasattr(n, "texpr"):
                continue
            out[k] = to_json(v)
        return out
    return repr(n)


def worker(out_json):
    sys.path.insert(0, os.path.join(HERE, "refshim", "stubs"))
    sys.path.insert(0, os.path.join(HERE, "refshim"))
    sys.path.insert(0, REF_ROOT)
    import antlr_v3_shim  # noqa: F401
    import antlr4 as antlr
    from constraintflow.ast_cflow import dslLexer, dslParser, astBuilder, astTC
    res = {}
    for prog in PROGRAMS:
        path = os.path.join(REF_ROOT, "examples", "compiler_examples", f"{prog}.cf")
        try:
            lexer = dslLexer.dslLexer(antlr.FileStream(path))
            tree = dslParser.dslParser(antlr.CommonTokenStream(lexer)).prog()
            ast = astBuilder.ASTBuilder().visit(tree)
            astTC.ASTTC().visit(ast)
            res[prog] = to_json(ast)
        except Exception as e:  # the reference front end refuses the program
            res[prog] = {"_front_end_error": f"{type(e).__name__}: {e}"}
    with open(out_json, "w") as f:
        json.dump(res, f)


def main():
    if not REF_ROOT or not os.path.isdir(os.path.join(REF_ROOT, "constraintflow")):
        sys.exit("set CF_REFERENCE_ROOT to the reference checkout (the directory holding constraintflow/)")
    import tempfile
    with tempfile.TemporaryDirectory() as tmp:
        out = os.path.join(tmp, "asts.json")
        code = "import sys; sys.path.insert(0, %r); import gen_codegen as g; g.worker(%r)" % (HERE, out)
        subprocess.run([sys.executable, "-c", code], cwd=tmp, check=True)
        asts = json.load(open(out))
    os.makedirs(os.path.join(HERE, "ast"), exist_ok=True)
    spec = importlib.util.spec_from_file_location("cfgpu_codegen", os.path.join(PKG, "cfgpu", "codegen.py"))
    cg = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(cg)
    sys.path.insert(0, HERE)
    import ast_json
    refused = {}
    for prog, tree in asts.items():
        if "_front_end_error" in tree:
            refused[prog] = "reference front end: " + tree["_front_end_error"]
            continue
        with open(os.path.join(HERE, "ast", f"{prog}.json"), "w") as f:
            json.dump(tree, f, indent=None, separators=(",", ":"))
        try:
            cg.write(ast_json.from_json(tree), os.path.join(HERE, "generated_cfgpu", prog), f"{prog}.cf")
            print(prog, "->", cg.analyse(ast_json.from_json(tree)).certifier)
        except cg.CodegenError as e:
            refused[prog] = str(e)
            print(prog, "refused:", e)
    with open(os.path.join(HERE, "generated_cfgpu", "refused.json"), "w") as f:
        json.dump(refused, f, indent=1, sort_keys=True)


if __name__ == "__main__":
    main()
