"""Semantic fingerprints of the certifier transformers the reference compiler generates.

Flow (flow_sparse.py) runs a generated program's whole layer loop in one fused driver call,
so it must know exactly which program the generated ``Affine`` / ``Relu`` methods compute.
A fingerprint is a hash of a canonical form of the two methods' syntax trees:

* local variables are renamed in order of first assignment (the compiler's CSE names, such
  as ``cse_var_38``, do not matter);
* the JIT bookkeeping keyword arguments (``layer_index``, ``counter``, ``inside_while``,
  ``while_number``, ``while_iteration``; constraintflow/gbcsr/tensor_ops.py) are dropped;
* every other token -- operators, called functions, constants, comparison thresholds,
  slope expressions, control flow -- is kept.

The reference compiler (constraintflow/compiler/compile.py:66-97, codeGen.py) is
deterministic, so its output for a given ``.cf`` program always has the same fingerprint,
while a program that differs in a threshold, a slope, an operator or the traversal has a
different one and is refused.  The constants the runtime takes as parameters (the stop depth
``get_start`` of the custom-stop programs, zid.cf's zonotope layer bound) are replaced by a
placeholder before hashing, after ``flow_sparse`` has read them.

``KNOWN`` maps the fingerprints of the reference compiler's output for the example programs
the runtime implements (examples/compiler_examples/*.cf) to (certifier, strict lower-slope
ReLU test).
"""
import ast
import hashlib
import inspect
import re
import textwrap

JIT_KWARGS = frozenset({"layer_index", "counter", "inside_while", "while_number", "while_iteration"})

# constants read as parameters: `curr[layer] - get_start` (the custom-stop traversal) and
# `curr[layer] <= K` (zid.cf) -- a const SparseTensor compared with the layer metadata
PARAM_RE = {
    "stop_depth": re.compile(r"(curr\.get_metadata\('layer'[^)]*\), SparseTensor\(\[\], \[\], 0, torch\.tensor\(\[\]\), "
                             r"dense_const=)(\d+)(, type= type\()(\d+)(\)\)(?:\.\w+\([^()]*(?:\([^()]*\))?[^()]*\))*, "
                             r"operator\.sub)"),
    "zono_upto": re.compile(r"(curr\.get_metadata\('layer'[^)]*\), SparseTensor\(\[\], \[\], 0, torch\.tensor\(\[\]\), "
                            r"dense_const=)(\d+)(, type= type\()(\d+)(\)\)(?:\.\w+\([^()]*(?:\([^()]*\))?[^()]*\))*, "
                            r"operator\.le)"),
}
PLACEHOLDER = "CF_PARAM"


def params(source, name):
    """The values of parameter `name` found in a method's source (a set of ints)."""
    return {int(m.group(2)) for m in PARAM_RE[name].finditer(source)}


def _strip_params(source):
    for rx in PARAM_RE.values():
        source = rx.sub(lambda m: m.group(1) + PLACEHOLDER + m.group(3) + PLACEHOLDER + m.group(5), source)
    return source


class _Canon:
    """Canonical text of a function definition: locals renamed by first assignment."""

    def __init__(self, args):
        self.names = {a: f"a{i}" for i, a in enumerate(args)}

    def _bind(self, target):
        if isinstance(target, ast.Name):
            if target.id not in self.names:
                self.names[target.id] = f"v{len(self.names)}"
        elif isinstance(target, (ast.Tuple, ast.List)):
            for t in target.elts:
                self._bind(t)

    def node(self, n):
        if isinstance(n, ast.Name):
            return self.names.get(n.id, n.id)
        if isinstance(n, ast.Constant):
            return f"{type(n.value).__name__}:{n.value!r}"
        if isinstance(n, ast.keyword):
            return f"{n.arg}={self.node(n.value)}"
        if isinstance(n, ast.Call):
            kws = [k for k in n.keywords if k.arg not in JIT_KWARGS]
            return "call(" + ",".join([self.node(n.func)] + [self.node(a) for a in n.args] +
                                      [self.node(k) for k in kws]) + ")"
        if isinstance(n, (ast.Assign, ast.AugAssign, ast.AnnAssign)):
            value = self.node(n.value) if n.value is not None else ""
            targets = n.targets if isinstance(n, ast.Assign) else [n.target]
            for t in targets:
                self._bind(t)
            return f"{type(n).__name__}(" + ",".join(self.node(t) for t in targets) + "=" + value + ")"
        if isinstance(n, ast.AST):
            parts = []
            for field, value in ast.iter_fields(n):
                if isinstance(value, list):
                    parts.append(field + "[" + ";".join(self.node(v) for v in value) + "]")
                elif isinstance(value, ast.AST):
                    parts.append(field + "=" + self.node(value))
                elif value is not None:
                    parts.append(f"{field}={value!r}")
            return type(n).__name__ + "(" + ",".join(parts) + ")"
        return repr(n)


def method_canon(method):
    """Canonical text of a generated method (its source with parameters replaced)."""
    src = _strip_params(textwrap.dedent(inspect.getsource(method)))
    fn = ast.parse(src).body[0]
    c = _Canon([a.arg for a in fn.args.args])
    return ";".join(c.node(stmt) for stmt in fn.body)


def fingerprint(cls):
    """Hash of the canonical Affine and Relu of a generated transformer class."""
    h = hashlib.sha256()
    for name in ("Affine", "Relu"):
        h.update(name.encode() + b"\0" + method_canon(getattr(cls, name)).encode() + b"\0")
    return h.hexdigest()[:32]


# fingerprint -> (certifier, strict ReLU lower-slope test).  Computed from the reference
# compiler's output for each example program (recomputed by tests/test_dropin_cpu.py).
KNOWN = {
    "c217fbe3fd1f963a832e6013f2d783f6": ("deeppoly", False),   # deeppoly.cf
    "ceea1c2469eebe12b609b707ccf90586": ("deeppoly", False),   # deeppoly_efficient.cf (composes to DeepPoly)
    "ac3b8ca0aedf356c7db8b2130f918e3b": ("deeppoly", True),    # deeppoly_custom_stop.cf, custom_stops/*.cf
    "cb714628d7d0bf800962c1313610c74f": ("crown", False),      # crown.cf
    "2894fc9428996c6c2672f769a12d2619": ("crownibp", False),   # crownibp.cf
    "a4c4f34561a0a6a17c5cf2fa7e35f4fa": ("zono", False),       # zono.cf
    "4cca3f85897a5185c8842f23c8a30689": ("ibp", False),        # ibp.cf
    "2bbe373f0ca98b2c7cc83383a47fd82f": ("polyzono", False),   # polyzono.cf
    "e5770c120f0fa8994e1c40311111ad79": ("zid", True),         # zid.cf
}
