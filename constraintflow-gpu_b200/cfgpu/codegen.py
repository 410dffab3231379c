"""Compiler backend for ConstraintFlow programs: emits Python that runs every transformer
operation as one fused libcfgpu call per layer, in place of the tensor_ops loop the
reference's code generator writes (constraintflow/compiler/codeGen.py).

Input: the program's AST as the reference front end builds it (ast_cflow/astBuilder.py,
type-checked by astTC.py) -- nodes are read by their class names and fields, so the
reference need not be importable here.  The backend decides, by evaluating the program's
own definitions, which fused kernel family implements each transformer operation:

  Affine  backsubstitution  members map(traverse(E; backward, P, S, R), G) for the bounds
                            and E, E for the linear expressions, E = prev . weight + bias,
                            with P ordering the lowest layer first, S never stopping,
                            R choosing L / U and G choosing l / u by the coefficient sign
          zonotope          map(Ez, g_low), map(Ez, g_up), Ez with Ez = prev[Z] . weight +
                            bias and g_low(c) = -|c|, g_up(c) = |c|
          interval          map(E, G_low), map(E, G_up) without a traversal
          backsubstitution  max(zonotope low, backsubstitution low), min(... up), E, E, Ez
          + zonotope        over the shape (l, u, L, U, Z) (polyzono.cf), either order
          backsubstitution  the backsubstitution tuple with S(n1, c) = n1[layer] < curr[layer] - d
          stopped           (the custom-stop programs): the traversal stops d layers down
          interval, then    curr[last_layer] == 1 ? backsubstitution tuple : (map(E, G_low),
          backsubstitution  map(E, G_up), E, E) (crownibp.cf); its traversal may take the
                            highest layer first (the runtime runs it on chains, where the
                            order does not change the bounds)
  Relu    DeepPoly          (relu(l), relu(u), 1[l+u>=0] x, l>=0 ? x : u<=0 ? 0 :
                            lam (x - l)), lam = u/(u-l), x the neuron (prev, prev[L] and
                            prev[U] all denote the affine input of the ReLU)
          CROWN             if l>=0 pass-through, elif u<=0 zero, else the all-crossing
                            tuple (whole-layer branches, crown.cf:25)
          zonotope          (0, 0, l>=0 ? Z : u<=0 ? 0 : lam Z + (u l / (2 (u-l))) (eps-1))
          DeepPoly, strict  the same with the lower slope where l + u > 0 (custom-stop programs)
          interval          (relu(l), relu(u))
          DeepPoly          DeepPoly's four members followed by the zonotope's Z member
          + zonotope        over the shape (l, u, L, U, Z)

Each candidate is checked on sample bounds (l, u) with exact arithmetic on affine forms
over the symbols x, L, U, Z, eps; a program whose operations match no family is refused
(CodegenError).  The emitted ``transformers.py`` declares the family (cf_certifier) and
calls cfgpu.layerwise per layer; ``main.py`` keeps the reference's ``run(...)`` signature
(codeGen.py:35), so ``constraintflow run`` drives it unchanged.
"""
import os

__all__ = ["CodegenError", "analyse", "generate", "write"]


class CodegenError(Exception):
    pass


# ------------------------------------------------------------------ values
class Form:
    """An affine form sum_s coef[s] * s + const over symbolic names."""

    def __init__(self, terms=None, const=0.0):
        self.t = {k: float(v) for k, v in (terms or {}).items() if v != 0}
        self.c = float(const)

    @staticmethod
    def of(v):
        return v if isinstance(v, Form) else Form({}, v)

    def __add__(self, o):
        o = Form.of(o)
        t = dict(self.t)
        for k, v in o.t.items():
            t[k] = t.get(k, 0.0) + v
        return Form(t, self.c + o.c)

    __radd__ = __add__

    def __neg__(self):
        return Form({k: -v for k, v in self.t.items()}, -self.c)

    def __sub__(self, o):
        return self + (-Form.of(o))

    def __rsub__(self, o):
        return Form.of(o) - self

    def scale(self, s):
        return Form({k: v * s for k, v in self.t.items()}, self.c * s)

    def merged(self, names, into):
        t = {}
        for k, v in self.t.items():
            key = into if k in names else k
            t[key] = t.get(key, 0.0) + v
        return Form(t, self.c)

    def close(self, o, tol=1e-9):
        o = Form.of(o)
        keys = set(self.t) | set(o.t)
        scale = 1.0 + abs(self.c) + sum(abs(v) for v in self.t.values())
        return abs(self.c - o.c) <= tol * scale and all(
            abs(self.t.get(k, 0.0) - o.t.get(k, 0.0)) <= tol * scale for k in keys)

    def __repr__(self):
        return " + ".join([f"{v:g}*{k}" for k, v in sorted(self.t.items())] + [f"{self.c:g}"])


class Neuron:
    """A neuron of the sample: its bounds and the symbols of its expressions."""

    def __init__(self, l, u, layer=1, sym="x"):
        self.l, self.u, self.layer, self.sym = l, u, layer, sym

    def element(self, name):
        if name == "l":
            return self.l
        if name == "u":
            return self.u
        if name in ("L", "U", "Z"):
            return Form({name if self.sym == "x" else f"{self.sym}.{name}": 1.0})
        raise CodegenError(f"unknown shape member {name!r}")

    def form(self):
        return Form({self.sym: 1.0})


class Opaque:
    """A value the evaluator does not model (a traversal, a dot product, ...)."""

    def __init__(self, node):
        self.node = node


def _val(v):
    return v.form() if isinstance(v, Neuron) else v


# ------------------------------------------------------------------ AST helpers
def _kind(n):
    return type(n).__name__


def _name(n):
    return n.name if _kind(n) == "VarNode" else str(n)


def _statements(stmt, out):
    if _kind(stmt) == "SeqNode":
        _statements(stmt.stmt1, out)
        _statements(stmt.stmt2, out)
    else:
        out.append(stmt)
    return out


class _Program:
    def __init__(self, ast):
        if _kind(ast) != "ProgramNode":
            raise CodegenError(f"expected a ProgramNode, got {_kind(ast)}")
        self.shape = [(_type_name(t), _name(v)) for t, v in ast.shape.elements.arglist]
        self.funcs, self.transformers, self.flows = {}, {}, []
        for s in _statements(ast.stmt, []):
            k = _kind(s)
            if k == "FuncNode":
                args = [_name(v) for _, v in s.decl.arglist.arglist]
                self.funcs[_name(s.decl.name)] = (args, s.expr)
            elif k == "TransformerNode":
                self.transformers[_name(s.name)] = {o.op.op_name: o.ret for o in s.oplist.olist}
            elif k == "FlowNode":
                self.flows.append(s)


def _type_name(t):
    return getattr(t, "name", str(t))


# ------------------------------------------------------------------ evaluator
class _Eval:
    """Evaluates an expression with numbers, booleans and affine forms."""

    def __init__(self, prog, env):
        self.prog, self.env = prog, env

    def call(self, fname, args):
        if fname not in self.prog.funcs:
            raise CodegenError(f"unknown function {fname!r}")
        params, body = self.prog.funcs[fname]
        if len(params) != len(args):
            raise CodegenError(f"{fname}: {len(args)} arguments for {len(params)} parameters")
        return _Eval(self.prog, dict(zip(params, args))).ev(body)

    def ev(self, n):
        k = _kind(n)
        if k in ("ConstIntNode", "ConstFloatNode"):
            return float(n.value)
        if k == "ConstBoolNode":
            return bool(n.value) if not isinstance(n.value, str) else n.value == "True"
        if k == "VarNode":
            if n.name in self.env:
                return self.env[n.name]
            raise CodegenError(f"free variable {n.name!r}")
        if k == "EpsilonNode":
            return Form({"eps": 1.0})
        if k == "GetElementNode":
            base = self.ev(n.expr)
            if not isinstance(base, Neuron):
                raise CodegenError("element access of a non-neuron")
            return base.element(_name(n.elem))
        if k == "GetMetadataNode":
            base = self.ev(n.expr)
            meta = getattr(n.metadata, "name", None) or _name(n.metadata)
            if isinstance(base, Neuron) and meta == "layer":
                return float(base.layer)
            return Opaque(n)
        if k == "UnOpNode":
            v = _val(self.ev(n.expr))
            if n.op == "-":
                return -v
            if n.op in ("not", "!", "~") and isinstance(v, bool):
                return not v
            raise CodegenError(f"unary {n.op!r}")
        if k == "BinOpNode":
            return self.binop(n.op, self.ev(n.left), self.ev(n.right))
        if k in ("TernaryNode", "IfNode"):
            c = self.ev(n.cond)
            if not isinstance(c, bool):
                raise CodegenError("condition is not a boolean")
            return self.ev(n.texpr if c else n.fexpr)
        if k == "FuncCallNode":
            return self.call(_name(n.name), [self.ev(a) for a in n.arglist.exprlist])
        if k == "MapNode":
            return self.map(self.ev(n.expr), _name(n.func))
        return Opaque(n)

    def binop(self, op, a, b):
        a, b = _val(a), _val(b)
        if op in ("and", "or"):
            if not (isinstance(a, bool) and isinstance(b, bool)):
                raise CodegenError(f"{op} of non-booleans")
            return (a and b) if op == "and" else (a or b)
        if isinstance(a, Opaque) or isinstance(b, Opaque):
            raise CodegenError("arithmetic on an unmodelled value")
        if op in ("<", "<=", ">", ">=", "==", "!="):
            if isinstance(a, Form) or isinstance(b, Form):
                raise CodegenError("comparison of symbolic expressions")
            return {"<": a < b, "<=": a <= b, ">": a > b, ">=": a >= b, "==": a == b, "!=": a != b}[op]
        if op == "+":
            return Form.of(a) + b if isinstance(a, Form) or isinstance(b, Form) else a + b
        if op == "-":
            return Form.of(a) - b if isinstance(a, Form) or isinstance(b, Form) else a - b
        if op == "*":
            if isinstance(a, Form) and isinstance(b, Form):
                raise CodegenError("product of symbolic expressions")
            if isinstance(a, Form):
                return a.scale(b)
            if isinstance(b, Form):
                return b.scale(a)
            return a * b
        if op == "/":
            if isinstance(b, Form):
                raise CodegenError("division by a symbolic expression")
            return a.scale(1.0 / b) if isinstance(a, Form) else a / b
        raise CodegenError(f"operator {op!r}")

    def map(self, v, fname):
        """map(e, f) over a polyexp with a single neuron symbol s: f(neuron s, coefficient)."""
        if not isinstance(v, Form) or len(v.t) != 1 or v.c != 0.0:
            raise CodegenError("map over an expression the evaluator does not model")
        (sym, coef), = v.t.items()
        res = self.call(fname, [Neuron(1.0, 2.0, sym=f"{sym}"), coef])
        return _val(res)


# ------------------------------------------------------------------ recognisers
_SAMPLES = [(0.5, 2.0), (-2.0, -0.5), (-1.0, 3.0), (-3.0, 1.0), (-1.0, 1.0), (0.0, 1.5), (-1.5, 0.0),
            (0.25, 0.75)]


def _ret_tuple(ret):
    if _kind(ret) != "TransRetBasicNode":
        return None
    return list(ret.exprlist.exprlist)


def _close(a, b):
    if isinstance(a, bool) or isinstance(b, bool):
        return a == b
    return Form.of(_val(a)).close(Form.of(_val(b)))


def _relu_env(l, u):
    return {"prev": Neuron(l, u, layer=2), "curr": Neuron(0.0, 0.0, layer=3)}


def _check_relu_basic(prog, ret, expect, merge):
    """Every sample: the tuple evaluates to expect(l, u) member by member."""
    exprs = _ret_tuple(ret)
    if exprs is None or len(exprs) != len(prog.shape):
        return False
    for l, u in _SAMPLES:
        want = expect(l, u)
        ev = _Eval(prog, _relu_env(l, u))
        for e, w in zip(exprs, want):
            got = _val(ev.ev(e))
            if isinstance(got, Opaque):
                return False
            if merge and isinstance(got, Form):
                got = got.merged(("x", "L", "U"), "x")
            if not _close(got, w):
                return False
    return True


def _deeppoly_relu(l, u):
    x = Form({"x": 1.0})
    lu = l + u >= 0.0
    if l >= 0.0:
        up = x
    elif u <= 0.0:
        up = Form()
    else:
        lam = u / (u - l)
        up = x.scale(lam) - lam * l
    return [max(l, 0.0), max(u, 0.0), x if lu else Form(), up]


def _deeppoly_relu_strict(l, u):
    """DeepPoly's Relu with relu_n testing l + u > 0 (the custom-stop programs)."""
    out = _deeppoly_relu(l, u)
    if l + u == 0.0:
        out[2] = Form()
    return out


def _zono_relu(l, u):
    z = Form({"Z": 1.0})
    if l >= 0.0:
        zz = z
    elif u <= 0.0:
        zz = Form()
    else:
        zz = z.scale(u / (u - l)) + Form({"eps": 1.0}, -1.0).scale(u * l / (2.0 * (u - l)))
    return [0.0, 0.0, zz]


def _ibp_relu(l, u):
    return [max(l, 0.0), max(u, 0.0)]


def _check_crown_relu(prog, ret):
    """if l>=0 (prev as is) elif u<=0 (zeros) else the all-crossing tuple, as whole-layer
    branches (TransRetIfNode)."""
    if _kind(ret) != "TransRetIfNode" or _kind(ret.fret) != "TransRetIfNode":
        return False
    t_pass, t_zero, t_cross = _ret_tuple(ret.tret), _ret_tuple(ret.fret.tret), _ret_tuple(ret.fret.fret)
    if None in (t_pass, t_zero, t_cross) or any(len(t) != 4 for t in (t_pass, t_zero, t_cross)):
        return False
    for l, u in _SAMPLES:
        ev = _Eval(prog, _relu_env(l, u))
        if ev.ev(ret.cond) != (l >= 0.0) or ev.ev(ret.fret.cond) != (u <= 0.0):
            return False
        want_pass = [l, u, Form({"L": 1.0}), Form({"U": 1.0})]
        if not all(_close(ev.ev(e), w) for e, w in zip(t_pass, want_pass)):
            return False
        if not all(_close(ev.ev(e), 0.0) for e in t_zero):
            return False
        if u - l == 0.0:
            continue
        c = (0.0 - l) > u
        lam = u / (u - l)
        want_cross = [0.0 if c else l, u, Form() if c else Form({"x": 1.0}),
                      Form({"U.U": lam}, (u * -1.0) * l / (u - l))]
        got = [_val(ev.ev(e)) for e in t_cross]
        # map(prev[U], replace_upper): prev[U]'s neurons replaced by their U (coefficient
        # >= 0); the sample coefficient is 1, so U.U
        if not all(_close(g, w) for g, w in zip(got, want_cross)):
            return False
    return True


def _affine_expr_ok(prog, n, member):
    """n is `prev<member> . curr[weight] + curr[bias]` (member '' for the neuron itself)."""
    if _kind(n) != "BinOpNode" or n.op != "+":
        return False
    d, b = n.left, n.right
    if _kind(d) != "DotNode" or _kind(b) != "GetMetadataNode":
        return False
    if getattr(b.metadata, "name", None) != "bias" or getattr(d.right, "metadata", None) is None:
        return False
    if getattr(d.right.metadata, "name", None) != "weight":
        return False
    left = d.left
    if member:
        return _kind(left) == "GetElementNode" and _name(left.expr) == "prev" and _name(left.elem) == member
    return _kind(left) == "VarNode" and left.name == "prev"


def _inline_call(prog, n):
    """A call of a program function with expression arguments, inlined one level."""
    while _kind(n) == "FuncCallNode" and _name(n.name) in prog.funcs:
        params, body = prog.funcs[_name(n.name)]
        n = _Subst(dict(zip(params, n.arglist.exprlist))).apply(body)
    return n


class _Subst:
    def __init__(self, m):
        self.m = m

    def apply(self, n):
        if _kind(n) == "VarNode" and n.name in self.m:
            return self.m[n.name]
        if not hasattr(n, "__dict__"):
            return n
        clone = object.__new__(type(n))
        for k, v in vars(n).items():
            if isinstance(v, list):
                v = [self.apply(x) for x in v]
            elif hasattr(v, "__dict__"):
                v = self.apply(v)
            setattr(clone, k, v)
        if hasattr(clone, "texpr"):
            clone.left, clone.right = clone.texpr, clone.fexpr
        return clone


def _sign_choice(prog, fname, pos, neg):
    """f(neuron, c) is c*pos for c >= 0 and c*neg for c < 0 (pos/neg: 'l', 'u', 'L', 'U')."""
    for c, want in ((2.0, pos), (-3.0, neg)):
        n = Neuron(-1.0, 4.0, sym="n")
        got = _val(_Eval(prog, {}).call(fname, [n, c]))
        w = n.element(want)
        w = Form.of(w).scale(c)
        if not _close(got, w):
            return False
    return True


_BAD = object()


def _stop_depth(prog, stop):
    """None when the traversal's stop is false for every neuron; d when it is a partial
    application stop_f(curr-dependent arguments) whose value for a neuron n1 is
    n1[layer] < curr[layer] - d (the custom-stop programs, deeppoly_custom_stop.cf:12-17);
    _BAD otherwise."""
    if _kind(stop) == "VarNode":
        return None if _Eval(prog, {}).call(_name(stop), [Neuron(0, 1, layer=1), 1.0]) is False else _BAD
    if _kind(stop) != "FuncCallNode":
        return _BAD
    depths = set()
    for K in (200, 233):   # layers of the bounded neuron; depths below K are identified
        bound = [_val(_Eval(prog, {"curr": Neuron(0, 1, layer=float(K))}).ev(a)) for a in stop.arglist.exprlist]
        flags = [_Eval(prog, {}).call(_name(stop.name), bound + [Neuron(0, 1, layer=float(L)), 1.0])
                 for L in range(K)]
        if not all(isinstance(f, bool) for f in flags):
            return _BAD
        d = K - sum(flags)
        if flags != [L < K - d for L in range(K)]:
            return _BAD
        depths.add(d)
    if len(depths) != 1:
        return _BAD
    return int(depths.pop())


def _check_backsub_member(prog, n, lower, any_order=False, depth_out=None):
    """n is map(traverse(E; backward, P, S, R), G) with E = prev . weight + bias, P taking
    the lowest layer first (or either order with any_order), R / G choosing L / U and l / u
    by the coefficient sign, and S never stopping -- or, when depth_out is given, stopping
    below curr[layer] - d (d appended to depth_out)."""
    n = _inline_call(prog, n)
    if _kind(n) != "MapNode" or _kind(n.expr) != "TraverseNode":
        return False
    t = n.expr
    if getattr(t.direction, "value", None) != "backward" or not _affine_expr_ok(prog, t.expr, ""):
        return False
    ev = _Eval(prog, {})
    # the lowest layer first: priority decreases with the layer index
    p1 = ev.call(_name(t.priority), [Neuron(0, 1, layer=1), 1.0])
    p2 = ev.call(_name(t.priority), [Neuron(0, 1, layer=2), 1.0])
    if not (isinstance(p1, float) and isinstance(p2, float) and (p1 > p2 or (any_order and p1 < p2))):
        return False
    depth = _stop_depth(prog, t.stop)
    if depth is _BAD or (depth is not None and depth_out is None):
        return False
    if depth_out is not None:
        depth_out.append(depth)
    pos, neg = ("L", "U") if lower else ("U", "L")
    bpos, bneg = ("l", "u") if lower else ("u", "l")
    return _sign_choice(prog, _name(t.func), pos, neg) and _sign_choice(prog, _name(n.func), bpos, bneg)


def _abs_map(prog, fname, sign):
    for c in (2.0, -3.0):
        got = _Eval(prog, {}).call(fname, [Neuron(0, 1, sym="eps"), c])
        if not _close(got, sign * abs(c)):
            return False
    return True


def _zono_bound(prog, n, lower):
    """n is map(prev[Z] . weight + bias, g) with g(c) = -|c| (lower) or |c| (upper)."""
    m = _inline_call(prog, n)
    return (_kind(m) == "MapNode" and _affine_expr_ok(prog, m.expr, "Z")
            and _abs_map(prog, _name(m.func), -1.0 if lower else 1.0))


def _met_bound(prog, n, lower):
    """n is max (lower) / min (upper) of the zonotope bound and the backsubstitution bound."""
    n = _inline_call(prog, n)
    if _kind(n) != "MaxOpNode" or getattr(n, "op", None) != ("max" if lower else "min"):
        return False
    a, b = n.expr1, n.expr2
    return any(_zono_bound(prog, x, lower) and _check_backsub_member(prog, y, lower) for x, y in ((a, b), (b, a)))


def _is_last_layer_test(n):
    """n is curr[last_layer] == 1."""
    return (_kind(n) == "BinOpNode" and n.op == "==" and _kind(n.left) == "GetMetadataNode"
            and _name(n.left.expr) == "curr" and getattr(n.left.metadata, "name", None) == "last_layer"
            and _kind(n.right) in ("ConstIntNode", "ConstFloatNode") and float(n.right.value) == 1.0)


def _classify_interval_then_backsub(prog, ret):
    """curr[last_layer] == 1 ? (backsubstitution bounds, E, E) : (map(E, G_low), map(E, G_up),
    E, E) over the shape (l, u, L, U)."""
    if [m for _, m in prog.shape] != ["l", "u", "L", "U"] or not _is_last_layer_test(ret.cond):
        return None
    t, f = _ret_tuple(ret.tret), _ret_tuple(ret.fret)
    if t is None or f is None or len(t) != 4 or len(f) != 4:
        return None
    if not (_check_backsub_member(prog, t[0], True, any_order=True)
            and _check_backsub_member(prog, t[1], False, any_order=True)
            and _affine_expr_ok(prog, t[2], "") and _affine_expr_ok(prog, t[3], "")):
        return None
    m0, m1 = _inline_call(prog, f[0]), _inline_call(prog, f[1])
    if (_kind(m0) == "MapNode" and _kind(m1) == "MapNode" and _affine_expr_ok(prog, m0.expr, "")
            and _affine_expr_ok(prog, m1.expr, "") and _sign_choice(prog, _name(m0.func), "l", "u")
            and _sign_choice(prog, _name(m1.func), "u", "l") and _affine_expr_ok(prog, f[2], "")
            and _affine_expr_ok(prog, f[3], "")):
        return "interval+backsub"
    return None


def _classify_affine(prog, ret):
    if _kind(ret) == "TransRetIfNode":
        return _classify_interval_then_backsub(prog, ret)
    exprs = _ret_tuple(ret)
    if exprs is None or len(exprs) != len(prog.shape):
        return None
    names = [m for _, m in prog.shape]
    if names == ["l", "u", "L", "U", "Z"]:
        if (_met_bound(prog, exprs[0], True) and _met_bound(prog, exprs[1], False)
                and _affine_expr_ok(prog, exprs[2], "") and _affine_expr_ok(prog, exprs[3], "")
                and _affine_expr_ok(prog, exprs[4], "Z")):
            return "backsub+zonotope"
        return None
    if names == ["l", "u", "L", "U"]:
        depths = []
        if (_check_backsub_member(prog, exprs[0], True, depth_out=depths)
                and _check_backsub_member(prog, exprs[1], False, depth_out=depths)
                and _affine_expr_ok(prog, exprs[2], "") and _affine_expr_ok(prog, exprs[3], "")
                and depths[0] == depths[1]):
            if depths[0] is None:
                return "backsub"
            prog.stop_depth = depths[0]
            return "backsub-stop"
        return None
    if names == ["l", "u", "Z"]:
        if (_zono_bound(prog, exprs[0], True) and _zono_bound(prog, exprs[1], False)
                and _affine_expr_ok(prog, exprs[2], "Z")):
            return "zonotope"
        return None
    if names == ["l", "u"]:
        m0, m1 = _inline_call(prog, exprs[0]), _inline_call(prog, exprs[1])
        if (_kind(m0) == "MapNode" and _kind(m1) == "MapNode" and _affine_expr_ok(prog, m0.expr, "")
                and _affine_expr_ok(prog, m1.expr, "") and _sign_choice(prog, _name(m0.func), "l", "u")
                and _sign_choice(prog, _name(m1.func), "u", "l")):
            return "interval"
    return None


def _classify_relu(prog, ret):
    names = [m for _, m in prog.shape]
    try:
        if names == ["l", "u", "L", "U"]:
            if _kind(ret) == "TransRetIfNode":
                return "crown" if _check_crown_relu(prog, ret) else None
            if _check_relu_basic(prog, ret, _deeppoly_relu, merge=True):
                return "deeppoly"
            return "deeppoly-strict" if _check_relu_basic(prog, ret, _deeppoly_relu_strict, merge=True) else None
        if names == ["l", "u", "Z"]:
            return "zonotope" if _check_relu_basic(prog, ret, _zono_relu, merge=False) else None
        if names == ["l", "u", "L", "U", "Z"]:
            both = _check_relu_basic(prog, ret, lambda l, u: _deeppoly_relu(l, u) + _zono_relu(l, u)[2:], merge=True)
            return "deeppoly+zonotope" if both else None
        if names == ["l", "u"]:
            return "interval" if _check_relu_basic(prog, ret, _ibp_relu, merge=False) else None
    except (CodegenError, ZeroDivisionError):
        return None
    return None


# certifier = (Affine family, Relu family)
_CERTIFIERS = {("backsub", "deeppoly"): "deeppoly", ("backsub", "crown"): "crown",
               ("zonotope", "zonotope"): "zono", ("interval", "interval"): "ibp",
               ("backsub+zonotope", "deeppoly+zonotope"): "polyzono", ("interval+backsub", "deeppoly"): "crownibp",
               ("backsub", "deeppoly-strict"): "deeppoly", ("backsub-stop", "deeppoly"): "deeppoly",
               ("backsub-stop", "deeppoly-strict"): "deeppoly"}


class Analysis:
    def __init__(self, name, certifier, shape, ops, stop_depth=None, relu_strict=False):
        self.name, self.certifier, self.shape, self.ops = name, certifier, shape, ops
        self.stop_depth, self.relu_strict = stop_depth, relu_strict


def analyse(ast):
    """The program's transformer and the fused kernel family of each of its operations."""
    prog = _Program(ast)
    if len(prog.transformers) != 1 or len(prog.flows) != 1:
        raise CodegenError("expected one transformer and one flow statement")
    flow = prog.flows[0]
    if getattr(flow.direction, "value", flow.direction) != "forward":
        raise CodegenError("only forward flows are run layer by layer")
    (name, ops), = prog.transformers.items()
    if _name(flow.trans) != name:
        raise CodegenError(f"flow runs {_name(flow.trans)!r}, the program defines {name!r}")
    if "Affine" not in ops or "Relu" not in ops:
        raise CodegenError("the transformer needs Affine and Relu operations")
    try:
        affine = _classify_affine(prog, ops["Affine"])
    except (CodegenError, ZeroDivisionError):
        affine = None
    relu = _classify_relu(prog, ops["Relu"])
    cert = _CERTIFIERS.get((affine, relu))
    if cert is None:
        raise CodegenError(f"transformer {name!r}: Affine ({affine or 'unrecognised'}) and Relu "
                           f"({relu or 'unrecognised'}) match no fused kernel family of libcfgpu")
    kinds = {"Affine": affine, "Relu": relu}
    for op in ops:
        kinds.setdefault(op, None)
    return Analysis(name, cert, prog.shape, kinds, stop_depth=getattr(prog, "stop_depth", None)
                    if affine == "backsub-stop" else None, relu_strict=relu == "deeppoly-strict")


# ------------------------------------------------------------------ emission
_SIG = ("self, abs_elem, prev, curr, poly_size, curr_size, prev_size, input_size, batch_size, "
        "layer_index=None")

_DOC = {"backsub": "backsubstitution of the layer's coefficient rows down to the input box",
        "zonotope": "zonotope step: symbol coefficients times the weights, concretised",
        "interval": "interval step: sign-split weights against the previous bounds",
        "deeppoly": "DeepPoly triangle relaxation", "crown": "CROWN whole-layer branches",
        "backsub+zonotope": "backsubstitution and zonotope step, bounds met (max / min)",
        "deeppoly+zonotope": "DeepPoly and zonotope relaxations from the met bounds",
        "interval+backsub": "interval bound; backsubstitution for the property layer only",
        "backsub-stop": "backsubstitution stopped below curr[layer] - get_start, concretised there",
        "deeppoly-strict": "DeepPoly triangle relaxation, lower slope where l + u > 0",
        None: "no fused kernel"}


def generate(ast, source_name="program.cf"):
    """{'transformers.py': ..., 'main.py': ...} for the program."""
    a = analyse(ast)
    lines = [f"# Generated by cfgpu.codegen from {source_name}: transformer {a.name!r}, certifier "
             f"{a.certifier!r}.",
             "# Every operation is one fused libcfgpu call per layer (cf_deeppoly_layer, cfgpu.layerwise);",
             "# Flow.flow calls the operations layer by layer.",
             "from cfgpu import layerwise", "", "",
             f"class {a.name}:",
             f"    cf_certifier = {a.certifier!r}",
             "    cf_layerwise = True"]
    if a.stop_depth is not None:
        lines.append(f"    cf_stop_depth = {a.stop_depth!r}")
    if a.relu_strict:
        lines.append("    cf_relu_strict = True")
    lines.append("")
    for op, kind in a.ops.items():
        lines.append(f"    def {op}({_SIG}):")
        lines.append(f"        # {_DOC.get(kind, kind)}")
        if kind is None:
            lines.append(f"        raise NotImplementedError({op + ': no fused kernel in libcfgpu'!r})")
        else:
            lines.append(f"        return layerwise.run_operation(abs_elem, {op!r}, layer_index)")
        lines.append("")
    transformers = "\n".join(lines).rstrip() + "\n"
    keys = ["llist"] + [m for _, m in a.shape]
    types = {m: t for t, m in a.shape}
    types["llist"] = "bool"
    spec_vars = {"l": "l", "u": "u", "L": "L", "U": "U", "Z": "Z", "llist": "llist"}
    d = ", ".join(f"{k!r}: {spec_vars.get(k, k)}" for k in keys)
    tp = ", ".join(f"{k!r}: {types[k]!r}" for k in keys)
    main = "\n".join([
        f"# Generated by cfgpu.codegen from {source_name}.",
        "from constraintflow.lib.abs_elem import Abs_elem_sparse",
        "from constraintflow.lib.flow_sparse import Flow",
        "from constraintflow.lib.spec import get_network_and_input_spec",
        f"from transformers import {a.name}",
        "",
        "",
        "def run(network_file, batch_size, eps, dataset_X, dataset_y, dataset, train, print_intermediate_results,",
        "        no_sparsity):",
        "    network, l, u, L, U, Z, llist = get_network_and_input_spec(network_file, batch_size, dataset_X, dataset_y,",
        "                                                               dataset, eps=eps, train=train,",
        "                                                               no_sparsity=no_sparsity)",
        f"    abs_elem = Abs_elem_sparse({{{d}}}, {{{tp}}}, network, batch_size=batch_size,",
        "                               no_sparsity=no_sparsity)",
        f"    return Flow(abs_elem, {a.name}(), network, print_intermediate_results, no_sparsity).flow()",
        ""])
    return {"transformers.py": transformers, "main.py": main}


def write(ast, out_dir, source_name="program.cf"):
    files = generate(ast, source_name)
    os.makedirs(out_dir, exist_ok=True)
    for fname, text in files.items():
        with open(os.path.join(out_dir, fname), "w") as f:
            f.write(text)
    return files

