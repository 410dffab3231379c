"""Rebuilds an AST stored by gen_codegen.py as objects whose class names and fields are
those of the reference front end's nodes (what cfgpu.codegen reads)."""

_CLASSES = {}


def _cls(name):
    if name not in _CLASSES:
        _CLASSES[name] = type(name, (), {})
    return _CLASSES[name]


def from_json(d):
    if isinstance(d, dict) and "_list" in d:
        items = [from_json(x) for x in d["_list"]]
        return tuple(items) if d.get("_tuple") else items
    if isinstance(d, dict) and "_" in d:
        obj = _cls(d["_"])()
        for k, v in d.items():
            if k != "_":
                setattr(obj, k, from_json(v))
        if hasattr(obj, "texpr"):
            obj.left, obj.right = obj.texpr, obj.fexpr
        return obj
    return d
