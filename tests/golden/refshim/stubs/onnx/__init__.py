# Test-infrastructure stand-in for the onnx package (absent offline): lets the reference's
# constraintflow/lib/parse.py:29-70 read an in-memory graph registered under a file name.
import types
_REG = {}
def register(name, graph): _REG[name] = types.SimpleNamespace(graph=graph)
def load(name): return _REG[name]
from . import numpy_helper
