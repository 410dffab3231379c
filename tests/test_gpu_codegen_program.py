"""Programs emitted by the compiler backend (cfgpu.codegen, tests/golden/generated_cfgpu/)
run through the drop-in constraintflow package: Flow.flow calls the emitted transformer
for every layer, each operation one fused cf_deeppoly_layer call, and the bounds match the
reference's own outputs (tests/golden/*.npz) and the whole-network driver."""
import importlib.util
import os
import sys

import numpy as np
import pytest
import torch

import parity
from golden_cases import Case

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
GEN = os.path.join(HERE, "golden", "generated_cfgpu")
_STUBS = os.path.join(HERE, "golden", "refshim", "stubs")
if _STUBS not in sys.path:
    sys.path.append(_STUBS)


def _load(program):
    d = os.path.join(GEN, program)
    saved = {k: sys.modules.pop(k) for k in ("transformers", "main") if k in sys.modules}
    spec = importlib.util.spec_from_file_location("transformers", os.path.join(d, "transformers.py"))
    tr = importlib.util.module_from_spec(spec)
    sys.modules["transformers"] = tr
    spec.loader.exec_module(tr)
    spec = importlib.util.spec_from_file_location("main", os.path.join(d, "main.py"))
    main = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(main)
    for k in ("transformers", "main"):
        sys.modules.pop(k, None)
    sys.modules.update(saved)
    return main, tr


CASES = [("deeppoly", "dp_w0_b4_e1e-3"), ("deeppoly", "dp_w2_b8_e2e-4"), ("deeppoly", "dp_w3_b4_e2e-3"),
         ("deeppoly_efficient", "dpe_w2_b4_e2e-4"), ("crown", "crown_w0_b4_e1e-3"), ("crown", "crown_w1_b2_e1e-1"),
         ("zono", "zono_w2_b4_e2e-3"), ("zono", "zono_w3_b2_e2e-3"), ("ibp", "ibp_w3_b2_e2e-3"),
         ("deeppoly", "dp_w5_b4_e2e-3"), ("polyzono", "pz_w0_b4_e1e-2"), ("polyzono", "pz_w2_b4_e2e-3"),
         ("crownibp", "cibp_w1_b8_e5e-4"), ("crownibp", "cibp_w3_b2_e2e-3"),
         ("deeppoly_custom_stop", "cs3_w2_b4_e2e-4"), ("deeppoly_custom_stop", "cs3_w0_b4_e1e-2")]


@pytest.mark.parametrize("program,name", CASES)
def test_emitted_program_matches_reference(program, name, monkeypatch):
    import onnx
    sys.path.insert(0, os.path.join(HERE, "golden"))
    import gen_golden
    from cfgpu import layerwise, nets
    calls = []
    orig = layerwise.run_operation

    def counting(abs_elem, op, layer_index):
        calls.append((op, layer_index))
        return orig(abs_elem, op, layer_index)
    monkeypatch.setattr(layerwise, "run_operation", counting)
    c = Case(name)
    main, _ = _load(program)
    net_name = f"cg_{name}.onnx"
    onnx.register(net_name, gen_golden._onnx_graph(nets, c.wl))
    lb, ub = main.run(net_name, c.B, c.eps, torch.from_numpy(c.X), torch.from_numpy(c.y), c.wl.dataset, False, False,
                      False)
    assert lb.dtype == torch.float64 and tuple(lb.shape) == (c.B, 9)
    lb, ub = lb.numpy(), ub.numpy()
    scale = np.maximum(np.abs(c.lb).max(axis=1, keepdims=True), np.abs(c.ub).max(axis=1, keepdims=True))
    tol = parity.RTOL * np.abs(c.lb) + parity.ATOL * scale
    assert (np.abs(lb - c.lb) <= tol).all() and (np.abs(ub - c.ub) <= tol).all()
    assert parity.verdicts_match(lb, c.lb, np.abs(c.lb).max(axis=1))[0]
    if nets.is_chain(c.wl.layers):
        # one call per layer, property layer included; the kinds follow the network
        kinds = ["Relu" if L.kind == "relu" else "Affine" for L in c.wl.layers] + ["Affine"]
        if not (program == "crown" and c.eps >= 0.1):
            assert [op for op, _ in calls] == kinds
            assert [i for _, i in calls] == list(range(1, len(kinds) + 1))
    else:
        assert calls == []      # Add / Concat networks run as a whole (general traversal)
