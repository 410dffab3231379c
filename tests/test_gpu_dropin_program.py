"""The reference compiler's own output for examples/compiler_examples/{deeppoly,crown,
deeppoly_efficient,zono,ibp,polyzono,crownibp}.cf (tests/golden/generated/<program>/{main.py,transformers.py}, saved
by tests/golden/gen_golden.py) runs UNCHANGED on this runtime's constraintflow package:
main.run(...) -> (lb, ub) float64, matching the reference's golden bounds (chain, residual
Add and Concat networks)."""
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
GEN = os.path.join(HERE, "golden", "generated")
_STUBS = os.path.join(HERE, "golden", "refshim", "stubs")
if _STUBS not in sys.path:
    sys.path.append(_STUBS)  # in-memory onnx stand-in; an installed onnx package comes first


def _load_program(program):
    """Import the generated main.py with its sibling transformers.py, as `constraintflow run` does."""
    d = os.path.join(GEN, program)
    saved = {k: sys.modules.pop(k) for k in ("transformers", "main") if k in sys.modules}
    stubs = os.path.join(HERE, "golden", "refshim", "stubs")
    if stubs not in sys.path:
        sys.path.append(stubs)  # the in-memory onnx stand-in (no onnx package offline)
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
    return main


PROGRAM_CASES = [("deeppoly", n) for n in ("dp_w0_b4_e1e-3", "dp_w1_b16_e5e-4", "dp_w2_b8_e2e-4", "dp_w3_b4_e2e-3")] + \
    [("crown", n) for n in ("crown_w0_b4_e1e-3", "crown_w2_b4_e2e-4")] + \
    [("deeppoly_efficient", n) for n in ("dpe_w0_b4_e1e-3", "dpe_w2_b4_e2e-4")] + \
    [("deeppoly", n) for n in ("dp_w5_b4_e2e-3", "dp_w6_b4_e2e-3")] + \
    [("crown", n) for n in ("crown_w5_b2_e2e-3", "crown_w6_b2_e1e-1")] + \
    [("zono", n) for n in ("zono_w0_b4_e1e-3", "zono_w2_b4_e2e-4")] + \
    [("ibp", n) for n in ("ibp_w0_b4_e1e-3", "ibp_w3_b2_e2e-3")] + \
    [("polyzono", n) for n in ("pz_w0_b4_e1e-2", "pz_w2_b4_e2e-4")] + \
    [("crownibp", n) for n in ("cibp_w0_b4_e1e-3", "cibp_w3_b2_e2e-3")] + \
    [("deeppoly_custom_stop", "cs3_w2_b4_e2e-4"), ("custom_stops/deeppoly_custom_stop05", "cs5_w2_b4_e2e-4")] + \
    [("zid", "zid_w2_b4_e2e-3"), ("zid", "zid_w3_b2_e2e-3")]


@pytest.mark.parametrize("program,name", PROGRAM_CASES)
def test_generated_program_runs_unchanged(program, name):
    import onnx
    sys.path.insert(0, os.path.join(HERE, "golden"))
    import gen_golden
    from cfgpu import nets
    c = Case(name)
    main = _load_program(program)
    net_name = f"{name}.onnx"
    onnx.register(net_name, gen_golden._onnx_graph(nets, c.wl))
    X = torch.from_numpy(c.X)
    y = torch.from_numpy(c.y)
    lb, ub = main.run(net_name, c.B, c.eps, X, y, c.wl.dataset, False, False, False)
    assert lb.dtype == torch.float64 and tuple(lb.shape) == (c.B, 9)
    lb, ub = lb.numpy(), ub.numpy()
    scale = np.maximum(np.abs(c.lb).max(axis=1, keepdims=True), np.abs(c.ub).max(axis=1, keepdims=True))
    tol = parity.RTOL * np.abs(c.lb) + parity.ATOL * scale
    assert (np.abs(lb - c.lb) <= tol).all() and (np.abs(ub - c.ub) <= tol).all()
    same, nd = parity.verdicts_match(lb, c.lb, np.abs(c.lb).max(axis=1))
    assert same


def test_programs_are_recognised():
    from constraintflow.lib.flow_sparse import certifier_of
    for program, expect in (("deeppoly", "deeppoly"), ("deeppoly_efficient", "deeppoly"), ("crown", "crown"),
                            ("zono", "zono"), ("ibp", "ibp"), ("polyzono", "polyzono"), ("crownibp", "crownibp")):
        main = _load_program(program)
        cls = program if program in ("zono", "ibp", "polyzono", "crownibp") else "deeppoly"
        assert certifier_of(getattr(main, cls)()) == expect

    class Other:   # some other certifier program: a ReLU without a recognised relaxation
        def Affine(self, abs_elem, prev, curr):
            return None

        def Relu(self, abs_elem, prev, curr):
            return None

    with pytest.raises(NotImplementedError):
        certifier_of(Other())
