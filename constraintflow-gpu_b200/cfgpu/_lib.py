"""ctypes binding of libcfgpu.so (the C ABI declared in include/cfgpu.h).

The library is the only compute path: importing this module fails loudly when the
shared object has not been built, and every wrapper raises on a non-zero status.
There is no CPU fallback.
"""
import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
# CF_LIB_PATH selects another build of the library (e.g. a -lineinfo debug build).
LIB_PATH = os.environ.get("CF_LIB_PATH") or os.path.join(_HERE, "libcfgpu.so")

CF_OK, CF_ERR_SHAPE, CF_ERR_UNSUPPORTED, CF_ERR_CUDA, CF_ERR_TIMEOUT, CF_ERR_NULL, CF_ERR_WORKSPACE, \
    CF_ERR_INJECTED = range(8)
CF_LAYER_LINEAR, CF_LAYER_CONV, CF_LAYER_RELU = 1, 2, 3
CF_RELAX_DEEPPOLY, CF_RELAX_CROWN, CF_RELAX_ZONO, CF_RELAX_IBP, CF_RELAX_CROWNIBP = 0, 1, 2, 3, 4
CF_RELAX_DEEPPOLY_STRICT, CF_RELAX_CROWNIBP_STRICT = 5, 6
CF_MAX_DIMS = 6
CF_STATIC_SCRATCH_BYTES = 32 << 20
CF_F32, CF_BOOL = 0, 1
OPS = dict(add=0, sub=1, mul=2, truediv=3, ge=4, gt=5, le=6, lt=7, eq=8, ne=9, and_=10, or_=11, max=12, min=13)
UOPS = dict(neg=0, not_=1, sigmoid=2, relu=3, to_f32=4)

_i32, _i64, _sz, _vp, _f32 = ctypes.c_int32, ctypes.c_int64, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_float
_p64 = ctypes.POINTER(ctypes.c_int64)


class CfError(RuntimeError):
    """A libcfgpu call returned a non-zero cf_status."""

    def __init__(self, status, msg):
        super().__init__(f"cfgpu status {status}: {msg}")
        self.status = status


class CfLayer(ctypes.Structure):
    _fields_ = [("kind", _i32), ("n_in", _i32), ("n_out", _i32),
                ("cin", _i32), ("ih", _i32), ("iw", _i32), ("cout", _i32), ("oh", _i32), ("ow", _i32),
                ("kh", _i32), ("kw", _i32), ("stride", _i32), ("pad", _i32),
                ("W_dev", _vp), ("b_dev", _vp)]


class CfProfileStats(ctypes.Structure):
    _fields_ = [("kernel_launches", _i64), ("step_launches", _i64), ("step_ms", ctypes.c_double),
                ("step_flops", ctypes.c_double), ("step_bytes", ctypes.c_double),
                ("mem_launches", _i64), ("mem_ms", ctypes.c_double), ("mem_bytes", ctypes.c_double)]


class CfConvGeom(ctypes.Structure):
    _fields_ = [(n, _i32) for n in ("K", "C", "ox", "oy", "ix", "iy", "kx", "ky", "sx", "sy", "px", "py")]


class CfNetwork(ctypes.Structure):
    _fields_ = [("n_layers", _i32), ("layers", ctypes.POINTER(CfLayer)), ("n_input", _i32),
                ("n_spec", _i32), ("relaxation", _i32), ("stop_depth", _i32)]


def _load():
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is missing: build it with `python -m cfgpu.build` "
                          "(constraintflow-gpu_b200/) or __graft_entry__.build(); there is no CPU fallback")
    lib = ctypes.CDLL(LIB_PATH)
    P = ctypes.POINTER
    sig = {
        "cf_network_neurons": (_i64, [P(CfNetwork)]),
        "cf_deeppoly_workspace_bytes": (_sz, [P(CfNetwork), _i64]),
        "cf_deeppoly_run": (_i32, [P(CfNetwork), _i64, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _sz, _vp]),
        "cf_deeppoly_layer": (_i32, [P(CfNetwork), _i32, _i64, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _sz, _vp]),
        "cf_signscale": (_i32, [_i64, _i64, _i64, _vp, _i64, _i64, _vp, _vp, _vp, _vp, _i64, _vp, _vp, _vp]),
        "cf_deeppoly_check": (_i32, [_vp, _vp]),
        "cf_deeppoly_run_static": (_i32, [P(CfNetwork), _i64, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
        "cf_deeppoly_check_static": (_i32, [_vp]),
        "cf_deeppoly_run_replay": (_i32, [P(CfNetwork), _i64, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _sz,
                                          _vp]),
        "cf_relu_relax": (_i32, [_i64, _i64, _vp, _vp, _i64, _vp, _vp, _i64, _vp, _vp, _vp, _i32, _vp]),
        "cf_backsub_step": (_i32, [_i64, _i64, _i64, _i64, _vp, _i64, _i64, _i64, _vp, _i64, _i64,
                                   _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
        "cf_concretize": (_i32, [_i64, _i64, _i64, _vp, _i64, _i64, _i64, _vp, _i64, _i64, _vp, _vp, _vp, _vp,
                                 _i64, _vp]),
        "cf_ew_binary": (_i32, [_i32, _i32, _p64, _vp, _i32, _p64, _vp, _i32, _p64, _vp, _i32, _vp]),
        "cf_ew_unary": (_i32, [_i32, _i32, _p64, _vp, _i32, _p64, _vp, _i32, _vp]),
        "cf_ew_where": (_i32, [_i32, _p64, _vp, _p64, _vp, _p64, _vp, _p64, _vp, _i32, _vp]),
        "cf_ew_clamp": (_i32, [_i32, _p64, _vp, _p64, _f32, _i32, _vp, _vp]),
        "cf_ew_any": (_i32, [_i32, _p64, _vp, _i32, _p64, _vp, _vp]),
        "cf_bounds_meet": (_i32, [_i64, _i64, _vp, _vp, _i64, _vp, _vp, _i64, _vp, _vp, _vp]),
        "cf_bmm": (_i32, [_i64, _i64, _i64, _i64, _vp, _i64, _i64, _i64, _vp, _i64, _i64, _i64, _vp, _i32, _vp]),
        "cf_input_box": (_i32, [_i64, _i32, _i64, _vp, _f32, ctypes.POINTER(_f32), ctypes.POINTER(_f32), _vp, _vp,
                                _vp]),
        "cf_spec_matrix": (_i32, [_i64, _i32, _vp, _vp, _vp]),
        "cf_conv_densify": (_i32, [P(CfConvGeom), _i64, _vp, _i64, _i64, _i64, _vp, _vp]),
        "cf_conv_apply": (_i32, [P(CfConvGeom), _i64, _i64, _vp, _i64, _i64, _i64, _vp, _i64, _i64, _i64, _vp, _i64,
                                 _i64, _i64, _vp]),
        "cf_conv_scale": (_i32, [P(CfConvGeom), _i64, _vp, _i64, _i64, _i64, _vp, _i64, _i64, _vp, _vp]),
        "cf_conv_transpose": (_i32, [P(CfConvGeom), _i64, _i64, _vp, _i64, _i64, _i64, _vp, _i32, _i32, _vp, _i64,
                                     _i64, _i64, _vp]),
        "cf_profile_enable": (_i32, [_i32]),
        "cf_profile_collect": (_i32, [P(CfProfileStats)]),
        "cf_last_error": (ctypes.c_char_p, []),
        "cf_version": (ctypes.c_char_p, []),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()

# Every symbol the C header declares (checked by the CPU test suite).
EXPORTED = ("cf_network_neurons", "cf_deeppoly_workspace_bytes", "cf_deeppoly_run", "cf_deeppoly_check",
            "cf_deeppoly_layer", "cf_signscale", "cf_bounds_meet",
            "cf_deeppoly_run_static", "cf_deeppoly_check_static", "cf_deeppoly_run_replay",
            "cf_relu_relax",
            "cf_backsub_step", "cf_concretize", "cf_ew_binary", "cf_ew_unary", "cf_ew_where", "cf_ew_clamp",
            "cf_ew_any", "cf_bmm", "cf_conv_densify", "cf_conv_apply", "cf_conv_scale", "cf_conv_transpose",
            "cf_input_box", "cf_spec_matrix", "cf_profile_enable", "cf_profile_collect",
            "cf_last_error", "cf_version")


def check(status, what=""):
    """Map a cf_status to the reference's exception types (tensor_ops.py:18-77)."""
    if status == CF_OK:
        return
    msg = (lib.cf_last_error() or b"").decode(errors="replace")
    if what:
        msg = f"{what}: {msg}"
    if status == CF_ERR_SHAPE:
        raise Exception(f"SHAPE MISMATCH ({msg})")
    if status == CF_ERR_UNSUPPORTED:
        raise NotImplementedError(msg)
    raise CfError(status, msg)


def f32_array(vals):
    return (ctypes.c_float * max(1, len(vals)))(*[float(v) for v in vals])


def i64_array(vals):
    arr = (ctypes.c_int64 * max(1, len(vals)))(*[int(v) for v in vals])
    return arr
