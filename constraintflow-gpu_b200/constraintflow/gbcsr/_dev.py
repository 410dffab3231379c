"""Device arithmetic of the gbcsr mirror: every value computed by the gbcsr ops goes
through libcfgpu's block kernels via cfgpu.ops (cf_ew_binary, cf_ew_unary, cf_ew_where,
cf_ew_clamp, cf_ew_any, cf_bmm)."""
from cfgpu.ops import (COMPARISONS, _OPS, any_nonzero, as_block_tensor, binary, bmm, clamp, device,  # noqa: F401
                       scalar_view, unary, where)
