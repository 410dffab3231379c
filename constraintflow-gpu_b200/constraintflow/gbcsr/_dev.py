"""Device arithmetic of the gbcsr mirror: every value computed by the gbcsr ops goes
through libcfgpu's block kernels via cfgpu.ops (cf_ew_binary, cf_ew_unary, cf_ew_where,
cf_ew_clamp, cf_ew_any, cf_bmm, cf_conv_densify, cf_conv_apply, cf_conv_scale,
cf_conv_transpose)."""
from cfgpu.ops import (COMPARISONS, _OPS, any_nonzero, as_block_tensor, binary, bmm, clamp, conv_apply,  # noqa: F401
                       conv_densify, conv_geom, conv_scale, conv_transpose, device, scalar_view, unary, where)
