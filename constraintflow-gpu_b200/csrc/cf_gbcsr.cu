// Elementwise block kernels of the gbcsr ops (binary / unary / where / clamp / any).
//
// One grid-stride kernel per op over the output block; each input is read through its
// own element strides (zero stride = broadcast), so RepeatBlock-style broadcast views
// (constraintflow/gbcsr/sparse_block.py:3797) and scalar fills need no materialisation.
// The op semantics follow operator.* on torch tensors as the reference applies them per
// block (sparse_block.py:49-60 `operation` / `unary_operation`).
#include "cf_common.cuh"

namespace cf {

struct Geo {
  int32_t ndim;
  int64_t shape[CF_MAX_DIMS];
  int64_t sx[CF_MAX_DIMS], sy[CF_MAX_DIMS], sz[CF_MAX_DIMS];
  int64_t total;
};

__device__ __forceinline__ void offsets(const Geo& g, int64_t t, int64_t& ox, int64_t& oy, int64_t& oz) {
  ox = oy = oz = 0;
  for (int d = g.ndim - 1; d >= 0; --d) {
    int64_t sz = g.shape[d];
    int64_t idx = t % sz;
    t /= sz;
    ox += idx * g.sx[d];
    oy += idx * g.sy[d];
    oz += idx * g.sz[d];
  }
}

__device__ __forceinline__ float ld(const void* p, int32_t dt, int64_t o) {
  return dt == CF_BOOL ? (float)(static_cast<const uint8_t*>(p)[o] != 0) : static_cast<const float*>(p)[o];
}
__device__ __forceinline__ void st(void* p, int32_t dt, int64_t o, float v) {
  if (dt == CF_BOOL) static_cast<uint8_t*>(p)[o] = (v != 0.0f);
  else static_cast<float*>(p)[o] = v;
}

__device__ __forceinline__ float apply(int32_t op, float a, float b) {
  switch (op) {
    case CF_OP_ADD: return __fadd_rn(a, b);
    case CF_OP_SUB: return __fsub_rn(a, b);
    case CF_OP_MUL: return __fmul_rn(a, b);
    case CF_OP_DIV: return __fdiv_rn(a, b);
    case CF_OP_GE: return a >= b;
    case CF_OP_GT: return a > b;
    case CF_OP_LE: return a <= b;
    case CF_OP_LT: return a < b;
    case CF_OP_EQ: return a == b;
    case CF_OP_NE: return a != b;
    case CF_OP_AND: return (a != 0.0f) && (b != 0.0f);
    case CF_OP_OR: return (a != 0.0f) || (b != 0.0f);
    case CF_OP_MAX: return fmaxf(a, b);
    case CF_OP_MIN: return fminf(a, b);
  }
  return 0.0f;
}

__global__ void k_ew_binary(int32_t op, Geo g, const void* x, int32_t xdt, const void* y, int32_t ydt, void* out,
                            int32_t odt) {
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < g.total; t += (int64_t)gridDim.x * blockDim.x) {
    int64_t ox, oy, oz;
    offsets(g, t, ox, oy, oz);
    st(out, odt, t, apply(op, ld(x, xdt, ox), ld(y, ydt, oy)));
  }
}

__global__ void k_ew_unary(int32_t op, Geo g, const void* x, int32_t xdt, void* out, int32_t odt) {
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < g.total; t += (int64_t)gridDim.x * blockDim.x) {
    int64_t ox, oy, oz;
    offsets(g, t, ox, oy, oz);
    float a = ld(x, xdt, ox), r;
    switch (op) {
      case CF_UOP_NEG: r = -a; break;
      case CF_UOP_NOT: r = (a == 0.0f); break;
      case CF_UOP_SIGMOID: r = 1.0f / (1.0f + expf(-a)); break;
      case CF_UOP_RELU: r = a > 0.0f ? a : 0.0f; break;
      default: r = a; break;
    }
    st(out, odt, t, r);
  }
}

__global__ void k_ew_where(Geo g, const uint8_t* c, const void* y, const void* z, void* out, int32_t odt) {
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < g.total; t += (int64_t)gridDim.x * blockDim.x) {
    int64_t oc, oy, oz;
    offsets(g, t, oc, oy, oz);
    st(out, odt, t, c[oc] ? ld(y, odt, oy) : ld(z, odt, oz));
  }
}

__global__ void k_ew_clamp(Geo g, const float* x, float c, int32_t min_true, float* out) {
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < g.total; t += (int64_t)gridDim.x * blockDim.x) {
    int64_t ox, oy, oz;
    offsets(g, t, ox, oy, oz);
    float v = x[ox];
    // torch clamp(min=c): NaN stays NaN; max(v, c) otherwise
    out[t] = min_true ? (v < c ? c : v) : (v > c ? c : v);
  }
}

__global__ void k_ew_any(Geo g, const void* x, int32_t xdt, uint32_t* flag) {
  bool found = false;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < g.total && !found;
       t += (int64_t)gridDim.x * blockDim.x) {
    int64_t ox, oy, oz;
    offsets(g, t, ox, oy, oz);
    found = ld(x, xdt, ox) != 0.0f;
  }
  if (__any_sync(0xffffffffu, found) && (threadIdx.x & 31) == 0) atomicOr(flag, 1u);
}

static cf_status make_geo(Geo& g, int32_t ndim, const int64_t* shape, const int64_t* sx, const int64_t* sy,
                          const int64_t* sz) {
  CF_REQUIRE(ndim >= 0 && ndim <= CF_MAX_DIMS, CF_ERR_SHAPE, "ew: ndim %d out of range", ndim);
  CF_REQUIRE(ndim == 0 || shape, CF_ERR_NULL, "ew: shape is NULL");
  g.ndim = ndim;
  g.total = 1;
  for (int d = 0; d < ndim; ++d) {
    CF_REQUIRE(shape[d] >= 0, CF_ERR_SHAPE, "ew: negative extent");
    g.shape[d] = shape[d];
    g.total *= shape[d];
    g.sx[d] = sx ? sx[d] : 0;
    g.sy[d] = sy ? sy[d] : 0;
    g.sz[d] = sz ? sz[d] : 0;
  }
  return CF_OK;
}

static inline unsigned grid_for(int64_t total) {
  int64_t b = ceil_div(total, 256);
  if (b > 148 * 16) b = 148 * 16;
  if (b < 1) b = 1;
  return (unsigned)b;
}

}  // namespace cf

using namespace cf;

extern "C" cf_status cf_ew_binary(int32_t op, int32_t ndim, const int64_t* shape, const void* x, int32_t xdt,
                                  const int64_t* xs, const void* y, int32_t ydt, const int64_t* ys, void* out,
                                  int32_t odt, void* stream) {
  clear_error();
  CF_INJECT("ew");
  CF_REQUIRE(op >= CF_OP_ADD && op <= CF_OP_MIN, CF_ERR_UNSUPPORTED, "ew_binary: op %d", op);
  Geo g;
  CF_TRY(make_geo(g, ndim, shape, xs, ys, nullptr));
  if (g.total == 0) return CF_OK;
  CF_REQUIRE(x && y && out, CF_ERR_NULL, "ew_binary: NULL argument");
  k_ew_binary<<<grid_for(g.total), 256, 0, as_stream(stream)>>>(op, g, x, xdt, y, ydt, out, odt);
  return check_launch("k_ew_binary");
}

extern "C" cf_status cf_ew_unary(int32_t op, int32_t ndim, const int64_t* shape, const void* x, int32_t xdt,
                                 const int64_t* xs, void* out, int32_t odt, void* stream) {
  clear_error();
  CF_INJECT("ew");
  CF_REQUIRE(op >= CF_UOP_NEG && op <= CF_UOP_TO_F32, CF_ERR_UNSUPPORTED, "ew_unary: op %d", op);
  Geo g;
  CF_TRY(make_geo(g, ndim, shape, xs, nullptr, nullptr));
  if (g.total == 0) return CF_OK;
  CF_REQUIRE(x && out, CF_ERR_NULL, "ew_unary: NULL argument");
  k_ew_unary<<<grid_for(g.total), 256, 0, as_stream(stream)>>>(op, g, x, xdt, out, odt);
  return check_launch("k_ew_unary");
}

extern "C" cf_status cf_ew_where(int32_t ndim, const int64_t* shape, const uint8_t* c, const int64_t* cs,
                                 const void* y, const int64_t* ys, const void* z, const int64_t* zs, void* out,
                                 int32_t odt, void* stream) {
  clear_error();
  CF_INJECT("ew");
  Geo g;
  CF_TRY(make_geo(g, ndim, shape, cs, ys, zs));
  if (g.total == 0) return CF_OK;
  CF_REQUIRE(c && y && z && out, CF_ERR_NULL, "ew_where: NULL argument");
  k_ew_where<<<grid_for(g.total), 256, 0, as_stream(stream)>>>(g, c, y, z, out, odt);
  return check_launch("k_ew_where");
}

extern "C" cf_status cf_ew_clamp(int32_t ndim, const int64_t* shape, const float* x, const int64_t* xs, float c,
                                 int32_t min_true, float* out, void* stream) {
  clear_error();
  CF_INJECT("ew");
  Geo g;
  CF_TRY(make_geo(g, ndim, shape, xs, nullptr, nullptr));
  if (g.total == 0) return CF_OK;
  CF_REQUIRE(x && out, CF_ERR_NULL, "ew_clamp: NULL argument");
  k_ew_clamp<<<grid_for(g.total), 256, 0, as_stream(stream)>>>(g, x, c, min_true, out);
  return check_launch("k_ew_clamp");
}

extern "C" cf_status cf_ew_any(int32_t ndim, const int64_t* shape, const void* x, int32_t xdt, const int64_t* xs,
                               uint32_t* flag, void* stream) {
  clear_error();
  CF_INJECT("ew");
  Geo g;
  CF_TRY(make_geo(g, ndim, shape, xs, nullptr, nullptr));
  if (g.total == 0) return CF_OK;
  CF_REQUIRE(x && flag, CF_ERR_NULL, "ew_any: NULL argument");
  k_ew_any<<<grid_for(g.total), 256, 0, as_stream(stream)>>>(g, x, xdt, flag);
  return check_launch("k_ew_any");
}
