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

// C[b] (+)= A[b] @ B[b] with arbitrary element strides (broadcast views included).
// 64x64 output tile per CTA, K staged 16 at a time, 4x4 register tile per thread.
constexpr int BM_M = 64, BM_N = 64, BM_K = 16;

__global__ void __launch_bounds__(256) k_bmm(int64_t nb, int64_t M, int64_t N, int64_t K, const float* __restrict__ A,
                                             int64_t a_bs, int64_t a_ms, int64_t a_ks, const float* __restrict__ B,
                                             int64_t b_bs, int64_t b_ks, int64_t b_ns, float* __restrict__ C,
                                             int accumulate) {
  __shared__ float As[BM_K][BM_M + 4];
  __shared__ float Bs[BM_K][BM_N + 4];
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  for (int64_t bt = blockIdx.z; bt < nb; bt += gridDim.z) {
    const float* Ab = A + bt * a_bs;
    const float* Bb = B + bt * b_bs;
    const int64_t m0 = (int64_t)blockIdx.y * BM_M, n0 = (int64_t)blockIdx.x * BM_N;
    float acc[4][4] = {};
    for (int64_t k0 = 0; k0 < K; k0 += BM_K) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int e = tid + 256 * q;
        const int kk = e & 15, mm = e >> 4;
        const int64_t mg = m0 + mm, kg = k0 + kk;
        As[kk][mm] = (mg < M && kg < K) ? Ab[mg * a_ms + kg * a_ks] : 0.0f;
        const int kk2 = e >> 6, nn = e & 63;
        const int64_t kg2 = k0 + kk2, ng = n0 + nn;
        Bs[kk2][nn] = (kg2 < K && ng < N) ? Bb[kg2 * b_ks + ng * b_ns] : 0.0f;
      }
      __syncthreads();
#pragma unroll
      for (int kk = 0; kk < BM_K; ++kk) {
        float a4[4], b4[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) a4[q] = As[kk][ty * 4 + q];
#pragma unroll
        for (int q = 0; q < 4; ++q) b4[q] = Bs[kk][tx * 4 + q];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a4[i], b4[j], acc[i][j]);
      }
      __syncthreads();
    }
    float* Cb = C + bt * M * N;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int64_t m = m0 + ty * 4 + i;
      if (m >= M) continue;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int64_t n = n0 + tx * 4 + j;
        if (n < N) Cb[m * N + n] = accumulate ? Cb[m * N + n] + acc[i][j] : acc[i][j];
      }
    }
  }
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

// Sign-selected column scaling of rows (the substitution of a ReLU layer's per-neuron
// relaxation into a coefficient matrix): out[b,m,n] = A[b,m,n] * (A >= 0 ? p[b,n] : q[b,n]),
// dc[b,m] = sum_n A[b,m,n] * (A >= 0 ? pc[b,n] : qc[b,n]).  One warp per row.
__global__ void k_signscale(int64_t nb, int64_t M, int64_t N, const float* __restrict__ A, int64_t a_bs,
                            int64_t a_ms, const float* __restrict__ p, const float* __restrict__ q,
                            const float* __restrict__ pc, const float* __restrict__ qc, int64_t v_bs,
                            float* __restrict__ out, float* __restrict__ dc) {
  const int64_t w = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= nb * M) return;
  const int64_t b = w / M, m = w - b * M;
  const float* a = A + b * a_bs + m * a_ms;
  const float *pb = p + b * v_bs, *qb = q + b * v_bs;
  const float* pcb = pc ? pc + b * v_bs : nullptr;
  const float* qcb = qc ? qc + b * v_bs : nullptr;
  float* o = out + w * N;
  float acc = 0.0f;
  for (int64_t n = lane; n < N; n += 32) {
    const float x = a[n];
    const bool pos = x >= 0.0f;
    o[n] = x * (pos ? pb[n] : qb[n]);
    const float* cv = pos ? pcb : qcb;
    if (cv) acc = fmaf(x, cv[n], acc);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (dc && lane == 0) dc[w] = acc;
}

extern "C" cf_status cf_signscale(int64_t nb, int64_t M, int64_t N, const float* A, int64_t a_bs, int64_t a_ms,
                                  const float* p, const float* q, const float* pc, const float* qc, int64_t v_bs,
                                  float* out, float* dc, void* stream) {
  clear_error();
  CF_INJECT("signscale");
  CF_REQUIRE(nb >= 0 && M >= 0 && N >= 0, CF_ERR_SHAPE, "signscale: negative size");
  if (nb * M == 0) return CF_OK;
  CF_REQUIRE(A && p && q && out, CF_ERR_NULL, "signscale: NULL argument");
  const int64_t warps = nb * M;
  const int64_t blocks = ceil_div(warps * 32, 256);
  CF_REQUIRE(blocks <= 0x7fffffff, CF_ERR_SHAPE, "signscale: too many rows");
  k_signscale<<<(unsigned)blocks, 256, 0, as_stream(stream)>>>(nb, M, N, A, a_bs, a_ms, p, q, pc, qc, v_bs, out, dc);
  return check_launch("k_signscale");
}

extern "C" cf_status cf_bmm(int64_t nb, int64_t M, int64_t N, int64_t K, const float* A, int64_t a_bs, int64_t a_ms,
                            int64_t a_ks, const float* B, int64_t b_bs, int64_t b_ks, int64_t b_ns, float* C,
                            int32_t accumulate, void* stream) {
  clear_error();
  CF_INJECT("bmm");
  CF_REQUIRE(nb >= 0 && M >= 0 && N >= 0 && K >= 0, CF_ERR_SHAPE, "bmm: negative size");
  if (nb * M * N == 0) return CF_OK;
  CF_REQUIRE(C && (K == 0 || (A && B)), CF_ERR_NULL, "bmm: NULL argument");
  const double flops = 2.0 * nb * M * N * K;
  const double bytes = 4.0 * ((double)nb * M * K + (double)(b_bs ? nb : 1) * K * N + (double)nb * M * N);
  // one matrix B shared by every batch (stride 0) and batch-contiguous A rows: a single
  // GEMM over nb*M rows (C is compact [nb, M, N], so its rows line up)
  if (nb > 1 && b_bs == 0 && a_bs == M * a_ms && ceil_div(nb * M, BM_M) <= 65535) {
    M *= nb;
    nb = 1;
    a_bs = 0;
  }
  const int64_t gx = ceil_div(N, BM_N), gy = ceil_div(M, BM_M);
  CF_REQUIRE(gx <= 0x7fffffff && gy <= 65535, CF_ERR_SHAPE, "bmm: %lld x %lld too large", (long long)M,
             (long long)N);
  dim3 grid((unsigned)gx, (unsigned)gy, (unsigned)(nb < 65535 ? nb : 65535));
  prof_step_begin(as_stream(stream));
  k_bmm<<<grid, 256, 0, as_stream(stream)>>>(nb, M, N, K, A, a_bs, a_ms, a_ks, B, b_bs, b_ks, b_ns, C, accumulate);
  prof_step_end(as_stream(stream), flops, bytes);
  return check_launch("k_bmm");
}
