// Chained backsubstitution on tcgen05 tensor cores (3xTF32), one launch per bounded layer
// (or per two independent layers: chain_launch_pair puts the output layer and the property
// rows in one grid, each CTA running one of the two parameter sets).
//
// For an affine layer m the DeepPoly bound of every neuron is obtained by pushing its
// coefficient row through ReLU_j + affine_j for j = m-1 .. 0 and folding the input box
// into the constant (generated deeppoly.Affine while-loop; the per-substitution sign
// split of constraintflow/gbcsr/tensor_ops.py:765 and inner_prod :370).  Rows are
// independent, so a CTA owns 128 coefficient rows for the whole chain:
//
//   TMEM (512 columns) = two fp32 accumulators of 128 lanes x 256 columns.  Step s writes
//   accumulator s%2; step s+1 reads it back (tcgen05.ld), applies the ReLU sign split
//   with the row's region relaxation, accumulates the constant in a register, splits the
//   result into tf32 hi + lo, and stages it in shared memory as the next A operand.
//   The coefficient matrix never leaves the SM between layers.
//
//   3xTF32: A*W ~= Ahi*Whi + Ahi*Wlo + Alo*Whi, fp32 accumulation in TMEM; W is split,
//   transposed to K-major and pre-swizzled into the UMMA shared-memory image once per
//   call, then streamed chunk by chunk with cp.async.bulk (TMA engine).
//
//   The last substitution (into the input layer) may be wider than 256 columns; it runs
//   in N tiles, each drained by the transform warps straight into the concretisation
//   sum_n (a>=0 ? a*box_s : a*box_{1-s}).  Only one float per row is written to HBM.
//
// Warp roles (320 threads): warps 0-7 transform/epilogue (thread t <-> TMEM lane t%128 <->
// tile row t%128; threads t and t+128 take the two 16-column halves of every chunk),
// warp 8 allocates TMEM and streams W chunks, warp 9 issues the MMAs.  Chunk g uses A stage
// and W stage g % 2; one commit after its MMAs releases both.
// Every mbarrier wait is bounded (cf_tc.cuh); a timeout is recorded in the device error
// word and all roles unwind.
#include <type_traits>

#include "cf_chain.cuh"
#include "cf_tc.cuh"

namespace cf {

using namespace tc;

constexpr uint32_t kAImg = 128 * 128;  // bytes of one 128-row x 32-fp32 A plane
constexpr int kTransformThreads = 256; // warps 0-7
constexpr int kTransformWarps = 8;
constexpr int kProducerWarp = 8;
constexpr int kMmaWarp = 9;
constexpr int kThreads = 320;

void chain_tile(int N, int& tile_n, int& n_tiles) {
  n_tiles = (N + 255) / 256;
  int per = (N + n_tiles - 1) / n_tiles;
  tile_n = ((per + 15) / 16) * 16;
}

size_t chain_wimg_bytes(int K, int N) {
  int tile_n, n_tiles;
  chain_tile(N, tile_n, n_tiles);
  int kchunks = (K + 31) / 32;
  return (size_t)n_tiles * kchunks * 2 * tile_n * 128;
}

// W [K, N] row-major -> per (n tile, k chunk): hi and lo tf32 planes of W^T (tile_n rows x
// 32 k), K-major with the 128-byte swizzle, zero outside [0,N) x [0,K).  One launch prepares
// the images of several layers: job blockIdx.y of the list.
struct PrepJob {
  const float* W;
  uint8_t* img;
  int32_t K, N, tile_n, n_tiles, kchunks;
};
constexpr int kPrepJobs = 32;
struct PrepList {
  PrepJob j[kPrepJobs];
};

__global__ void k_prep_wimg(const __grid_constant__ PrepList L) {
  const PrepJob& J = L.j[blockIdx.y];
  const float* __restrict__ W = J.W;
  uint8_t* __restrict__ img = J.img;
  const int K = J.K, N = J.N, tile_n = J.tile_n, kchunks = J.kchunks;
  int64_t total = (int64_t)J.n_tiles * kchunks * tile_n * 32;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    int kl = (int)(e & 31);
    int64_t q = e >> 5;
    int nl = (int)(q % tile_n);
    q /= tile_n;
    int c = (int)(q % kchunks);
    int t = (int)(q / kchunks);
    int n = t * tile_n + nl, k = c * 32 + kl;
    float v = (n < N && k < K) ? W[(int64_t)k * N + n] : 0.0f;
    float hi = to_tf32(v);
    float lo = to_tf32(v - hi);
    size_t plane = (size_t)tile_n * 128;
    uint8_t* base = img + ((size_t)t * kchunks + c) * 2 * plane;
    uint32_t off = sw128_offset(nl, kl);
    *reinterpret_cast<float*>(base + off) = hi;
    *reinterpret_cast<float*>(base + plane + off) = lo;
  }
}

cf_status chain_prep_weights_batch(const float* const* W, const int* K, const int* N, uint8_t* const* img, int n,
                                   cudaStream_t st) {
  for (int j0 = 0; j0 < n; j0 += kPrepJobs) {
    PrepList L;
    memset(&L, 0, sizeof(L));
    const int m = n - j0 < kPrepJobs ? n - j0 : kPrepJobs;
    int64_t most = 0;
    double bytes = 0.0;
    for (int j = 0; j < m; ++j) {
      PrepJob& J = L.j[j];
      J.W = W[j0 + j];
      J.img = img[j0 + j];
      J.K = K[j0 + j];
      J.N = N[j0 + j];
      chain_tile(J.N, J.tile_n, J.n_tiles);
      J.kchunks = (J.K + 31) / 32;
      const int64_t total = (int64_t)J.n_tiles * J.kchunks * J.tile_n * 32;
      if (total > most) most = total;
      bytes += 4.0 * J.K * J.N + (double)chain_wimg_bytes(J.K, J.N);   // W in, the hi / lo image out
    }
    int64_t blocks = ceil_div(most, 256);
    if (blocks > 148 * 8 / m + 1) blocks = 148 * 8 / m + 1;
    prof_mem_begin(st);
    k_prep_wimg<<<dim3((unsigned)blocks, (unsigned)m), 256, 0, st>>>(L);
    prof_mem_end(st, bytes);
    CF_TRY(check_launch("k_prep_wimg"));
  }
  return CF_OK;
}

cf_status chain_prep_weights(const float* W, int K, int N, uint8_t* img, cudaStream_t st) {
  return chain_prep_weights_batch(&W, &K, &N, &img, 1, st);
}

// Columns of N tile t of a step: tile_n, except the last tile, which covers the remaining
// columns rounded up to 16.
__device__ __forceinline__ int tile_width(const ChainStep& S, int t) {
  const int rest = S.N - t * S.tile_n;
  return rest >= S.tile_n ? S.tile_n : ((rest + 15) / 16) * 16;
}

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~(uintptr_t)1023);
}

// 16 consecutive floats p[k0 .. k0+16) with zeros at k >= K; four 16-byte loads when
// `vec` (16-byte aligned rows and K % 4 == 0), scalar loads otherwise (read-only global memory).
__device__ __forceinline__ void load16g(const float* __restrict__ p, int k0, int K, bool vec, float (&o)[16]) {
  if (vec && k0 + 16 <= K) {
    const float4* q = reinterpret_cast<const float4*>(p + k0);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float4 v = __ldg(q + j);
      o[4 * j] = v.x;
      o[4 * j + 1] = v.y;
      o[4 * j + 2] = v.z;
      o[4 * j + 3] = v.w;
    }
  } else {
#pragma unroll
    for (int e = 0; e < 16; ++e) o[e] = (k0 + e < K) ? __ldg(p + k0 + e) : 0.0f;
  }
}

// Bounded wait by every lane of a warp with a warp-uniform result, so that warp-collective
// code after it (__syncwarp, tcgen05.ld) is reached by all lanes or by none.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, int* err, int site,
                                          uint32_t max_polls = kMaxPolls) {
  const bool ok = mbar_wait(bar, parity, err, site, max_polls);
  return __all_sync(0xffffffffu, ok);
}

// 16 consecutive floats at shared-memory byte address `saddr` (16-byte aligned): four
// ld.shared.v4.  Ordered after the mbarrier waits that publish them (asm volatile).
__device__ __forceinline__ void lds16(uint32_t saddr, float (&o)[16]) {
#pragma unroll
  for (int j = 0; j < 4; ++j)
    asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(o[4 * j]), "=f"(o[4 * j + 1]), "=f"(o[4 * j + 2]), "=f"(o[4 * j + 3])
                 : "r"(saddr + 16u * j));
}
// Elements k0 .. k0+15 of a staged row with zeros at k >= K (bytes past K are not written).
__device__ __forceinline__ void lds16_row(uint32_t row_saddr, int k0, int K, float (&o)[16]) {
  if (k0 + 16 <= K) {
    lds16(row_saddr + 4u * (uint32_t)k0, o);
  } else {
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      float x = 0.0f;
      if (k0 + e < K) asm volatile("ld.shared.f32 %0, [%1];" : "=f"(x) : "r"(row_saddr + 4u * (uint32_t)(k0 + e)));
      o[e] = x;
    }
  }
}

// Column sums over the 32 lanes of a warp of the 16 values every lane holds (lane <->
// row): four halving exchange rounds and a last pair exchange; afterwards v[0] of lanes
// 2c and 2c+1 is the sum of column c.
__device__ __forceinline__ void warp_colsum16(float (&v)[16]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int o = 16 >> r, m = 8 >> r;
    const bool hi = (lane & o) != 0;
#pragma unroll
    for (int j = 0; j < m; ++j) {
      const float send = hi ? v[j] : v[j + m];
      const float recv = __shfl_xor_sync(0xffffffffu, send, o);
      v[j] = (hi ? v[j + m] : v[j]) + recv;
    }
  }
  v[0] += __shfl_xor_sync(0xffffffffu, v[0], 1);
}

// The warp's per-slot column sums of the positive / negative parts of 16 columns n0 ..
// n0+15 (lane <-> row) into zpos / zneg[((cta*4 + w)*2 + slot)*N + n], w = warp % 4.
__device__ __forceinline__ void zono_colsums(float* zpos, float* zneg, int64_t cta, int N, int n0,
                                             const float (&x)[16], bool valid, int slot, bool two_slots) {
  const int lane = threadIdx.x & 31, w = (threadIdx.x >> 5) & 3;
  for (int sl = 0; sl < (two_slots ? 2 : 1); ++sl) {
    float p[16], q[16];
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      const float v = (valid && (!two_slots || slot == sl)) ? x[e] : 0.0f;
      p[e] = fmaxf(v, 0.0f);
      q[e] = fminf(v, 0.0f);
    }
    warp_colsum16(p);
    warp_colsum16(q);
    const int c = n0 + (lane >> 1);
    if ((lane & 1) == 0 && c < N) {
      const size_t idx = (((size_t)cta * 4 + w) * 2 + sl) * (size_t)N + c;
      zpos[idx] = p[0];
      zneg[idx] = q[0];
    }
  }
}

// Zonotope drain of 16 columns n0 .. n0+15 of this thread's row: store the row's values
// (columns below N) and, unless zpos is null (a plain product), the warp's per-slot column
// sums.
__device__ __forceinline__ void zono_drain(float* zout, int64_t zo_bs, int zo_vec, float* zpos, float* zneg,
                                           int64_t cta, int N, int n0, const float (&x)[16], bool valid,
                                           int64_t b, int64_t i, int slot, bool two_slots) {
  if (valid) {
    float* o = zout + b * zo_bs + i * N + n0;
    if (zo_vec && n0 + 16 <= N) {
#pragma unroll
      for (int j = 0; j < 4; ++j)
        reinterpret_cast<float4*>(o)[j] = make_float4(x[4 * j], x[4 * j + 1], x[4 * j + 2], x[4 * j + 3]);
    } else {
#pragma unroll
      for (int e = 0; e < 16; ++e)
        if (n0 + e < N) o[e] = x[e];
    }
  }
  if (zpos) zono_colsums(zpos, zneg, cta, N, n0, x, valid, slot, two_slots);
}

// Shared-memory pieces the transform warps use.
struct ChainSmem {
  uint32_t a_region;     // A stages (shared-memory byte address)
  uint32_t coef;         // two step buffers of relaxation vectors
  uint32_t box;          // input-box rows
  uint64_t* full_a;
  uint64_t* empty_a;
  uint64_t* coef_full;
  uint64_t* coef_empty;
  uint64_t* box_full;
  uint64_t* acc_full;
  float* red;
};

// Transform / epilogue warps (threads 0-255).  Thread -> tile row (TMEM lane) r; the two
// halves take the two 16-column halves of every 32-column chunk.  kStaged: relaxation
// vectors come from the shared-memory step buffers; kBox: the input box from shared memory.
template <bool kStaged, bool kBox, bool kZono>
__device__ __forceinline__ void chain_transform(const ChainParams& P, const ChainSmem& M, uint32_t tbase,
                                                int64_t p0, int64_t tile) {
  const int warp = threadIdx.x >> 5;
  int* err = P.err;
  const int r = threadIdx.x & 127, half = threadIdx.x >> 7;
  bool valid;
  int64_t sb_ = 0, b = 0, i = 0;
  int slot = 0;
  if constexpr (kZono) {
    const int64_t row = tile * 128 + r;
    valid = row < P.rows;
    if (valid) {
      sb_ = row / (P.B * P.R);
      int64_t rem = row - sb_ * P.B * P.R;
      b = rem / P.R;
      i = rem - b * P.R;
      slot = (int)(row / P.R - p0);
    }
  } else {
    // pair q of the tile: lane r & 63, lower bound in lanes 0-63, upper in 64-127
    const int64_t q = tile * 64 + (r & 63);
    valid = q < P.B * P.R;
    sb_ = r >> 6;
    if (valid) {
      b = q / P.R;
      i = q - b * P.R;
      slot = (int)(b - p0);
    }
  }
  const bool lower = sb_ == 0;
  // zonotope mode: does the CTA's row range reach into a second region
  const bool two_slots = kZono && ((P.rows - 1 < tile * 128 + 127 ? P.rows - 1 : tile * 128 + 127) / P.R) != p0;
  float cacc = (valid && P.c0 && half == 0) ? P.c0[i] : 0.0f;
  float conc = 0.0f;
  const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
  // this thread's four 16-byte slots of a swizzled 128-byte A row (the same every chunk)
  uint32_t soff[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) soff[q] = (uint32_t)r * 128u + ((((uint32_t)(half * 4 + q)) ^ ((uint32_t)r & 7u)) << 4);
  const float* a0row = P.A0 + sb_ * P.a_ss + b * P.a_bs + i * P.a_rs;
  // input box: staged rows (l0 then u0 per slot) or global memory
  const uint32_t box_pos = M.box + 4u * (uint32_t)((size_t)slot * 2 * P.n0 + (lower ? 0 : P.n0));
  const uint32_t box_neg = M.box + 4u * (uint32_t)((size_t)slot * 2 * P.n0 + (lower ? P.n0 : 0));
  const float* gpos = (lower ? P.l0 : P.u0) + b * P.ld_box;
  const float* gneg = (lower ? P.u0 : P.l0) + b * P.ld_box;
  uint32_t g = 0, nacc = 0;
  bool ok = true;
  for (int s = 0; s < P.S && ok; ++s) {
    const ChainStep& S = P.st[s];
    const int K = S.K;
    const bool cvec = (K & 3) == 0;
    if (s > 0) {
      if (!warp_wait(M.acc_full, nacc & 1, err, 31, P.max_polls)) { ok = false; break; }
      ++nacc;
      tc_fence_after();
    }
    // relaxation rows of this step: staged (shared-memory byte addresses) or global pointers
    uint32_t s_pf = 0, s_nf = 0, s_mu = 0, s_bias = 0;
    const float *g_pf = nullptr, *g_nf = nullptr, *g_mu = nullptr, *g_bias = S.bias;
    if (kStaged) {
      if (!warp_wait(&M.coef_full[s & 1], (s >> 1) & 1, err, 34, P.max_polls)) { ok = false; break; }
      const uint32_t cbuf = M.coef + 4u * (uint32_t)((s & 1) * kCoefBufFloats);
      const uint32_t al = cbuf + 4u * (uint32_t)(slot * 3 * kCoefRow), la = al + 4u * kCoefRow;
      s_pf = lower ? al : la;
      s_nf = lower ? la : al;
      s_mu = al + 8u * kCoefRow;
      s_bias = cbuf + 4u * (uint32_t)(kCoefSlots * 3 * kCoefRow);
    } else if (S.alpha != nullptr) {
      g_pf = (lower ? S.alpha : S.lam) + b * K;
      g_nf = (lower ? S.lam : S.alpha) + b * K;
      g_mu = S.mu + b * K;
    }
    const uint32_t src_acc = tbase + (uint32_t)((s - 1) & 1) * 256u + lane_off;
    const int src_cols = s > 0 ? P.st[s - 1].tile_n : 0;

    // one tile of chunks, specialised on the ReLU and on the first N tile (which also
    // accumulates the constant: mu and bias terms)
    auto tile_chunks = [&](auto relu_c, auto first_c) -> bool {
      constexpr bool kRelu = decltype(relu_c)::value, kFirst = decltype(first_c)::value;
      // zonotope mode: every chunk's rows come from global memory; the next chunk's values
      // are loaded one chunk ahead so that their latency overlaps this chunk's transform
      float vnext[16];
      if constexpr (kZono) load16g(a0row, half * 16, valid ? K : 0, P.a0_vec, vnext);
      for (int c = 0; c < S.kchunks; ++c, ++g) {
        const uint32_t stage = g % kAStages, round = g / kAStages;
        const int k0 = c * 32 + half * 16;
        float pv[16], nv[16], mv[16], bv[16], v[16];
        if (kStaged) {
          if (kRelu) {
            lds16_row(s_pf, k0, K, pv);
            lds16_row(s_nf, k0, K, nv);
            if (kFirst) lds16_row(s_mu, k0, K, mv);
          }
          if (kFirst) lds16_row(s_bias, k0, K, bv);
        } else {
          if (kRelu) {
            load16g(g_pf, k0, K, cvec, pv);
            load16g(g_nf, k0, K, cvec, nv);
            if (kFirst) load16g(g_mu, k0, K, cvec, mv);
          }
          if (kFirst) load16g(g_bias, k0, K, cvec, bv);
        }
        if (kZono) {
#pragma unroll
          for (int e = 0; e < 16; ++e) v[e] = vnext[e];
          if (c + 1 < S.kchunks) load16g(a0row, k0 + 32, valid ? K : 0, P.a0_vec, vnext);
        } else if (s == 0) {
          load16g(a0row, k0, valid ? K : 0, P.a0_vec, v);
        } else if (k0 < src_cols) {
          // columns [K, tile_n) of the previous accumulator are exact zeros (zero-padded W);
          // a half-chunk past tile_n was never written and is skipped
          tmem_ld16(src_acc + (uint32_t)k0, v);
          tmem_ld_wait();
        } else {
#pragma unroll
          for (int e = 0; e < 16; ++e) v[e] = 0.0f;
        }
        float hi[16], lo[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          float tr = v[e];
          if (kRelu) {
            const float pos = fmaxf(v[e], 0.0f), neg = fminf(v[e], 0.0f);
            tr = fmaf(pos, pv[e], neg * nv[e]);
            if (kFirst) cacc = fmaf(lower ? neg : pos, mv[e], cacc);
          }
          if (kFirst) cacc = fmaf(tr, bv[e], cacc);
          split_tf32(tr, hi[e], lo[e]);
        }
        // only the stage write waits for the MMAs that read this stage kAStages chunks ago
        if (!warp_wait(&M.empty_a[stage], (round & 1) ^ 1, err, 32, P.max_polls)) return false;
        const uint32_t sbase = M.a_region + stage * 2 * kAImg;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(sbase + soff[q]), "f"(hi[4 * q]),
                       "f"(hi[4 * q + 1]), "f"(hi[4 * q + 2]), "f"(hi[4 * q + 3])
                       : "memory");
          asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(sbase + kAImg + soff[q]), "f"(lo[4 * q]),
                       "f"(lo[4 * q + 1]), "f"(lo[4 * q + 2]), "f"(lo[4 * q + 3])
                       : "memory");
        }
        // this thread's stores are made visible to the tensor core (async proxy)
        fence_proxy_async_smem();
        tc_fence_before();
        mbar_arrive(&M.full_a[stage]);
      }
      return true;
    };

    const bool relu = S.alpha != nullptr;
    for (int t = 0; t < S.n_tiles && ok; ++t) {
      using T = std::true_type;
      using F = std::false_type;
      if (relu)
        ok = t == 0 ? tile_chunks(T{}, T{}) : tile_chunks(T{}, F{});
      else
        ok = t == 0 ? tile_chunks(F{}, T{}) : tile_chunks(F{}, F{});
      if (!ok) break;
      if (s == P.S - 1) {
        // drain output tile t straight into the concretisation; halves take alternate
        // 16-column groups
        const int ng = tile_width(S, t) / 16, nlim = valid ? S.N : 0;
        if (kBox && !warp_wait(M.box_full, 0, err, 35, P.max_polls)) { ok = false; break; }
        if (!warp_wait(M.acc_full, nacc & 1, err, 33, P.max_polls)) { ok = false; break; }
        ++nacc;
        tc_fence_after();
        const uint32_t dst = tbase + (uint32_t)(s & 1) * 256u + lane_off;
        for (int q = half; q < ng; q += 2) {
          const int n0 = t * S.tile_n + q * 16;
          if constexpr (kZono) {
            float x[16];
            tmem_ld16(dst + (uint32_t)(q * 16), x);
            tmem_ld_wait();
            zono_drain(P.zout, P.zo_bs, P.zo_vec, P.zpos, P.zneg, tile, S.N, n0, x, valid, b, i, slot,
                       two_slots);
            continue;
          }
          float pb[16], nb[16], x[16];
          if (kBox) {
            lds16_row(box_pos, n0, nlim, pb);
            lds16_row(box_neg, n0, nlim, nb);
          } else {
            load16g(gpos, n0, nlim, P.box_vec, pb);
            load16g(gneg, n0, nlim, P.box_vec, nb);
          }
          tmem_ld16(dst + (uint32_t)(q * 16), x);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 16; ++e) conc = fmaf(x[e], x[e] >= 0.0f ? pb[e] : nb[e], conc);
        }
        tc_fence_before();
      }
    }
    // step buffer s%2 may be refilled (for step s+2)
    if (kStaged && ok) {
      __syncwarp();
      if ((threadIdx.x & 31) == 0) mbar_arrive(&M.coef_empty[s & 1]);
    }
  }
  if constexpr (kZono) return;   // rows and column sums were written by the drain
  // combine the two halves of every row
  if (half == 1) M.red[r] = conc + cacc;
  asm volatile("bar.sync 1, %0;" ::"r"(kTransformThreads) : "memory");
  float res = 0.0f;
  if (half == 0 && valid && ok) {
    res = (conc + cacc) + M.red[r];
    (lower ? P.out_l : P.out_u)[b * P.ld_out + i] = res;
    if (P.out_l64) (lower ? P.out_l64 : P.out_u64)[b * P.ld_out64 + i] = (double)res;
  }
  if (P.relu.alpha != nullptr) {
    // both bounds of neuron (b, i) are in this tile (lanes r and r + 64): relax the ReLU above
    if (half == 0) M.red[128 + r] = res;
    asm volatile("bar.sync 1, %0;" ::"r"(kTransformThreads) : "memory");
    if (half == 0 && r < 64 && valid && ok) relu_relax_store(P.relu, b, i, M.red[128 + r], M.red[192 + r]);
  }
}

// One CTA of k_chain on parameter set kWhich of the launch (a compile-time choice, so that
// every parameter is read at a fixed offset of the parameter space), tile `tile` of its rows.
template <bool kZono, int kWhich>
__device__ __forceinline__ void chain_cta(const ChainPair& PP, int64_t tile) {
  const ChainParams& P = PP.p[kWhich];
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  // shared memory: kAStages A-operand stages (hi, lo planes), kWStages weight stages (hi, lo
  // planes of tile_n rows), two step buffers of relaxation vectors, the input-box rows of
  // the CTA's regions, then the mbarriers.  Chunk g uses A stage and W stage g % 2; the
  // commit after its MMAs (empty_a) releases both.
  static_assert(kAStages == kWStages, "one barrier releases an A stage and a W stage");
  const uint32_t w_stage_bytes = P.stage_bytes;
  uint8_t* a_region = smem;
  uint8_t* w_region = smem + kAStages * 2 * kAImg;
  float* coef_region = reinterpret_cast<float*>(w_region + kWStages * w_stage_bytes);
  float* box_region = coef_region + 2 * kCoefBufFloats;
  uint64_t* full_a = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(box_region) + P.box_smem_bytes);
  uint64_t* empty_a = full_a + kAStages;
  uint64_t* full_w = empty_a + kAStages;
  uint64_t* coef_full = full_w + kWStages;
  uint64_t* coef_empty = coef_full + 2;
  uint64_t* box_full = coef_empty + 2;
  uint64_t* acc_full = box_full + 1;
  uint64_t* mma_done = acc_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  float* red = reinterpret_cast<float*>(tmem_slot + 4);  // [256]: second-half sums, then the rows' bounds
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int* err = P.err;
  // the slots of this CTA's rows: regions p0 .. p0+n_pairs-1 (bounding mode) or (bound,
  // region) pairs p = row / R (zonotope mode).  With at most kCoefSlots of them, their
  // relaxation vectors and box rows are staged in shared memory.
  int64_t p0;
  int n_pairs;
  if (kZono) {
    const int64_t row_first = tile * 128;
    const int64_t row_last = (row_first + 127 < P.rows ? row_first + 127 : P.rows - 1);
    p0 = row_first / P.R;
    n_pairs = (int)(row_last / P.R - p0 + 1);
  } else {
    const int64_t q_first = tile * 64, q_all = P.B * P.R;
    const int64_t q_last = (q_first + 63 < q_all ? q_first + 63 : q_all - 1);
    p0 = q_first / P.R;
    n_pairs = (int)(q_last / P.R - p0 + 1);
  }
  const bool staged = P.coef_ok && n_pairs <= kCoefSlots;
  const bool box_staged = staged && P.box_smem_bytes > 0;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kAStages; ++i) {
      mbar_init(&full_a[i], kTransformThreads);
      mbar_init(&empty_a[i], 1);
    }
    for (int i = 0; i < kWStages; ++i) mbar_init(&full_w[i], 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&coef_full[i], 1);
      mbar_init(&coef_empty[i], kTransformWarps);
    }
    mbar_init(box_full, 1);
    mbar_init(acc_full, 1);
    mbar_init(mma_done, 1);
    fence_mbar_init();
  }
  if (warp == kProducerWarp) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  // an earlier launch of this pass recorded an error (a timeout, or a CROWN layer that
  // took the all-crossing branch): do nothing, before any copy or MMA is issued
  if (threadIdx.x == 0) tmem_slot[1] = *(volatile int*)err != 0 ? 1u : 0u;
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;
  if (tmem_slot[1] != 0) {
    if (warp == kProducerWarp) tmem_dealloc(tbase, 512);
    return;
  }

  if (warp == kProducerWarp) {
    // ---------------------------------------------------------------- W producer
    if (lane == 0) {
      uint32_t g = 0;
      int coef_n = 0;  // step buffers of relaxation vectors issued
      if (box_staged) {
        // input-box rows (l0 then u0) of every (bound, region) pair of the CTA
        const uint32_t rb = (uint32_t)P.n0 * 4u;
        mbar_arrive_expect_tx(box_full, 2u * rb * (uint32_t)n_pairs);
        for (int j = 0; j < n_pairs; ++j) {
          const int64_t b = (p0 + j) % P.B;
          bulk_g2s(box_region + (size_t)j * 2 * P.n0, P.l0 + b * P.ld_box, rb, box_full);
          bulk_g2s(box_region + (size_t)j * 2 * P.n0 + P.n0, P.u0 + b * P.ld_box, rb, box_full);
        }
      }
      for (int s = 0; s < P.S; ++s) {
        const ChainStep& S = P.st[s];
        const uint32_t plane = (uint32_t)S.tile_n * 128u;  // image plane stride
        if (staged) {
          // step s's alpha / lambda / mu rows of the CTA's regions and the layer bias, into
          // step buffer s%2 once the transform warps have finished step s-2
          const int cb = s & 1;
          if (!mbar_wait(&coef_empty[cb], ((s >> 1) & 1) ^ 1, err, 13, P.max_polls)) goto done_w;
          const uint32_t kb = (uint32_t)S.K * 4u;
          const bool relu = S.alpha != nullptr;
          float* dst = coef_region + cb * kCoefBufFloats;
          mbar_arrive_expect_tx(&coef_full[cb], kb * (relu ? 3u * (uint32_t)n_pairs + 1u : 1u));
          if (relu) {
            for (int j = 0; j < n_pairs; ++j) {
              const int64_t b = (p0 + j) % P.B;
              bulk_g2s(dst + j * 3 * kCoefRow, S.alpha + b * S.K, kb, &coef_full[cb]);
              bulk_g2s(dst + j * 3 * kCoefRow + kCoefRow, S.lam + b * S.K, kb, &coef_full[cb]);
              bulk_g2s(dst + j * 3 * kCoefRow + 2 * kCoefRow, S.mu + b * S.K, kb, &coef_full[cb]);
            }
          }
          bulk_g2s(dst + kCoefSlots * 3 * kCoefRow, S.bias, kb, &coef_full[cb]);
          ++coef_n;
        }
        for (int t = 0; t < S.n_tiles; ++t) {
          for (int c = 0; c < S.kchunks; ++c, ++g) {
            const uint32_t stage = g % kWStages, round = g / kWStages;
            // chunk g's A stage and W stage are released together (empty_a, one commit)
            if (!mbar_wait(&empty_a[stage], (round & 1) ^ 1, err, 11, P.max_polls)) goto done_w;
            uint8_t* sb = w_region + stage * w_stage_bytes;
            const uint8_t* src = S.wimg + ((size_t)t * S.kchunks + c) * 2 * plane;
            const uint32_t bytes = (uint32_t)tile_width(S, t) * 128u;  // rows the MMAs read
            mbar_arrive_expect_tx(&full_w[stage], 2 * bytes);
            bulk_g2s(sb, src, bytes, &full_w[stage]);
            bulk_g2s(sb + P.w_lo_off, src + plane, bytes, &full_w[stage]);
          }
        }
      }
    done_w:
      // copies still in flight (error path) land before the CTA can exit
      for (uint32_t x = 0; x < kWStages && x < g; ++x) {
        const uint32_t gl = g - 1 - x, stage = gl % kWStages, round = gl / kWStages;
        mbar_wait_drain(&full_w[stage], round & 1, err, 12, P.max_polls);
      }
      for (int x = 0; x < 2 && x < coef_n; ++x) {
        const int sl = coef_n - 1 - x;
        mbar_wait_drain(&coef_full[sl & 1], (sl >> 1) & 1, err, 14, P.max_polls);
      }
      if (box_staged) mbar_wait_drain(box_full, 0, err, 15, P.max_polls);
    }
  } else if (warp == kMmaWarp) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      uint32_t g = 0;
      for (int s = 0; s < P.S; ++s) {
        const ChainStep& S = P.st[s];
        const uint32_t acc = tbase + (uint32_t)(s & 1) * 256u;
        for (int t = 0; t < S.n_tiles; ++t) {
          // the last N tile is only as wide as the columns left (a multiple of 16)
          const uint32_t idesc = idesc_tf32((uint32_t)tile_width(S, t));
          for (int c = 0; c < S.kchunks; ++c, ++g) {
            // k-steps of 8 that reach below K (the rest of the chunk is zero padding)
            const int nks = min(4, (S.K - c * 32 + 7) / 8);
            const uint32_t as = g % kAStages, ar = g / kAStages, ws = g % kWStages, wr = g / kWStages;
            if (!mbar_wait(&full_a[as], ar & 1, err, 21, P.max_polls)) goto done_m;
            if (!mbar_wait(&full_w[ws], wr & 1, err, 22, P.max_polls)) goto done_m;
            tc_fence_after();
            const uint32_t sa = smem_u32(a_region + as * 2 * kAImg), sw = smem_u32(w_region + ws * w_stage_bytes);
            const uint32_t a_hi = sa, a_lo = sa + kAImg, w_hi = sw, w_lo = sw + P.w_lo_off;
#pragma unroll
            for (int ks = 0; ks < 4; ++ks) {
              if (ks >= nks) break;
              const uint64_t dah = sw128_desc(a_hi + ks * 32), dal = sw128_desc(a_lo + ks * 32);
              const uint64_t dwh = sw128_desc(w_hi + ks * 32), dwl = sw128_desc(w_lo + ks * 32);
              mma_tf32(acc, dal, dwh, idesc, (c | ks) != 0);
              mma_tf32(acc, dah, dwl, idesc, 1);
              mma_tf32(acc, dah, dwh, idesc, 1);
            }
            // one commit releases both stages (a second commit per chunk cost ~1% of the launch)
            mma_commit(&empty_a[as]);
          }
          // (failure-path test: the first step's accumulator-ready arrival is withheld, so the
          // transform warps' bounded wait for it gives up)
          if (!(P.withhold_acc && s == 0)) mma_commit(acc_full);
        }
      }
    done_m:
      // every MMA issued above has completed before TMEM is released
      mma_commit(mma_done);
      mbar_wait_drain(mma_done, 0, err, 23, P.max_polls);
    }
  } else {
    // ---------------------------------------------------------------- transform warps
    const ChainSmem M{smem_u32(a_region), smem_u32(coef_region), smem_u32(box_region), full_a, empty_a,
                      coef_full, coef_empty, box_full, acc_full, red};
    if constexpr (kZono) {
      if (staged)
        chain_transform<true, false, true>(P, M, tbase, p0, tile);
      else
        chain_transform<false, false, true>(P, M, tbase, p0, tile);
    } else {
      if (box_staged)
        chain_transform<true, true, false>(P, M, tbase, p0, tile);
      else if (staged)
        chain_transform<true, false, false>(P, M, tbase, p0, tile);
      else
        chain_transform<false, false, false>(P, M, tbase, p0, tile);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kProducerWarp) tmem_dealloc(tbase, 512);
}

// CTAs [0, split) run parameter set 0, the rest set 1 (two independent layers in one launch;
// the zonotope mode uses set 0 only)
template <bool kZono>
__global__ void __launch_bounds__(kThreads, 1) k_chain(const __grid_constant__ ChainPair PP) {
  if constexpr (kZono) {
    chain_cta<true, 0>(PP, (int64_t)blockIdx.x);
  } else {
    if ((int64_t)blockIdx.x < PP.split) chain_cta<false, 0>(PP, (int64_t)blockIdx.x);
    else chain_cta<false, 1>(PP, (int64_t)blockIdx.x - PP.split);
  }
}

// Checks P and fills the launch fields of its copy Q; smem: the dynamic shared memory its
// CTAs need, tiles: its CTA count.
static cf_status chain_prepare(const ChainParams& P, ChainParams& Q, size_t& smem, int64_t& tiles) {
  CF_REQUIRE(P.S >= 1 && P.S <= kChainMaxSteps, CF_ERR_UNSUPPORTED, "chain: %d steps", P.S);
  int tn_max = 0;
  for (int s = 0; s < P.S; ++s) {
    const ChainStep& S = P.st[s];
    CF_REQUIRE(S.tile_n >= 16 && S.tile_n <= 256 && S.tile_n % 16 == 0, CF_ERR_SHAPE, "chain: tile_n %d", S.tile_n);
    CF_REQUIRE(s == P.S - 1 || S.n_tiles == 1, CF_ERR_UNSUPPORTED, "chain: wide intermediate layer");
    CF_REQUIRE(s == 0 || S.K <= 256, CF_ERR_UNSUPPORTED, "chain: K %d > 256", S.K);
    CF_REQUIRE(s == 0 || S.K == P.st[s - 1].N, CF_ERR_SHAPE, "chain: K/N mismatch at step %d", s);
    if (S.tile_n > tn_max) tn_max = S.tile_n;
  }
  CF_REQUIRE(P.st[P.S - 1].N == P.n0, CF_ERR_SHAPE, "chain: last step does not reach the input");
  Q = P;
  if (Q.ld_box == 0) Q.ld_box = Q.n0;
  // bounded-wait limit: kMaxPolls, or CF_WAIT_POLLS (>= 256) for the failure-path test;
  // CF_FAULT=chain_withhold_acc withholds one arrival so that a wait runs out
  Q.max_polls = kMaxPolls;
  if (const char* e = getenv("CF_WAIT_POLLS")) {
    const long v = strtol(e, nullptr, 10);
    if (v >= 256 && v < (long)kMaxPolls) Q.max_polls = (uint32_t)v;
  }
  Q.withhold_acc = fault_injected("chain_withhold_acc") ? 1 : 0;
  CF_REQUIRE(Q.ld_box >= Q.n0, CF_ERR_SHAPE, "chain: box row stride %lld < %lld", (long long)Q.ld_box,
             (long long)Q.n0);
  // weight stage: hi plane then lo plane, each tn_max rows x 128 bytes (1024-aligned)
  Q.w_lo_off = (uint32_t)tn_max * 128u;
  Q.stage_bytes = 2u * (uint32_t)tn_max * 128u;
  // relaxation vectors are staged through shared memory (bulk copies: 16-byte aligned rows
  // of K <= 256 floats, K % 4 == 0); otherwise the transform warps read them from global memory
  auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  bool coef_ok = true;
  for (int s = 0; s < P.S; ++s) {
    const ChainStep& S = P.st[s];
    coef_ok = coef_ok && S.K <= kCoefRow && S.K % 4 == 0 && S.bias != nullptr && a16(S.bias);
    if (S.alpha) coef_ok = coef_ok && a16(S.alpha) && a16(S.lam) && a16(S.mu);
  }
  Q.coef_ok = coef_ok ? 1 : 0;
  const size_t fixed = 1024 + (size_t)kAStages * 2 * kAImg + (size_t)kWStages * Q.stage_bytes +
                       (size_t)2 * kCoefBufFloats * 4 + (2 * kAStages + kWStages + 4 + 3) * 8 + 16 + 256 * 4;
  // input-box rows of up to kCoefSlots (bound, region) pairs, when they fit
  const size_t box_bytes = (size_t)kCoefSlots * 2 * P.n0 * 4;
  const bool box_ok = !P.zono && coef_ok && P.n0 % 4 == 0 && Q.ld_box % 4 == 0 && a16(P.l0) && a16(P.u0) &&
                      fixed + box_bytes <= 227 * 1024;
  Q.box_smem_bytes = box_ok ? (uint32_t)box_bytes : 0u;
  smem = fixed + Q.box_smem_bytes;
  // at least 116 KB so that one CTA (which holds all 512 TMEM columns) runs per SM
  if (smem < 116 * 1024) smem = 116 * 1024;
  if (P.zono) {
    CF_REQUIRE(P.S == 1 && P.R >= 128 && P.rows % P.R == 0 && P.zout && (P.zpos != nullptr) == (P.zneg != nullptr),
               CF_ERR_UNSUPPORTED, "chain: zonotope mode needs one step, >= 128 rows per region and its outputs");
    Q.zo_vec = (P.st[0].N % 4 == 0 && a16(P.zout) && (P.zo_bs % 4) == 0) ? 1 : 0;
  }
  CF_REQUIRE(smem <= 227 * 1024, CF_ERR_UNSUPPORTED, "chain: %zu bytes of shared memory", smem);
  tiles = P.zono ? ceil_div(P.rows, 128) : ceil_div(P.B * P.R, 64);
  CF_REQUIRE(tiles <= 0x3fffffff, CF_ERR_SHAPE, "chain: too many rows");
  return CF_OK;
}

static cf_status chain_run(const ChainPair& PP, bool zono, int64_t grid, size_t smem, cudaStream_t st) {
  auto kern = zono ? k_chain<true> : k_chain<false>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
  if (e != cudaSuccess) {
    set_error("chain: cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    return CF_ERR_CUDA;
  }
  if (grid == 0) return CF_OK;
  kern<<<(unsigned)grid, kThreads, smem, st>>>(PP);
  return check_launch(zono ? "k_chain (zonotope)" : "k_chain");
}

cf_status chain_launch(const ChainParams& P, cudaStream_t st) {
  ChainPair PP;
  memset(&PP, 0, sizeof(PP));
  size_t smem = 0;
  int64_t tiles = 0;
  CF_TRY(chain_prepare(P, PP.p[0], smem, tiles));
  PP.split = tiles;
  return chain_run(PP, P.zono != 0, tiles, smem, st);
}

cf_status chain_launch_pair(const ChainParams& P0, const ChainParams& P1, cudaStream_t st) {
  CF_REQUIRE(!P0.zono && !P1.zono, CF_ERR_UNSUPPORTED, "chain: paired launches are bounding-mode only");
  ChainPair PP;
  memset(&PP, 0, sizeof(PP));
  size_t smem0 = 0, smem1 = 0;
  int64_t tiles0 = 0, tiles1 = 0;
  CF_TRY(chain_prepare(P0, PP.p[0], smem0, tiles0));
  CF_TRY(chain_prepare(P1, PP.p[1], smem1, tiles1));
  PP.split = tiles0;
  return chain_run(PP, false, tiles0 + tiles1, smem0 > smem1 ? smem0 : smem1, st);
}

// ------------------------------------------------------------------ persistent zonotope GEMM
// 448 threads: warps 0-7 stage the A operand (coalesced 16-byte pieces of the chunk's rows
// and of lam loaded from global memory one chunk ahead, scaled, split into tf32 hi + lo,
// written at their SW128 positions), warp 8 allocates TMEM
// and streams the W^T chunks (bulk copies), warp 9 issues the 3xTF32 MMAs, warps 10-13
// drain (thread <-> TMEM lane).  A CTA loops over the row tiles blockIdx.x, +gridDim.x,
// ...; tile i accumulates in TMEM buffer i % 2, so the drain of tile i overlaps the MMAs
// of tile i+1.  Every wait is bounded.  (Staging the 128 rows of a chunk through per-row
// bulk copies instead was 2.8x slower: the copy engine handles 128-byte copies slowly.)
constexpr int kZtThreads = 448;

__global__ void __launch_bounds__(kZtThreads, 1) k_zono_persist(const __grid_constant__ ZonoTcParams P) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* a_region = smem;                               // 2 stages x (hi, lo) planes
  uint8_t* w_region = smem + 2 * 2 * kAImg;               // 2 stages x stage_bytes
  uint64_t* bars = reinterpret_cast<uint64_t*>(w_region + 2 * P.stage_bytes);
  uint64_t* full_a = bars;
  uint64_t* empty_a = bars + 2;
  uint64_t* full_w = bars + 4;     // (chunk g's W stage is released with its A stage: empty_a)
  uint64_t* acc_full = bars + 6;
  uint64_t* acc_empty = bars + 8;
  uint64_t* mma_done = bars + 10;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 11);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int* err = P.err;
  const int64_t n_tiles = (P.rows + 127) / 128;
  const int64_t my_tiles = (int64_t)blockIdx.x < n_tiles ? (n_tiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&full_a[i], kTransformThreads);
      mbar_init(&empty_a[i], 1);
      mbar_init(&full_w[i], 1);
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 4);
    }
    mbar_init(mma_done, 1);
    fence_mbar_init();
  }
  if (warp == kProducerWarp) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  if (threadIdx.x == 0) tmem_slot[1] = *(volatile int*)err != 0 ? 1u : 0u;
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;
  if (tmem_slot[1] != 0) {
    if (warp == kProducerWarp) tmem_dealloc(tbase, 512);
    return;
  }
  const uint32_t plane = (uint32_t)P.tile_n * 128u;

  if (warp == kProducerWarp) {
    // ---------------------------------------------------------------- W^T chunks
    if (lane == 0) {
      uint32_t g = 0;
      for (int64_t i = 0; i < my_tiles; ++i) {
        for (int c = 0; c < P.kchunks; ++c, ++g) {
          const uint32_t stage = g & 1u, round = g >> 1;
          if (!mbar_wait(&empty_a[stage], (round & 1u) ^ 1u, err, 51)) goto done_w;
          uint8_t* sb = w_region + stage * P.stage_bytes;
          const uint8_t* src = P.wimg + (size_t)c * 2 * plane;
          mbar_arrive_expect_tx(&full_w[stage], 2 * plane);
          bulk_g2s(sb, src, plane, &full_w[stage]);
          bulk_g2s(sb + P.w_lo_off, src + plane, plane, &full_w[stage]);
        }
      }
    done_w:
      for (uint32_t x = 0; x < 2 && x < g; ++x) {
        const uint32_t gl = g - 1 - x;
        mbar_wait_drain(&full_w[gl & 1u], (gl >> 1) & 1u, err, 52);
      }
    }
  } else if (warp == kMmaWarp) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_tf32((uint32_t)P.tile_n);
      uint32_t g = 0;
      for (int64_t i = 0; i < my_tiles; ++i) {
        const uint32_t buf = (uint32_t)(i & 1);
        if (i >= 2 && !mbar_wait(&acc_empty[buf], (uint32_t)((i >> 1) & 1) ^ 1u, err, 53)) goto done_m;
        tc_fence_after();
        const uint32_t acc = tbase + buf * 256u;
        for (int c = 0; c < P.kchunks; ++c, ++g) {
          const int nks = min(4, (P.K - c * 32 + 7) / 8);
          const uint32_t stage = g & 1u, round = g >> 1;
          if (!mbar_wait(&full_a[stage], round & 1u, err, 54)) goto done_m;
          if (!mbar_wait(&full_w[stage], round & 1u, err, 55)) goto done_m;
          tc_fence_after();
          const uint32_t sa = smem_u32(a_region + stage * 2 * kAImg), sw = smem_u32(w_region + stage * P.stage_bytes);
          const uint32_t a_hi = sa, a_lo = sa + kAImg, w_hi = sw, w_lo = sw + P.w_lo_off;
#pragma unroll
          for (int ks = 0; ks < 4; ++ks) {
            if (ks >= nks) break;
            const uint64_t dah = sw128_desc(a_hi + ks * 32), dal = sw128_desc(a_lo + ks * 32);
            const uint64_t dwh = sw128_desc(w_hi + ks * 32), dwl = sw128_desc(w_lo + ks * 32);
            mma_tf32(acc, dal, dwh, idesc, (c | ks) != 0);
            mma_tf32(acc, dah, dwl, idesc, 1);
            mma_tf32(acc, dah, dwh, idesc, 1);
          }
          mma_commit(&empty_a[stage]);   // releases the A stage and the W stage
        }
        mma_commit(&acc_full[buf]);
      }
    done_m:
      mma_commit(mma_done);
      mbar_wait_drain(mma_done, 0, err, 56);
    }
  } else if (warp < kTransformWarps) {
    // ---------------------------------------------------------------- A operand
    // Thread t handles the 16-byte pieces f = t + 256*q (q < 4) of the 128-row x 128-byte
    // chunk: row f / 8, piece f % 8 -- eight consecutive threads read one row's 128 bytes
    // (coalesced), scale by the row's region's lam, split, and write the piece to its SW128
    // position (row*128 + ((piece ^ row%8) << 4)) in the hi and lo planes.  Requires K % 4 == 0.
    const int t = threadIdx.x;
    uint32_t g = 0;
    bool ok = true;
    const float* prow[4];
    const float* plam[4];
    bool pval[4];
    auto tile_rows = [&](int64_t i) {
      const int64_t first = ((int64_t)blockIdx.x + i * gridDim.x) * 128;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int64_t row = first + ((t + 256 * q) >> 3);
        pval[q] = row < P.rows;
        const int64_t b = pval[q] ? row / P.E : 0, e = pval[q] ? row - b * P.E : 0;
        prow[q] = P.A + b * P.a_bs + e * P.K;
        plam[q] = P.lam ? P.lam + b * P.K : nullptr;
      }
    };
    // chunk c's pieces (and lam) of the current rows; zeros past the rows or columns
    auto load_chunk = [&](int c, float4 (&v)[4], float4 (&l)[4]) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int k = c * 32 + ((t + 256 * q) & 7) * 4;
        const bool in = pval[q] && k < P.K;
        v[q] = in ? __ldg(reinterpret_cast<const float4*>(prow[q] + k)) : make_float4(0.f, 0.f, 0.f, 0.f);
        l[q] = (in && plam[q]) ? __ldg(reinterpret_cast<const float4*>(plam[q] + k)) : make_float4(1.f, 1.f, 1.f, 1.f);
      }
    };
    float4 vnext[4], lnext[4];
    if (my_tiles > 0) {
      tile_rows(0);
      load_chunk(0, vnext, lnext);
    }
    for (int64_t i = 0; i < my_tiles && ok; ++i) {
      for (int c = 0; c < P.kchunks; ++c, ++g) {
        const uint32_t stage = g & 1u, round = g >> 1;
        float4 hi[4], lo[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float4 v = vnext[q], l = lnext[q];
          split_tf32(v.x * l.x, hi[q].x, lo[q].x);
          split_tf32(v.y * l.y, hi[q].y, lo[q].y);
          split_tf32(v.z * l.z, hi[q].z, lo[q].z);
          split_tf32(v.w * l.w, hi[q].w, lo[q].w);
        }
        if (c + 1 < P.kchunks) {
          load_chunk(c + 1, vnext, lnext);
        } else if (i + 1 < my_tiles) {
          tile_rows(i + 1);
          load_chunk(0, vnext, lnext);
        }
        if (!warp_wait(&empty_a[stage], (round & 1u) ^ 1u, err, 57)) {
          ok = false;
          break;
        }
        const uint32_t sbase = smem_u32(a_region) + stage * 2 * kAImg;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint32_t f = (uint32_t)(t + 256 * q), row = f >> 3, piece = f & 7u;
          const uint32_t off = row * 128u + ((piece ^ (row & 7u)) << 4);
          asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(sbase + off), "f"(hi[q].x), "f"(hi[q].y),
                       "f"(hi[q].z), "f"(hi[q].w)
                       : "memory");
          asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(sbase + kAImg + off), "f"(lo[q].x),
                       "f"(lo[q].y), "f"(lo[q].z), "f"(lo[q].w)
                       : "memory");
        }
        fence_proxy_async_smem();
        mbar_arrive(&full_a[stage]);
      }
    }
  } else {
    // ---------------------------------------------------------------- drain (warps 10-13)
    const int q4 = warp & 3;
    const uint32_t lane_off = (uint32_t)(q4 * 32) << 16;
    for (int64_t i = 0; i < my_tiles; ++i) {
      const uint32_t buf = (uint32_t)(i & 1);
      const int64_t tile = (int64_t)blockIdx.x + i * gridDim.x;
      const int64_t first = tile * 128, last = first + 127 < P.rows ? first + 127 : P.rows - 1;
      const int64_t p0 = first / P.E;
      const bool two_slots = last / P.E != p0;
      const int64_t row = first + q4 * 32 + lane;
      const bool valid = row < P.rows;
      const int64_t b = valid ? row / P.E : 0, e = valid ? row - b * P.E : 0;
      const int slot = valid ? (int)(b - p0) : 0;
      if (!warp_wait(&acc_full[buf], (uint32_t)((i >> 1) & 1), err, 58)) break;
      tc_fence_after();
      const uint32_t src = tbase + buf * 256u + lane_off;
      for (int q = 0; q < P.tile_n / 16; ++q) {
        float x[16];
        tmem_ld16(src + (uint32_t)(q * 16), x);
        tmem_ld_wait();
        zono_drain(P.out, P.o_bs, P.o_vec, P.zpos, P.zneg, tile, P.N, q * 16, x, valid, b, e, slot, two_slots);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kProducerWarp) tmem_dealloc(tbase, 512);
}

cf_status zono_tc_launch(const ZonoTcParams& P, cudaStream_t st) {
  int tile_n, nt;
  chain_tile(P.N, tile_n, nt);
  CF_REQUIRE(nt == 1 && P.N >= 1 && P.K >= 1 && P.K % 4 == 0 && P.E >= 128 && P.rows == P.B * P.E && P.out &&
                 P.zpos && P.zneg && P.wimg && P.A && P.err,
             CF_ERR_UNSUPPORTED, "zono_tc: N %d, K %d, E %lld", P.N, P.K, (long long)P.E);
  ZonoTcParams Q = P;
  Q.tile_n = tile_n;
  Q.kchunks = (P.K + 31) / 32;
  Q.w_lo_off = (uint32_t)tile_n * 128u;
  Q.stage_bytes = 2u * (uint32_t)tile_n * 128u;
  auto a16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
  Q.a_vec = (P.K % 4 == 0 && P.a_bs % 4 == 0 && a16(P.A)) ? 1 : 0;
  Q.lam_vec = (P.lam && P.K % 4 == 0 && a16(P.lam)) ? 1 : 0;
  Q.o_vec = (P.N % 4 == 0 && P.o_bs % 4 == 0 && a16(P.out)) ? 1 : 0;
  size_t smem = 1024 + (size_t)4 * kAImg + (size_t)2 * Q.stage_bytes + 11 * 8 + 16;
  if (smem < 116 * 1024) smem = 116 * 1024;  // one CTA per SM: it holds all 512 TMEM columns
  CF_REQUIRE(smem <= 227 * 1024, CF_ERR_UNSUPPORTED, "zono_tc: %zu bytes of shared memory", smem);
  static int sms = 0;
  if (sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
  }
  cudaError_t e = cudaFuncSetAttribute(k_zono_persist, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
  if (e != cudaSuccess) {
    set_error("zono_tc: cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    return CF_ERR_CUDA;
  }
  const int64_t tiles = (P.rows + 127) / 128;
  const int64_t grid = tiles < sms ? tiles : sms;
  k_zono_persist<<<(unsigned)grid, kZtThreads, smem, st>>>(Q);
  return check_launch("k_zono_persist");
}

}  // namespace cf
