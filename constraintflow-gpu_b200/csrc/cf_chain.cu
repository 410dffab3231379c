// Chained backsubstitution on tcgen05 tensor cores (3xTF32), one launch per bounded layer.
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
// warp 8 allocates TMEM and streams W chunks, warp 9 issues the MMAs.
// Every mbarrier wait is bounded (cf_tc.cuh); a timeout is recorded in the device error
// word and all roles unwind.
#include "cf_chain.cuh"
#include "cf_tc.cuh"

namespace cf {

using namespace tc;

constexpr uint32_t kAImg = 128 * 128;  // bytes of one 128-row x 32-fp32 A plane
constexpr int kTransformThreads = 256; // warps 0-7
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
// 32 k), K-major with the 128-byte swizzle, zero outside [0,N) x [0,K).
__global__ void k_prep_wimg(const float* __restrict__ W, int K, int N, int tile_n, int n_tiles, int kchunks,
                            uint8_t* __restrict__ img) {
  int64_t total = (int64_t)n_tiles * kchunks * tile_n * 32;
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

cf_status chain_prep_weights(const float* W, int K, int N, uint8_t* img, cudaStream_t st) {
  int tile_n, n_tiles;
  chain_tile(N, tile_n, n_tiles);
  int kchunks = (K + 31) / 32;
  int64_t total = (int64_t)n_tiles * kchunks * tile_n * 32;
  int64_t blocks = ceil_div(total, 256);
  if (blocks > 148 * 8) blocks = 148 * 8;
  k_prep_wimg<<<(unsigned)blocks, 256, 0, st>>>(W, K, N, tile_n, n_tiles, kchunks, img);
  return check_launch("k_prep_wimg");
}

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~(uintptr_t)1023);
}

// 16 consecutive floats p[k0 .. k0+16) with zeros at k >= K; four 16-byte loads when
// `vec` (16-byte aligned rows and K % 4 == 0), scalar loads otherwise.
__device__ __forceinline__ void load16(const float* __restrict__ p, int k0, int K, bool vec, float (&o)[16]) {
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

__global__ void __launch_bounds__(kThreads, 1) k_chain(const __grid_constant__ ChainParams P) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  const uint32_t stage_bytes = P.stage_bytes;
  uint64_t* full_a = reinterpret_cast<uint64_t*>(smem + kChainStages * stage_bytes);
  uint64_t* full_w = full_a + kChainStages;
  uint64_t* empty = full_w + kChainStages;
  uint64_t* acc_full = empty + kChainStages;
  uint64_t* mma_done = acc_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  float* red = reinterpret_cast<float*>(tmem_slot + 4);  // [128] partial sums of the second half
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int* err = P.err;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kChainStages; ++i) {
      mbar_init(&full_a[i], kTransformThreads);
      mbar_init(&full_w[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(mma_done, 1);
    fence_mbar_init();
  }
  if (warp == kProducerWarp) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;

  if (warp == kProducerWarp) {
    // ---------------------------------------------------------------- W producer
    if (lane == 0) {
      uint32_t g = 0;
      for (int s = 0; s < P.S; ++s) {
        const ChainStep& S = P.st[s];
        const uint32_t plane = (uint32_t)S.tile_n * 128u;
        for (int t = 0; t < S.n_tiles; ++t) {
          for (int c = 0; c < S.kchunks; ++c, ++g) {
            const uint32_t stage = g % kChainStages, round = g / kChainStages;
            if (!mbar_wait(&empty[stage], (round & 1) ^ 1, err, 11)) goto done_w;
            uint8_t* sb = smem + stage * stage_bytes;
            const uint8_t* src = S.wimg + ((size_t)t * S.kchunks + c) * 2 * plane;
            mbar_arrive_expect_tx(&full_w[stage], 2 * plane);
            bulk_g2s(sb + 2 * kAImg, src, plane, &full_w[stage]);
            bulk_g2s(sb + P.w_lo_off, src + plane, plane, &full_w[stage]);
          }
        }
      }
    done_w:
      // copies still in flight (error path) land before the CTA can exit
      for (uint32_t x = 0; x < kChainStages && x < g; ++x) {
        const uint32_t gl = g - 1 - x, stage = gl % kChainStages, round = gl / kChainStages;
        mbar_wait(&full_w[stage], round & 1, err, 12);
      }
    }
  } else if (warp == kMmaWarp) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      uint32_t g = 0;
      for (int s = 0; s < P.S; ++s) {
        const ChainStep& S = P.st[s];
        const uint32_t acc = tbase + (uint32_t)(s & 1) * 256u;
        const uint32_t idesc = idesc_tf32((uint32_t)S.tile_n);
        for (int t = 0; t < S.n_tiles; ++t) {
          for (int c = 0; c < S.kchunks; ++c, ++g) {
            const uint32_t stage = g % kChainStages, round = g / kChainStages;
            if (!mbar_wait(&full_a[stage], round & 1, err, 21)) goto done_m;
            if (!mbar_wait(&full_w[stage], round & 1, err, 22)) goto done_m;
            tc_fence_after();
            const uint32_t sb = smem_u32(smem + stage * stage_bytes);
            const uint32_t a_hi = sb, a_lo = sb + kAImg, w_hi = sb + 2 * kAImg, w_lo = sb + P.w_lo_off;
#pragma unroll
            for (uint32_t ks = 0; ks < 4; ++ks) {
              const uint64_t dah = sw128_desc(a_hi + ks * 32), dal = sw128_desc(a_lo + ks * 32);
              const uint64_t dwh = sw128_desc(w_hi + ks * 32), dwl = sw128_desc(w_lo + ks * 32);
              mma_tf32(acc, dal, dwh, idesc, (c | ks) != 0);
              mma_tf32(acc, dah, dwl, idesc, 1);
              mma_tf32(acc, dah, dwh, idesc, 1);
            }
            mma_commit(&empty[stage]);
          }
          mma_commit(acc_full);
        }
      }
    done_m:
      // every MMA issued above has completed before TMEM is released
      mma_commit(mma_done);
      mbar_wait(mma_done, 0, err, 23);
    }
  } else {
    // ---------------------------------------------------------------- transform warps
    // thread -> tile row (TMEM lane) `r`; the two halves split each 32-column chunk
    const int r = threadIdx.x & 127, half = threadIdx.x >> 7;
    const int64_t row = (int64_t)blockIdx.x * 128 + r;
    const bool valid = row < P.rows;
    int64_t sb_ = 0, b = 0, i = 0;
    if (valid) {
      sb_ = row / (P.B * P.R);
      int64_t rem = row - sb_ * P.B * P.R;
      b = rem / P.R;
      i = rem - b * P.R;
    }
    const bool lower = sb_ == 0;
    float cacc = (valid && P.c0 && half == 0) ? P.c0[i] : 0.0f;
    float conc = 0.0f;
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    uint32_t g = 0, nacc = 0;
    const float* a0row = P.A0 + sb_ * P.a_ss + b * P.a_bs + i * P.a_rs;
    const float* pos_box = (lower ? P.l0 : P.u0) + b * P.n0;
    const float* neg_box = (lower ? P.u0 : P.l0) + b * P.n0;
    bool ok = true;
    for (int s = 0; s < P.S && ok; ++s) {
      const ChainStep& S = P.st[s];
      const int K = S.K;
      const bool cvec = (K & 3) == 0;
      if (s > 0) {
        if (!mbar_wait(acc_full, nacc & 1, err, 31)) { ok = false; break; }
        ++nacc;
        tc_fence_after();
      }
      const uint32_t src_acc = tbase + (uint32_t)((s - 1) & 1) * 256u + lane_off;
      const int src_cols = s > 0 ? P.st[s - 1].tile_n : 0;
      const bool relu = S.alpha != nullptr;
      const float* pf = (lower ? S.alpha : S.lam) + b * K;
      const float* nf = (lower ? S.lam : S.alpha) + b * K;
      const float* muv = S.mu + b * K;
      for (int t = 0; t < S.n_tiles && ok; ++t) {
        for (int c = 0; c < S.kchunks; ++c, ++g) {
          const uint32_t stage = g % kChainStages, round = g / kChainStages;
          const int k0 = c * 32 + half * 16;
          // coefficient loads first: they depend on nothing the barriers protect
          float pv[16], nv[16], mv[16], bv[16];
          if (relu) {
            load16(pf, k0, K, cvec, pv);
            load16(nf, k0, K, cvec, nv);
            if (t == 0) load16(muv, k0, K, cvec, mv);
          }
          if (t == 0) load16(S.bias, k0, K, cvec, bv);
          float v[16];
          if (s == 0) load16(a0row, k0, valid ? K : 0, P.a0_vec, v);
          if (!mbar_wait(&empty[stage], (round & 1) ^ 1, err, 32)) { ok = false; break; }
          if (s > 0) {
            // columns [K, tile_n) of the previous accumulator are exact zeros (zero-padded
            // W); a half-chunk past tile_n was never written and is skipped
            if (k0 < src_cols) {
              tmem_ld16(src_acc + (uint32_t)k0, v);
              tmem_ld_wait();
            } else {
#pragma unroll
              for (int e = 0; e < 16; ++e) v[e] = 0.0f;
            }
          }
          float hi[16], lo[16];
          if (relu && t == 0) {
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              const float pos = fmaxf(v[e], 0.0f), neg = fminf(v[e], 0.0f);
              const float tr = fmaf(pos, pv[e], neg * nv[e]);
              cacc = fmaf(lower ? neg : pos, mv[e], cacc);
              cacc = fmaf(tr, bv[e], cacc);
              split_tf32(tr, hi[e], lo[e]);
            }
          } else if (relu) {
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              const float tr = fmaf(fmaxf(v[e], 0.0f), pv[e], fminf(v[e], 0.0f) * nv[e]);
              split_tf32(tr, hi[e], lo[e]);
            }
          } else if (t == 0) {
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              cacc = fmaf(v[e], bv[e], cacc);
              split_tf32(v[e], hi[e], lo[e]);
            }
          } else {
#pragma unroll
            for (int e = 0; e < 16; ++e) split_tf32(v[e], hi[e], lo[e]);
          }
          uint8_t* sbase = smem + stage * stage_bytes;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint32_t qq = (uint32_t)(half * 4 + q);
            const uint32_t off = (uint32_t)r * 128u + ((qq ^ ((uint32_t)r & 7u)) << 4);
            *reinterpret_cast<float4*>(sbase + off) = make_float4(hi[4 * q], hi[4 * q + 1], hi[4 * q + 2], hi[4 * q + 3]);
            *reinterpret_cast<float4*>(sbase + kAImg + off) =
                make_float4(lo[4 * q], lo[4 * q + 1], lo[4 * q + 2], lo[4 * q + 3]);
          }
          fence_proxy_async_smem();
          tc_fence_before();
          mbar_arrive(&full_a[stage]);
        }
        if (!ok) break;
        if (s == P.S - 1) {
          // drain output tile t straight into the concretisation; halves take alternate 16-column groups
          if (!mbar_wait(acc_full, nacc & 1, err, 33)) { ok = false; break; }
          ++nacc;
          tc_fence_after();
          const uint32_t dst = tbase + (uint32_t)(s & 1) * 256u + lane_off;
          for (int q = half; q < S.tile_n / 16; q += 2) {
            const int n0 = t * S.tile_n + q * 16;
            float pb[16], nb[16], x[16];
            load16(pos_box, n0, valid ? S.N : 0, P.box_vec, pb);
            load16(neg_box, n0, valid ? S.N : 0, P.box_vec, nb);
            tmem_ld16(dst + (uint32_t)(q * 16), x);
            tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 16; ++e) conc = fmaf(x[e], x[e] >= 0.0f ? pb[e] : nb[e], conc);
          }
          tc_fence_before();
        }
      }
    }
    // combine the two halves of every row
    if (half == 1) red[r] = conc + cacc;
    asm volatile("bar.sync 1, %0;" ::"r"(kTransformThreads) : "memory");
    if (half == 0 && valid && ok) {
      const float res = (conc + cacc) + red[r];
      (lower ? P.out_l : P.out_u)[b * P.ld_out + i] = res;
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kProducerWarp) tmem_dealloc(tbase, 512);
}

cf_status chain_launch(const ChainParams& P, cudaStream_t st) {
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
  ChainParams Q = P;
  Q.w_lo_off = 2 * kAImg + (uint32_t)tn_max * 128u;
  Q.stage_bytes = (2 * kAImg + 2u * (uint32_t)tn_max * 128u + 1023u) & ~1023u;
  size_t smem = 1024 + (size_t)kChainStages * Q.stage_bytes + (3 * kChainStages + 2) * 8 + 16 + 128 * 4;
  // at least 116 KB so that one CTA (which holds all 512 TMEM columns) runs per SM
  if (smem < 116 * 1024) smem = 116 * 1024;
  cudaError_t e = cudaFuncSetAttribute(k_chain, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
  if (e != cudaSuccess) {
    set_error("chain: cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    return CF_ERR_CUDA;
  }
  CF_REQUIRE(smem <= 227 * 1024, CF_ERR_UNSUPPORTED, "chain: %zu bytes of shared memory", smem);
  const int64_t tiles = ceil_div(P.rows, 128);
  CF_REQUIRE(tiles <= 0x7fffffff, CF_ERR_SHAPE, "chain: too many rows");
  k_chain<<<(unsigned)tiles, kThreads, smem, st>>>(Q);
  return check_launch("k_chain");
}

}  // namespace cf
