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
// Warp roles (192 threads): warps 0-3 transform/epilogue (thread t <-> TMEM lane t <->
// tile row t), warp 4 allocates TMEM and streams W chunks, warp 5 issues the MMAs.
// Every mbarrier wait is bounded (cf_tc.cuh); a timeout is recorded in the device error
// word and all roles unwind.
#include "cf_chain.cuh"
#include "cf_tc.cuh"

namespace cf {

using namespace tc;

constexpr uint32_t kAImg = 128 * 128;  // bytes of one 128-row x 32-fp32 A plane
constexpr int kThreads = 192;

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
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int* err = P.err;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kChainStages; ++i) {
      mbar_init(&full_a[i], 128);
      mbar_init(&full_w[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(mma_done, 1);
    fence_mbar_init();
  }
  if (warp == 4) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;

  if (warp == 4) {
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
  } else if (warp == 5) {
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
    const int tid = threadIdx.x;  // 0..127: tile row and TMEM lane
    const int64_t row = (int64_t)blockIdx.x * 128 + tid;
    const bool valid = row < P.rows;
    int64_t sb_ = 0, b = 0, i = 0;
    if (valid) {
      sb_ = row / (P.B * P.R);
      int64_t rem = row - sb_ * P.B * P.R;
      b = rem / P.R;
      i = rem - b * P.R;
    }
    const bool lower = sb_ == 0;
    float cacc = (valid && P.c0) ? P.c0[i] : 0.0f;
    float conc = 0.0f;
    const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
    uint32_t g = 0, nacc = 0;
    const float* a0row = P.A0 + sb_ * P.a_ss + b * P.a_bs + i * P.a_rs;
    const float* pos_box = (lower ? P.l0 : P.u0) + b * P.n0;
    const float* neg_box = (lower ? P.u0 : P.l0) + b * P.n0;
    bool ok = true;
    for (int s = 0; s < P.S && ok; ++s) {
      const ChainStep& S = P.st[s];
      const int K = S.K;
      if (s > 0) {
        if (!mbar_wait(acc_full, nacc & 1, err, 31)) { ok = false; break; }
        ++nacc;
        tc_fence_after();
      }
      const uint32_t src_acc = tbase + (uint32_t)((s - 1) & 1) * 256u + lane_off;
      const float* pf = nullptr;
      const float* nf = nullptr;
      const float* muv = nullptr;
      if (S.alpha && valid) {
        pf = (lower ? S.alpha : S.lam) + b * K;
        nf = (lower ? S.lam : S.alpha) + b * K;
        muv = S.mu + b * K;
      }
      for (int t = 0; t < S.n_tiles && ok; ++t) {
        for (int c = 0; c < S.kchunks; ++c, ++g) {
          const uint32_t stage = g % kChainStages, round = g / kChainStages;
          if (!mbar_wait(&empty[stage], (round & 1) ^ 1, err, 32)) { ok = false; break; }
          float v[32];
          if (s == 0) {
#pragma unroll
            for (int e = 0; e < 32; ++e) {
              int k = c * 32 + e;
              v[e] = (valid && k < K) ? a0row[k] : 0.0f;
            }
          } else {
            float h0[16], h1[16];
            tmem_ld16(src_acc + (uint32_t)(c * 32), h0);
            tmem_ld16(src_acc + (uint32_t)(c * 32 + 16), h1);
            tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              v[e] = (c * 32 + e < K) ? h0[e] : 0.0f;
              v[16 + e] = (c * 32 + 16 + e < K) ? h1[e] : 0.0f;
            }
          }
          uint8_t* sbase = smem + stage * stage_bytes;
          float hi[32], lo[32];
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const int k = c * 32 + e;
            float a = valid ? v[e] : 0.0f;
            float tr = a;
            if (pf && k < K) {
              tr = a >= 0.0f ? a * pf[k] : a * nf[k];
              if (t == 0 && (lower ? (a < 0.0f) : (a > 0.0f))) cacc = fmaf(a, muv[k], cacc);
            }
            if (t == 0 && k < K && valid) cacc = fmaf(tr, S.bias[k], cacc);
            hi[e] = to_tf32(tr);
            lo[e] = to_tf32(tr - hi[e]);
          }
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const uint32_t off = (uint32_t)tid * 128u + ((((uint32_t)q) ^ ((uint32_t)tid & 7u)) << 4);
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
          // drain output tile t straight into the concretisation
          if (!mbar_wait(acc_full, nacc & 1, err, 33)) { ok = false; break; }
          ++nacc;
          tc_fence_after();
          const uint32_t dst = tbase + (uint32_t)(s & 1) * 256u + lane_off;
          for (int q = 0; q < S.tile_n / 16; ++q) {
            float x[16];
            tmem_ld16(dst + (uint32_t)(q * 16), x);
            tmem_ld_wait();
            const int n_base = t * S.tile_n + q * 16;
            if (valid) {
#pragma unroll
              for (int e = 0; e < 16; ++e) {
                const int n = n_base + e;
                if (n < S.N) conc += x[e] >= 0.0f ? x[e] * pos_box[n] : x[e] * neg_box[n];
              }
            }
          }
          tc_fence_before();
        }
      }
    }
    if (valid && ok) {
      const float res = conc + cacc;
      (lower ? P.out_l : P.out_u)[b * P.ld_out + i] = res;
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 4) tmem_dealloc(tbase, 512);
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
  size_t smem = 1024 + (size_t)kChainStages * Q.stage_bytes + (3 * kChainStages + 2) * 8 + 16;
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
