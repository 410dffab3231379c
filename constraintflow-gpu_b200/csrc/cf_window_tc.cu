// Transposed convolution of receptive-field windows on tcgen05 tensor cores (3xTF32).
//
// One stride phase of the transposed convolution that substitutes a conv layer into the
// coefficient windows (the adjoint of the conv, constraintflow/gbcsr/sparse_block.py:839-928
// conv_transpose2d; cf_window.cu describes the phase decomposition) is the implicit GEMM
//   out[m, ci] = sum_k A[m, k] * B[k, ci]
//   m = (row r, phase position iy, ix)       M = rows * ny * nx
//   k = (co, ty, tx)                         K = Cout * tyn * txn
//   A[m, k] = in[r, co, q0y + iy - ty, q0x + ix - tx]   (0 outside the input window)
//   B[k, ci] = W[co, ci, py + ty*s, px + tx*s]
// written to out[r, ci, u0 + iy*s, v0 + ix*s] (0 where that position lies outside the
// level image: the conv's zero padding).
//
// One launch covers all stride phases; each persistent CTA works on one phase and loops over
// that phase's 128-row M tiles.  The phase's weight image B (tf32 hi and lo planes of B^T,
// K-major, 128-byte swizzle; N = Cin padded to 16) is copied into shared memory once per CTA
// and stays there.  Warps 0-7 gather the A operand chunk by chunk
// (32 k columns; thread <-> tile row, the two halves take 16 columns each; a per-thread tap
// mask replaces the window bounds test), split it into tf32 hi + lo and store it at its
// SW128 position; warp 8 allocates TMEM and loads the weights, warp 9 issues the
// 3xTF32 MMAs (Alo*Bhi + Ahi*Blo + Ahi*Bhi) into one of two TMEM accumulators, and warps
// 10-13 drain the other accumulator (tile i-1) into the output windows while tile i
// computes.  Every mbarrier wait is bounded (cf_tc.cuh); a timeout is recorded in the
// device error word and every role unwinds.
#include "cf_tc.cuh"
#include "cf_window.cuh"

namespace cf {

using namespace tc;

namespace {

constexpr uint32_t kWAImg = 128 * 128;  // one 128-row x 32-fp32 A plane
constexpr int kWTransformWarps = 8;
constexpr int kWTransformThreads = 256;
constexpr int kWProducerWarp = 8;
constexpr int kWMmaWarp = 9;
constexpr int kWThreads = 448;           // + 4 drain warps (10-13)
constexpr int kWMaxTaps = 31;            // tap index 31 marks padded k columns

constexpr int kWMaxPhases = 9;          // stride <= 3

// One launch covers every stride phase of the step.  CTA c works on phase c % S2 only (the
// grid is a multiple of S2), on that phase's tiles c / S2, + gridDim.x / S2, ...: the S2
// phase tiles of the same output block run at the same time on neighbouring CTAs, so the
// interleaved output elements of a 32-byte sector are written together (merged in L2) and
// the input window every phase reads is fetched from DRAM once.
struct WinTcParams {
  RowGeom rg;
  WinGeom gi, go;
  ConvGeom cv;
  int32_t S2;                      // number of phases
  ConvPhase phs[kWMaxPhases];
  int32_t Ks[kWMaxPhases], kch[kWMaxPhases], tapsv[kWMaxPhases];
  uint32_t woff[kWMaxPhases], wbytes[kWMaxPhases];   // weight image of each phase in `wimg`
  int64_t Mp[kWMaxPhases];         // M of each phase
  const float* in;
  float* out;
  const uint8_t* wimg;   // per phase: kchunks x (hi plane, lo plane) of n_pad rows x 128 B
  int32_t N, n_pad, kchunks_max;
  int32_t a_stages;
  uint32_t wimg_max;     // shared-memory bytes reserved for one phase's image
  int* err;
};

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~(uintptr_t)1023);
}

__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, int* err, int site) {
  const bool ok = mbar_wait(bar, parity, err, site);
  return __all_sync(0xffffffffu, ok);
}

// B^T image of one phase: element (n, k) -> plane c = k / 32 of the hi / lo image at the
// SW128 position of (n, k % 32); zero outside [0, N) x [0, K).
__global__ void k_win_prep_wimg(const float* __restrict__ W, ConvGeom cv, ConvPhase ph, int N, int n_pad, int K,
                                int kchunks, uint8_t* __restrict__ img) {
  const int taps = ph.tyn * ph.txn;
  const int64_t total = (int64_t)kchunks * n_pad * 32;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int kl = (int)(e & 31);
    const int64_t q = e >> 5;
    const int nl = (int)(q % n_pad);
    const int c = (int)(q / n_pad);
    const int k = c * 32 + kl;
    float v = 0.0f;
    if (nl < N && k < K) {
      const int co = k / taps, t = k - co * taps, ty = t / ph.txn, tx = t - ty * ph.txn;
      const int ky = ph.py + ty * cv.s, kx = ph.px + tx * cv.s;
      v = W[(((int64_t)co * cv.cin + nl) * cv.kh + ky) * cv.kw + kx];
    }
    float hi, lo;
    split_tf32(v, hi, lo);
    const size_t plane = (size_t)n_pad * 128;
    uint8_t* base = img + (size_t)c * 2 * plane;
    const uint32_t off = sw128_offset((uint32_t)nl, (uint32_t)kl);
    *reinterpret_cast<float*>(base + off) = hi;
    *reinterpret_cast<float*>(base + plane + off) = lo;
  }
}

__global__ void __launch_bounds__(kWThreads, 1) k_win_convT_tc(const __grid_constant__ WinTcParams P) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* w_region = smem;                                        // resident weight image
  uint8_t* a_region = smem + ((P.wimg_max + 1023u) & ~1023u);      // A stages (hi, lo planes)
  int2* ktab = reinterpret_cast<int2*>(a_region + (size_t)P.a_stages * 2 * kWAImg);  // per k: (offset, tap)
  uint64_t* bars = reinterpret_cast<uint64_t*>(ktab + P.kchunks_max * 32);
  uint64_t* full_a = bars;                 // [a_stages]
  uint64_t* empty_a = bars + 4;            // [a_stages]
  uint64_t* w_full = bars + 8;
  uint64_t* acc_full = bars + 9;           // [2]
  uint64_t* acc_empty = bars + 11;         // [2]
  uint64_t* mma_done = bars + 13;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 14);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int* err = P.err;
  // this CTA's phase and its tiles first, + stride, + 2*stride, ...
  const int phase = (int)(blockIdx.x % (unsigned)P.S2);
  const ConvPhase ph = P.phs[phase];
  const int K = P.Ks[phase], kchunks = P.kch[phase], taps = P.tapsv[phase];
  const int64_t M = P.Mp[phase];
  const uint8_t* wimg = P.wimg + P.woff[phase];
  const uint32_t wimg_bytes = P.wbytes[phase];
  const int64_t first = blockIdx.x / P.S2, stride = gridDim.x / P.S2;
  const int64_t n_tiles = (M + 127) / 128;
  const int64_t my_tiles = first < n_tiles ? (n_tiles - 1 - first) / stride + 1 : 0;
  // two accumulators of n_pad columns, each at a power-of-two column stride >= 32
  uint32_t acc_cols = 32;
  while (acc_cols < (uint32_t)P.n_pad) acc_cols <<= 1;
  const uint32_t tmem_cols = 2 * acc_cols;
  const int plane_in = P.gi.Ph * P.gi.Pw;

  if (threadIdx.x == 0) {
    for (int i = 0; i < P.a_stages; ++i) {
      mbar_init(&full_a[i], kWTransformThreads);
      mbar_init(&empty_a[i], 1);
    }
    mbar_init(w_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 4);
    }
    mbar_init(mma_done, 1);
    fence_mbar_init();
  }
  // k table: k -> (window offset co*plane - ty*Pw - tx, tap index; 31 for padded columns)
  for (int k = threadIdx.x; k < kchunks * 32; k += blockDim.x) {
    int2 e = make_int2(0, kWMaxTaps);
    if (k < K) {
      const int co = k / taps, t = k - co * taps, ty = t / ph.txn, tx = t - ty * ph.txn;
      e = make_int2(co * plane_in - ty * P.gi.Pw - tx, t);
    }
    ktab[k] = e;
  }
  if (warp == kWProducerWarp) {
    tmem_alloc(tmem_slot, tmem_cols);
    tmem_relinquish();
  }
  if (threadIdx.x == 0) tmem_slot[1] = *(volatile int*)err != 0 ? 1u : 0u;
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;
  if (tmem_slot[1] != 0 || my_tiles == 0) {
    tc_fence_before();
    __syncthreads();
    if (warp == kWProducerWarp) tmem_dealloc(tbase, tmem_cols);
    return;
  }
  const uint32_t wplane = (uint32_t)P.n_pad * 128u;

  if (warp == kWProducerWarp) {
    // ---------------------------------------------------------------- weights, once
    if (lane == 0) {
      mbar_arrive_expect_tx(w_full, wimg_bytes);
      // bulk copies of at most 64 KB each (the image is a multiple of 16 bytes)
      for (uint32_t o = 0; o < wimg_bytes; o += 65536u) {
        const uint32_t nb = wimg_bytes - o < 65536u ? wimg_bytes - o : 65536u;
        bulk_g2s(w_region + o, wimg + o, nb, w_full);
      }
      mbar_wait_drain(w_full, 0, err, 61);
    }
  } else if (warp == kWMmaWarp) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_tf32((uint32_t)P.n_pad);
      uint32_t g = 0;
      if (!mbar_wait(w_full, 0, err, 62)) goto done_m;
      for (int64_t i = 0; i < my_tiles; ++i) {
        const uint32_t buf = (uint32_t)(i & 1);
        if (i >= 2 && !mbar_wait(&acc_empty[buf], (uint32_t)((i >> 1) & 1) ^ 1u, err, 63)) goto done_m;
        tc_fence_after();
        const uint32_t acc = tbase + buf * acc_cols;
        for (int c = 0; c < kchunks; ++c, ++g) {
          const int nks = min(4, (K - c * 32 + 7) / 8);
          const uint32_t stage = g % (uint32_t)P.a_stages, round = g / (uint32_t)P.a_stages;
          if (!mbar_wait(&full_a[stage], round & 1u, err, 64)) goto done_m;
          tc_fence_after();
          const uint32_t sa = smem_u32(a_region + stage * 2 * kWAImg);
          const uint32_t sw = smem_u32(w_region + (size_t)c * 2 * wplane);
          const uint32_t a_hi = sa, a_lo = sa + kWAImg, w_hi = sw, w_lo = sw + wplane;
#pragma unroll
          for (int ks = 0; ks < 4; ++ks) {
            if (ks >= nks) break;
            const uint64_t dah = sw128_desc(a_hi + ks * 32), dal = sw128_desc(a_lo + ks * 32);
            const uint64_t dwh = sw128_desc(w_hi + ks * 32), dwl = sw128_desc(w_lo + ks * 32);
            mma_tf32(acc, dal, dwh, idesc, (c | ks) != 0);
            mma_tf32(acc, dah, dwl, idesc, 1);
            mma_tf32(acc, dah, dwh, idesc, 1);
          }
          mma_commit(&empty_a[stage]);
        }
        mma_commit(&acc_full[buf]);
      }
    done_m:
      // every MMA issued above has completed before TMEM is released
      mma_commit(mma_done);
      mbar_wait_drain(mma_done, 0, err, 65);
    }
  } else if (warp < kWTransformWarps) {
    // ---------------------------------------------------------------- A operand (gather)
    const int r = threadIdx.x & 127, half = threadIdx.x >> 7;
    uint32_t soff[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) soff[q] = (uint32_t)r * 128u + ((((uint32_t)(half * 4 + q)) ^ ((uint32_t)r & 7u)) << 4);
    const int pos = ph.ny * ph.nx;
    const int64_t per_in = (int64_t)P.gi.C * plane_in;
    uint32_t g = 0;
    bool ok = true;
    // this row's window base (at its phase position) and the taps whose input position lies
    // inside the input window, for tile i
    const float* base = P.in;
    uint32_t tapmask = 0;
    auto tile_row = [&](int64_t i) {
      const int64_t m = (first + i * stride) * 128 + r;
      base = P.in;
      tapmask = 0;
      if (m < M) {
        const int64_t rr = m / pos;
        const int rem = (int)(m - rr * pos);
        const int iy = rem / ph.nx, ix = rem - iy * ph.nx;
        const int qy = ph.q0y + iy, qx = ph.q0x + ix;
        base = P.in + rr * per_in + (int64_t)qy * P.gi.Pw + qx;
        for (int t = 0; t < taps; ++t) {
          const int ty = t / ph.txn, tx = t - ty * ph.txn;
          const int u = qy - ty, v = qx - tx;
          if (u >= 0 && u < P.gi.Ph && v >= 0 && v < P.gi.Pw) tapmask |= 1u << t;
        }
      }
    };
    // the 16 values of chunk c of the current tile row (loaded one chunk ahead, so that their
    // latency overlaps the split and the store of the chunk before)
    auto load_chunk = [&](int c, float (&v)[16]) {
      const int kb = c * 32 + half * 16;
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        const int2 te = ktab[kb + e];
        v[e] = ((tapmask >> te.y) & 1u) ? __ldg(base + te.x) : 0.0f;
      }
    };
    float vnext[16];
    tile_row(0);
    load_chunk(0, vnext);
    for (int64_t i = 0; i < my_tiles && ok; ++i) {
      for (int c = 0; c < kchunks; ++c, ++g) {
        const uint32_t stage = g % (uint32_t)P.a_stages, round = g / (uint32_t)P.a_stages;
        float hi[16], lo[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) split_tf32(vnext[e], hi[e], lo[e]);
        if (c + 1 < kchunks) {
          load_chunk(c + 1, vnext);
        } else if (i + 1 < my_tiles) {
          tile_row(i + 1);
          load_chunk(0, vnext);
        }
        if (!warp_wait(&empty_a[stage], (round & 1u) ^ 1u, err, 66)) {
          ok = false;
          break;
        }
        const uint32_t sbase = smem_u32(a_region) + stage * 2 * kWAImg;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(sbase + soff[q]), "f"(hi[4 * q]),
                       "f"(hi[4 * q + 1]), "f"(hi[4 * q + 2]), "f"(hi[4 * q + 3])
                       : "memory");
          asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(sbase + kWAImg + soff[q]), "f"(lo[4 * q]),
                       "f"(lo[4 * q + 1]), "f"(lo[4 * q + 2]), "f"(lo[4 * q + 3])
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
    const int pos = ph.ny * ph.nx;
    const int plane_out = P.go.Ph * P.go.Pw;
    const int64_t per_out = (int64_t)P.go.C * plane_out;
    for (int64_t i = 0; i < my_tiles; ++i) {
      const uint32_t buf = (uint32_t)(i & 1);
      const int64_t m = (first + i * stride) * 128 + q4 * 32 + lane;
      const bool valid = m < M;
      float* o = nullptr;
      bool inside = false;
      if (valid) {
        const int64_t rr = m / pos;
        const int rem = (int)(m - rr * pos);
        const int iy = rem / ph.nx, ix = rem - iy * ph.nx;
        const int uo = ph.u0 + iy * P.cv.s, vo = ph.v0 + ix * P.cv.s;
        // row rr = (bound, region, i); i's position (oy, ox) in the bounded layer's image
        const int64_t BR = P.rg.B * P.rg.R;
        const int64_t rem2 = rr - (rr / BR) * BR;
        const int64_t ri = rem2 - (rem2 / P.rg.R) * P.rg.R;
        const int64_t hw = (int64_t)P.rg.Hm * P.rg.Wm;
        const int64_t pp = ri - (ri / hw) * hw;
        const int oy = (int)(pp / P.rg.Wm), ox = (int)(pp - (int64_t)oy * P.rg.Wm);
        const int Y = oy * P.go.sig_h - P.go.pi_h + uo, X = ox * P.go.sig_w - P.go.pi_w + vo;
        inside = Y >= 0 && Y < P.go.H && X >= 0 && X < P.go.W;
        o = P.out + rr * per_out + (int64_t)uo * P.go.Pw + vo;
      }
      if (!warp_wait(&acc_full[buf], (uint32_t)((i >> 1) & 1), err, 67)) break;
      tc_fence_after();
      const uint32_t src = tbase + buf * acc_cols + lane_off;
      for (int q = 0; q < P.n_pad / 16; ++q) {
        float x[16];
        tmem_ld16(src + (uint32_t)(q * 16), x);
        tmem_ld_wait();
        if (valid) {
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const int n = q * 16 + e;
            if (n < P.N) o[(int64_t)n * plane_out] = inside ? x[e] : 0.0f;
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kWProducerWarp) tmem_dealloc(tbase, tmem_cols);
}

}  // namespace

// Bytes of one phase's weight image (kchunks x 2 planes x n_pad rows x 128 B).
static size_t phase_wimg_bytes(int K, int n_pad) { return (size_t)((K + 31) / 32) * 2 * n_pad * 128; }

size_t win_convT_tc_scratch_bytes(const ConvGeom& cv, int cout) {
  // every phase's image, each at most the largest one (taps ceil(kh/s) x ceil(kw/s))
  const int tyn = (cv.kh + cv.s - 1) / cv.s, txn = (cv.kw + cv.s - 1) / cv.s;
  const int n_pad = ((cv.cin + 15) / 16) * 16;
  return (size_t)cv.s * cv.s * ((phase_wimg_bytes(cout * tyn * txn, n_pad) + 1023) & ~(size_t)1023);
}

bool win_convT_tc_applicable(const ConvGeom& cv, int cout) {
  const int tyn = (cv.kh + cv.s - 1) / cv.s, txn = (cv.kw + cv.s - 1) / cv.s;
  const int n_pad = ((cv.cin + 15) / 16) * 16;
  const size_t wb = phase_wimg_bytes(cout * tyn * txn, n_pad);
  const size_t smem = 1024 + ((wb + 1023) & ~(size_t)1023) + (size_t)2 * 2 * kWAImg +
                      (size_t)((cout * tyn * txn + 31) / 32) * 32 * 8 + 16 * 8 + 16;
  return cv.cin >= 1 && cv.s * cv.s <= kWMaxPhases && n_pad <= 256 && tyn * txn <= kWMaxTaps && smem <= 227 * 1024;
}

cf_status win_convT_tc(const RowGeom& rg, const WinGeom& gi, const WinGeom& go, const ConvGeom& cv, int cout,
                       const float* in, const float* W, float* out, uint8_t* scratch, int* err, cudaStream_t st) {
  const int64_t rows = 2 * rg.B * rg.R;
  if (rows * go.C * go.Ph * go.Pw == 0) return CF_OK;
  CF_REQUIRE(win_convT_tc_applicable(cv, cout), CF_ERR_UNSUPPORTED, "convT_tc: geometry");
  static int sms = 0;
  if (sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
  }
  cudaError_t e = cudaFuncSetAttribute(k_win_convT_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
  if (e != cudaSuccess) {
    set_error("convT_tc: cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    return CF_ERR_CUDA;
  }
  const int s = cv.s;
  CF_REQUIRE(s * s <= kWMaxPhases, CF_ERR_UNSUPPORTED, "convT_tc: stride %d", s);
  const int Dy = gi.pi_h * s + cv.pad - go.pi_h, Dx = gi.pi_w * s + cv.pad - go.pi_w;
  const int n_pad = ((cv.cin + 15) / 16) * 16;
  WinTcParams P;
  memset(&P, 0, sizeof(P));
  P.rg = rg;
  P.gi = gi;
  P.go = go;
  P.cv = cv;
  P.in = in;
  P.out = out;
  P.N = cv.cin;
  P.n_pad = n_pad;
  P.wimg = scratch;
  P.err = err;
  int64_t t_max = 0;
  uint32_t off = 0;
  for (int py = 0; py < s; ++py) {
    const int u0 = ((py - Dy) % s + s) % s;
    const int ny = u0 < go.Ph ? (go.Ph - u0 + s - 1) / s : 0;
    const int tyn = cv.kh > py ? (cv.kh - py + s - 1) / s : 0;
    for (int px = 0; px < s; ++px) {
      const int v0 = ((px - Dx) % s + s) % s;
      const int nx = v0 < go.Pw ? (go.Pw - v0 + s - 1) / s : 0;
      const int txn = cv.kw > px ? (cv.kw - px + s - 1) / s : 0;
      if (ny == 0 || nx == 0) continue;
      CF_REQUIRE(tyn >= 1 && txn >= 1, CF_ERR_UNSUPPORTED, "convT_tc: a phase without taps");
      const int q = P.S2++;
      P.phs[q] = ConvPhase{py, px, ny, nx, tyn, txn, u0, v0, (u0 + Dy - py) / s, (v0 + Dx - px) / s};
      P.tapsv[q] = tyn * txn;
      P.Ks[q] = cout * P.tapsv[q];
      P.kch[q] = (P.Ks[q] + 31) / 32;
      P.Mp[q] = rows * ny * nx;
      P.woff[q] = off;
      P.wbytes[q] = (uint32_t)phase_wimg_bytes(P.Ks[q], n_pad);
      off += (P.wbytes[q] + 1023u) & ~1023u;
      if (P.wbytes[q] > P.wimg_max) P.wimg_max = P.wbytes[q];
      if (P.kch[q] > P.kchunks_max) P.kchunks_max = P.kch[q];
      const int64_t tiles = (P.Mp[q] + 127) / 128;
      if (tiles > t_max) t_max = tiles;
    }
  }
  if (P.S2 == 0) return CF_OK;
  const size_t fixed = 1024 + ((P.wimg_max + 1023u) & ~1023u) + (size_t)P.kchunks_max * 32 * 8 + 16 * 8 + 16;
  P.a_stages = fixed + (size_t)4 * 2 * kWAImg <= 227 * 1024 ? 4
               : (fixed + (size_t)3 * 2 * kWAImg <= 227 * 1024 ? 3 : 2);
  const size_t smem = fixed + (size_t)P.a_stages * 2 * kWAImg;
  CF_REQUIRE(smem <= 227 * 1024, CF_ERR_UNSUPPORTED, "convT_tc: %zu bytes of shared memory", smem);
  // every phase's weight image (stream-ordered before the GEMM that reads them)
  for (int q = 0; q < P.S2; ++q) {
    const int64_t total = (int64_t)P.kch[q] * n_pad * 32;
    k_win_prep_wimg<<<(unsigned)ceil_div(total, 256), 256, 0, st>>>(W, cv, P.phs[q], P.N, n_pad, P.Ks[q], P.kch[q],
                                                                     scratch + P.woff[q]);
    CF_TRY(check_launch("k_win_prep_wimg"));
  }
  // a multiple of S2 CTAs (each CTA works on one phase), at most one per SM
  int64_t per_phase = sms / P.S2;
  if (per_phase < 1) per_phase = 1;
  if (per_phase > t_max) per_phase = t_max;
  const int64_t grid = per_phase * P.S2;
  k_win_convT_tc<<<(unsigned)grid, kWThreads, smem, st>>>(P);
  return check_launch("k_win_convT_tc");
}

}  // namespace cf
