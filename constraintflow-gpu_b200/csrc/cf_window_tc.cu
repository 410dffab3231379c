// Transposed convolution of receptive-field windows on tcgen05 tensor cores (3xTF32).
//
// The substitution of a conv layer (weights [Cout, Cin, kh, kw], stride s, pad) into the
// coefficient windows is the adjoint of the conv (constraintflow/gbcsr/sparse_block.py:
// 839-928 conv_transpose2d).  An output-window position u' (window-relative) receives tap
// ky from input-window position u when u' + D = u*s + ky, with D = gi.pi*s + pad - go.pi
// (0 for receptive-field windows, pad for whole-image ones).  Writing u' + D = i*s + py
// (py = the stride phase), the taps of phase py are ky = py + ty*s and they read the input
// rows u = i - ty for every phase alike.  So one implicit GEMM covers all s*s phases, with
// the phases stacked along N:
//   out[m, n] = sum_k A[m, k] * B[k, n]
//   m = (row r, grid position iy, ix), i = i0 + iy, j = j0 + ix     M = rows * ny * nx
//   k = (co, ty, tx)                    K = Cout * TY * TX, TY = ceil(kh/s), TX = ceil(kw/s)
//   n = (py, px, ci)                    N = s*s * Cin
//   A[m, k] = in[r, co, i - ty, j - tx]     (0 outside the input window)
//   B[k, n] = W[co, ci, py + ty*s, px + tx*s] (0 past the kernel)
// written to out[r, ci, i*s + py - D, j*s + px - D] where that lies inside the output
// window (0 where it lies outside the level image: the conv's zero padding).  A small Cin
// becomes an N of 4*Cin for a stride-2 conv: an M=128, K=8 tf32 MMA costs about the same
// issue time for N = 32 as for N = 208 (measured with clock64 stamps of the issuing
// thread), so N is what makes the tensor core pay.  The s*s phase outputs of a position
// are adjacent in memory, so a tile writes whole sectors.
//
// A stride-1 layer has one phase, so N would be Cin alone.  There the output positions are
// blocked f x f (f = 2): with S = s*f and u' + D = i*S + py, py = qy*s + ry (qy < f,
// ry < s), the taps are ky = ry + ty*s and the input rows u = i*f + (f-1) - ty' with
// ty' = ty - qy + (f-1) in [0, TY + f - 1) for every phase alike, so
//   k = (co, ty', tx'), K = Cout * (TY + f - 1) * (TX + f - 1);  n = (py, px, ci), N = S*S*Cin
//   A[m, k] = in[r, co, i*f + f-1 - ty', j*f + f-1 - tx']
//   B[k, n] = W[co, ci, ry + (ty' + qy - (f-1))*s, rx + (tx' + qx - (f-1))*s] (0 off the kernel)
// and the output goes to out[r, ci, i*S + py - D, j*S + px - D].  f = 1 is the phase-stacked
// form above.  For a 3x3 stride-1 layer this takes 2.25x fewer MMAs and gathered loads.
//
// Persistent CTAs loop over 128-row M tiles.  Warps 0-7 gather the A operand chunk by chunk
// (32 k columns; thread <-> tile row, two threads per row take 16 columns each, two chunks
// loaded ahead; a per-thread tap mask replaces the window bounds test), split it into tf32
// hi + lo and store it at its SW128 position; warp 8 allocates TMEM and copies the weight
// image (tf32 hi and lo planes of B^T, K-major, 128-byte swizzle, prepared once per call in
// the workspace) into shared memory with bulk copies: all of it once when it fits, else
// chunk by chunk through a ring of stages; warp 9 issues the 3xTF32 MMAs (Alo*Bhi + Ahi*Blo +
// Ahi*Bhi) into one of two TMEM accumulators, and warps 10-13 drain the other accumulator
// (tile i-1) into the output windows while tile i computes.  Every mbarrier wait is bounded
// (cf_tc.cuh); a timeout is recorded in the device error word and every role unwinds.
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
constexpr int kWCols = 32 / (kWTransformThreads / 128);   // k columns of a chunk per transform thread
constexpr int kWMaxTaps = 31;            // tap index 31 marks padded k columns
constexpr int kWStages = 4;              // max A / W stages (barrier slots)

struct WinTcParams {
  RowGeom rg;
  WinGeom gi, go;
  ConvGeom cv;
  int32_t TY, TX;        // k taps per dimension (the conv's taps per phase + f - 1)
  int32_t f, S;          // output blocking factor (1, or 2 for stride 1) and S = s*f
  int32_t i0, j0;        // grid origin: i = i0 + iy
  int32_t ny, nx;        // grid size
  int32_t Dy, Dx;
  int32_t K, kchunks, taps;
  int32_t N, n_pad;      // N = S*S*Cin
  int64_t M;
  const float* in;
  float* out;
  const uint8_t* wimg;   // kchunks x (hi plane, lo plane) of n_pad rows x 128 B
  int32_t a_stages, w_stages;
  int* err;
};

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~(uintptr_t)1023);
}

__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, int* err, int site) {
  const bool ok = mbar_wait(bar, parity, err, site);
  return __all_sync(0xffffffffu, ok);
}

// B^T image: element (n, k) -> plane c = k / 32 of the hi / lo image at the SW128 position
// of (n, k % 32); zero outside [0, N) x [0, K) and past the kernel.  TY, TX: k taps per
// dimension; f: the output blocking factor (S = s*f phases per dimension).
__global__ void k_win_prep_wimg(const float* __restrict__ W, ConvGeom cv, int TY, int TX, int f, int N, int n_pad,
                                int K, int kchunks, uint8_t* __restrict__ img) {
  const int64_t total = (int64_t)kchunks * n_pad * 32;
  const int taps = TY * TX;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int kl = (int)(e & 31);
    const int64_t q = e >> 5;
    const int nl = (int)(q % n_pad);
    const int c = (int)(q / n_pad);
    const int k = c * 32 + kl;
    float v = 0.0f;
    if (nl < N && k < K) {
      const int S = cv.s * f;
      const int co = k / taps, t = k - co * taps, tyk = t / TX, txk = t - tyk * TX;
      const int p = nl / cv.cin, ci = nl - p * cv.cin, py = p / S, px = p - py * S;
      const int ty = tyk + py / cv.s - (f - 1), tx = txk + px / cv.s - (f - 1);
      const int ky = py % cv.s + ty * cv.s, kx = px % cv.s + tx * cv.s;
      if (ty >= 0 && tx >= 0 && ky < cv.kh && kx < cv.kw)
        v = W[(((int64_t)co * cv.cin + ci) * cv.kh + ky) * cv.kw + kx];
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
  const uint32_t wplane = (uint32_t)P.n_pad * 128u;
  uint8_t* a_region = smem;                                               // A stages (hi, lo planes)
  uint8_t* w_region = smem + (size_t)P.a_stages * 2 * kWAImg;             // W stages (hi, lo planes)
  // W: w_stages streamed stages, or (w_stages == 0) the whole image resident
  const size_t w_bytes = (size_t)(P.w_stages ? P.w_stages : P.kchunks) * 2 * wplane;
  int2* ktab = reinterpret_cast<int2*>(w_region + w_bytes);  // per k: (offset, tap)
  uint64_t* bars = reinterpret_cast<uint64_t*>(ktab + P.kchunks * 32);
  uint64_t* full_a = bars;                         // [a_stages]
  uint64_t* empty_a = bars + kWStages;             // [a_stages]
  uint64_t* full_w = bars + 2 * kWStages;          // [w_stages]
  uint64_t* empty_w = bars + 3 * kWStages;         // [w_stages]
  uint64_t* acc_full = bars + 4 * kWStages;        // [2]
  uint64_t* acc_empty = acc_full + 2;              // [2]
  uint64_t* mma_done = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int* err = P.err;
  const int64_t n_tiles = (P.M + 127) / 128;
  const int64_t my_tiles = (int64_t)blockIdx.x < n_tiles ? (n_tiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;
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
    for (int i = 0; i < (P.w_stages ? P.w_stages : 1); ++i) {
      mbar_init(&full_w[i], 1);
      mbar_init(&empty_w[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 4);
    }
    mbar_init(mma_done, 1);
    fence_mbar_init();
  }
  // k table: k -> (window offset co*plane - ty*Pw - tx, tap index; 31 for padded columns)
  for (int k = threadIdx.x; k < P.kchunks * 32; k += blockDim.x) {
    int2 e = make_int2(0, kWMaxTaps);
    if (k < P.K) {
      const int co = k / P.taps, t = k - co * P.taps, ty = t / P.TX, tx = t - ty * P.TX;
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

  if (warp == kWProducerWarp && P.w_stages == 0) {
    // ---------------------------------------------------------------- weights, once
    if (lane == 0) {
      const uint32_t bytes = (uint32_t)P.kchunks * 2 * wplane;
      mbar_arrive_expect_tx(&full_w[0], bytes);
      for (uint32_t o = 0; o < bytes; o += 65536u) {
        const uint32_t nb = bytes - o < 65536u ? bytes - o : 65536u;
        bulk_g2s(w_region + o, P.wimg + o, nb, &full_w[0]);
      }
      mbar_wait_drain(&full_w[0], 0, err, 69);
    }
  } else if (warp == kWProducerWarp) {
    // ---------------------------------------------------------------- weight chunks
    if (lane == 0) {
      uint32_t g = 0;
      for (int64_t i = 0; i < my_tiles; ++i) {
        for (int c = 0; c < P.kchunks; ++c, ++g) {
          const uint32_t stage = g % (uint32_t)P.w_stages, round = g / (uint32_t)P.w_stages;
          if (!mbar_wait(&empty_w[stage], (round & 1u) ^ 1u, err, 61)) goto done_w;
          uint8_t* sb = w_region + (size_t)stage * 2 * wplane;
          const uint8_t* src = P.wimg + (size_t)c * 2 * wplane;
          mbar_arrive_expect_tx(&full_w[stage], 2 * wplane);
          bulk_g2s(sb, src, wplane, &full_w[stage]);
          bulk_g2s(sb + wplane, src + wplane, wplane, &full_w[stage]);
        }
      }
    done_w:
      // copies still in flight (error path) land before the CTA can exit
      for (uint32_t x = 0; x < (uint32_t)P.w_stages && x < g; ++x) {
        const uint32_t gl = g - 1 - x;
        mbar_wait_drain(&full_w[gl % (uint32_t)P.w_stages], (gl / (uint32_t)P.w_stages) & 1u, err, 62);
      }
    }
  } else if (warp == kWMmaWarp) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_tf32((uint32_t)P.n_pad);
      uint32_t g = 0;
      for (int64_t i = 0; i < my_tiles; ++i) {
        const uint32_t buf = (uint32_t)(i & 1);
        if (i >= 2 && !mbar_wait(&acc_empty[buf], (uint32_t)((i >> 1) & 1) ^ 1u, err, 63)) goto done_m;
        tc_fence_after();
        const uint32_t acc = tbase + buf * acc_cols;
        for (int c = 0; c < P.kchunks; ++c, ++g) {
          const int nks = min(4, (P.K - c * 32 + 7) / 8);
          const uint32_t as = g % (uint32_t)P.a_stages, ar = g / (uint32_t)P.a_stages;
          const bool resident = P.w_stages == 0;
          const uint32_t ws = resident ? 0u : g % (uint32_t)P.w_stages;
          const uint32_t wr = resident ? 0u : g / (uint32_t)P.w_stages;
          if (!mbar_wait(&full_a[as], ar & 1u, err, 64)) goto done_m;
          if ((!resident || g == 0) && !mbar_wait(&full_w[ws], wr & 1u, err, 68)) goto done_m;
          tc_fence_after();
          const uint32_t sa = smem_u32(a_region + as * 2 * kWAImg);
          const uint32_t sw = smem_u32(w_region + (size_t)(resident ? c : (int)ws) * 2 * wplane);
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
          mma_commit(&empty_a[as]);
          if (!resident) mma_commit(&empty_w[ws]);
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
    // thread -> tile row r and the kWCols columns [part*kWCols, +kWCols) of every chunk
    const int r = threadIdx.x & 127, part = threadIdx.x >> 7;
    constexpr int kQ = kWCols / 4;   // 16-byte pieces per thread and plane
    uint32_t soff[kQ];
#pragma unroll
    for (int q = 0; q < kQ; ++q)
      soff[q] = (uint32_t)r * 128u + ((((uint32_t)(part * kQ + q)) ^ ((uint32_t)r & 7u)) << 4);
    const int pos = P.ny * P.nx;
    const int64_t per_in = (int64_t)P.gi.C * plane_in;
    uint32_t g = 0;
    bool ok = true;
    // load cursor (tile li, chunk lc): two chunks ahead of the chunk being stored; its row's
    // window base (at its grid position) and the taps whose input position lies inside the
    // input window
    int64_t li = 0;
    int lc = 0;
    const float* base = P.in;
    uint32_t tapmask = 0;
    auto tile_row = [&](int64_t i) {
      const int64_t m = ((int64_t)blockIdx.x + i * gridDim.x) * 128 + r;
      base = P.in;
      tapmask = 0;
      if (i < my_tiles && m < P.M) {
        const int64_t rr = m / pos;
        const int rem = (int)(m - rr * pos);
        const int iy = rem / P.nx, ix = rem - iy * P.nx;
        const int qy = (P.i0 + iy) * P.f + P.f - 1, qx = (P.j0 + ix) * P.f + P.f - 1;
        base = P.in + rr * per_in + (int64_t)qy * P.gi.Pw + qx;
        for (int t = 0; t < P.taps; ++t) {
          const int ty = t / P.TX, tx = t - ty * P.TX;
          const int u = qy - ty, v = qx - tx;
          if (u >= 0 && u < P.gi.Ph && v >= 0 && v < P.gi.Pw) tapmask |= 1u << t;
        }
      }
    };
    auto load_next = [&](float (&v)[kWCols]) {
      const int kb = lc * 32 + part * kWCols;
#pragma unroll
      for (int e = 0; e < kWCols; ++e) {
        const int2 te = ktab[kb + e];
        v[e] = ((tapmask >> te.y) & 1u) ? __ldg(base + te.x) : 0.0f;
      }
      if (++lc == P.kchunks) {
        lc = 0;
        tile_row(++li);
      }
    };
    // chunk g of the flattened (tile, chunk) sequence: split the values of buffer v, reuse v
    // for chunk g + 2, store the split values into stage g % a_stages
    auto process = [&](float (&v)[kWCols]) -> bool {
      const uint32_t stage = g % (uint32_t)P.a_stages, round = g / (uint32_t)P.a_stages;
      float hi[kWCols], lo[kWCols];
#pragma unroll
      for (int e = 0; e < kWCols; ++e) split_tf32(v[e], hi[e], lo[e]);
      load_next(v);   // past the last tile the cursor's tapmask is 0: no loads
      if (!warp_wait(&empty_a[stage], (round & 1u) ^ 1u, err, 66)) return false;
      const uint32_t sbase = smem_u32(a_region) + stage * 2 * kWAImg;
#pragma unroll
      for (int q = 0; q < kQ; ++q) {
        asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(sbase + soff[q]), "f"(hi[4 * q]),
                     "f"(hi[4 * q + 1]), "f"(hi[4 * q + 2]), "f"(hi[4 * q + 3])
                     : "memory");
        asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(sbase + kWAImg + soff[q]), "f"(lo[4 * q]),
                     "f"(lo[4 * q + 1]), "f"(lo[4 * q + 2]), "f"(lo[4 * q + 3])
                     : "memory");
      }
      fence_proxy_async_smem();
      mbar_arrive(&full_a[stage]);
      ++g;
      return true;
    };
    float va[kWCols], vb[kWCols];
    tile_row(0);
    load_next(va);
    load_next(vb);
    const uint32_t total = (uint32_t)(my_tiles * P.kchunks);
    while (ok && g < total) {
      ok = process(va);
      if (ok && g < total) ok = process(vb);
    }
  } else {
    // ---------------------------------------------------------------- drain (warps 10-13)
    const int q4 = warp & 3;
    const uint32_t lane_off = (uint32_t)(q4 * 32) << 16;
    const int pos = P.ny * P.nx;
    const int plane_out = P.go.Ph * P.go.Pw;
    const int64_t per_out = (int64_t)P.go.C * plane_out;
    const int s = P.S, cin = P.cv.cin;
    // 8-byte pair stores: stride 2, even offsets (output x of phase 0 even), whole 16-column
    // channel groups, even plane and row lengths (8-byte aligned rows)
    const bool pair_ok = s == 2 && cin % 16 == 0 && (P.go.Pw & 1) == 0 && (plane_out & 1) == 0 &&
                         (per_out & 1) == 0 && (reinterpret_cast<uintptr_t>(P.out) & 7) == 0;
    const bool pairs = pair_ok && (P.Dx & 1) == 0;
    const bool pairs_odd = pair_ok && (P.Dx & 1) == 1;
    for (int64_t i = 0; i < my_tiles; ++i) {
      const uint32_t buf = (uint32_t)(i & 1);
      const int64_t m = ((int64_t)blockIdx.x + i * gridDim.x) * 128 + q4 * 32 + lane;
      const bool valid = m < P.M;
      float* o = nullptr;
      int ub = 0, vb = 0, Yb = 0, Xb = 0;   // output-window and image coordinates of phase (0, 0)
      if (valid) {
        const int64_t rr = m / pos;
        const int rem = (int)(m - rr * pos);
        const int iy = rem / P.nx, ix = rem - iy * P.nx;
        ub = (P.i0 + iy) * s - P.Dy;
        vb = (P.j0 + ix) * s - P.Dx;
        // row rr = (bound, region, i); i's position (oy, ox) in the bounded layer's image
        const int64_t BR = P.rg.B * P.rg.R;
        const int64_t rem2 = rr - (rr / BR) * BR;
        const int64_t ri = rem2 - (rem2 / P.rg.R) * P.rg.R;
        const int64_t hw = (int64_t)P.rg.Hm * P.rg.Wm;
        const int64_t pp = ri - (ri / hw) * hw;
        const int oy = (int)(pp / P.rg.Wm), ox = (int)(pp - (int64_t)oy * P.rg.Wm);
        Yb = oy * P.go.sig_h - P.go.pi_h + ub;
        Xb = ox * P.go.sig_w - P.go.pi_w + vb;
        o = P.out + rr * per_out;
      }
      if (!warp_wait(&acc_full[buf], (uint32_t)((i >> 1) & 1), err, 67)) break;
      tc_fence_after();
      const uint32_t src = tbase + buf * acc_cols + lane_off;
      if (pairs) {
        // stride 2, even offset: the px = 0 and px = 1 outputs of a position are one aligned
        // 8-byte pair; columns (py, 0, c0..c0+15) and (py, 1, c0..c0+15) give 16 pairs
        for (int py = 0; py < 2; ++py) {
          for (int c0 = 0; c0 < cin; c0 += 16) {
            float x0[16], x1[16];
            tmem_ld16(src + (uint32_t)((2 * py) * cin + c0), x0);
            tmem_ld16(src + (uint32_t)((2 * py + 1) * cin + c0), x1);
            tmem_ld_wait();
            const int uo = ub + py;
            if (!valid || uo < 0 || uo >= P.go.Ph) continue;
            const bool yin = Yb + py >= 0 && Yb + py < P.go.H;
            const bool in0 = yin && Xb >= 0 && Xb < P.go.W, in1 = yin && Xb + 1 >= 0 && Xb + 1 < P.go.W;
            const bool v1 = vb + 1 < P.go.Pw;   // vb itself is inside the window (even, >= 0)
            float* orow = o + (int64_t)uo * P.go.Pw + vb;
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              float* q = orow + (int64_t)(c0 + e) * plane_out;
              const float a = in0 ? x0[e] : 0.0f, b = in1 ? x1[e] : 0.0f;
              if (v1) *reinterpret_cast<float2*>(q) = make_float2(a, b);
              else *q = a;
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[buf]);
        continue;
      }
      if (pairs_odd) {
        // stride 2, odd offset: px = 1 of position (i, j) (even x) and px = 0 of (i, j+1) form
        // the aligned pair; the neighbour's value comes from the next lane when that lane
        // holds the next position of the same grid row, else both are stored singly
        const int ix = valid ? (int)((m % pos) % P.nx) : 0;
        const bool partner = lane < 31 && valid && ix < P.nx - 1 && m + 1 < P.M;
        const bool left_in_warp = lane > 0 && ix > 0;
        for (int py = 0; py < 2; ++py) {
          for (int c0 = 0; c0 < cin; c0 += 16) {
            float x0[16], x1[16], n0[16];
            tmem_ld16(src + (uint32_t)((2 * py) * cin + c0), x0);
            tmem_ld16(src + (uint32_t)((2 * py + 1) * cin + c0), x1);
            tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 16; ++e) n0[e] = __shfl_down_sync(0xffffffffu, x0[e], 1);
            const int uo = ub + py;
            if (!valid || uo < 0 || uo >= P.go.Ph) continue;
            const bool yin = Yb + py >= 0 && Yb + py < P.go.H;
            const bool in0 = yin && Xb >= 0 && Xb < P.go.W, in1 = yin && Xb + 1 >= 0 && Xb + 1 < P.go.W;
            const bool inp = yin && Xb + 2 >= 0 && Xb + 2 < P.go.W;
            const int v0 = vb, v1 = vb + 1;     // px = 0 (odd x) and px = 1 (even x)
            float* orow = o + (int64_t)uo * P.go.Pw;
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              float* q = orow + (int64_t)(c0 + e) * plane_out;
              if (v1 < P.go.Pw) {
                const float b = in1 ? x1[e] : 0.0f;
                if (partner) *reinterpret_cast<float2*>(q + v1) = make_float2(b, inp ? n0[e] : 0.0f);
                else q[v1] = b;
              }
              if (!left_in_warp && v0 >= 0 && v0 < P.go.Pw) q[v0] = in0 ? x0[e] : 0.0f;
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[buf]);
        continue;
      }
      // column n = (py, px, ci) decoded incrementally (ci fastest)
      int ci = 0, px = 0, py = 0;
      for (int q = 0; q < P.n_pad / 16; ++q) {
        float x[16];
        tmem_ld16(src + (uint32_t)(q * 16), x);
        tmem_ld_wait();
        if (valid) {
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            if (q * 16 + e >= P.N) break;
            const int uo = ub + py, vo = vb + px;
            if (uo >= 0 && uo < P.go.Ph && vo >= 0 && vo < P.go.Pw) {
              const int Y = Yb + py, X = Xb + px;
              const bool inside = Y >= 0 && Y < P.go.H && X >= 0 && X < P.go.W;
              o[(int64_t)ci * plane_out + (int64_t)uo * P.go.Pw + vo] = inside ? x[e] : 0.0f;
            }
            if (++ci == cin) {
              ci = 0;
              if (++px == s) {
                px = 0;
                ++py;
              }
            }
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

// Geometry of the phase-stacked GEMM of one conv step.
struct TcGeom {
  int TY, TX, f, S, i0, j0, ny, nx, Dy, Dx, K, kchunks, N, n_pad;
};

int floor_div(int a, int b) { return a >= 0 ? a / b : -((-a + b - 1) / b); }

// output blocking factor: 2x2 output blocks for a stride-1 layer (N = 4*Cin <= 256) unless
// CF_CONV_BLOCK=0; 1 otherwise
int tc_blocking(const ConvGeom& cv) {
  static int off = -1;
  if (off < 0) {
    const char* e = getenv("CF_CONV_BLOCK");
    off = (e && e[0] == '0') ? 1 : 0;
  }
  return (!off && cv.s == 1 && cv.kh >= 2 && cv.kw >= 2 && 4 * cv.cin <= 256 &&
          (cv.kh + 1) * (cv.kw + 1) <= kWMaxTaps)
             ? 2
             : 1;
}

// k taps per dimension, K, N of the GEMM of a conv step
void tc_dims(const ConvGeom& cv, int cout, int& f, int& TY, int& TX, int& K, int& N, int& n_pad) {
  f = tc_blocking(cv);
  TY = (cv.kh + cv.s - 1) / cv.s + f - 1;
  TX = (cv.kw + cv.s - 1) / cv.s + f - 1;
  K = cout * TY * TX;
  N = cv.s * f * cv.s * f * cv.cin;
  n_pad = ((N + 15) / 16) * 16;
}

TcGeom tc_geom(const WinGeom& gi, const WinGeom& go, const ConvGeom& cv, int cout) {
  TcGeom t;
  const int s = cv.s;
  tc_dims(cv, cout, t.f, t.TY, t.TX, t.K, t.N, t.n_pad);
  t.S = s * t.f;
  t.Dy = gi.pi_h * s + cv.pad - go.pi_h;
  t.Dx = gi.pi_w * s + cv.pad - go.pi_w;
  // grid rows i with some phase position u' = i*S + py - D inside [0, Ph)
  t.i0 = floor_div(t.Dy, t.S);
  t.j0 = floor_div(t.Dx, t.S);
  t.ny = floor_div(go.Ph - 1 + t.Dy, t.S) - t.i0 + 1;
  t.nx = floor_div(go.Pw - 1 + t.Dx, t.S) - t.j0 + 1;
  t.kchunks = (t.K + 31) / 32;
  return t;
}

size_t tc_smem_fixed(int kchunks) { return 1024 + (size_t)kchunks * 32 * 8 + (4 * kWStages + 5) * 8 + 16; }

}  // namespace

size_t win_convT_tc_scratch_bytes(const ConvGeom& cv, int cout) {
  // the weight image: kchunks x 2 planes x n_pad rows x 128 B
  int f, TY, TX, K, N, n_pad;
  tc_dims(cv, cout, f, TY, TX, K, N, n_pad);
  return (size_t)((K + 31) / 32) * 2 * n_pad * 128;
}

bool win_convT_tc_applicable(const ConvGeom& cv, int cout) {
  int f, TY, TX, K, N, n_pad;
  tc_dims(cv, cout, f, TY, TX, K, N, n_pad);
  const size_t smem = tc_smem_fixed((K + 31) / 32) + (size_t)2 * (2 * kWAImg + 2 * n_pad * 128);
  return cv.cin >= 1 && n_pad <= 256 && TY * TX <= kWMaxTaps && smem <= 227 * 1024;
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
  const TcGeom t = tc_geom(gi, go, cv, cout);
  CF_REQUIRE(t.ny >= 1 && t.nx >= 1, CF_ERR_SHAPE, "convT_tc: empty grid");
  WinTcParams P;
  memset(&P, 0, sizeof(P));
  P.rg = rg;
  P.gi = gi;
  P.go = go;
  P.cv = cv;
  P.TY = t.TY;
  P.TX = t.TX;
  P.f = t.f;
  P.S = t.S;
  P.i0 = t.i0;
  P.j0 = t.j0;
  P.ny = t.ny;
  P.nx = t.nx;
  P.Dy = t.Dy;
  P.Dx = t.Dx;
  P.K = t.K;
  P.kchunks = t.kchunks;
  P.taps = t.TY * t.TX;
  P.N = t.N;
  P.n_pad = t.n_pad;
  P.M = rows * t.ny * t.nx;
  P.in = in;
  P.out = out;
  P.wimg = scratch;
  P.err = err;
  // the whole weight image resident with as many A stages (2..kWStages) as fit, else
  // streamed W stages beside the A stages
  const size_t fixed = tc_smem_fixed(t.kchunks);
  const size_t a_st = (size_t)2 * kWAImg, w_st = (size_t)2 * t.n_pad * 128;
  const size_t w_all = (size_t)t.kchunks * w_st;
  size_t smem;
  if (fixed + w_all + 2 * a_st <= 227 * 1024) {
    int stages = kWStages;
    while (stages > 2 && fixed + w_all + stages * a_st > 227 * 1024) --stages;
    P.a_stages = stages;
    P.w_stages = 0;
    smem = fixed + w_all + stages * a_st;
  } else {
    int stages = kWStages;
    while (stages > 2 && fixed + stages * (a_st + w_st) > 227 * 1024) --stages;
    P.a_stages = P.w_stages = stages;
    smem = fixed + stages * (a_st + w_st);
  }
  CF_REQUIRE(smem <= 227 * 1024, CF_ERR_UNSUPPORTED, "convT_tc: %zu bytes of shared memory", smem);
  // the phase-stacked weight image (stream-ordered before the GEMM that reads it)
  const int64_t total = (int64_t)t.kchunks * t.n_pad * 32;
  k_win_prep_wimg<<<(unsigned)ceil_div(total, 256), 256, 0, st>>>(W, cv, t.TY, t.TX, t.f, t.N, t.n_pad, t.K,
                                                                   t.kchunks, scratch);
  CF_TRY(check_launch("k_win_prep_wimg"));
  const int64_t tiles = (P.M + 127) / 128;
  const int64_t grid = tiles < sms ? tiles : sms;
  k_win_convT_tc<<<(unsigned)grid, kWThreads, smem, st>>>(P);
  return check_launch("k_win_convT_tc");
}

}  // namespace cf
