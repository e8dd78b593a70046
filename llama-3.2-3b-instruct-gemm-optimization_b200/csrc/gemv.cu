// gemv.cu -- stream-K decode GEMV for sm_100a.
//
// y[m, n] = epilogue( s[n] * sum_k x[m, k] * W[k, n] ),  m < M <= 8.
//
// This computes what the reference's run_gemv computes
// (kernels/gemv_fp8.cu:276-283 -> gemv_chunk_kernel :91-151 -> cast :153-173;
// kernels/gemv_fp16.cu:134-156), but is organised for B200:
//
//  * One CTA per SM.  The packed weight stream (gemv.h) is cut into `grid`
//    equal contiguous byte ranges (stream-K), so every SM streams the same
//    number of bytes whatever the shape -- no wave quantisation, no tail.
//  * A producer warp streams the CTA's range into a shared-memory ring with
//    1-D bulk TMA copies (cp.async.bulk, L2 evict-first), several stages in
//    flight; it never waits on the previous kernel (weights are constant), so
//    under programmatic dependent launch the stream starts while the previous
//    kernel drains.
//  * Eight consumer warps take units round-robin.  A unit is 16 output
//    channels x 32 k (E4M3) or 16 k (FP16); each lane's 16 B are exactly its
//    m16n8k16 A-fragment, so E4M3 is widened with cvt.rn.f16x2.e4m3x2 in
//    registers and fed to mma.sync with x^T (k x 8 tokens) as the B operand:
//    the M <= 8 decode rows fill the n = 8 side of the tile.  A CUDA-core
//    FFMA variant of the same loop (kMathFfma) exists for comparison.
//  * Split-K partial sums are combined deterministically: per virtual tile,
//    the warps' partials are summed in warp order by the last warp to finish
//    it; a tile split across CTAs is summed in (k-range, CTA) order by the
//    last CTA to arrive (a counter per tile, reset by that CTA).  No float
//    atomics (the reference atomically adds into y_acc, gemv_fp8.cu:143-150),
//    no memset, no separate cast kernel.
//  * Epilogues: per-channel/tensor scale, fp16 rounding, SiLU(gate)*up for the
//    fused gate||up op, residual add; RMSNorm of the input rows in the
//    prologue.
#include <cstdio>
#include <type_traits>

#include "device.cuh"
#include "gemv.h"

namespace b2g {

__device__ int g_device_error;

int* device_error_word() {
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_device_error) != cudaSuccess) return nullptr;
  return static_cast<int*>(p);
}

namespace {

constexpr int W = kConsumerWarps;
constexpr int kUnitsPerWarpStage = 2;
constexpr int kStageUnits = W * kUnitsPerWarpStage;

__device__ __forceinline__ long long cta_of(long long u, long long T, int G) {
  return ((u + 1) * G + T - 1) / T - 1;
}

__device__ __forceinline__ float channel_scale(const GemvParams& p, int plane, int n) {
  switch (p.scale_mode) {
    case 1:
      return __half2float(reinterpret_cast<const __half*>(p.scales)[plane]);
    case 2:
      return __half2float(reinterpret_cast<const __half*>(p.scales)[(size_t)plane * p.N + n]);
    case 3:
      return reinterpret_cast<const float*>(p.scales)[(size_t)plane * p.N + n];
    default:
      return 1.0f;
  }
}

__device__ __forceinline__ float2 h2_to_f2(uint32_t v) {
  __half2 h;
  *reinterpret_cast<uint32_t*>(&h) = v;
  return __half22float2(h);
}

__device__ __forceinline__ uint32_t f2_to_h2(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Lane layout of a finished tile (the m16n8 accumulator): entry i of lane
// (g = lane/4, q = lane%4) is channel g + 8*(i/2), token 2q + (i%2).
template <int P>
__device__ void epilogue(const GemvParams& p, int tile, const float (&v)[P][4], int lane) {
  const int g = lane >> 2, q = lane & 3;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int m = 2 * q + (i & 1);
    const int n = tile * kTileCh + g + 8 * (i >> 1);
    if (m < p.M && n < p.N) {
      __half out;
      if constexpr (P == 1) {
        out = __float2half_rn(v[0][i] * channel_scale(p, 0, n));
        if (p.residual_add)
          out = __float2half_rn(__half2float(__ldcg(p.residual + (size_t)m * p.ldr + n)) +
                                __half2float(out));
      } else {
        const float gf = __half2float(__float2half_rn(v[0][i] * channel_scale(p, 0, n)));
        const float uf = __half2float(__float2half_rn(v[1][i] * channel_scale(p, 1, n)));
        out = __float2half_rn(gf / (1.0f + expf(-gf)) * uf);
      }
      p.y[(size_t)m * p.ldy + n] = out;
    }
  }
}

// A virtual tile's CTA-level partial is complete in v: finish it here if this
// CTA is the tile's only contributor, else publish it and let the last
// contributing CTA sum all partials in (k-range, CTA) order.
template <int P>
__device__ void finish_vt(const GemvParams& p, long long vt, const float (&v)[P][4], int lane) {
  const long long T = p.total_units;
  const int G = p.grid;
  const int cta = blockIdx.x;
  const int ks = (int)(vt / p.n_tiles);
  const int tile = (int)(vt - (long long)ks * p.n_tiles);
  int total = 0;
  for (int k = 0; k < p.ksplit; ++k) {
    const long long a = ((long long)k * p.n_tiles + tile) * p.kbpv;
    total += (int)(cta_of(a + p.kbpv - 1, T, G) - cta_of(a, T, G)) + 1;
  }
  if (total == 1) {
    epilogue<P>(p, tile, v, lane);
    return;
  }
  const long long c_first = cta_of(vt * p.kbpv, T, G);
  float4* dst = reinterpret_cast<float4*>(p.partials) +
                ((size_t)vt * p.max_contrib + (size_t)(cta - c_first)) * P * 32;
#pragma unroll
  for (int pl = 0; pl < P; ++pl)
    __stcg(&dst[pl * 32 + lane], make_float4(v[pl][0], v[pl][1], v[pl][2], v[pl][3]));
  __threadfence();
  __syncwarp();
  int old = 0;
  if (lane == 0) old = atomicAdd(&p.counters[tile], 1);
  old = __shfl_sync(0xffffffffu, old, 0);
  if (old != total - 1) return;
  __threadfence();
  float s[P][4];
#pragma unroll
  for (int pl = 0; pl < P; ++pl) s[pl][0] = s[pl][1] = s[pl][2] = s[pl][3] = 0.f;
  for (int k = 0; k < p.ksplit; ++k) {
    const long long vt2 = (long long)k * p.n_tiles + tile;
    const long long a = vt2 * p.kbpv;
    const long long cf = cta_of(a, T, G), cl = cta_of(a + p.kbpv - 1, T, G);
    for (long long c = cf; c <= cl; ++c) {
      const float4* src = reinterpret_cast<const float4*>(p.partials) +
                          ((size_t)vt2 * p.max_contrib + (size_t)(c - cf)) * P * 32;
#pragma unroll
      for (int pl = 0; pl < P; ++pl) {
        const float4 t = __ldcg(&src[pl * 32 + lane]);
        s[pl][0] += t.x;
        s[pl][1] += t.y;
        s[pl][2] += t.z;
        s[pl][3] += t.w;
      }
    }
  }
  if (lane == 0) p.counters[tile] = 0;
  epilogue<P>(p, tile, s, lane);
}

// ---------------------------------------------------------------------------
// x (the M activation rows) -> shared memory in B-fragment order:
// [k32 block][m][quad q][16 B], the 16 B holding, for k16 steps s = 0, 1,
// the f16 pairs (16s + 2q, +1) and (16s + 8 + 2q, +1).
// ---------------------------------------------------------------------------
__device__ __forceinline__ void load8(const __half* row, int c, int K, bool vec, float (&f)[8]) {
  const int k0 = c * 8;
  if (vec && k0 + 8 <= K) {
    const uint4 v = __ldcg(reinterpret_cast<const uint4*>(row + k0));
    const float2 a = h2_to_f2(v.x), b = h2_to_f2(v.y), cc = h2_to_f2(v.z), d = h2_to_f2(v.w);
    f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y;
    f[4] = cc.x; f[5] = cc.y; f[6] = d.x; f[7] = d.y;
  } else {
#pragma unroll
    for (int e = 0; e < 8; ++e) f[e] = (k0 + e < K) ? __half2float(__ldcg(row + k0 + e)) : 0.f;
  }
}

__device__ void load_x(const GemvParams& p, uint8_t* xs, int kx_lo, int nkx, float* rms_r,
                       float* red, int tid) {
  constexpr int NT = W * 32;
  const int M = p.M, K = p.K;
  const bool vec = ((reinterpret_cast<uintptr_t>(p.x) & 15) == 0) && ((p.ldx & 7) == 0);
  if (p.rmsnorm) {
    const int nch = (K + 7) / 8;
    for (int m = 0; m < M; ++m) {
      const __half* xr = p.x + (size_t)m * p.ldx;
      float s = 0.f;
      for (int c = tid; c < nch; c += NT) {
        float f[8];
        load8(xr, c, K, vec, f);
#pragma unroll
        for (int e = 0; e < 8; ++e) s = fmaf(f[e], f[e], s);
      }
#pragma unroll
      for (int off = 16; off; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
      if ((tid & 31) == 0) red[(tid >> 5) * 8 + m] = s;
    }
    named_sync(1, NT);
    if (tid < M) {
      float t = 0.f;
      for (int w = 0; w < W; ++w) t += red[w * 8 + tid];
      rms_r[tid] = 1.0f / sqrtf(t / (float)K + p.rms_eps);
    }
    named_sync(1, NT);
  }
  const int c_lo = kx_lo * 4, nch = nkx * 4;
  for (int idx = tid; idx < M * nch; idx += NT) {
    const int m = idx / nch, cr = idx - m * nch;
    float f[8];
    load8(p.x + (size_t)m * p.ldx, c_lo + cr, K, vec, f);
    if (p.rmsnorm) {
      const float r = rms_r[m];
#pragma unroll
      for (int e = 0; e < 8; ++e) f[e] *= r;
    }
    uint32_t* base = reinterpret_cast<uint32_t*>(xs + (size_t)((cr >> 2) * M + m) * 64) + (cr & 3);
#pragma unroll
    for (int j = 0; j < 4; ++j) base[j * 4] = f2_to_h2(f[2 * j], f[2 * j + 1]);
  }
}

// ---------------------------------------------------------------------------
// Per-unit math
// ---------------------------------------------------------------------------
template <int P, int WB>
struct MmaMath {
  float acc[P][4];
  __device__ __forceinline__ void zero() {
#pragma unroll
    for (int pl = 0; pl < P; ++pl) acc[pl][0] = acc[pl][1] = acc[pl][2] = acc[pl][3] = 0.f;
  }
  // xq = xs + (kx * M) * 64 + q * 16 (the lane's quad column of block kx)
  __device__ __forceinline__ void unit(const uint4 (&wv)[P], const uint8_t* xq, int g, int M,
                                       int kg) {
    if constexpr (WB == 1) {
      uint4 xb = make_uint4(0, 0, 0, 0);
      if (g < M) xb = lds128(xq + g * 64);
#pragma unroll
      for (int pl = 0; pl < P; ++pl) {
        const uint4 w = wv[pl];
        mma_16816(acc[pl], e4m3x2_to_f16x2((uint16_t)(w.x & 0xFFFF)),
                  e4m3x2_to_f16x2((uint16_t)(w.x >> 16)), e4m3x2_to_f16x2((uint16_t)(w.y & 0xFFFF)),
                  e4m3x2_to_f16x2((uint16_t)(w.y >> 16)), xb.x, xb.y);
        mma_16816(acc[pl], e4m3x2_to_f16x2((uint16_t)(w.z & 0xFFFF)),
                  e4m3x2_to_f16x2((uint16_t)(w.z >> 16)), e4m3x2_to_f16x2((uint16_t)(w.w & 0xFFFF)),
                  e4m3x2_to_f16x2((uint16_t)(w.w >> 16)), xb.z, xb.w);
      }
    } else {
      uint2 xb = make_uint2(0, 0);
      if (g < M) xb = lds64(xq + g * 64 + (kg & 1) * 8);
#pragma unroll
      for (int pl = 0; pl < P; ++pl) {
        const uint4 w = wv[pl];
        mma_16816(acc[pl], w.x, w.y, w.z, w.w, xb.x, xb.y);
      }
    }
  }
  __device__ __forceinline__ void result(float (&v)[P][4], int) const {
#pragma unroll
    for (int pl = 0; pl < P; ++pl)
#pragma unroll
      for (int i = 0; i < 4; ++i) v[pl][i] = acc[pl][i];
  }
};

template <int P, int WB>
struct FfmaMath {
  float acc[P][2][8];  // [plane][channel g or g+8][token]
  __device__ __forceinline__ void zero() {
#pragma unroll
    for (int pl = 0; pl < P; ++pl)
#pragma unroll
      for (int c = 0; c < 2; ++c)
#pragma unroll
        for (int m = 0; m < 8; ++m) acc[pl][c][m] = 0.f;
  }
  __device__ __forceinline__ void unit(const uint4 (&wv)[P], const uint8_t* xq, int, int M,
                                       int kg) {
    // weights as float pairs: wf[pl][s][r], r = (which << 1) | channel
    constexpr int S = (WB == 1) ? 2 : 1;
    float2 wf[P][S][4];
#pragma unroll
    for (int pl = 0; pl < P; ++pl) {
      const uint4 w = wv[pl];
      if constexpr (WB == 1) {
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int s = 0; s < 2; ++s)
#pragma unroll
          for (int r = 0; r < 4; ++r) {
            const uint32_t word = ws[s * 2 + (r >> 1)];
            const uint16_t pr = (r & 1) ? (uint16_t)(word >> 16) : (uint16_t)(word & 0xFFFF);
            wf[pl][s][r] = h2_to_f2(e4m3x2_to_f16x2(pr));
          }
      } else {
        wf[pl][0][0] = h2_to_f2(w.x);
        wf[pl][0][1] = h2_to_f2(w.y);
        wf[pl][0][2] = h2_to_f2(w.z);
        wf[pl][0][3] = h2_to_f2(w.w);
      }
    }
#pragma unroll
    for (int m = 0; m < 8; ++m) {
      if (m < M) {
        float2 xf[S][2];
        if constexpr (WB == 1) {
          const uint4 xv = lds128(xq + m * 64);
          xf[0][0] = h2_to_f2(xv.x);
          xf[0][1] = h2_to_f2(xv.y);
          xf[1][0] = h2_to_f2(xv.z);
          xf[1][1] = h2_to_f2(xv.w);
        } else {
          const uint2 xv = lds64(xq + m * 64 + (kg & 1) * 8);
          xf[0][0] = h2_to_f2(xv.x);
          xf[0][1] = h2_to_f2(xv.y);
        }
#pragma unroll
        for (int pl = 0; pl < P; ++pl)
#pragma unroll
          for (int s = 0; s < S; ++s)
#pragma unroll
            for (int r = 0; r < 4; ++r) {
              const float2 a = wf[pl][s][r], b = xf[s][r >> 1];
              float& d = acc[pl][r & 1][m];
              d = fmaf(a.x, b.x, d);
              d = fmaf(a.y, b.y, d);
            }
      }
    }
  }
  __device__ __forceinline__ void result(float (&v)[P][4], int lane) {
    const int q = lane & 3;
#pragma unroll
    for (int pl = 0; pl < P; ++pl)
#pragma unroll
      for (int c = 0; c < 2; ++c)
#pragma unroll
        for (int m = 0; m < 8; ++m) {
          float t = acc[pl][c][m];
          t += __shfl_xor_sync(0xffffffffu, t, 1);
          t += __shfl_xor_sync(0xffffffffu, t, 2);
          acc[pl][c][m] = t;
        }
#pragma unroll
    for (int pl = 0; pl < P; ++pl)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float t = 0.f;
#pragma unroll
        for (int m = 0; m < 8; ++m)
          if (m == 2 * q + (i & 1)) t = acc[pl][i >> 1][m];
        v[pl][i] = t;
      }
  }
};

// ---------------------------------------------------------------------------
// The kernel
// ---------------------------------------------------------------------------
template <int P, int WB, int MATH>
__global__ void __launch_bounds__(kThreads, 1) gemv_streamk_kernel(const __grid_constant__ GemvParams p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  constexpr int UNIT = P * kUnitPlaneBytes;
  const int NS = p.n_stages;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + NS;
  int* slot_count = reinterpret_cast<int*>(smem + p.off_misc);
  volatile int* abort_flag = slot_count + p.n_slots;
  float* rms_r = reinterpret_cast<float*>(slot_count + p.n_slots + 1);
  float* red = rms_r + 8;
  uint8_t* ring = smem + p.off_ring;
  float4* slots = reinterpret_cast<float4*>(smem + p.off_slots);
  uint8_t* xs = smem + p.off_x;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const long long T = p.total_units;
  const int G = p.grid;
  const long long u0 = (long long)blockIdx.x * T / G;
  const long long u1 = (long long)(blockIdx.x + 1) * T / G;
  const long long n_units = u1 - u0;
  const int n_st = (int)((n_units + kStageUnits - 1) / kStageUnits);

  if (tid == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], W);
    }
    fence_mbarrier_init();
    pdl_launch_dependents();
  }
  for (int i = tid; i <= p.n_slots; i += blockDim.x) slot_count[i] = 0;
  for (int i = tid; i < p.n_slots * W * P * 32; i += blockDim.x) slots[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  __syncthreads();

  if (warp == W) {
    // ---------------- producer: TMA bulk stream of [u0, u1) ----------------
    if (lane == 0 && n_st > 0) {
      const uint64_t pol = l2_policy_evict_first();
      int s = 0, err = kErrNone;
      for (; s < n_st; ++s) {
        const int slot = s % NS;
        if (s >= NS && !mbar_wait_bounded(&empty[slot], ((s / NS) - 1) & 1)) {
          err = kErrEmptyWait;
          break;
        }
        if (*abort_flag) break;
        const long long us = u0 + (long long)s * kStageUnits;
        const int nu = (int)min((long long)kStageUnits, u1 - us);
        const uint32_t bytes = (uint32_t)nu * UNIT;
        mbar_arrive_expect_tx(&full[slot], bytes);
        bulk_g2s(ring + (size_t)slot * kStageUnits * UNIT, p.packed + us * UNIT, bytes, &full[slot], pol);
      }
      if (err != kErrNone || *abort_flag) {
        if (err != kErrNone) atomicCAS(p.error, 0, err);
        *abort_flag = 1;
        // every copy this CTA issued must land before the CTA exits
        for (int s2 = max(0, s - NS); s2 < s; ++s2)
          if (!mbar_wait_bounded(&full[s2 % NS], (s2 / NS) & 1)) {
            atomicCAS(p.error, 0, kErrDrainWait);
            break;
          }
      }
    }
    return;
  }

  // ---------------- consumers ----------------
  const int g = lane >> 2, q = lane & 3;
  const int M = p.M;
  const int kbpv = p.kbpv;
  long long vt_first = 0;
  int kx_lo = 0, nkx = 0;
  if (n_units > 0) {
    vt_first = u0 / kbpv;
    const long long vt_last = (u1 - 1) / kbpv;
    const int ks_lo = (int)(vt_first / p.n_tiles), ks_hi = (int)(vt_last / p.n_tiles);
    const int kx_per_ks = kbpv * (WB == 1 ? 32 : 16) / 32;
    kx_lo = ks_lo * kx_per_ks;
    nkx = (ks_hi + 1) * kx_per_ks - kx_lo;
  }
  pdl_wait();
  load_x(p, xs, kx_lo, nkx, rms_r, red, tid);
  named_sync(1, W * 32);
  if (n_units <= 0) return;

  using Math = typename std::conditional<MATH == kMathMma, MmaMath<P, WB>, FfmaMath<P, WB>>::type;
  Math math;
  math.zero();

  // This warp's units are u0 + warp + j*W.
  long long u = u0 + warp;
  long long vt = u / kbpv;
  int kbl = (int)(u - vt * kbpv);
  int kg = (int)(vt / p.n_tiles) * kbpv + kbl;  // k-block index over padded K
  bool touched = false;

  // Flush the warp's partial for virtual tile `fvt` into its smem slot; the
  // last warp of the CTA to do so sums the slot (warp order) and finishes it.
  auto flush = [&](long long fvt) {
    float v[P][4];
    math.result(v, lane);
    const int j = (int)(fvt - vt_first);
    float4* sl = slots + (size_t)(j * W + warp) * P * 32;
#pragma unroll
    for (int pl = 0; pl < P; ++pl) sl[pl * 32 + lane] = make_float4(v[pl][0], v[pl][1], v[pl][2], v[pl][3]);
    __threadfence_block();
    __syncwarp();
    int old = 0;
    if (lane == 0) old = atomicAdd(&slot_count[j], 1);
    old = __shfl_sync(0xffffffffu, old, 0);
    const long long a = max(fvt * kbpv, u0), b = min((fvt + 1) * kbpv, u1);
    const int expected = (int)min((long long)W, b - a);
    if (old == expected - 1) {
      __threadfence_block();
      float s[P][4];
#pragma unroll
      for (int pl = 0; pl < P; ++pl) s[pl][0] = s[pl][1] = s[pl][2] = s[pl][3] = 0.f;
      for (int w = 0; w < W; ++w) {
        const float4* src = slots + (size_t)(j * W + w) * P * 32;
#pragma unroll
        for (int pl = 0; pl < P; ++pl) {
          const float4 t = src[pl * 32 + lane];
          s[pl][0] += t.x;
          s[pl][1] += t.y;
          s[pl][2] += t.z;
          s[pl][3] += t.w;
        }
      }
      finish_vt<P>(p, fvt, s, lane);
    }
  };

  for (int s = 0; s < n_st; ++s) {
    const int slot = s % NS;
    const bool ok = mbar_wait_bounded(&full[slot], (s / NS) & 1);
    if (!__all_sync(0xffffffffu, ok)) {
      if (lane == 0) {
        atomicCAS(p.error, 0, kErrFullWait);
        *abort_flag = 1;
      }
      return;
    }
    const long long us = u0 + (long long)s * kStageUnits;
    const int nu = (int)min((long long)kStageUnits, u1 - us);
    const uint8_t* stage = ring + (size_t)slot * kStageUnits * UNIT;
    uint4 wv[kUnitsPerWarpStage][P];
#pragma unroll
    for (int jj = 0; jj < kUnitsPerWarpStage; ++jj) {
      const int i = warp + jj * W;
      if (i < nu) {
#pragma unroll
        for (int pl = 0; pl < P; ++pl) wv[jj][pl] = lds128(stage + (size_t)i * UNIT + pl * kUnitPlaneBytes + lane * 16);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);
#pragma unroll
    for (int jj = 0; jj < kUnitsPerWarpStage; ++jj) {
      const int i = warp + jj * W;
      if (i < nu) {
        const int kx = (WB == 1 ? kg : (kg >> 1)) - kx_lo;
        math.unit(wv[jj], xs + (size_t)kx * M * 64 + q * 16, g, M, kg);
        touched = true;
        kbl += W;
        kg += W;
        if (kbl >= kbpv) {
          flush(vt);
          math.zero();
          touched = false;
          do {
            kbl -= kbpv;
            ++vt;
          } while (kbl >= kbpv);
          kg = (int)(vt / p.n_tiles) * kbpv + kbl;
        }
      }
    }
  }
  if (touched) flush(vt);
}

template <int P, int WB, int MATH>
cudaError_t launch_variant(const GemvParams& p, size_t smem, bool pdl, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, gemv_streamk_kernel<P, WB, MATH>, p);
}

template <int P, int WB, int MATH>
cudaError_t set_limit(int bytes) {
  return cudaFuncSetAttribute(gemv_streamk_kernel<P, WB, MATH>,
                              cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
}

}  // namespace

cudaError_t launch_gemv(const GemvParams& p, int planes, int wbytes, int math, size_t smem, bool pdl,
                        cudaStream_t stream) {
#define B2G_CASE(PP, WBB, MM) \
  if (planes == PP && wbytes == WBB && math == MM) return launch_variant<PP, WBB, MM>(p, smem, pdl, stream);
  B2G_CASE(1, 1, kMathMma)
  B2G_CASE(2, 1, kMathMma)
  B2G_CASE(1, 2, kMathMma)
  B2G_CASE(2, 2, kMathMma)
  B2G_CASE(1, 1, kMathFfma)
  B2G_CASE(2, 1, kMathFfma)
  B2G_CASE(1, 2, kMathFfma)
  B2G_CASE(2, 2, kMathFfma)
#undef B2G_CASE
  return cudaErrorInvalidValue;
}

cudaError_t gemv_set_smem_limit(int bytes) {
  cudaError_t e = cudaSuccess, r;
#define B2G_LIM(PP, WBB, MM) \
  if ((r = set_limit<PP, WBB, MM>(bytes)) != cudaSuccess) e = r;
  B2G_LIM(1, 1, kMathMma)
  B2G_LIM(2, 1, kMathMma)
  B2G_LIM(1, 2, kMathMma)
  B2G_LIM(2, 2, kMathMma)
  B2G_LIM(1, 1, kMathFfma)
  B2G_LIM(2, 1, kMathFfma)
  B2G_LIM(1, 2, kMathFfma)
  B2G_LIM(2, 2, kMathFfma)
#undef B2G_LIM
  return e;
}

}  // namespace b2g
