// gemv.cu -- stream-K decode GEMV for sm_100a.
//
// y[m, n] = epilogue( s[n] * sum_k x[m, k] * W[k, n] ),  m < M <= 8.
//
// This computes what the reference's run_gemv computes
// (kernels/gemv_fp8.cu:276-283 -> gemv_chunk_kernel :91-151 -> cast :153-173;
// kernels/gemv_fp16.cu:134-156), organised for B200:
//
//  * One CTA of 16 warps per SM.  The packed weight stream (gemv.h) is cut
//    into `grid` equal contiguous ranges (stream-K), so every SM streams the
//    same number of bytes whatever the shape: no wave quantisation, no tail.
//  * Weights go straight from HBM into registers: each lane's 16 B of a unit
//    (16 output channels x 32 k for E4M3, x 16 k for FP16) is exactly its
//    m16n8k16 A fragment, loaded with ld.global.nc.L1::no_allocate (L2
//    evict-first) 8-16 units ahead, 128 KB in flight per SM.  The first loads
//    are issued before waiting on the previous kernel (weights are
//    constant), and the tail of the stream warms L2 for the next kernel.
//  * The M <= 8 activation rows are staged once per CTA in shared memory by
//    bulk copy (RMSNorm applied there when fused), with the k order inside each
//    32-block permuted by the prepack so a lane's B fragment is one 16 B load;
//    the decode rows fill the n = 8 side of mma.sync.m16n8k16 (x^T as B).
//  * E4M3 is widened to f16 in registers (cvt.rn.f16x2.e4m3x2).  A CUDA-core
//    FFMA variant of the same loop (kMathFfma) exists for comparison.
//  * Each warp's partial per virtual tile goes to a shared-memory slot.  After
//    the stream the slots are summed in warp order, and a tile split across
//    CTAs is summed in (k-range, CTA) order by the last CTA to arrive (one
//    counter per tile, reset by that CTA).  Deterministic; no float atomics
//    (the reference atomically adds into y_acc, gemv_fp8.cu:143-150), no
//    memset, no separate cast kernel.
//  * Epilogues: per-channel/tensor scale, fp16 rounding, SiLU(gate)*up for the
//    fused gate||up op, residual add.
#include <cstdio>
#include <type_traits>

#include "device.cuh"
#include "gemv.h"

namespace b2g {

__device__ int g_device_error;

#ifdef B2G_TRACE
// Per-CTA phase timestamps (%globaltimer), debug builds only.
__device__ unsigned long long g_trace[1024][16];
#define TRACE(i) do { g_trace[blockIdx.x][(i)] = globaltimer_ns(); } while (0)
#else
#define TRACE(i) do { } while (0)
#endif

int* device_error_word() {
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_device_error) != cudaSuccess) return nullptr;
  return static_cast<int*>(p);
}

namespace {

constexpr int W = kWarps;
constexpr int NT = kThreads;

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

// Address of the idx-th partial of output tile `tile`, contributions ordered
// by (k-range, CTA).
template <int P>
__device__ __forceinline__ const float4* contrib_ptr(const GemvParams& p, int tile, int idx) {
  const long long T = p.total_units;
  for (int k = 0; k < p.ksplit; ++k) {
    const long long vt = (long long)k * p.n_tiles + tile;
    const long long a = vt * p.kbpv;
    const int n = (int)(cta_of(a + p.kbpv - 1, T, p.grid) - cta_of(a, T, p.grid)) + 1;
    if (idx < n)
      return reinterpret_cast<const float4*>(p.partials) + ((size_t)vt * p.max_contrib + idx) * P * 32;
    idx -= n;
  }
  return nullptr;
}

// A virtual tile's CTA-level sum is complete in v: finish it here if this CTA
// is the tile's only contributor, else publish it and let the last
// contributing CTA sum all partials in (k-range, CTA) order.
template <int P>
__device__ void finish_vt(const GemvParams& p, long long vt, const float (&v)[P][4], int lane) {
  const long long T = p.total_units;
  const int G = p.grid;
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
                ((size_t)vt * p.max_contrib + (size_t)(blockIdx.x - c_first)) * P * 32;
#pragma unroll
  for (int pl = 0; pl < P; ++pl)
    __stcg(&dst[pl * 32 + lane], make_float4(v[pl][0], v[pl][1], v[pl][2], v[pl][3]));
  fence_acq_rel_gpu();
  __syncwarp();
  int old = 0;
  if (lane == 0) old = atomicAdd(&p.counters[tile], 1);
  old = __shfl_sync(0xffffffffu, old, 0);
  if (old != total - 1) return;
  fence_acq_rel_gpu();
  float s[P][4];
#pragma unroll
  for (int pl = 0; pl < P; ++pl) s[pl][0] = s[pl][1] = s[pl][2] = s[pl][3] = 0.f;
  constexpr int B = 4;  // partials fetched per round trip
  for (int base = 0; base < total; base += B) {
    float4 t[B][P];
#pragma unroll
    for (int b = 0; b < B; ++b) {
      if (base + b < total) {
        const float4* src = contrib_ptr<P>(p, tile, base + b);
#pragma unroll
        for (int pl = 0; pl < P; ++pl) t[b][pl] = __ldcg(&src[pl * 32 + lane]);
      }
    }
#pragma unroll
    for (int b = 0; b < B; ++b) {
      if (base + b < total) {
#pragma unroll
        for (int pl = 0; pl < P; ++pl) {
          s[pl][0] += t[b][pl].x;
          s[pl][1] += t[b][pl].y;
          s[pl][2] += t[b][pl].z;
          s[pl][3] += t[b][pl].w;
        }
      }
    }
  }
  if (lane == 0) p.counters[tile] = 0;
  epilogue<P>(p, tile, s, lane);
}

// ---------------------------------------------------------------------------
// Activation rows in shared memory: row m at xs + m * x_rs (halves), holding
// k in [k_lo, k_lo + krange).  The row stride is = 8 (mod 64) halves so the
// eight rows of a B fragment fall in different banks.
// ---------------------------------------------------------------------------
__device__ void stage_x_manual(const GemvParams& p, __half* xs, int k_lo, int krange, int tid) {
  const int M = p.M, K = p.K;
  const bool vec = ((reinterpret_cast<uintptr_t>(p.x) & 15) == 0) && ((p.ldx & 7) == 0);
  const int nch = krange / 8;
  for (int idx = tid; idx < M * nch; idx += NT * 4) {
    uint4 v[4];
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int id = idx + r * NT;
      v[r] = make_uint4(0, 0, 0, 0);
      if (id < M * nch) {
        const int m = id / nch, c = id - m * nch;
        const int k0 = k_lo + c * 8;
        const __half* row = p.x + (size_t)m * p.ldx;
        if (vec && k0 + 8 <= K) {
          v[r] = __ldcg(reinterpret_cast<const uint4*>(row + k0));
        } else {
          uint32_t e[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) e[j] = (k0 + j < K) ? __half_as_ushort(__ldcg(row + k0 + j)) : 0u;
          v[r] = make_uint4(e[0] | (e[1] << 16), e[2] | (e[3] << 16), e[4] | (e[5] << 16),
                            e[6] | (e[7] << 16));
        }
      }
    }
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int id = idx + r * NT;
      if (id < M * nch) {
        const int m = id / nch, c = id - m * nch;
        sts128(xs + (size_t)m * p.x_rs + c * 8, v[r]);
      }
    }
  }
}

// In-place RMSNorm of the staged rows (gamma = 1): x <- fp16(x / sqrt(mean(x^2) + eps)).
// Requires the full row in shared memory (k_lo == 0, K % 8 == 0; host-checked).
__device__ void rmsnorm_rows(const GemvParams& p, __half* xs, float* rms_r, float* red, int tid) {
  const int M = p.M, K = p.K;
  const int nch = K / 8;
  for (int m = 0; m < M; ++m) {
    const __half* row = xs + (size_t)m * p.x_rs;
    float s = 0.f;
    for (int c = tid; c < nch; c += NT) {
      const uint4 v = lds128(row + c * 8);
      const float2 a = h2_to_f2(v.x), b = h2_to_f2(v.y), cc = h2_to_f2(v.z), d = h2_to_f2(v.w);
      s = fmaf(a.x, a.x, s); s = fmaf(a.y, a.y, s); s = fmaf(b.x, b.x, s); s = fmaf(b.y, b.y, s);
      s = fmaf(cc.x, cc.x, s); s = fmaf(cc.y, cc.y, s); s = fmaf(d.x, d.x, s); s = fmaf(d.y, d.y, s);
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
  for (int idx = tid; idx < M * nch; idx += NT) {
    const int m = idx / nch, c = idx - m * nch;
    __half* at = xs + (size_t)m * p.x_rs + c * 8;
    const uint4 v = lds128(at);
    const float r = rms_r[m];
    const float2 a = h2_to_f2(v.x), b = h2_to_f2(v.y), cc = h2_to_f2(v.z), d = h2_to_f2(v.w);
    sts128(at, make_uint4(f2_to_h2(a.x * r, a.y * r), f2_to_h2(b.x * r, b.y * r),
                          f2_to_h2(cc.x * r, cc.y * r), f2_to_h2(d.x * r, d.y * r)));
  }
}

// ---------------------------------------------------------------------------
// Per-unit math.  `xk` points at the unit's first k in row 0 of the staged x.
// ---------------------------------------------------------------------------
template <int P, int WB>
struct MmaMath {
  float acc[P][4];
  __device__ __forceinline__ void zero() {
#pragma unroll
    for (int pl = 0; pl < P; ++pl) acc[pl][0] = acc[pl][1] = acc[pl][2] = acc[pl][3] = 0.f;
  }
  // xf: this lane's B fragment for the unit (b0..b3 for E4M3; b0, b1 for FP16).
  __device__ __forceinline__ void unit(const uint4 (&wv)[P], const uint4& xf) {
    if constexpr (WB == 1) {
#pragma unroll
      for (int pl = 0; pl < P; ++pl) {
        const uint4 w = wv[pl];
        mma_16816(acc[pl], e4m3x2_to_f16x2(w.x), e4m3x2_to_f16x2(w.x >> 16), e4m3x2_to_f16x2(w.y),
                  e4m3x2_to_f16x2(w.y >> 16), xf.x, xf.y);
        mma_16816(acc[pl], e4m3x2_to_f16x2(w.z), e4m3x2_to_f16x2(w.z >> 16), e4m3x2_to_f16x2(w.w),
                  e4m3x2_to_f16x2(w.w >> 16), xf.z, xf.w);
      }
    } else {
#pragma unroll
      for (int pl = 0; pl < P; ++pl) {
        const uint4 w = wv[pl];
        mma_16816(acc[pl], w.x, w.y, w.z, w.w, xf.x, xf.y);
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
  // xk: this lane's x slice of the unit in row 0 (row m at xk + m * rs).
  __device__ __forceinline__ void unit(const uint4 (&wv)[P], const __half* xk, int M, int rs) {
    constexpr int S = (WB == 1) ? 2 : 1;  // k16 steps per unit
    float2 wf[P][S][4];                   // [plane][step][register r]
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
            wf[pl][s][r] = h2_to_f2(e4m3x2_to_f16x2((r & 1) ? (word >> 16) : word));
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
        const __half* xr = xk + (size_t)m * rs;
        float2 xf[S][2];  // [step][which: k or k+8]
        if constexpr (WB == 1) {
          const uint4 v = lds128(xr);
          xf[0][0] = h2_to_f2(v.x);
          xf[0][1] = h2_to_f2(v.y);
          xf[1][0] = h2_to_f2(v.z);
          xf[1][1] = h2_to_f2(v.w);
        } else {
          const uint2 v = lds64(xr);
          xf[0][0] = h2_to_f2(v.x);
          xf[0][1] = h2_to_f2(v.y);
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
__global__ void __launch_bounds__(kThreads, 1)
    gemv_streamk_kernel(const __grid_constant__ GemvParams p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  constexpr int UNIT = P * kUnitPlaneBytes;
  // Units each lane keeps in flight: 16 B x 512 threads x D x P = 128 KB per SM.
  constexpr int D = (MATH == kMathMma) ? (P == 1 ? 16 : 8) : (P == 1 ? 8 : 4);
  constexpr int KPB = (WB == 1) ? 32 : 16;  // k per k-block
  uint64_t* xbar = reinterpret_cast<uint64_t*>(smem);
  volatile int* abort_flag = reinterpret_cast<int*>(smem + kOffMisc);
  float* rms_r = reinterpret_cast<float*>(smem + kOffMisc + 16);
  float* red = reinterpret_cast<float*>(smem + 128);
  float4* slots = reinterpret_cast<float4*>(smem + kOffSlots);  // [n_slots][W][P][32]
  __half* xs = reinterpret_cast<__half*>(smem + p.off_x);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, q = lane & 3;
  const int M = p.M;
  const int kbpv = p.kbpv;
  const long long T = p.total_units;
  const int G = p.grid;
  const int u0 = (int)((long long)blockIdx.x * T / G);
  const int u1 = (int)((long long)(blockIdx.x + 1) * T / G);
  const int n_units = u1 - u0;
  if (n_units <= 0) return;  // whole CTA: no barrier is reached
  if (tid == 0) TRACE(0);
  const int n_mine = n_units > warp ? (n_units - warp + W - 1) / W : 0;  // units u0 + warp + j*W

  // ---- weight stream: the first D units, before waiting on the previous kernel
  const uint64_t pol = l2_policy_evict_first();
  const uint8_t* wlane = p.packed + ((size_t)u0 + warp) * UNIT + lane * 16;
  constexpr size_t WSTEP = (size_t)W * UNIT;
  uint4 buf[D][P];
#pragma unroll
  for (int d = 0; d < D; ++d)
    if (d < n_mine) {
#pragma unroll
      for (int pl = 0; pl < P; ++pl) buf[d][pl] = ldg_stream(wlane + d * WSTEP + pl * kUnitPlaneBytes, pol);
    }

  if (tid == 0) {
    mbar_init(xbar, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
    pdl_launch_dependents();
  }
  for (int i = tid; i < p.n_slots * W * P * 32; i += NT) slots[i] = make_float4(0.f, 0.f, 0.f, 0.f);

  // ---- the x rows this CTA needs
  const int vt_first = u0 / kbpv;
  const int vt_last = (u1 - 1) / kbpv;
  const int ks_lo = vt_first / p.n_tiles, ks_hi = vt_last / p.n_tiles;
  const int k_lo = ks_lo * kbpv * KPB;
  const int krange = (ks_hi + 1 - ks_lo) * kbpv * KPB;
  __syncthreads();
  pdl_wait();
  if (tid == 0) TRACE(1);
  if (p.x_tma) {
    if (tid == 0) {
      fence_proxy_async_global();
      const uint32_t row_bytes = (uint32_t)krange * 2;
      mbar_arrive_expect_tx(xbar, row_bytes * M);
      const uint64_t keep = l2_policy_evict_last();
      for (int m = 0; m < M; ++m)
        bulk_g2s(xs + (size_t)m * p.x_rs, p.x + (size_t)m * p.ldx + k_lo, row_bytes, xbar, keep);
    }
    if (!__all_sync(0xffffffffu, mbar_wait_bounded(xbar, 0))) {
      if (lane == 0) {
        atomicCAS(p.error, 0, kErrFullWait);
        *abort_flag = 1;
      }
    }
  } else {
    stage_x_manual(p, xs, k_lo, krange, tid);
  }
  __syncthreads();
  if (p.rmsnorm) {
    rmsnorm_rows(p, xs, rms_r, red, tid);
    __syncthreads();
  }
  if (tid == 0) TRACE(2);

  // ---- stream: compute unit j while units j+1 .. j+D-1 are in flight
  using Math = typename std::conditional<MATH == kMathMma, MmaMath<P, WB>, FfmaMath<P, WB>>::type;
  Math math;
  math.zero();
  // Segment bookkeeping: this warp's units in the current virtual tile are
  // counted down (seg_left) instead of re-deriving the tile per unit.
  int vt = (u0 + warp) / kbpv;
  int kbl = (u0 + warp) - vt * kbpv;  // k-block (within vt) of the segment's first unit
  int seg_n = (kbpv - kbl + W - 1) / W;  // this warp's units in vt
  int seg_left = seg_n;
  int cur_j = vt - vt_first;
  // This lane's slice of the staged x: the prepack permutes k inside each
  // block so the B fragment is one 16 B (E4M3) or 8 B (FP16) load at
  // k-offset 8q (4q) of row g.  xoff: k offset of the warp's next unit.
  const __half* xlane = xs + (size_t)(g < M ? g : 0) * p.x_rs + (WB == 1 ? 8 * q : 4 * q);
  const __half* xq = xs + (WB == 1 ? 8 * q : 4 * q);  // row 0, for the FFMA variant
  int xoff = ((vt / p.n_tiles) * kbpv + kbl) * KPB - k_lo;
  const uint8_t* lp = wlane + D * WSTEP;  // address of unit j + D
  int loads_left = n_mine - D;

  auto flush = [&](int j) {
    float v[P][4];
    math.result(v, lane);
#pragma unroll
    for (int pl = 0; pl < P; ++pl)
      slots[((size_t)(j * W + warp) * P + pl) * 32 + lane] = make_float4(v[pl][0], v[pl][1], v[pl][2], v[pl][3]);
  };

  for (int j0 = 0; j0 < n_mine; j0 += D) {
#pragma unroll
    for (int d = 0; d < D; ++d) {
      if (j0 + d < n_mine) {
        uint4 xf = make_uint4(0, 0, 0, 0);
        if constexpr (MATH == kMathMma) {
          if (g < M) {
            if constexpr (WB == 1) {
              xf = lds128(xlane + xoff);
            } else {
              const uint2 t = lds64(xlane + xoff);
              xf.x = t.x;
              xf.y = t.y;
            }
          }
          math.unit(buf[d], xf);
        } else {
          math.unit(buf[d], xq + xoff, M, p.x_rs);
        }
        if (loads_left > 0) {
#pragma unroll
          for (int pl = 0; pl < P; ++pl) buf[d][pl] = ldg_stream(lp + pl * kUnitPlaneBytes, pol);
          lp += WSTEP;
        }
        --loads_left;
        xoff += W * KPB;
        if (--seg_left == 0) {
          // this warp's next virtual tile: unit vt*kbpv + kbl + seg_n*W
          flush(cur_j);
          math.zero();
          kbl += seg_n * W - kbpv;
          ++vt;
          while (kbl >= kbpv) {
            kbl -= kbpv;
            ++vt;
          }
          seg_n = (kbpv - kbl + W - 1) / W;
          seg_left = seg_n;
          cur_j = vt - vt_first;
          xoff = ((vt / p.n_tiles) * kbpv + kbl) * KPB - k_lo;
        }
      }
    }
  }
  if (n_mine > 0 && seg_left != seg_n) flush(cur_j);
  if (tid == 0) {
    TRACE(3);
    // Warm L2 with the start of the range the next kernel's CTA of the same
    // index will stream.
    if (p.pf_packed != nullptr && (int)blockIdx.x < p.pf_grid) {
      const long long a = (long long)blockIdx.x * p.pf_total_units / p.pf_grid;
      const long long b = (long long)(blockIdx.x + 1) * p.pf_total_units / p.pf_grid;
      const long long bytes = min((long long)p.pf_bytes, (b - a) * p.pf_unit_bytes);
      const uint8_t* src = p.pf_packed + a * p.pf_unit_bytes;
      for (long long off = 0; off < bytes; off += 32768)
        bulk_prefetch_l2(src + off, (uint32_t)min(32768LL, bytes - off));
    }
  }

  // ---- combine: the warps' partials in warp order, then finish each tile
  __syncthreads();
  if (*abort_flag) return;
  const int nvt = vt_last - vt_first + 1;
  for (int j = warp; j < nvt; j += W) {
    float v[P][4];
#pragma unroll
    for (int pl = 0; pl < P; ++pl) v[pl][0] = v[pl][1] = v[pl][2] = v[pl][3] = 0.f;
    for (int w = 0; w < W; ++w) {
#pragma unroll
      for (int pl = 0; pl < P; ++pl) {
        const float4 t = slots[((size_t)(j * W + w) * P + pl) * 32 + lane];
        v[pl][0] += t.x;
        v[pl][1] += t.y;
        v[pl][2] += t.z;
        v[pl][3] += t.w;
      }
    }
    finish_vt<P>(p, vt_first + j, v, lane);
  }
  if (tid == 0) TRACE(4);
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

#ifdef B2G_TRACE
extern "C" int b2g_debug_trace(unsigned long long* out, int n_ctas) {
  return (int)cudaMemcpyFromSymbol(out, g_trace, sizeof(unsigned long long) * 16 * n_ctas);
}

#endif

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
