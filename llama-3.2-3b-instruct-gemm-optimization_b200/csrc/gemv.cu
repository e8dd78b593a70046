// gemv.cu -- stream-K decode GEMV and the persistent decode-MLP stack for sm_100a.
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
//    evict-first) 16 (one plane) or 8 (two planes) units ahead: 128 KB in
//    flight per SM.  A phase's first loads are issued before its activations
//    exist (before the previous kernel is waited on, or before the stack
//    kernel's grid barrier), since weights are constant.
//  * The M <= 8 activation rows are staged once per phase in shared memory
//    with one round of 16 B loads.  RMSNorm is linear in x, so a fused norm
//    scales the accumulators by each row's factor in the epilogue; the factors
//    are summed from the staged rows while other warps finish streaming.  The
//    prepack permutes k inside each block so a lane's B fragment is one 16 B
//    (E4M3) or 8 B (FP16) shared load; the decode rows fill the n = 8 side of
//    mma.sync.m16n8k16 (x^T as B).  E4M3 is widened with cvt.rn.f16x2.e4m3x2.
//    A CUDA-core FFMA variant of the same loop (kMathFfma) exists for
//    comparison.
//  * Each warp's partial per virtual tile goes to a shared-memory slot.  After
//    the stream the slots are summed in warp order, and a tile split across
//    CTAs is summed in (k-range, CTA) order by the last CTA to arrive (one
//    counter per tile, reset by that CTA).  Deterministic; no float atomics
//    (the reference atomically adds into y_acc, gemv_fp8.cu:143-150), no
//    memset, no separate cast kernel.
//  * Epilogues: per-channel/tensor scale, fp16 rounding, SiLU(gate)*up for the
//    fused gate||up op, residual add.
//  * stack_kernel runs the layers of the decode MLP in one cooperative launch:
//    phases [RMSNorm + gate||up + SiLU*up] and [down + residual] per layer,
//    separated by bounded grid barriers, each phase's first weights already in
//    flight while the barrier and the activation staging complete.
#include <cstdio>
#include <type_traits>

#include "device.cuh"
#include "gemv.h"

namespace b2g {

__device__ int g_device_error;

#ifdef B2G_TRACE
// Per-CTA phase timestamps (%globaltimer), trace builds only.  g_tl: the
// single-op kernels' points 0 start, 1 past the dependency wait, 2 inputs
// staged, 3 weights streamed, 4 end, per launch slot (the host's launch
// count mod kTraceLaunches) and CTA; g_strace: 4 points per stack phase.
constexpr int kTracePts = 256;
constexpr int kTraceLaunches = 64;
constexpr int kTraceCtas = 160;
__device__ unsigned long long g_tl[kTraceLaunches][kTraceCtas][8];
__device__ unsigned long long g_strace[160][kTracePts];
#define TRACE(i) \
  do { \
    if (blockIdx.x < kTraceCtas) g_tl[p.trace_slot % kTraceLaunches][blockIdx.x][(i)] = globaltimer_ns(); \
  } while (0)
#define STRACE(i) \
  do { if ((i) >= 0 && (i) < kTracePts && blockIdx.x < 160) g_strace[blockIdx.x][(i)] = globaltimer_ns(); } while (0)
#else
#define TRACE(i) do { } while (0)
#define STRACE(i) do { } while (0)
#endif

int* device_error_word() {
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_device_error) != cudaSuccess) return nullptr;
  return static_cast<int*>(p);
}

namespace {

constexpr int W = kWarps;
constexpr int NT = kThreads;

// The buffers one GEMV phase reads and writes.
struct Io {
  const uint8_t* packed;
  const void* scales;
  const __half* x;
  long long ldx;
  const __half* residual;
  long long ldr;
  __half* y;
  long long ldy;
};

__device__ __forceinline__ Io io_of_params(const GemvParams& p) {
  return Io{p.packed, p.scales, p.x, p.ldx, p.residual, p.ldr, p.y, p.ldy};
}

// x / d for 0 <= x < 2^31 with the host-computed constants of d (FastDiv).
__device__ __forceinline__ int fdiv(int x, const FastDiv& f) {
  return (int)((__umulhi((uint32_t)x, f.mul) + (uint32_t)x) >> f.shift);
}

// The partition: CTA c streams granules [c*Tg/G, (c+1)*Tg/G) of gran units
// each (Tg = total_gran); cta_of(u) is the CTA whose range holds unit u.
// All operands stay below 2^31 (host-checked).
__device__ __forceinline__ int cta_of(const GemvParams& p, int u) {
  const int gi = fdiv(u, p.div_gran);
  return fdiv((gi + 1) * p.grid + p.total_gran - 1, p.div_tg) - 1;
}

// First unit of CTA c's range.
__device__ __forceinline__ int range_start(const GemvParams& p, int c) {
  return fdiv(c * p.total_gran, p.div_grid) * p.gran;
}

__device__ __forceinline__ float channel_scale(const GemvParams& p, const Io& io, int plane, int n) {
  switch (p.scale_mode) {
    case 1:
      return __half2float(reinterpret_cast<const __half*>(io.scales)[plane]);
    case 2:
      return __half2float(reinterpret_cast<const __half*>(io.scales)[(size_t)plane * p.N + n]);
    case 3:
      return reinterpret_cast<const float*>(io.scales)[(size_t)plane * p.N + n];
    default:
      return 1.0f;
  }
}

__device__ __forceinline__ float2 h2_to_f2(uint32_t v) {
  __half2 h;
  *reinterpret_cast<uint32_t*>(&h) = v;
  return __half22float2(h);
}

// Lane layout of a finished tile (the m16n8 accumulator): entry i of lane
// (g = lane/4, q = lane%4) is channel g + 8*(i/2), token 2q + (i%2).
// Per-slot epilogue inputs in shared memory, loaded with the activations:
// the scales of the slot's 16 channels (per plane) and, for a residual op,
// the residual rows.  Slot j is the CTA's j-th virtual tile.
struct Epi {
  float* scale;  // [n_slots][P][16]
  __half* res;   // [n_slots][8][16], as stored in memory
};

__device__ __forceinline__ Epi epi_of(const GemvParams& p, uint8_t* smem, int P) {
  float* base = reinterpret_cast<float*>(smem + p.off_epi);
  return Epi{base, reinterpret_cast<__half*>(base + p.n_slots * P * 16)};
}

// The scales of the CTA's tiles (constants: may load before the previous
// kernel is waited on).  ASYNC: FP32 per-channel scales go global -> shared
// with cp.async, so no thread stalls on them before the dependency wait (a
// load issued behind the start of the L2 prefetch waits microseconds); the
// caller completes them (cp_async_wait_all) before the epilogue reads them.
template <int P, bool ASYNC = false>
__device__ __forceinline__ void load_scales(const GemvParams& p, const Io& io, const Epi& e, int vt_first, int nvt,
                                            int tid) {
  const int ns = nvt * P * 16;
  for (int i = tid; i < ns; i += NT) {
    const int j = i / (P * 16), pl = (i / 16) % P, c = i % 16;
    const int tile = fdiv(vt_first + j, p.div_tiles);
    const int n = (vt_first + j - tile * p.n_tiles) * kTileCh + c;
    if (ASYNC && p.scale_mode == 3 && n < p.N)
      cp_async4(e.scale + i, reinterpret_cast<const float*>(io.scales) + (size_t)pl * p.N + n);
    else
      e.scale[i] = n < p.N ? channel_scale(p, io, pl, n) : 0.f;
  }
}

// The residual rows of the CTA's tiles (written by an earlier kernel or phase).
template <int P>
__device__ __forceinline__ void load_residual(const GemvParams& p, const Io& io, const Epi& e, int vt_first,
                                              int nvt, int tid) {
  if (P == 1 && p.residual_add) {
    const int nr = nvt * 8 * 16;
    for (int i = tid; i < nr; i += NT) {
      const int j = i / 128, m = (i / 16) % 8, c = i % 16;
      const int vt = vt_first + j;
      const int n = (vt - fdiv(vt, p.div_tiles) * p.n_tiles) * kTileCh + c;
      e.res[i] = (m < p.M && n < p.N) ? __ldcg(io.residual + (size_t)m * io.ldr + n) : __float2half(0.f);
    }
  }
}

// The same rows without stalling a thread: 16-byte pieces (8 channels of one
// row of a tile) global -> shared with cp.async, issued before the
// activations are staged so that the two round trips overlap; a piece that
// would cross N goes element by element.  Rows are 16-byte aligned (lean
// flavor, host-checked); the caller completes the copies before the epilogue.
template <int P>
__device__ __forceinline__ void load_residual_async(const GemvParams& p, const Io& io, const Epi& e, int vt_first,
                                                    int nvt, int tid) {
  if (P == 1 && p.residual_add) {
    const int np = nvt * p.M * 2;
    for (int i = tid; i < np; i += NT) {
      const int j = i / (p.M * 2), r = i - j * (p.M * 2), m = r >> 1, h = r & 1;
      const int vt = vt_first + j;
      const int n0 = (vt - fdiv(vt, p.div_tiles) * p.n_tiles) * kTileCh + h * 8;
      __half* dst = e.res + (j * 8 + m) * 16 + h * 8;
      const __half* src = io.residual + (size_t)m * io.ldr + n0;
      if (n0 + 8 <= p.N) {
        cp_async16(dst, src);
      } else {
        for (int c = 0; c < 8; ++c) dst[c] = n0 + c < p.N ? __ldcg(src + c) : __float2half(0.f);
      }
    }
  }
}

template <int P>
__device__ __forceinline__ void load_epi(const GemvParams& p, const Io& io, const Epi& e, int vt_first, int nvt,
                                         int tid) {
  const int ns = nvt * P * 16;
  for (int i = tid; i < ns; i += NT) {
    const int j = i / (P * 16), pl = (i / 16) % P, c = i % 16;
    const int tile = fdiv(vt_first + j, p.div_tiles);
    const int n = (vt_first + j - tile * p.n_tiles) * kTileCh + c;
    e.scale[i] = n < p.N ? channel_scale(p, io, pl, n) : 0.f;
  }
  if (P == 1 && p.residual_add) {
    const int nr = nvt * 8 * 16;
    for (int i = tid; i < nr; i += NT) {
      const int j = i / 128, m = (i / 16) % 8, c = i % 16;
      const int vt = vt_first + j;
      const int n = (vt - fdiv(vt, p.div_tiles) * p.n_tiles) * kTileCh + c;
      e.res[i] = (m < p.M && n < p.N) ? __ldcg(io.residual + (size_t)m * io.ldr + n) : __float2half(0.f);
    }
  }
}

// RMSNorm factor of row m from the per-warp sums of squares (see stage_x).
__device__ __forceinline__ float rms_of(const GemvParams& p, const float* red, int m) {
  float s = 0.f;
#pragma unroll
  for (int w = 0; w < W; ++w) s += red[w * 8 + m];
  return rsqrtf(s / (float)p.K + p.rms_eps);
}

// REDUCE: this launch's exchange round (this CTA's previous count, staged
// in shared memory by thread 0, plus one).
__device__ __forceinline__ unsigned tp_round() {
  extern __shared__ __align__(1024) uint8_t dyn_smem[];
  return *reinterpret_cast<volatile unsigned*>(dyn_smem + kOffRound) + 1u;
}

// REDUCE: a finished tile's rows (in the warp's stage) as flag-in-data
// words (round << 32 | two channels) into this rank's slot of every other
// rank's inbox (peer stores over NVLink); the rows stay in the stage for
// this rank's own share of the sum.
__device__ __noinline__ void tp_reduce_push(const GemvParams& p, const __half* stage, int tile, int lane) {
  const unsigned long long flag = (unsigned long long)tp_round() << 32;
  const int half_w = p.tp.width / 2;
  for (int w = lane; w < p.M * 8; w += 32) {
    const int m = w >> 3, i = w & 7;
    const unsigned long long word = flag | *reinterpret_cast<const uint32_t*>(stage + m * 16 + 2 * i);
    const size_t off = (((size_t)p.tp.buf * p.tp.world + p.tp.rank) * p.tp.inbox_m + m) * half_w + tile * 8 + i;
    for (int r = 0; r < p.tp.world; ++r)
      if (r != p.tp.rank) st_relaxed_sys_u64(reinterpret_cast<unsigned long long*>(p.tp.inbox[r]) + off, word);
  }
}

// red: RMSNorm partial sums (nullptr when the op has no RMSNorm); the
// normalisation is linear, so it scales the accumulator: y = fp16(acc * r_m * s_n).
// stage: 256 B of this warp's own shared memory, for PUSH rows.  TPX: the
// launch may exchange rows with other ranks (the TP code is compiled only
// into those kernels).
template <int P, bool TPX>
__device__ __forceinline__ void epilogue(const GemvParams& p, const Io& io, int j, int tile, const float (&v)[P][4],
                                         int lane, const float* red, const Epi& e, __half* stage, bool write) {
  if (!write) return;  // a tensor-parallel gather whose wait expired: rows void, nothing written
  const int g = lane >> 2, q = lane & 3;
  // this lane's two token rows, 2q and 2q + 1
  const float r0 = (red && 2 * q < p.M) ? rms_of(p, red, 2 * q) : 1.0f;
  const float r1 = (red && 2 * q + 1 < p.M) ? rms_of(p, red, 2 * q + 1) : 1.0f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int m = 2 * q + (i & 1);
    const int c = g + 8 * (i >> 1);
    const int n = tile * kTileCh + c;
    if (m < p.M && n < p.N) {
      const float r = (i & 1) ? r1 : r0;
      __half out;
      if constexpr (P == 1) {
        out = __float2half_rn(v[0][i] * r * e.scale[j * 16 + c]);
        if (p.residual_add) out = __float2half_rn(__half2float(e.res[(j * 8 + m) * 16 + c]) + __half2float(out));
      } else {
        const float gf = __half2float(__float2half_rn(v[0][i] * r * e.scale[(j * 2) * 16 + c]));
        const float uf = __half2float(__float2half_rn(v[1][i] * r * e.scale[(j * 2 + 1) * 16 + c]));
        out = __float2half_rn(gf / (1.0f + __expf(-gf)) * uf);
      }
      if (TPX && P == 1 && tp_pushes(p.tp.mode))
        stage[m * 16 + c] = out;
      else
        io.y[(size_t)m * io.ldy + n] = out;
    }
  }
  if (TPX && P == 1 && p.tp.mode == kTpReduce) {
    __syncwarp();
    tp_reduce_push(p, stage, tile, lane);
  }
  if (TPX && P == 1 && p.tp.mode == kTpPush) {
    // The tile's rows are 32 B each: two lanes per row store 16 B into this
    // rank's slot of every rank's inbox (peer stores over NVLink).
    __syncwarp();
    if (lane < 2 * p.M) {
      const int m = lane >> 1, h = lane & 1;
      const uint4 v16 = lds128(stage + m * 16 + h * 8);
      const size_t off =
          (((size_t)p.tp.buf * p.tp.world + p.tp.rank) * p.tp.inbox_m + m) * p.tp.width + tile * kTileCh + h * 8;
      for (int r = 0; r < p.tp.world; ++r) *reinterpret_cast<uint4*>(p.tp.inbox[r] + off) = v16;
    }
  }
}

// A virtual tile's CTA-level sum is complete in v: finish it here if this CTA
// is the tile's only contributor, else publish it and let the last
// contributing CTA sum all partials in (k-range, CTA) order.
// SPLIT: the plan may share a virtual tile between CTAs (else every tile has
// one contributor and the handshake code is not compiled in).
template <int P, bool TPX, bool SPLIT = true>
__device__ __forceinline__ void finish_vt(const GemvParams& p, const Io& io, int vt, int j, const float (&v)[P][4],
                                          int lane, const float* red, const Epi& e, __half* stage,
                                          bool write = true) {
  const int ks = fdiv(vt, p.div_tiles);
  const int tile = vt - ks * p.n_tiles;
  // Contributors of k-range k: CTAs cta_of(a_k) .. cta_of(a_k + kbpv - 1).
  auto first_of = [&](int k) { return cta_of(p, (k * p.n_tiles + tile) * p.kbpv); };
  auto count_of = [&](int k) {
    const int a = (k * p.n_tiles + tile) * p.kbpv;
    return cta_of(p, a + p.kbpv - 1) - cta_of(p, a) + 1;
  };
  int total = 1;
  if constexpr (SPLIT) {
    total = 0;
#pragma unroll 1
    for (int k = 0; k < p.ksplit; ++k) total += count_of(k);
  }
  float s[P][4];
#pragma unroll
  for (int pl = 0; pl < P; ++pl)
#pragma unroll
    for (int i = 0; i < 4; ++i) s[pl][i] = v[pl][i];
  if (total > 1) {
    float4* parts = reinterpret_cast<float4*>(p.partials);
    auto src = [&](int k, int c) {
      return parts + ((size_t)(k * p.n_tiles + tile) * p.max_contrib + c) * P * 32 + lane;
    };
    float4* dst = src(ks, blockIdx.x - first_of(ks));
#pragma unroll
    for (int pl = 0; pl < P; ++pl) __stcg(dst + pl * 32, make_float4(v[pl][0], v[pl][1], v[pl][2], v[pl][3]));
    __syncwarp();
    int old = 0;
    if (lane == 0) old = atom_add_acq_rel_gpu(&p.counters[tile], 1);
    old = __shfl_sync(0xffffffffu, old, 0);
    if (old != total - 1) return;
    fence_acq_rel_gpu();
    // Last to arrive: sum every partial in (k-range, CTA) order, B per round trip.
    constexpr int B = (P == 1) ? 8 : 4;
#pragma unroll
    for (int pl = 0; pl < P; ++pl) s[pl][0] = s[pl][1] = s[pl][2] = s[pl][3] = 0.f;
    int k = 0, c = 0, n = count_of(0);
#pragma unroll 1
    for (int base = 0; base < total; base += B) {
      float4 t[B][P];
#pragma unroll
      for (int b = 0; b < B; ++b) {
        const bool have = base + b < total;
#pragma unroll
        for (int pl = 0; pl < P; ++pl) t[b][pl] = have ? __ldcg(src(k, c) + pl * 32) : make_float4(0.f, 0.f, 0.f, 0.f);
        if (have && ++c == n) {
          ++k;
          c = 0;
          n = k < p.ksplit ? count_of(k) : 0;
        }
      }
#pragma unroll
      for (int b = 0; b < B; ++b)
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
    if (lane == 0) p.counters[tile] = 0;
  }
  epilogue<P, TPX>(p, io, j, tile, s, lane, red, e, stage, write);
}

// Sum of squares of 8 halves, in one fixed order (stage_x and gather_x share
// it, so the plain and the all-reduced staging give bitwise the same norm).
__device__ __forceinline__ float sumsq8(const uint4& v) {
  const float2 a = h2_to_f2(v.x), b = h2_to_f2(v.y), c = h2_to_f2(v.z), d = h2_to_f2(v.w);
  float t = a.x * a.x;
  t = fmaf(a.y, a.y, t); t = fmaf(b.x, b.x, t); t = fmaf(b.y, b.y, t);
  t = fmaf(c.x, c.x, t); t = fmaf(c.y, c.y, t); t = fmaf(d.x, d.x, t); t = fmaf(d.y, d.y, t);
  return t;
}

// Per-thread row sums -> red[warp][m] (shuffle tree over the warp).
__device__ __forceinline__ void reduce_rows(float (&ss)[8], int tid, float* red) {
  const int lane = tid & 31, warp = tid >> 5;
#pragma unroll
  for (int off = 16; off; off >>= 1)
#pragma unroll
    for (int m = 0; m < 8; ++m) ss[m] += __shfl_xor_sync(0xffffffffu, ss[m], off);
  if (lane < 8) {
    float t = ss[0];
#pragma unroll
    for (int m = 1; m < 8; ++m) t = lane == m ? ss[m] : t;
    red[warp * 8 + lane] = t;
  }
}

// ---------------------------------------------------------------------------
// Activation rows in shared memory: row m at xs + m * x_rs (halves), holding
// k in [k_lo, k_lo + krange), zero beyond K.  All threads load 16 B pieces,
// up to 8 each in flight (M = 8 rows of 3072 halves is one round).  L2 loads
// (ld.cg): x may have been written by another CTA of the same launch.
// ---------------------------------------------------------------------------
// With `red` non-null (RMSNorm ops, whole rows staged) the loaded values also
// give each row's sum of squares: every thread sums its own chunks, each warp
// reduces across its lanes and writes red[warp * 8 + m]; rms_of() adds the
// warps in order (deterministic).
// VEC_ONLY: the host has checked that every row piece is 16-byte aligned and
// inside K (the element path is then not compiled in).
template <bool VEC_ONLY = false>
__device__ void stage_x(const GemvParams& p, const Io& io, __half* xs, int k_lo, int krange, int tid,
                        float* red) {
  const int M = p.M, K = p.K;
  const int nch = krange / 8;
  const bool vec =
      VEC_ONLY || (((reinterpret_cast<uintptr_t>(io.x) & 15) == 0) && ((io.ldx & 7) == 0) && k_lo + krange <= K);
  float ss[8];
#pragma unroll
  for (int m = 0; m < 8; ++m) ss[m] = 0.f;
  if (vec) {
    // Chunk c of every row per thread: up to 8 loads in flight, no index division.
#pragma unroll 1
    for (int c = tid; c < nch; c += NT) {
      uint4 v[8];
#pragma unroll
      for (int m = 0; m < 8; ++m)
        if (m < M) v[m] = __ldcg(reinterpret_cast<const uint4*>(io.x + (size_t)m * io.ldx + k_lo + c * 8));
#pragma unroll
      for (int m = 0; m < 8; ++m)
        if (m < M) {
          sts128(xs + (size_t)m * p.x_rs + c * 8, v[m]);
          if (red) ss[m] += sumsq8(v[m]);
        }
    }
  } else {
    // Unaligned rows or a range past K: element loads, zero past K.
#pragma unroll
    for (int m = 0; m < 8; ++m) {
      if (m < M) {
        const __half* row = io.x + (size_t)m * io.ldx;
#pragma unroll 1
        for (int k = k_lo + tid; k < k_lo + krange; k += NT) {
          const __half v = k < K ? __ldcg(row + k) : __float2half(0.f);
          xs[(size_t)m * p.x_rs + (k - k_lo)] = v;
          const float f = __half2float(v);
          ss[m] = fmaf(f, f, ss[m]);
        }
      }
    }
  }
  if (red) reduce_rows(ss, tid, red);
}

// Bounded wait (thread 0) until this rank's arrival counters all reach
// epoch * push_grid: every rank's pushing launch of this round has finished
// its stores.  Counters only grow; the comparison tolerates wrap-around.
__device__ __forceinline__ bool tp_wait_arrivals(const TpParams& tp, int* err) {
  if (*reinterpret_cast<volatile int*>(err) != 0) return false;  // an earlier wait failed: fail fast
  const unsigned target = *reinterpret_cast<volatile unsigned*>(tp.epoch) * (unsigned)tp.push_grid;
  const unsigned* cnt = tp.counters[tp.rank];
  const unsigned long long t0 = globaltimer_ns();
  for (int r = 0; r < tp.world; ++r) {
    while ((int)(ld_acquire_sys(cnt + r) - target) < 0) {
      if (globaltimer_ns() - t0 > kWaitBudgetNs) {
        atomicCAS(err, 0, kErrPeerWait);
        return false;
      }
      __nanosleep(64);
    }
  }
  return true;
}

// Slot r of buffer buf at row m, halves [k0, k0 + 8).
__device__ __forceinline__ const uint4* tp_slot(const TpParams& tp, int r, int m, int k0) {
  const size_t slot = (size_t)tp.inbox_m * tp.width;
  return reinterpret_cast<const uint4*>(tp.inbox[tp.rank] + ((size_t)tp.buf * tp.world + r) * slot +
                                        (size_t)m * tp.width + k0);
}

__device__ __forceinline__ void add8(float (&a)[8], const uint4& v) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 f = h2_to_f2(w[j]);
    a[2 * j] += f.x;
    a[2 * j + 1] += f.y;
  }
}

__device__ __forceinline__ uint4 round8(const float (&a)[8]) {
  uint32_t o[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    __half2 h = __floats2half2_rn(a[2 * j], a[2 * j + 1]);
    o[j] = *reinterpret_cast<uint32_t*>(&h);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// Sum of inbox slots 0..world-1 at row m, halves [k0, k0 + 8), in rank order
// in fp32, rounded once to fp16.
__device__ __forceinline__ uint4 tp_sum8(const TpParams& tp, int m, int k0) {
  float a[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) a[j] = 0.f;
  for (int r = 0; r < tp.world; ++r) add8(a, __ldcg(tp_slot(tp, r, m, k0)));
  return round8(a);
}

// GATHER staging: x = the all-reduced rows, written to tp.h_out as well (each
// CTA writes the chunks c with c % grid == its index).  Same thread -> chunk
// assignment, layout and sums of squares as stage_x (so the norm is bitwise
// the plain path's); rows are whole (k_lo = 0, host-checked).  Rows go in
// batches of 4, every rank's slot load of a batch issued before its sums.
template <class Sync>
__device__ void gather_x(const GemvParams& p, __half* xs, int krange, int tid, float* red, volatile int* verdict,
                         Sync sync) {
  const int M = p.M;
  if (tid == 0) *verdict = tp_wait_arrivals(p.tp, p.error) ? 1 : 0;
  sync();
  const bool ok = *verdict != 0;  // false: the wait expired; h_out is left as it was
  const int nch = krange / 8;
  constexpr int B = 4;
  float ss[8];
#pragma unroll
  for (int m = 0; m < 8; ++m) ss[m] = 0.f;
#pragma unroll 1
  for (int c = tid; c < nch; c += NT) {
#pragma unroll
    for (int m0 = 0; m0 < 8; m0 += B) {
      if (m0 < M) {
        float a[B][8];
#pragma unroll
        for (int b = 0; b < B; ++b)
#pragma unroll
          for (int j = 0; j < 8; ++j) a[b][j] = 0.f;
#pragma unroll
        for (int r = 0; r < kMaxTp; ++r) {
          if (r < p.tp.world) {
            uint4 v[B];
#pragma unroll
            for (int b = 0; b < B; ++b)
              if (m0 + b < M) v[b] = __ldcg(tp_slot(p.tp, r, m0 + b, c * 8));
#pragma unroll
            for (int b = 0; b < B; ++b)
              if (m0 + b < M) add8(a[b], v[b]);
          }
        }
#pragma unroll
        for (int b = 0; b < B; ++b) {
          const int m = m0 + b;
          if (m < M) {
            const uint4 v = round8(a[b]);
            sts128(xs + (size_t)m * p.x_rs + c * 8, v);
            if (ok && c % p.grid == (int)blockIdx.x)
              *reinterpret_cast<uint4*>(p.tp.h_out + (size_t)m * p.tp.ldh + c * 8) = v;
            if (red) ss[m] += sumsq8(v);
          }
        }
      }
    }
  }
  if (red) reduce_rows(ss, tid, red);
}

// REDUCE tail (after every tile's epilogue; the CTA synchronised): the CTA
// reads the words of its own tiles from the other ranks' slots of buffer
// `buf` in its inbox, polling each (bounded) until it carries this launch's
// round, and adds this rank's rows from the tiles' stages in rank order
// (fp32 from 0, one fp16 rounding: the order tp_sum8 uses, so every rank
// gets bitwise the same rows).  A CTA one of whose polls expires, or that
// finds the error word set, writes none of its rows.  Tiles are whole (one
// contributor each, K not split: host-checked), so tile j of the CTA's range
// was finished by this CTA and its rows are in slot j's stage.
__device__ __noinline__ void tp_reduce_tail(const GemvParams& p, uint8_t* smem, int tid) {
  const unsigned v = tp_round();
  const int u0 = range_start(p, blockIdx.x), u1 = range_start(p, blockIdx.x + 1);
  const int t0 = fdiv(u0, p.div_kbpv);
  const int nt = u1 > u0 ? fdiv(u1 - 1, p.div_kbpv) - t0 + 1 : 0;
  const int per_tile = p.M * 8;  // 4-byte words (two channels) per tile
  const int half_w = p.tp.width / 2;
  bool expired = false;
  float a0 = 0.f, a1 = 0.f;
  int j = 0, m = 0, i = 0;
  if (tid < nt * per_tile) {  // nt <= kMaxSlots, so at most kThreads words
    j = tid / per_tile;
    const int rem = tid - j * per_tile;
    m = rem >> 3;
    i = rem & 7;
    const uint32_t own = *reinterpret_cast<const uint32_t*>(
        reinterpret_cast<const __half*>(smem + kOffSlots + (size_t)j * kWarps * kUnitPlaneBytes) + m * 16 + 2 * i);
    const unsigned long long* box = reinterpret_cast<const unsigned long long*>(p.tp.inbox[p.tp.rank]) +
                                    (size_t)m * half_w + (t0 + j) * 8 + i;
    unsigned long long t_start = 0;
    for (int r = 0; r < p.tp.world && !expired; ++r) {
      uint32_t d = own;
      if (r != p.tp.rank) {
        const unsigned long long* src = box + ((size_t)p.tp.buf * p.tp.world + r) * p.tp.inbox_m * half_w;
        unsigned long long w = ld_relaxed_sys_u64(src);
        while ((unsigned)(w >> 32) != v) {
          if (t_start == 0) t_start = globaltimer_ns();
          if (*reinterpret_cast<volatile int*>(p.error) != 0 || globaltimer_ns() - t_start > kWaitBudgetNs) {
            expired = true;
            break;
          }
          __nanosleep(32);
          w = ld_relaxed_sys_u64(src);
        }
        d = (uint32_t)w;
      }
      const float2 f = h2_to_f2(d);
      a0 += f.x;
      a1 += f.y;
    }
  }
  if (__syncthreads_or(expired)) {
    if (tid == 0) atomicCAS(p.error, 0, kErrPeerWait);
  } else if (tid < nt * per_tile) {
    *reinterpret_cast<__half2*>(p.y + (size_t)m * p.ldy + (t0 + j) * kTileCh + 2 * i) = __floats2half2_rn(a0, a1);
  }
  if (tid == 0) {
    volatile unsigned* rc = p.tp.rounds;
    rc[blockIdx.x] = v;
    if (blockIdx.x == 0)
      for (int c = p.grid; c < kTpMaxCtas; ++c) rc[c] = v;  // every entry advances, whatever the grid
  }
}

// REDUCE: thread 0 completes the copy of the CTA's round count into shared
// memory (issued after the dependency wait) before the combine phase.
struct RoundHook {
  template <class T>
  __device__ __forceinline__ void operator()(T&) const {
    if (threadIdx.x == 0) cp_async_wait_all();
  }
};

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
  // w: this lane's A fragments (one uint4 per plane); xf: its B fragment
  // (b0..b3 for E4M3, two k16 steps; b0, b1 for FP16).
  __device__ __forceinline__ void unit(const uint4* w, const uint4& xf) {
#pragma unroll
    for (int pl = 0; pl < P; ++pl) {
      const uint4 a = w[pl];
      if constexpr (WB == 1) {
        uint32_t h0, h1, h2, h3;
        e4m3x4_to_f16x2x2(a.x, h0, h1);
        e4m3x4_to_f16x2x2(a.y, h2, h3);
        mma_16816(acc[pl], h0, h1, h2, h3, xf.x, xf.y);
        e4m3x4_to_f16x2x2(a.z, h0, h1);
        e4m3x4_to_f16x2x2(a.w, h2, h3);
        mma_16816(acc[pl], h0, h1, h2, h3, xf.z, xf.w);
      } else {
        mma_16816(acc[pl], a.x, a.y, a.z, a.w, xf.x, xf.y);
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
  __device__ __forceinline__ void unit(const uint4* w, const __half* xk, int M, int rs) {
    constexpr int S = (WB == 1) ? 2 : 1;  // k16 steps per unit
    float2 wf[P][S][4];                   // [plane][step][register r]
#pragma unroll
    for (int pl = 0; pl < P; ++pl) {
      const uint4 a = w[pl];
      if constexpr (WB == 1) {
        const uint32_t ws[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
        for (int s = 0; s < 2; ++s)
#pragma unroll
          for (int r = 0; r < 4; ++r) {
            const uint32_t word = ws[s * 2 + (r >> 1)];
            wf[pl][s][r] = h2_to_f2(e4m3x2_to_f16x2((r & 1) ? (word >> 16) : word));
          }
      } else {
        wf[pl][0][0] = h2_to_f2(a.x);
        wf[pl][0][1] = h2_to_f2(a.y);
        wf[pl][0][2] = h2_to_f2(a.z);
        wf[pl][0][3] = h2_to_f2(a.w);
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
// Phase pieces.  A phase is one GEMV over this CTA's range of the stream.
// The ring holds R uint4 per lane: unit d of the warp's next D = R / P units
// in ring[d*P .. d*P + P - 1].
// ---------------------------------------------------------------------------
struct Range {
  int u0, u1, n_mine;  // CTA's units [u0, u1); this warp's count (units u0 + warp + j*W)
};

__device__ __forceinline__ Range cta_range(const GemvParams& p, int warp) {
  Range r;
  if ((int)blockIdx.x >= p.grid) {  // a launch wider than this phase's plan
    r.u0 = r.u1 = r.n_mine = 0;
    return r;
  }
  r.u0 = range_start(p, blockIdx.x);
  r.u1 = range_start(p, blockIdx.x + 1);
  const int n = r.u1 - r.u0;
  r.n_mine = n > warp ? (n - warp + W - 1) / W : 0;
  return r;
}

// Issue the loads of units [D0, D1) of this warp's first D units of a phase
// into their ring slots.  Every entry in the range is written (zero past the
// warp's units), so the compiler sees the old contents die here and does not
// keep them live across a phase's combine.
template <int P, int R, int D0 = 0, int D1 = R / P>
__device__ __forceinline__ void prefetch_phase(const GemvParams& p, const uint8_t* packed,
                                               uint4 (&ring)[R], int warp, int lane, uint64_t pol) {
  constexpr int UNIT = P * kUnitPlaneBytes;
  constexpr size_t WSTEP = (size_t)W * UNIT;
  const Range r = cta_range(p, warp);
  const uint8_t* wl = packed + ((size_t)r.u0 + warp) * UNIT + lane * 16;
#pragma unroll
  for (int d = D0; d < D1; ++d) {
#pragma unroll
    for (int pl = 0; pl < P; ++pl)
      ring[d * P + pl] = d < r.n_mine ? ldg_stream(wl + d * WSTEP + pl * kUnitPlaneBytes, pol)
                                      : make_uint4(0, 0, 0, 0);
  }
}

// Warm L2 with the first `bytes` of this CTA's range of a phase (one thread
// issues bulk prefetches; no registers, no completion to wait for).
__device__ __forceinline__ void l2_prefetch_phase(const GemvParams& p, const uint8_t* packed, int unit_bytes,
                                                  long long bytes) {
  if (threadIdx.x != 0 || (int)blockIdx.x >= p.grid) return;
  const long long a = range_start(p, blockIdx.x);
  const long long b = range_start(p, blockIdx.x + 1);
  bytes = min(bytes, (b - a) * unit_bytes);
  const uint8_t* src = packed + a * unit_bytes;
  for (long long off = 0; off < bytes; off += 32768)
    bulk_prefetch_l2(src + off, (uint32_t)min(32768LL, bytes - off));
}

// One phase with the ring pre-filled by prefetch_phase: stage x (and
// RMSNorm it), stream the rest of the range, leave each warp's partial per
// virtual tile in a shared slot, run after_stream(ring) (the ring is idle
// then: e.g. prefetch the next phase), then combine and finish the tiles.
// Entry requires every thread of the CTA to be past its last read of the
// shared slots and x rows of any earlier phase.
struct NoHook {
  template <class T>
  __device__ __forceinline__ void operator()(T&) const {}
};

// SCALES_LOADED: the caller loaded the tiles' scales already (before the
// dependency wait); the phase loads only the residual rows.
// LEAN: whole virtual tiles per CTA and aligned activation rows (the
// host-checked common case: no split-tile handshake, vector staging only).
// TP: the PUSH epilogue is compiled in; GATHERX: the GATHER staging is.
template <int P, int WB, int MATH, int R, class AfterStream, bool TP, bool SCALES_LOADED = false, bool LEAN = false,
          bool GATHERX = TP>
__device__ __forceinline__ void run_phase(const GemvParams& p, const Io& io, uint8_t* smem,
                                          uint4 (&ring)[R], uint64_t pol, AfterStream after_stream,
                                          int trace_base = -1) {
  constexpr int D = R / P;
  constexpr int UNIT = P * kUnitPlaneBytes;
  constexpr size_t WSTEP = (size_t)W * UNIT;
  constexpr int KPB = (WB == 1) ? 32 : 16;  // k per k-block
  float* red = reinterpret_cast<float*>(smem + kOffRed);  // RMSNorm sums of squares [W][8]
  const Epi epi = epi_of(p, smem, P);
  float4* slots = reinterpret_cast<float4*>(smem + kOffSlots);  // [n_slots][W][P][32]
  __half* xs = reinterpret_cast<__half*>(smem + p.off_x);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, q = lane & 3;
  const int M = p.M, kbpv = p.kbpv;
  const Range r = cta_range(p, warp);
  const int u0 = r.u0, n_mine = r.n_mine;
  const bool active = r.u1 > r.u0;
  const int vt_first = fdiv(u0, p.div_kbpv);
  const int vt_last = active ? fdiv(r.u1 - 1, p.div_kbpv) : vt_first - 1;
  const int ks_first = fdiv(vt_first, p.div_tiles);
  const int k_lo = ks_first * kbpv * KPB;
  const int krange = active ? (fdiv(vt_last, p.div_tiles) + 1 - ks_first) * kbpv * KPB : 0;

  // ---- activations
  if (tid == 0) STRACE(trace_base);
  const bool gather = GATHERX && p.tp.mode == kTpGather;
  if (gather) {
    // every CTA takes part (the wait and the write-back of the reduced rows)
    gather_x(p, xs, active ? krange : p.K / 8 * 8, tid, p.rmsnorm ? red : nullptr,
             reinterpret_cast<volatile int*>(smem + kOffMisc), [] { __syncthreads(); });
  }
  if (active) {
    if (LEAN && SCALES_LOADED) load_residual_async<P>(p, io, epi, vt_first, vt_last - vt_first + 1, tid);
    if (!gather) stage_x<LEAN>(p, io, xs, k_lo, krange, tid, p.rmsnorm ? red : nullptr);
    if (!SCALES_LOADED)
      load_epi<P>(p, io, epi, vt_first, vt_last - vt_first + 1, tid);
    else if (!LEAN)
      load_residual<P>(p, io, epi, vt_first, vt_last - vt_first + 1, tid);
  }
  for (int i = tid; i < p.n_slots * W * P * 32; i += NT) slots[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  __syncthreads();
  if (threadIdx.x == 0) {
    TRACE(2);
    STRACE(trace_base + 1);
  }

  // ---- stream: compute unit j while units j+1 .. j+D-1 are in flight
  using Math = typename std::conditional<MATH == kMathMma, MmaMath<P, WB>, FfmaMath<P, WB>>::type;
  Math math;
  math.zero();
  // Segment bookkeeping: this warp's units in the current virtual tile are
  // counted down; the tile is re-derived only at a segment end.
  int vt = fdiv(u0 + warp, p.div_kbpv);
  int kbl = (u0 + warp) - vt * kbpv;     // k-block (within vt) of the segment's first unit
  int seg_n = (kbpv - kbl + W - 1) / W;  // this warp's units in vt
  int seg_left = seg_n;
  int cur_j = vt - vt_first;
  // This lane's B fragment: row g of the staged x at k-offset 8q (E4M3) or
  // 4q (FP16) of each block (the prepack's k permutation).  Rows g >= M read
  // row 0: those token columns are computed but never stored.
  const __half* xlane = xs + (size_t)(g < M ? g : 0) * p.x_rs + (WB == 1 ? 8 * q : 4 * q);
  const __half* xq = xs + (WB == 1 ? 8 * q : 4 * q);  // row 0, for the FFMA variant
  int xoff = (fdiv(vt, p.div_tiles) * kbpv + kbl) * KPB - k_lo;  // k offset (halves) of the next unit
  uint32_t xa = smem_addr(xlane) + 2 * xoff;                  // its shared address
  const uint8_t* lp = io.packed + ((size_t)u0 + warp) * UNIT + lane * 16 + D * WSTEP;  // unit j0 + D

  auto flush = [&](int j) {
    float v[P][4];
    math.result(v, lane);
#pragma unroll
    for (int pl = 0; pl < P; ++pl)
      slots[((size_t)(j * W + warp) * P + pl) * 32 + lane] = make_float4(v[pl][0], v[pl][1], v[pl][2], v[pl][3]);
  };
  // Unit d of the current block: math on ring slot d, then (if `load`) refill
  // the slot with the unit D ahead.
  auto unit = [&](const int d, const bool load) {
    if constexpr (MATH == kMathMma) {
      uint4 xf;
      if constexpr (WB == 1) {
        xf = lds128_at(xa);
      } else {
        const uint2 t = lds64_at(xa);
        xf = make_uint4(t.x, t.y, 0u, 0u);
      }
      math.unit(&ring[d * P], xf);
    } else {
      math.unit(&ring[d * P], xq + xoff, M, p.x_rs);
    }
    if (load) {
#pragma unroll
      for (int pl = 0; pl < P; ++pl)
        ring[d * P + pl] = ldg_stream(lp + (size_t)d * WSTEP + pl * kUnitPlaneBytes, pol);
    }
    xoff += W * KPB;
    xa += 2 * W * KPB;
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
      xoff = (fdiv(vt, p.div_tiles) * kbpv + kbl) * KPB - k_lo;
      xa = smem_addr(xlane) + 2 * xoff;
    }
  };
  // Blocks of D units: slot d of a block is used while unit j0 + d exists and
  // refills with unit j0 + D + d while that exists.
  for (int j0 = 0; j0 < n_mine; j0 += D) {
    const int use = n_mine - j0, refill = use - D;
#pragma unroll
    for (int d = 0; d < D; ++d)
      if (d < use) unit(d, d < refill);
    lp += (size_t)D * WSTEP;
  }
  if (n_mine > 0 && seg_left != seg_n) flush(cur_j);
  if (threadIdx.x == 0) {
    TRACE(3);
    STRACE(trace_base + 2);
  }
  after_stream(ring);
  if constexpr (SCALES_LOADED) cp_async_wait_all();  // the scales (and lean residual rows) copied asynchronously

  // ---- combine: the warps' partials in warp order, then finish each tile
  __syncthreads();
  const int nvt = vt_last - vt_first + 1;
  // A tensor-parallel gather whose wait expired: the tiles' handshakes still
  // run, their rows are not written.
  const bool write = !(gather && *reinterpret_cast<volatile int*>(smem + kOffMisc) == 0);
  for (int j = warp; j < nvt; j += W) {
    float v[P][4];
#pragma unroll
    for (int pl = 0; pl < P; ++pl) v[pl][0] = v[pl][1] = v[pl][2] = v[pl][3] = 0.f;
#pragma unroll
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
    // slot j's shared memory is this warp's alone once summed: the PUSH stage
    __syncwarp();
    finish_vt<P, TP, !LEAN>(p, io, vt_first + j, j, v, lane, p.rmsnorm ? red : nullptr, epi,
                 reinterpret_cast<__half*>(slots + (size_t)j * W * P * 32), write);
  }
#ifdef B2G_TRACE
  __syncthreads();
  if (tid == 0) STRACE(trace_base + 3);
#endif
}

// ---------------------------------------------------------------------------
// One GEMV per launch
// ---------------------------------------------------------------------------
// FLAVOR: kFlavorLean (whole tiles, aligned rows, no exchange),
// kFlavorGeneral (any plan and rows, no exchange), kFlavorPush (the
// tensor-parallel PUSH epilogue compiled in) or kFlavorGather (the GATHER
// staging compiled in).  Code size shows up as instruction-fetch stalls in
// every launch, so each launch takes the smallest flavor that covers it.
// kFlavorReduce: the lean flavor with the REDUCE epilogue and tail (one
// plane only).
enum : int { kFlavorLean = 0, kFlavorGeneral = 1, kFlavorPush = 2, kFlavorGather = 3, kFlavorReduce = 4 };

template <int P, int WB, int MATH, int FLAVOR>
__global__ void __launch_bounds__(kThreads, 1) gemv_streamk_kernel(const __grid_constant__ GemvParams p) {
  constexpr bool REDUCEX = FLAVOR == kFlavorReduce;
  constexpr bool TPX = FLAVOR == kFlavorPush || REDUCEX;  // the pushing epilogue and arrivals
  constexpr bool GATHERX = FLAVOR == kFlavorGather;
  constexpr bool LEAN = FLAVOR == kFlavorLean || REDUCEX;
  extern __shared__ __align__(1024) uint8_t smem[];
  // 128 KB of weights in flight per SM (16 B x 512 threads x 16); the FFMA
  // variant needs the registers for its accumulators and keeps half.
  constexpr int R = (MATH == kMathMma) ? kRing : kRing / 2;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) TRACE(0);
  const uint64_t pol = l2_policy_evict_first();
  uint4 ring[R];
  // Weights are constant: the first loads go out before the previous kernel
  // in the stream is waited on.
  prefetch_phase<P, R>(p, p.packed, ring, warp, lane, pol);
  // Warm L2 with the start of the ranges the next kernel's CTAs will stream
  // (next CTAs blockIdx.x, blockIdx.x + grid, ...), so HBM keeps working
  // through this kernel's tail and the launch gap, and the next kernel's
  // first loads hit L2.
  if (tid == 0 && p.pf_packed != nullptr) {
    const long long tg = p.pf_total_units / p.pf_gran;
    for (int c = blockIdx.x; c < p.pf_grid; c += p.grid) {
      const long long a = (long long)c * tg / p.pf_grid * p.pf_gran;
      const long long b = (long long)(c + 1) * tg / p.pf_grid * p.pf_gran;
      const long long bytes = min((long long)p.pf_bytes, (b - a) * p.pf_unit_bytes);
      const uint8_t* src = p.pf_packed + a * p.pf_unit_bytes;
      for (long long off = 0; off < bytes; off += 32768)
        bulk_prefetch_l2(src + off, (uint32_t)min(32768LL, bytes - off));
    }
  }
  pdl_launch_dependents();
  // The scales are constants: into shared memory before the wait, off the
  // critical path (an HBM round trip after it otherwise).
  if ((int)blockIdx.x < p.grid) {
    const int u0 = range_start(p, blockIdx.x), u1 = range_start(p, blockIdx.x + 1);
    if (u1 > u0) {
      const int vt_first = fdiv(u0, p.div_kbpv);
      load_scales<P, true>(p, io_of_params(p), epi_of(p, smem, P), vt_first, fdiv(u1 - 1, p.div_kbpv) - vt_first + 1,
                           tid);
    }
  }
  pdl_wait();
  if (tid == 0) TRACE(1);
  if constexpr (REDUCEX) {
    // the previous launch's round count (that launch is complete now)
    if (tid == 0) cp_async4(smem + kOffRound, p.tp.rounds + blockIdx.x);
    run_phase<P, WB, MATH, R, RoundHook, TPX, true, LEAN, GATHERX>(p, io_of_params(p), smem, ring, pol, RoundHook{});
    __syncthreads();  // every tile's rows staged and pushed
    tp_reduce_tail(p, smem, tid);
  } else {
    if (TPX && p.tp.mode == kTpPush && blockIdx.x == 0 && tid == 0) atomicAdd(p.tp.epoch, 1u);
    run_phase<P, WB, MATH, R, NoHook, TPX, true, LEAN, GATHERX>(p, io_of_params(p), smem, ring, pol, NoHook{});
    if (TPX && p.tp.mode == kTpPush) {
      // This CTA's peer stores are done: one arrival on every rank.
      __syncthreads();
      if (tid == 0) {
        fence_acq_rel_sys();  // the CTA's peer stores (ordered by the barrier) before the arrivals
        for (int r = 0; r < p.tp.world; ++r) red_relaxed_sys_add(p.tp.counters[r] + p.tp.rank, 1u);
      }
    }
  }
  if (tid == 0) TRACE(4);
}


// ---------------------------------------------------------------------------
// TMA pipeline: weights through a ring of stages in shared memory
// ---------------------------------------------------------------------------
// Warp 16 (lane 0, the producer) streams a CTA's contiguous range of the
// packed weights into a ring of n_stages stages with 1-D bulk copies
// (cp.async.bulk, one CTA's own copies from this GPU's memory).  Warps 0..15 (the
// consumers) take the units as the register-ring kernel does (warp w: units
// w, w + 16, ... of the range) and read each lane's 16-byte A fragment from
// the ring.  Stage s of the ring's life fills slot s % n_stages; full[slot]
// completes when its bytes land, empty[slot] when all 16 consumer warps have
// passed it.  The copies never wait for activations: while the consumers
// wait for the previous kernel (or grid phase) and stage x, the ring fills.
__device__ __forceinline__ void consumer_sync() { named_sync(1, kThreads); }

struct Ring {
  uint8_t* base;
  uint64_t* full;
  uint64_t* empty;
  int n_stages, stage_bytes;
  int slot;        // next stage's slot
  uint32_t round;  // times the ring has wrapped before the next stage
  __device__ __forceinline__ void advance() {
    if (++slot == n_stages) {
      slot = 0;
      ++round;
    }
  }
};

__device__ __forceinline__ Ring ring_at(uint8_t* smem, int off_ring, int n_stages, int stage_bytes) {
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kOffBars);
  return Ring{smem + off_ring, full, full + kMaxStages, n_stages, stage_bytes, 0, 0u};
}

// Thread 0 of a CTA: the ring's mbarriers (followed by a CTA-wide barrier).
__device__ __forceinline__ void ring_init(const Ring& r) {
  for (int i = 0; i < r.n_stages; ++i) {
    mbar_init(&r.full[i], 1);
    mbar_init(&r.empty[i], W);
  }
  fence_mbarrier_init();
}

// Producer: units [u0, u1) of `packed` into the next stages.  False if a
// wait for a free slot expired (the error word is set; nothing more is issued).
__device__ bool ring_produce(Ring& r, const uint8_t* packed, int unit_bytes, int u0, int u1, uint64_t pol,
                             int* err) {
  const long long all = (long long)(u1 - u0) * unit_bytes;
  const uint8_t* src = packed + (size_t)u0 * unit_bytes;
  for (long long off = 0; off < all; off += r.stage_bytes) {
    if (r.round > 0 && !mbar_wait_bounded(&r.empty[r.slot], (r.round - 1) & 1)) {
      atomicCAS(err, 0, kErrEmptyWait);
      return false;
    }
    const uint32_t bytes = (uint32_t)min((long long)r.stage_bytes, all - off);
    mbar_arrive_expect_tx(&r.full[r.slot], bytes);
    bulk_g2s(r.base + (size_t)r.slot * r.stage_bytes, src + off, bytes, &r.full[r.slot], pol);
    r.advance();
  }
  return true;
}

// Producer, before it leaves: every stage it issued has landed (bounded), so
// no copy into this CTA's shared memory is in flight once it exits.
__device__ void ring_drain(const Ring& r, long long issued, int* err) {
  Ring q = r;
  for (long long i = 0; i < min(issued, (long long)r.n_stages); ++i) {
    if (q.slot == 0) {
      q.slot = r.n_stages - 1;
      --q.round;
    } else {
      --q.slot;
    }
    if (!mbar_wait_bounded(&q.full[q.slot], q.round & 1)) {
      atomicCAS(err, 0, kErrDrainWait);
      return;
    }
  }
}

// L2 prefetch of CTA c's range of a partition (units of unit_bytes in
// granules of gran over `grid` CTAs), up to `bytes`.
__device__ __forceinline__ void l2_prefetch_range(const uint8_t* packed, long long total_units, int gran,
                                                  int unit_bytes, int grid, int c, long long bytes) {
  const long long tg = total_units / gran;
  const long long a = (long long)c * tg / grid * gran;
  const long long b = (long long)(c + 1) * tg / grid * gran;
  bytes = min(bytes, (b - a) * unit_bytes);
  const uint8_t* src = packed + a * unit_bytes;
  for (long long off = 0; off < bytes; off += 32768) bulk_prefetch_l2(src + off, (uint32_t)min(32768LL, bytes - off));
}

struct Geom {
  Range r;
  bool active;
  int vt_first, vt_last, k_lo, krange;
};

template <int WB>
__device__ __forceinline__ Geom geom_of(const GemvParams& p, int warp) {
  constexpr int KPB = (WB == 1) ? 32 : 16;
  Geom g;
  g.r = cta_range(p, warp);
  g.active = g.r.u1 > g.r.u0;
  g.vt_first = fdiv(g.r.u0, p.div_kbpv);
  g.vt_last = g.active ? fdiv(g.r.u1 - 1, p.div_kbpv) : g.vt_first - 1;
  const int ks_first = fdiv(g.vt_first, p.div_tiles);
  g.k_lo = ks_first * p.kbpv * KPB;
  g.krange = g.active ? (fdiv(g.vt_last, p.div_tiles) + 1 - ks_first) * p.kbpv * KPB : 0;
  return g;
}

// Consumers, before the activations exist: zeroed partial slots, the scales.
template <int P>
__device__ __forceinline__ void tma_setup(const GemvParams& p, const Io& io, uint8_t* smem, const Geom& g, int tid) {
  float4* slots = reinterpret_cast<float4*>(smem + kOffSlots);
  for (int i = tid; i < p.n_slots * W * P * 32; i += NT) slots[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  if (g.active) load_scales<P>(p, io, epi_of(p, smem, P), g.vt_first, g.vt_last - g.vt_first + 1, tid);
}

// Consumers, once the activations exist: x (staged, or all-reduced by the
// tensor-parallel gather), the residual rows; a consumer barrier at the end.
template <int P, bool TPX>
__device__ __forceinline__ void tma_inputs(const GemvParams& p, const Io& io, uint8_t* smem, const Geom& g, int tid) {
  float* red = reinterpret_cast<float*>(smem + kOffRed);
  __half* xs = reinterpret_cast<__half*>(smem + p.off_x);
  if (TPX && p.tp.mode == kTpGather) {
    gather_x(p, xs, g.active ? g.krange : p.K / 8 * 8, tid, p.rmsnorm ? red : nullptr,
             reinterpret_cast<volatile int*>(smem + kOffMisc), [] { consumer_sync(); });
  } else if (g.active) {
    stage_x(p, io, xs, g.k_lo, g.krange, tid, p.rmsnorm ? red : nullptr);
  }
  if (g.active) load_residual<P>(p, io, epi_of(p, smem, P), g.vt_first, g.vt_last - g.vt_first + 1, tid);
  consumer_sync();
}

// Consumers: this CTA's range from the ring (every stage of it, in order:
// every warp waits for and then releases every stage, so the producer can
// refill it), then the combine and the epilogue.
template <int P, int WB, bool TPX>
__device__ void tma_stream(const GemvParams& p, const Io& io, uint8_t* smem, const Geom& geo, Ring& ring, bool& live,
                           int trace_base = -1) {
  constexpr int UNIT = P * kUnitPlaneBytes;
  constexpr int KPB = (WB == 1) ? 32 : 16;
  float* red = reinterpret_cast<float*>(smem + kOffRed);
  const Epi epi = epi_of(p, smem, P);
  float4* slots = reinterpret_cast<float4*>(smem + kOffSlots);  // [n_slots][W][P][32]
  __half* xs = reinterpret_cast<__half*>(smem + p.off_x);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, q = lane & 3;
  const int M = p.M, kbpv = p.kbpv;
  const int u0 = geo.r.u0, n_mine = geo.r.n_mine;
  const int vt_first = geo.vt_first, k_lo = geo.k_lo;
  const int nvt = geo.vt_last - vt_first + 1;
  const int SU = ring.stage_bytes / UNIT;  // units per stage (a multiple of 16)
  const int UPW = SU / W;                  // each warp's units per full stage
  const int n_st = (geo.r.u1 - geo.r.u0 + SU - 1) / SU;
  if (tid == 0) STRACE(trace_base + 1);

  MmaMath<P, WB> math;
  math.zero();
  int vt = fdiv(u0 + warp, p.div_kbpv);
  int kbl = (u0 + warp) - vt * kbpv;
  int seg_n = (kbpv - kbl + W - 1) / W;
  int seg_left = seg_n;
  int cur_j = vt - vt_first;
  const __half* xlane = xs + (size_t)(g < M ? g : 0) * p.x_rs + (WB == 1 ? 8 * q : 4 * q);
  int xoff = (fdiv(vt, p.div_tiles) * kbpv + kbl) * KPB - k_lo;
  uint32_t xa = smem_addr(xlane) + 2 * xoff;
  const uint32_t wbase = smem_addr(ring.base) + warp * UNIT + lane * 16;
  auto flush = [&](int j) {
    float v[P][4];
    math.result(v, lane);
#pragma unroll
    for (int pl = 0; pl < P; ++pl)
      slots[((size_t)(j * W + warp) * P + pl) * 32 + lane] = make_float4(v[pl][0], v[pl][1], v[pl][2], v[pl][3]);
  };
  int j = 0;
#pragma unroll 1
  for (int s = 0; s < n_st; ++s) {
    const int jend = min((s + 1) * UPW, n_mine);
    // Every warp waits for every stage, even one it has no units in (the
    // last stage of a range may be short): its arrival on empty must count
    // for this round of the slot, which has begun only once the producer
    // has refilled it.
    if (live && !mbar_wait_bounded(&ring.full[ring.slot], ring.round & 1)) {
      atomicCAS(p.error, 0, kErrFullWait);
      live = false;
    }
    const uint32_t sa = wbase + (uint32_t)(ring.slot * ring.stage_bytes);
#pragma unroll 1
    for (int k = 0; j < jend; ++j, ++k) {
      uint4 w[P];
#pragma unroll
      for (int pl = 0; pl < P; ++pl) w[pl] = lds128_at(sa + (uint32_t)(k * W * UNIT + pl * kUnitPlaneBytes));
      uint4 xf;
      if constexpr (WB == 1) {
        xf = lds128_at(xa);
      } else {
        const uint2 t = lds64_at(xa);
        xf = make_uint4(t.x, t.y, 0u, 0u);
      }
      math.unit(w, xf);
      xoff += W * KPB;
      xa += 2 * W * KPB;
      if (--seg_left == 0) {
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
        xoff = (fdiv(vt, p.div_tiles) * kbpv + kbl) * KPB - k_lo;
        xa = smem_addr(xlane) + 2 * xoff;
      }
    }
    // this warp is done with the stage: one arrival frees the slot
    __syncwarp();
    if (lane == 0) mbar_arrive(&ring.empty[ring.slot]);
    ring.advance();
  }
  if (n_mine > 0 && seg_left != seg_n) flush(cur_j);
  if (tid == 0) STRACE(trace_base + 2);

  // ---- combine the warps' partials in warp order, then finish each tile
  consumer_sync();
  // A tensor-parallel gather whose wait expired: the tiles' handshakes still
  // run, their rows are not written.
  const bool write = !(TPX && p.tp.mode == kTpGather && *reinterpret_cast<volatile int*>(smem + kOffMisc) == 0);
  for (int jj = warp; jj < nvt; jj += W) {
    float v[P][4];
#pragma unroll
    for (int pl = 0; pl < P; ++pl) v[pl][0] = v[pl][1] = v[pl][2] = v[pl][3] = 0.f;
#pragma unroll
    for (int w2 = 0; w2 < W; ++w2) {
#pragma unroll
      for (int pl = 0; pl < P; ++pl) {
        const float4 t = slots[((size_t)(jj * W + w2) * P + pl) * 32 + lane];
        v[pl][0] += t.x;
        v[pl][1] += t.y;
        v[pl][2] += t.z;
        v[pl][3] += t.w;
      }
    }
    __syncwarp();
    finish_vt<P, TPX>(p, io, vt_first + jj, jj, v, lane, p.rmsnorm ? red : nullptr, epi,
                      reinterpret_cast<__half*>(slots + (size_t)jj * W * P * 32), write);
  }
  if (tid == 0) STRACE(trace_base + 3);
}

// ---------------------------------------------------------------------------
// One GEMV per launch on the TMA pipeline
// ---------------------------------------------------------------------------
template <int P, int WB, bool TPX>
__global__ void __launch_bounds__(kTmaThreads, 1) gemv_tma_kernel(const __grid_constant__ GemvParams p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  constexpr int UNIT = P * kUnitPlaneBytes;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  Ring ring = ring_at(smem, p.off_ring, p.n_stages, p.stage_bytes);
  if (tid == 0) ring_init(ring);
  __syncthreads();  // the barriers are initialised before anyone uses them
  pdl_launch_dependents();
  if (warp == W) {
    // ---- producer: weights are constant, so no dependency wait
    if (lane == 0) {
      const Range rg = cta_range(p, 0);
      ring_produce(ring, p.packed, UNIT, rg.u0, rg.u1, l2_policy_evict_first(), p.error);
      // Every copy of this range is issued: HBM goes on with the next
      // kernel's weights (the ranges its CTAs blockIdx.x, blockIdx.x + grid,
      // ... will stream) while this kernel's math, its epilogue, the launch
      // gap and the next kernel's activation staging run.
      if (p.pf_packed != nullptr)
        for (int c = blockIdx.x; c < p.pf_grid; c += p.grid)
          l2_prefetch_range(p.pf_packed, p.pf_total_units, p.pf_gran, p.pf_unit_bytes, p.pf_grid, c, p.pf_bytes);
      ring_drain(ring, (long long)ring.round * ring.n_stages + ring.slot, p.error);
    }
    return;
  }
  // ---- consumers (warps 0..15)
  if (tid == 0) TRACE(0);
  const Io io = io_of_params(p);
  const Geom geo = geom_of<WB>(p, warp);
  tma_setup<P>(p, io, smem, geo, tid);
  pdl_wait();
  if (tid == 0) TRACE(1);
  if (TPX && p.tp.mode == kTpPush && blockIdx.x == 0 && tid == 0) atomicAdd(p.tp.epoch, 1u);
  tma_inputs<P, TPX>(p, io, smem, geo, tid);
  if (tid == 0) TRACE(2);
  bool live = true;
  tma_stream<P, WB, TPX>(p, io, smem, geo, ring, live);
  if (tid == 0) TRACE(3);
  if (TPX && p.tp.mode == kTpPush) {
    // This CTA's peer stores are done: one arrival on every rank.
    consumer_sync();
    if (tid == 0) {
      fence_acq_rel_sys();
      for (int r = 0; r < p.tp.world; ++r) red_relaxed_sys_add(p.tp.counters[r] + p.tp.rank, 1u);
    }
  }
  if (tid == 0) TRACE(4);
}

// ---------------------------------------------------------------------------
// The decode-MLP stack in one cooperative launch
// ---------------------------------------------------------------------------
// Grid barrier on a counter that is zero at launch and counts one arrival per
// CTA per barrier: barrier b (1-based) completes when it reaches b * grid.
// The wait is bounded; on expiry the error word is set and false returned.
__device__ bool grid_barrier(unsigned* counter, unsigned target, int* err, volatile int* verdict) {
  __syncthreads();
  if (threadIdx.x == 0) {
    fence_acq_rel_gpu();
    atomicAdd(counter, 1u);
    const unsigned long long t0 = globaltimer_ns();
    int ok = 1;
    while (true) {
      unsigned v;
      asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(counter) : "memory");
      if (v >= target) break;
      if (globaltimer_ns() - t0 > kWaitBudgetNs) {
        atomicCAS(err, 0, kErrGridWait);
        ok = 0;
        break;
      }
      __nanosleep(32);
    }
    *verdict = ok;
  }
  __syncthreads();
  return *verdict != 0;
}

// Last arrival of the launch: the CTA that brings the counter to `total`
// (every CTA has passed every barrier) resets it for the next launch.
__device__ void grid_exit(unsigned* counter, unsigned total) {
  if (threadIdx.x == 0) {
    const unsigned old = atomicAdd(counter, 1u);
    if (old == total - 1) atomicExch(counter, 0u);
  }
}

// The stack kernel keeps HBM busy independently of its phase structure: at
// the start of each phase every CTA asks L2 to fetch its whole range of the
// NEXT phase's weights (bulk prefetch through the TMA unit: no registers, no
// L1 miss slots).  By the time the next phase streams, most of its weights
// are L2 hits, and HBM works through the following phase meanwhile.  L2 holds
// at most two phases (75 MB of a Llama-3.2-3B layer) at once.
constexpr long long kWholeRange = 1LL << 40;

template <int WB>
__global__ void __launch_bounds__(kThreads, 1) stack_kernel(const __grid_constant__ StackParams sp) {
  extern __shared__ __align__(1024) uint8_t smem[];
  constexpr int R = kRing;
  volatile int* verdict = reinterpret_cast<int*>(smem + kOffMisc);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint64_t pol = l2_policy_evict_first();
  const GemvParams& gu = sp.gu;
  const GemvParams& dn = sp.dn;
  const unsigned G = gridDim.x;
  uint4 ring[R];
  unsigned nbar = 0;
  l2_prefetch_phase(gu, sp.layers[0].pgu, 2 * kUnitPlaneBytes, kWholeRange);
  prefetch_phase<2, R>(gu, sp.layers[0].pgu, ring, warp, lane, pol);
  for (int l = 0; l < sp.n_layers; ++l) {
    const StackLayer& L = sp.layers[l];
    const bool more = l + 1 < sp.n_layers;
    const uint8_t* next_gu = more ? sp.layers[l + 1].pgu : nullptr;
    // act = SiLU(RMSNorm(h) . Wg) * (RMSNorm(h) . Wu); this layer's down
    // weights go to L2 meanwhile.
    l2_prefetch_phase(dn, L.pd, kUnitPlaneBytes, kWholeRange);
    const Io io_gu{L.pgu, L.sgu, sp.h, sp.ldh, nullptr, 0, sp.act, sp.ldact};
    run_phase<2, WB, kMathMma, R, NoHook, false>(gu, io_gu, smem, ring, pol, NoHook{}, 8 * l);
    // The ring is free again: the down phase's first units load while the
    // barrier completes.
    prefetch_phase<1, R>(dn, L.pd, ring, warp, lane, pol);
    if (!grid_barrier(sp.barrier, (++nbar) * G, gu.error, verdict)) return;
    // h = h + act . Wd; the next layer's gate||up weights go to L2 meanwhile.
    if (more) l2_prefetch_phase(gu, next_gu, 2 * kUnitPlaneBytes, kWholeRange);
    const Io io_dn{L.pd, L.sd, sp.act, sp.ldact, sp.h, sp.ldh, sp.h, sp.ldh};
    run_phase<1, WB, kMathMma, R, NoHook, false>(dn, io_dn, smem, ring, pol, NoHook{}, 8 * l + 4);
    if (more) {
      prefetch_phase<2, R>(gu, next_gu, ring, warp, lane, pol);
      if (!grid_barrier(sp.barrier, (++nbar) * G, gu.error, verdict)) return;
    }
  }
  grid_exit(sp.barrier, (nbar + 1) * G);
}


// ---------------------------------------------------------------------------
// The decode-MLP stack in one cooperative launch on the TMA pipeline
// ---------------------------------------------------------------------------
// The producer streams every phase's range of this CTA in order -- layer l's
// gate||up, then its down, then layer l + 1's gate||up ... -- through one
// ring, bounded only by free slots, and asks L2 for the phase after the one
// it streams (so HBM keeps working while the consumers sit at a grid barrier
// or stage activations).  The consumers run the phases; a grid barrier
// (consumer threads only) separates each phase from the next, since every
// tile of a phase reads all of the previous phase's rows.
__device__ __forceinline__ void cgrid_arrive(unsigned* counter) {
  if (threadIdx.x == 0) {
    fence_acq_rel_gpu();  // this CTA's rows (ordered by the consumer barrier) before the arrival
    atomicAdd(counter, 1u);
  }
}

// Waits (thread 0, bounded) until the counter reaches target, then releases
// the consumers.  False once a wait expired (or the error word was already
// set); the phase still runs, on void data.
__device__ __forceinline__ bool cgrid_wait(unsigned* counter, unsigned target, int* err, volatile int* verdict) {
  if (threadIdx.x == 0) {
    int ok = *reinterpret_cast<volatile int*>(err) == 0;
    const unsigned long long t0 = globaltimer_ns();
    while (ok) {
      unsigned v;
      asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(counter) : "memory");
      if (v >= target) break;
      if (globaltimer_ns() - t0 > kWaitBudgetNs) {
        atomicCAS(err, 0, kErrGridWait);
        ok = 0;
      }
      __nanosleep(32);
    }
    *verdict = ok;
  }
  consumer_sync();
  return *verdict != 0;
}

template <int WB>
__global__ void __launch_bounds__(kTmaThreads, 1) stack_tma_kernel(const __grid_constant__ StackParams sp) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const GemvParams& gu = sp.gu;
  const GemvParams& dn = sp.dn;
  const unsigned G = gridDim.x;
  Ring ring = ring_at(smem, gu.off_ring, gu.n_stages, gu.stage_bytes);
  if (tid == 0) ring_init(ring);
  __syncthreads();
  if (warp == W) {
    if (lane == 0) {
      const uint64_t pol = l2_policy_evict_first();
      const Range rg = cta_range(gu, 0), rd = cta_range(dn, 0);
      for (int l = 0; l < sp.n_layers; ++l) {
        const StackLayer& L = sp.layers[l];
        if (!ring_produce(ring, L.pgu, 2 * kUnitPlaneBytes, rg.u0, rg.u1, pol, gu.error)) break;
        if (rd.u1 > rd.u0)
          l2_prefetch_range(L.pd, dn.total_units, dn.gran, kUnitPlaneBytes, dn.grid, blockIdx.x, kWholeRange);
        if (!ring_produce(ring, L.pd, kUnitPlaneBytes, rd.u0, rd.u1, pol, gu.error)) break;
        if (l + 1 < sp.n_layers && rg.u1 > rg.u0)
          l2_prefetch_range(sp.layers[l + 1].pgu, gu.total_units, gu.gran, 2 * kUnitPlaneBytes, gu.grid, blockIdx.x,
                            kWholeRange);
      }
      ring_drain(ring, (long long)ring.round * ring.n_stages + ring.slot, gu.error);
    }
    return;
  }
  // ---- consumers
  volatile int* verdict = reinterpret_cast<volatile int*>(smem + kOffMisc);
  unsigned nbar = 0;
  bool live = true;
  for (int l = 0; l < sp.n_layers; ++l) {
    const StackLayer& L = sp.layers[l];
    // act = SiLU(RMSNorm(h) . Wg) * (RMSNorm(h) . Wu)
    const Io io_gu{L.pgu, L.sgu, sp.h, sp.ldh, nullptr, 0, sp.act, sp.ldact};
    const Geom g1 = geom_of<WB>(gu, warp);
    if (tid == 0) STRACE(8 * l);
    tma_setup<2>(gu, io_gu, smem, g1, tid);
    if (l > 0) cgrid_wait(sp.barrier, (++nbar) * G, gu.error, verdict);
    tma_inputs<2, false>(gu, io_gu, smem, g1, tid);
    tma_stream<2, WB, false>(gu, io_gu, smem, g1, ring, live, 8 * l);
    consumer_sync();
    cgrid_arrive(sp.barrier);
    // h = h + act . Wd
    const Io io_dn{L.pd, L.sd, sp.act, sp.ldact, sp.h, sp.ldh, sp.h, sp.ldh};
    const Geom g2 = geom_of<WB>(dn, warp);
    if (tid == 0) STRACE(8 * l + 4);
    tma_setup<1>(dn, io_dn, smem, g2, tid);
    cgrid_wait(sp.barrier, (++nbar) * G, gu.error, verdict);
    tma_inputs<1, false>(dn, io_dn, smem, g2, tid);
    tma_stream<1, WB, false>(dn, io_dn, smem, g2, ring, live, 8 * l + 4);
    if (l + 1 < sp.n_layers) {
      consumer_sync();
      cgrid_arrive(sp.barrier);
    }
  }
  grid_exit(sp.barrier, (nbar + 1) * G);
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
  // The smallest flavor that covers the launch.  Measured on B200 per decode
  // layer (28 layers, M = 8 / 1): gate||up on the exchange flavor 22.9 /
  // 22.1 us, on the general one 21.2 / 20.5, both ops on the lean one
  // 20.6 / 19.6.
  if constexpr (P == 1)
    if (p.tp.mode == kTpReduce) return cudaLaunchKernelEx(&cfg, gemv_streamk_kernel<P, WB, MATH, kFlavorReduce>, p);
  if (p.tp.mode == kTpPush) return cudaLaunchKernelEx(&cfg, gemv_streamk_kernel<P, WB, MATH, kFlavorPush>, p);
  if (p.tp.mode == kTpGather) return cudaLaunchKernelEx(&cfg, gemv_streamk_kernel<P, WB, MATH, kFlavorGather>, p);
  if (p.lean) return cudaLaunchKernelEx(&cfg, gemv_streamk_kernel<P, WB, MATH, kFlavorLean>, p);
  return cudaLaunchKernelEx(&cfg, gemv_streamk_kernel<P, WB, MATH, kFlavorGeneral>, p);
}

template <int P, int WB>
cudaError_t launch_tma_variant(const GemvParams& p, size_t smem, bool pdl, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.grid);
  cfg.blockDim = dim3(kTmaThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  if (p.tp.mode != kTpNone) return cudaLaunchKernelEx(&cfg, gemv_tma_kernel<P, WB, true>, p);
  return cudaLaunchKernelEx(&cfg, gemv_tma_kernel<P, WB, false>, p);
}

}  // namespace

cudaError_t launch_gemv_tma(const GemvParams& p, int planes, int wbytes, size_t smem, bool pdl,
                            cudaStream_t stream) {
  if (planes == 1 && wbytes == 1) return launch_tma_variant<1, 1>(p, smem, pdl, stream);
  if (planes == 2 && wbytes == 1) return launch_tma_variant<2, 1>(p, smem, pdl, stream);
  if (planes == 1 && wbytes == 2) return launch_tma_variant<1, 2>(p, smem, pdl, stream);
  if (planes == 2 && wbytes == 2) return launch_tma_variant<2, 2>(p, smem, pdl, stream);
  return cudaErrorInvalidValue;
}

cudaError_t launch_stack_tma(const StackParams& sp, int grid, int wbytes, size_t smem, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kTmaThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (wbytes == 1) return cudaLaunchKernelEx(&cfg, stack_tma_kernel<1>, sp);
  if (wbytes == 2) return cudaLaunchKernelEx(&cfg, stack_tma_kernel<2>, sp);
  return cudaErrorInvalidValue;
}

cudaError_t stack_tma_max_coresident(int wbytes, size_t smem, int num_sms, int* max_grid) {
  int per_sm = 0;
  const cudaError_t e =
      wbytes == 1 ? cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, stack_tma_kernel<1>, kTmaThreads, smem)
                  : cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, stack_tma_kernel<2>, kTmaThreads, smem);
  *max_grid = per_sm * num_sms;
  return e;
}

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

cudaError_t launch_stack(const StackParams& sp, int grid, int wbytes, size_t smem, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (wbytes == 1) return cudaLaunchKernelEx(&cfg, stack_kernel<1>, sp);
  if (wbytes == 2) return cudaLaunchKernelEx(&cfg, stack_kernel<2>, sp);
  return cudaErrorInvalidValue;
}

cudaError_t stack_max_coresident(int wbytes, size_t smem, int num_sms, int* max_grid) {
  int per_sm = 0;
  const cudaError_t e =
      wbytes == 1 ? cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, stack_kernel<1>, kThreads, smem)
                  : cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, stack_kernel<2>, kThreads, smem);
  *max_grid = per_sm * num_sms;
  return e;
}

namespace {
__global__ void __launch_bounds__(256) tp_gather_kernel(const __grid_constant__ TpParams tp, int m_rows, int* err) {
  __shared__ int verdict;
  // A launch chained after this one (programmatic dependent launch) may start
  // its weight stream now; it reads h only after its own dependency wait.
  pdl_launch_dependents();
  if (threadIdx.x == 0) verdict = tp_wait_arrivals(tp, err) ? 1 : 0;
  __syncthreads();
  if (!verdict) return;  // reported through the error word; h is left as it was
  const int nch = tp.width / 8;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < m_rows * nch; i += gridDim.x * blockDim.x) {
    const int m = i / nch, c = i - m * nch;
    *reinterpret_cast<uint4*>(tp.h_out + (size_t)m * tp.ldh + c * 8) = tp_sum8(tp, m, c * 8);
  }
}
}  // namespace

cudaError_t launch_tp_gather(const TpParams& tp, int m, int* error, cudaStream_t stream) {
  const int chunks = m * (tp.width / 8);
  const int blocks = min(148, (chunks + 255) / 256);
  tp_gather_kernel<<<blocks, 256, 0, stream>>>(tp, m, error);
  return cudaGetLastError();
}

#ifdef B2G_TRACE
// The whole per-launch timeline: [kTraceLaunches][kTraceCtas][8] u64 (bytes
// must be at least its size).
extern "C" int b2g_debug_trace(unsigned long long* out, size_t bytes) {
  if (bytes < sizeof(g_tl)) return (int)cudaErrorInvalidValue;
  return (int)cudaMemcpyFromSymbol(out, g_tl, sizeof(g_tl));
}
extern "C" int b2g_debug_stack_trace(unsigned long long* out, int n_ctas) {
  return (int)cudaMemcpyFromSymbol(out, g_strace, sizeof(unsigned long long) * kTracePts * n_ctas);
}
#endif

cudaError_t gemv_set_smem_limit(int bytes) {
  cudaError_t e = cudaSuccess, r;
#define B2G_LIM(K) \
  if ((r = cudaFuncSetAttribute(K, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes)) != cudaSuccess) e = r;
  B2G_LIM((gemv_streamk_kernel<1, 1, kMathMma, kFlavorLean>))
  B2G_LIM((gemv_streamk_kernel<1, 1, kMathMma, kFlavorGeneral>))
  B2G_LIM((gemv_streamk_kernel<1, 1, kMathMma, kFlavorPush>))
  B2G_LIM((gemv_streamk_kernel<1, 1, kMathMma, kFlavorGather>))
  B2G_LIM((gemv_streamk_kernel<1, 1, kMathMma, kFlavorReduce>))
  B2G_LIM((gemv_streamk_kernel<1, 1, kMathFfma, kFlavorReduce>))
  B2G_LIM((gemv_streamk_kernel<1, 2, kMathMma, kFlavorReduce>))
  B2G_LIM((gemv_streamk_kernel<1, 2, kMathFfma, kFlavorReduce>))
  B2G_LIM((gemv_streamk_kernel<1, 1, kMathFfma, kFlavorLean>))
  B2G_LIM((gemv_streamk_kernel<1, 1, kMathFfma, kFlavorGeneral>))
  B2G_LIM((gemv_streamk_kernel<1, 1, kMathFfma, kFlavorPush>))
  B2G_LIM((gemv_streamk_kernel<1, 1, kMathFfma, kFlavorGather>))
  B2G_LIM((gemv_streamk_kernel<1, 2, kMathMma, kFlavorLean>))
  B2G_LIM((gemv_streamk_kernel<1, 2, kMathMma, kFlavorGeneral>))
  B2G_LIM((gemv_streamk_kernel<1, 2, kMathMma, kFlavorPush>))
  B2G_LIM((gemv_streamk_kernel<1, 2, kMathMma, kFlavorGather>))
  B2G_LIM((gemv_streamk_kernel<1, 2, kMathFfma, kFlavorLean>))
  B2G_LIM((gemv_streamk_kernel<1, 2, kMathFfma, kFlavorGeneral>))
  B2G_LIM((gemv_streamk_kernel<1, 2, kMathFfma, kFlavorPush>))
  B2G_LIM((gemv_streamk_kernel<1, 2, kMathFfma, kFlavorGather>))
  B2G_LIM((gemv_streamk_kernel<2, 1, kMathMma, kFlavorLean>))
  B2G_LIM((gemv_streamk_kernel<2, 1, kMathMma, kFlavorGeneral>))
  B2G_LIM((gemv_streamk_kernel<2, 1, kMathMma, kFlavorPush>))
  B2G_LIM((gemv_streamk_kernel<2, 1, kMathMma, kFlavorGather>))
  B2G_LIM((gemv_streamk_kernel<2, 1, kMathFfma, kFlavorLean>))
  B2G_LIM((gemv_streamk_kernel<2, 1, kMathFfma, kFlavorGeneral>))
  B2G_LIM((gemv_streamk_kernel<2, 1, kMathFfma, kFlavorPush>))
  B2G_LIM((gemv_streamk_kernel<2, 1, kMathFfma, kFlavorGather>))
  B2G_LIM((gemv_streamk_kernel<2, 2, kMathMma, kFlavorLean>))
  B2G_LIM((gemv_streamk_kernel<2, 2, kMathMma, kFlavorGeneral>))
  B2G_LIM((gemv_streamk_kernel<2, 2, kMathMma, kFlavorPush>))
  B2G_LIM((gemv_streamk_kernel<2, 2, kMathMma, kFlavorGather>))
  B2G_LIM((gemv_streamk_kernel<2, 2, kMathFfma, kFlavorLean>))
  B2G_LIM((gemv_streamk_kernel<2, 2, kMathFfma, kFlavorGeneral>))
  B2G_LIM((gemv_streamk_kernel<2, 2, kMathFfma, kFlavorPush>))
  B2G_LIM((gemv_streamk_kernel<2, 2, kMathFfma, kFlavorGather>))
  B2G_LIM((stack_kernel<1>))
  B2G_LIM((stack_kernel<2>))
  B2G_LIM((gemv_tma_kernel<1, 1, false>))
  B2G_LIM((gemv_tma_kernel<1, 1, true>))
  B2G_LIM((gemv_tma_kernel<2, 1, false>))
  B2G_LIM((gemv_tma_kernel<2, 1, true>))
  B2G_LIM((gemv_tma_kernel<1, 2, false>))
  B2G_LIM((gemv_tma_kernel<1, 2, true>))
  B2G_LIM((gemv_tma_kernel<2, 2, false>))
  B2G_LIM((gemv_tma_kernel<2, 2, true>))
  B2G_LIM((stack_tma_kernel<1>))
  B2G_LIM((stack_tma_kernel<2>))
#undef B2G_LIM
  return e;
}

}  // namespace b2g
