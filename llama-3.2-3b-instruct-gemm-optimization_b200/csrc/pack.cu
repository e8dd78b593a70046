// pack.cu -- one-off weight preparation kernels:
//   * E4M3 quantisation with the reference's scale rules
//     (pack_e4m3, kernels/gemv_fp8.cu:297-304; check_real's fp16 scale and
//     pre-divide, :515-543) and the per-channel FP32 absmax/448 rule;
//   * the repack of [K, N] / [N, K] weights into the stream-K tile layout
//     described in gemv.h.
#include "device.cuh"
#include "gemv.h"

namespace b2g {
namespace {

__device__ __forceinline__ size_t widx(int layout, long long ld, int k, int n) {
  return layout == 0 ? (size_t)k * ld + n : (size_t)n * ld + k;
}

// One thread per (unit, lane): writes that lane's 16 bytes of one plane.
__global__ void prepack_kernel(const uint8_t* __restrict__ w, long long ld, int layout, int wbytes,
                               int K, int N, int plane, int planes, int ksplit, int kbpv,
                               int n_tiles, long long total_units, uint8_t* __restrict__ packed) {
  const long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= total_units * 32) return;
  const long long u = t >> 5;
  const int lane = (int)(t & 31);
  const long long vt = u / kbpv;
  const int kbl = (int)(u - vt * kbpv);
  const int ks = (int)(vt / n_tiles);
  const int tile = (int)(vt - (long long)ks * n_tiles);
  const int kb = ks * kbpv + kbl;
  const int g = lane >> 2, q = lane & 3;
  uint8_t out[16];
  if (wbytes == 1) {
    // Byte j: A-register pair pr = j/2 (element e = j%2) -> k16 step s = pr/4,
    // register r = pr%4: channel g + 8*(r&1), MMA k-slot 16s + 8*(r>>1) + 2q + e.
    // Slots are mapped to k inside the 32-block so that lane q's B fragment is
    // x[8q .. 8q+7]: k = 32kb + 8q + 4s + 2*(r>>1) + e.
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int pr = j >> 1, e = j & 1, s = pr >> 2, r = pr & 3;
      const int n = tile * kTileCh + g + 8 * (r & 1);
      const int k = kb * 32 + 8 * q + 4 * s + 2 * (r >> 1) + e;
      out[j] = (k < K && n < N) ? w[widx(layout, ld, k, n)] : 0;
    }
  } else {
    // half j: register r = j/2, element e = j%2 of one k16 step; k-slot
    // 8*(r>>1) + 2q + e maps to k = 16kb + 4q + 2*(r>>1) + e, so lane q's B
    // fragment is x[4q .. 4q+3].
    const uint16_t* w16 = reinterpret_cast<const uint16_t*>(w);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int r = j >> 1, e = j & 1;
      const int n = tile * kTileCh + g + 8 * (r & 1);
      const int k = kb * 16 + 4 * q + 2 * (r >> 1) + e;
      const uint16_t v = (k < K && n < N) ? w16[widx(layout, ld, k, n)] : 0;
      out[2 * j] = (uint8_t)(v & 0xFF);
      out[2 * j + 1] = (uint8_t)(v >> 8);
    }
  }
  uint4 v;
  memcpy(&v, out, 16);
  reinterpret_cast<uint4*>(packed + ((size_t)u * planes + plane) * kUnitPlaneBytes)[lane] = v;
}

// Per-output-channel absmax -> scale (fp16: half(max(a,1e-12)/448);
// fp32: max(a,1e-12)/448).
__global__ void channel_scale_kernel(const __half* __restrict__ w, int K, int N, int layout,
                                     int scale_mode, void* scales) {
  const int n = blockIdx.x * blockDim.x + threadIdx.x;
  if (n >= N) return;
  const long long ld = layout == 0 ? N : K;
  float a = 0.f;
  for (int k = 0; k < K; ++k) {
    const float v = fabsf(__half2float(w[widx(layout, ld, k, n)]));
    if (v > a) a = v;
  }
  const float s = fmaxf(a, 1e-12f) / 448.0f;
  if (scale_mode == 2)
    reinterpret_cast<__half*>(scales)[n] = __float2half_rn(s);
  else
    reinterpret_cast<float*>(scales)[n] = s;
}

// Whole-tensor absmax -> fp16 scale in scales[0].  One block.
__global__ void tensor_scale_kernel(const __half* __restrict__ w, long long elems, void* scales) {
  __shared__ float red[32];
  float a = 0.f;
  for (long long i = threadIdx.x; i < elems; i += blockDim.x) {
    const float v = fabsf(__half2float(w[i]));
    if (v > a) a = v;
  }
  for (int off = 16; off; off >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, off));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = a;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) t = fmaxf(t, red[i]);
    reinterpret_cast<__half*>(scales)[0] = __float2half_rn(fmaxf(t, 1e-12f) / 448.0f);
  }
}

__global__ void quantize_kernel(const __half* __restrict__ w, int K, int N, int layout,
                                int scale_mode, const void* scales, uint8_t* __restrict__ q) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long elems = (long long)K * N;
  if (i >= elems) return;
  const int n = layout == 0 ? (int)(i % N) : (int)(i / K);
  const __half h = w[i];
  uint8_t code;
  switch (scale_mode) {
    case 1:
    case 2: {
      const __half s = reinterpret_cast<const __half*>(scales)[scale_mode == 1 ? 0 : n];
      code = f16_to_e4m3(__float2half_rn(__half2float(h) / __half2float(s)));
      break;
    }
    case 3:
      code = f32_to_e4m3(__half2float(h) / reinterpret_cast<const float*>(scales)[n]);
      break;
    default:
      code = f16_to_e4m3(h);
  }
  q[i] = code;
}

}  // namespace

cudaError_t launch_prepack(const void* w, long long ld, int layout, int wbytes, int K, int N,
                           int plane, int planes, int ksplit, int kbpv, int n_tiles, int kb_total,
                           uint8_t* packed, cudaStream_t stream) {
  const long long total_units = (long long)n_tiles * kb_total;
  const long long threads = total_units * 32;
  const int block = 256;
  const long long blocks = (threads + block - 1) / block;
  prepack_kernel<<<(unsigned)blocks, block, 0, stream>>>(static_cast<const uint8_t*>(w), ld, layout,
                                                          wbytes, K, N, plane, planes, ksplit, kbpv,
                                                          n_tiles, total_units, packed);
  return cudaGetLastError();
}

cudaError_t launch_quantize(const __half* w16, int K, int N, int layout, int scale_mode, uint8_t* w8,
                            void* scales, cudaStream_t stream) {
  if (scale_mode == 2 || scale_mode == 3)
    channel_scale_kernel<<<(N + 127) / 128, 128, 0, stream>>>(w16, K, N, layout, scale_mode, scales);
  else if (scale_mode == 1)
    tensor_scale_kernel<<<1, 1024, 0, stream>>>(w16, (long long)K * N, scales);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const long long elems = (long long)K * N;
  quantize_kernel<<<(unsigned)((elems + 255) / 256), 256, 0, stream>>>(w16, K, N, layout, scale_mode,
                                                                       scales, w8);
  return cudaGetLastError();
}

}  // namespace b2g
