// ref_host_shim.cu -- exposes the reference project's own host-side
// functions through a C ABI.  TEST INFRASTRUCTURE ONLY (the checker and the
// CPU baseline); the product never loads it.
//
// Nothing here is a copy: the reference sources are #included from where they
// lie (path given on the command line by oracle/Makefile), each wrapped in its
// own namespace so the two files' identically named statics do not collide.
// The output goes to oracle/_ref/ only.
//
// Wrapped reference functions (kernels/gemv_fp8.cu unless noted):
//   fill_host              :285-295
//   pack_e4m3              :297-304
//   e4m3_to_double         :306-310
//   cpu_reference_e4m3     :313-323
//   cpu_reference_fp16     :325-335
//   cosine_stats           :337-355
//   cpu_reference_scaled   :470-482
//   fill_x (checkreal's synthetic activations) :408-413
//   cpu_reference (fp16)   kernels/gemv_fp16.cu:287-297
#include <cstdio>
#include <cstdlib>
#include <cstdint>
#include <cstring>
#include <cmath>
#include <string>
#include <thread>
#include <vector>
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>

#define main ref8_program_main
namespace ref8 {
#include REF_FP8_SRC
}
#undef main
#undef DISPATCH
#undef DISPATCH_KU
#define main ref16_program_main
namespace ref16 {
#include REF_FP16_SRC
}
#undef main

namespace {
std::vector<__half> as_half(const uint16_t* p, size_t n) {
  std::vector<__half> v(n);
  std::memcpy(v.data(), p, n * sizeof(uint16_t));
  return v;
}
}  // namespace

extern "C" {

void ref_fill_host(uint16_t* W, size_t w_elems, uint16_t* x, int K, int N) {
  std::vector<__half> w(w_elems), xv(K);
  ref8::fill_host(w, xv, K, N);
  std::memcpy(W, w.data(), w_elems * sizeof(uint16_t));
  std::memcpy(x, xv.data(), (size_t)K * sizeof(uint16_t));
}

void ref_fill_x(uint16_t* x, int K, unsigned seed) {
  std::vector<__half> xv(K);
  ref8::fill_x(xv, K, seed);
  std::memcpy(x, xv.data(), (size_t)K * sizeof(uint16_t));
}

void ref_pack_e4m3(const uint16_t* w16, size_t n, uint8_t* q) {
  std::vector<uint8_t> out;
  ref8::pack_e4m3(as_half(w16, n), out);
  std::memcpy(q, out.data(), n);
}

double ref_e4m3_to_double(uint8_t b) { return ref8::e4m3_to_double(b); }

void ref_cpu_reference_e4m3(const uint8_t* W, const uint16_t* x, double* y, int K, int N) {
  std::vector<uint8_t> w(W, W + (size_t)K * N);
  std::vector<double> yv;
  ref8::cpu_reference_e4m3(w, as_half(x, K), yv, K, N);
  std::memcpy(y, yv.data(), (size_t)N * sizeof(double));
}

void ref_cpu_reference_fp16(const uint16_t* W, const uint16_t* x, double* y, int K, int N) {
  std::vector<double> yv;
  ref8::cpu_reference_fp16(as_half(W, (size_t)K * N), as_half(x, K), yv, K, N);
  std::memcpy(y, yv.data(), (size_t)N * sizeof(double));
}

void ref16_cpu_reference(const uint16_t* W, const uint16_t* x, double* y, int K, int N) {
  std::vector<double> yv;
  ref16::cpu_reference(as_half(W, (size_t)K * N), as_half(x, K), yv, K, N);
  std::memcpy(y, yv.data(), (size_t)N * sizeof(double));
}

void ref_cpu_reference_scaled(const uint8_t* W, const uint16_t* x, const uint16_t* s,
                              double* y, int K, int N) {
  std::vector<uint8_t> w(W, W + (size_t)K * N);
  std::vector<double> yv;
  ref8::cpu_reference_scaled(w, as_half(x, K), as_half(s, N), yv, K, N);
  std::memcpy(y, yv.data(), (size_t)N * sizeof(double));
}

void ref_cosine_stats(const uint16_t* got, const double* want, int N, double* out3) {
  std::vector<double> wv(want, want + N);
  ref8::cosine_stats(as_half(got, N), wv, N, out3[0], out3[1], out3[2]);
}

// ---------------------------------------------------------------------------
// Multi-threaded driver around the reference's own fp64 loop, for the CPU
// baseline.  The K rows are cut into one contiguous slab per thread (set up
// once, outside any timed region); each thread runs cpu_reference_e4m3 or
// cpu_reference_fp16 unchanged on its slab, and the slab results are summed
// in slab order.
// ---------------------------------------------------------------------------
struct RefCpuPlan {
  int K, N, nthreads, wtype;
  std::vector<int> k0;
  std::vector<std::vector<uint8_t>> w8;
  std::vector<std::vector<__half>> w16;
};

void* ref_cpu_plan_create(const void* W, int wtype, int K, int N, int nthreads) {
  if (nthreads < 1) nthreads = 1;
  if (nthreads > K) nthreads = K;
  auto* p = new RefCpuPlan{K, N, nthreads, wtype, {}, {}, {}};
  for (int t = 0; t <= nthreads; ++t) p->k0.push_back((int)((long)K * t / nthreads));
  for (int t = 0; t < nthreads; ++t) {
    const size_t a = (size_t)p->k0[t] * N, b = (size_t)p->k0[t + 1] * N;
    if (wtype == 1) {
      const uint8_t* w = (const uint8_t*)W;
      p->w8.emplace_back(w + a, w + b);
    } else {
      p->w16.push_back(as_half((const uint16_t*)W + a, b - a));
    }
  }
  return p;
}

// x is [M, K] fp16 bits; y is [M, N] doubles.
void ref_cpu_plan_run(void* plan, const uint16_t* x, int M, double* y) {
  auto* p = (RefCpuPlan*)plan;
  std::vector<std::vector<double>> part(p->nthreads);
  for (int m = 0; m < M; ++m) {
    std::vector<std::thread> th;
    for (int t = 0; t < p->nthreads; ++t) {
      th.emplace_back([p, t, m, x, &part]() {
        const int ks = p->k0[t], kn = p->k0[t + 1] - p->k0[t];
        std::vector<__half> xs = as_half(x + (size_t)m * p->K + ks, kn);
        if (p->wtype == 1) ref8::cpu_reference_e4m3(p->w8[t], xs, part[t], kn, p->N);
        else ref8::cpu_reference_fp16(p->w16[t], xs, part[t], kn, p->N);
      });
    }
    for (auto& t : th) t.join();
    double* yr = y + (size_t)m * p->N;
    for (int n = 0; n < p->N; ++n) yr[n] = 0.0;
    for (int t = 0; t < p->nthreads; ++t)
      for (int n = 0; n < p->N; ++n) yr[n] += part[t][n];
  }
}

void ref_cpu_plan_destroy(void* plan) { delete (RefCpuPlan*)plan; }

}  // extern "C"
