// ref_gpu_shim.cu -- the reference project's own GPU GEMV path
// (kernels/gemv_fp8.cu run_gemv :276-283 -> gemv_chunk_kernel :91-151 ->
// cast_f32_to_f16_kernel :153-157; kernels/gemv_fp16.cu run_gemv :262-271),
// compiled unmodified for sm_100a and exposed through a C ABI so the
// benchmark can time it beside this library.  Baseline only: the library
// never loads it.
//
// The reference sources are #included from where they lie (paths given by
// baseline/Makefile), each in its own namespace; nothing is copied.  Output
// goes to baseline/_ref/ only.
#include <cstdio>
#include <cstdlib>
#include <cstdint>
#include <cstring>
#include <cmath>
#include <string>
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

extern "C" {

// One reference FP8 GEMV (M = 1) on the legacy default stream: memset of
// y_acc, gemv_chunk_kernel<variant>, cast.  N must be 8192 or 3072 (the
// reference exits otherwise, kernels/gemv_fp8.cu:270-273, so this checks
// first).  Returns the CUDA error of the launches.
int ref_gpu_gemv_fp8(const void* w, const void* x, float* y_acc, void* y, int K, int N, int variant,
                     int grid, int ku) {
  if (N != 8192 && N != 3072) return (int)cudaErrorInvalidValue;
  ref8::run_gemv(w, static_cast<const __half*>(x), y_acc, static_cast<__half*>(y), K, N, variant, grid, ku);
  return (int)cudaGetLastError();
}

// One reference FP16 GEMV (M = 1), kernels/gemv_fp16.cu:262-271.
int ref_gpu_gemv_fp16(const void* w, const void* x, float* y_acc, void* y, int K, int N, int variant,
                      int grid) {
  if (N != 8192 && N != 3072) return (int)cudaErrorInvalidValue;
  ref16::run_gemv(w, static_cast<const __half*>(x), y_acc, static_cast<__half*>(y), K, N, variant, grid);
  return (int)cudaGetLastError();
}

// The reference's shipped configuration (tuned on an L4):
// kernels/gemv_fp8.cu:232-234, kernels/gemv_fp16.cu:226-227.
int ref_gpu_fp8_best_variant(void) { return ref8::kBestVariant; }
int ref_gpu_fp8_best_grid(int N) { return ref8::best_grid(N); }
int ref_gpu_fp8_best_ku(int N) { return ref8::best_ku(N); }
int ref_gpu_fp16_best_variant(void) { return ref16::kBestVariant; }
int ref_gpu_fp16_best_grid(int N) { return ref16::best_grid(N); }

}  // extern "C"
