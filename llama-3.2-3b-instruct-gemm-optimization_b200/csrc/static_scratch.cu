// static_scratch.cu -- the fixed device scratch behind b2g_enqueue_static.
//
// The GEMV kernels need a workspace (tile counters + split-K partials).  The
// regular entry points take it from the caller; b2g_enqueue_static uses this
// file-scope array instead, so a caller that cannot allocate device memory
// can still run an op.  The array is zero-filled when the module loads; the
// host clears the tile counters before every launch anyway, since a launch
// that was abandoned may have left them non-zero.  There is one array per
// device and no lock around it: calls that overlap on the device (other
// streams, other host threads) race on it.
#include "../../include/b200gemv.h"
#include "gemv.h"

namespace b2g {

static_assert(B2G_STATIC_SCRATCH_BYTES % 256 == 0, "scratch size must keep 256-byte alignment");
static_assert(B2G_STATIC_SCRATCH_BYTES > kCounterRegionBytes, "scratch must hold the counter region");

static __device__ __align__(256) uint8_t g_static_scratch[B2G_STATIC_SCRATCH_BYTES];

cudaError_t static_scratch_address(void** ptr) {
  return cudaGetSymbolAddress(ptr, g_static_scratch);
}

}  // namespace b2g
