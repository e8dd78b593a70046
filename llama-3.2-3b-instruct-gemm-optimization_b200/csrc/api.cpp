// api.cpp -- the C ABI (include/b200gemv.h): op planning, validation,
// prepack/quantise, enqueue and the decode-MLP stack driver.
//
// Host-side replacement of the reference's launch plumbing
// (kernels/gemv_fp8.cu:192-283, kernels/gemv_fp16.cu:198-271): instead of a
// compile-time table of (threads, rows, vectors) variants for N in
// {8192, 3072} and a tuned split count, the plan below derives the stream-K
// partition, pipeline depth and shared-memory layout from the shape and the
// device (SM count, shared memory per block).
#include <algorithm>
#include <atomic>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <new>
#include <vector>

#include "../../include/b200gemv.h"
#include "gemv.h"

using namespace b2g;

struct b2g_op {
  b2g_fields f;
  int planes, wbytes, kpb;
  int K, N, Kp, n_tiles, kb_total, ksplit, kbpv;
  long long total_units;
  int unit_bytes;
  size_t packed_bytes;
  int device, num_sms, smem_optin, smem_per_sm;
  int grid, grid_override, ksplit_override;
  int partition, gran;  // B2G_PARTITION_* requested; units per granule in use
  long long total_gran;
  int max_contrib, n_slots, xk_cap;
  int math;
  int pipe;  // B2G_PIPE_* requested
};

struct b2g_stack {
  b2g_stack_fields f;
  b2g_op* gu;
  b2g_op* dn;
  int mode;  // B2G_STACK_MODE_*
  struct Layer {
    const void *pgu, *sgu, *pd, *sd;
  };
  std::vector<Layer> layers;
};

namespace {

constexpr int kMaxM = 8;

b2g_status cuda_status(cudaError_t e) { return e == cudaSuccess ? B2G_OK : B2G_ERR_CUDA; }

std::mutex g_mu;
bool g_limit_set[64];
int* g_err_word[64];
// Launches enqueued so far (a trace build files each launch's phase
// timestamps under this count).
std::atomic<unsigned> g_launch_count{0};

// L2 prefetch depth: the first bytes of each next-launch CTA's range that a
// launch warms (the start is what the next CTA's register ring asks for
// first).  The fills compete with the launch's own critical path (its late
// CTAs' first loads, the activation staging), so deeper is not better.  Per
// decode layer (gate||up on 128 CTAs, down on 96), 128 / 256 / 512 KB:
// M = 8 20.29 / 20.12 / 20.88 us; M = 1 18.90 / 19.34 / 19.60.  What pays
// at small M is warming less of a fused gate||up launch (393 KB per CTA)
// while the down launch runs; down's own 256 KB ranges are best warmed
// whole.  128 KB for a next gate||up launch up to M = 4, 256 KB otherwise:
// M = 1 / 2 / 4 / 8 18.69 / 19.19 / 19.57 / 20.10 us, against 19.27 /
// 19.64 / 19.81 / 20.12 with 256 KB everywhere, and a chain of down GEMVs
// at M = 1 keeps its 7.13 us (7.84 with 128 KB).
constexpr int kPrefetchBytesPerCta = 256 * 1024;
constexpr int kPrefetchBytesSmallM = 128 * 1024;  // a next two-plane launch at M <= 4
// The TMA pipeline issues its prefetch once its own copies are all issued,
// and asks for whole ranges (the next launch then streams from L2).
constexpr int kPrefetchBytesTma = 1 << 30;

b2g_status ensure_device_setup(int dev, int smem_optin) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (dev < 0 || dev >= 64) return B2G_ERR_UNSUPPORTED;
  if (!g_limit_set[dev]) {
    if (gemv_set_smem_limit(smem_optin) != cudaSuccess) return B2G_ERR_CUDA;
    int* w = device_error_word();
    if (!w) return B2G_ERR_CUDA;
    g_err_word[dev] = w;
    g_limit_set[dev] = true;
  }
  return B2G_OK;
}

// K ranges: `want` if it is valid (0 = automatic).  Automatic keeps K whole
// while max_m activation rows fit in 128 KB of shared memory (whole rows cost
// one staging copy but need no cross-range reduction; measured faster on
// B200), else the largest of 8/4/2 that leaves each range >= 2048 k.  A range
// must hold whole k-blocks and a multiple of 32 k; RMSNorm needs whole rows in
// one CTA, so no split.
int choose_ksplit(const b2g_op* op, int want) {
  auto ok = [&](int ks) {
    return ks >= 1 && op->kb_total % ks == 0 && ((op->kb_total / ks) * op->kpb) % 32 == 0;
  };
  if (op->f.fuse & B2G_FUSE_RMSNORM_INPUT) return want <= 1 ? 1 : -1;
  if (want > 0) return ok(want) ? want : -1;
  if ((long long)op->f.max_m * op->Kp * 2 <= 128 * 1024) return 1;
  for (int ks : {8, 4, 2})
    if (op->K / ks >= 2048 && ok(ks)) return ks;
  return 1;
}

// The partition (mirrors cta_of / range_start in gemv.cu): CTA c streams
// granules [c*Tg/G, (c+1)*Tg/G) of gran units each.
long long range_start(const b2g_op* op, long long c) { return c * op->total_gran / op->grid * op->gran; }
long long cta_of(const b2g_op* op, long long u) {
  const long long Tg = op->total_gran;
  return ((u / op->gran + 1) * op->grid + Tg - 1) / Tg - 1;
}

// Partition statistics for the op's grid.
void plan_partition(b2g_op* op) {
  const int G = op->grid;
  int max_slots = 0, max_kx = 0;
  const int kx_per_ks = op->kbpv * op->kpb / 32;
  for (int c = 0; c < G; ++c) {
    const long long u0 = range_start(op, c), u1 = range_start(op, c + 1);
    if (u1 <= u0) continue;
    const long long vf = u0 / op->kbpv, vl = (u1 - 1) / op->kbpv;
    max_slots = std::max(max_slots, (int)(vl - vf + 1));
    const int ks_lo = (int)(vf / op->n_tiles), ks_hi = (int)(vl / op->n_tiles);
    max_kx = std::max(max_kx, (ks_hi + 1 - ks_lo) * kx_per_ks);
  }
  int max_contrib = 1;
  const long long n_vt = (long long)op->ksplit * op->n_tiles;
  for (long long vt = 0; vt < n_vt; ++vt) {
    const long long a = vt * op->kbpv;
    max_contrib = std::max(max_contrib, (int)(cta_of(op, a + op->kbpv - 1) - cta_of(op, a)) + 1);
  }
  op->n_slots = max_slots;
  op->xk_cap = max_kx;
  op->max_contrib = max_contrib;
}

struct LaunchPlan {
  int off_epi, off_x, x_rs;
  size_t smem;
  // TMA pipeline: the weight ring after the x rows (0 stages: does not fit)
  int off_ring, n_stages;
  size_t smem_tma;
};

// Shared memory per CTA (one CTA per SM): flags, the per-warp partial slots,
// and the M staged activation rows.
bool plan_launch(const b2g_op* op, int m, LaunchPlan* lp) {
  // Row stride = 32 (E4M3) or 16 (FP16) halves mod 64, so the eight rows of a
  // B fragment load fall in distinct banks.
  const int krange = op->xk_cap * 32;
  const int x_rs = (krange + 63) / 64 * 64 + (op->wbytes == 1 ? 32 : 16);
  const size_t xbytes = ((size_t)m * x_rs * 2 + 127) / 128 * 128;
  const size_t slot_bytes = (size_t)op->n_slots * kWarps * op->planes * kUnitPlaneBytes;
  const size_t epi_bytes = ((size_t)op->n_slots * (op->planes * 16 + 8 * 16) * 4 + 127) / 128 * 128;
  lp->off_epi = (int)(kOffSlots + slot_bytes);
  lp->off_x = (int)(lp->off_epi + epi_bytes);
  lp->x_rs = x_rs;
  lp->smem = lp->off_x + xbytes;
  // TMA pipeline: as many 16 KB stages as the rest of the opt-in shared
  // memory holds (at least 2, at most kMaxStages).
  lp->off_ring = (int)((lp->smem + 1023) / 1024 * 1024);
  const long long room = (long long)op->smem_optin - lp->off_ring;
  lp->n_stages = room >= 2LL * kStageBytes ? (int)std::min<long long>(kMaxStages, room / kStageBytes) : 0;
  lp->smem_tma = (size_t)lp->off_ring + (size_t)lp->n_stages * kStageBytes;
  return lp->smem <= (size_t)op->smem_optin;
}

// Whether calls with m rows run on the TMA pipeline.  AUTO keeps the
// register pipeline: measured per decode layer on B200 (28 layers,
// per-layer launches, both kernels loading their scales before the
// dependency wait), both ops on registers 22.9 us at M = 8 and 22.1 at
// M = 1; gate||up on TMA 23.2-23.3 / 22.0-22.2; both on TMA 25.0 / 21.5.
bool use_tma(const b2g_op* op, const LaunchPlan& lp) {
  if (op->math != kMathMma || lp.n_stages < 2) return false;
  return op->pipe == B2G_PIPE_TMA;
}

// One planning pass for `want` CTAs.  *slots_full: the CTAs' ranges touch
// more virtual tiles than their shared slots hold.
b2g_status plan_at(b2g_op* op, long long want, bool* slots_full) {
  *slots_full = false;
  const long long n_vt = (long long)op->ksplit * op->n_tiles;
  bool aligned = op->partition == B2G_PARTITION_TILES;
  if (op->partition == B2G_PARTITION_AUTO) {
    // Whole virtual tiles per CTA remove the cross-CTA handshake of split
    // tiles, and the SMs the shrunk grid leaves idle take the next launch's
    // CTAs early (programmatic dependent launch), which start their weight
    // stream there.  Taken when nothing is split along K anyway and the
    // largest share is at most 1.6x the even share: down 8192->3072 (192
    // tiles, 2 per CTA on 96 CTAs against 1.3 on 148) measured 10.6 vs
    // 11.0 us per launch and 25.6 vs 27.2 us per decode layer.
    const long long g = std::min<long long>(n_vt, want);
    aligned = op->ksplit == 1 && (double)((n_vt + g - 1) / g) / ((double)n_vt / g) <= 1.6;
  }
  op->gran = aligned ? op->kbpv : 1;
  op->total_gran = op->total_units / op->gran;
  op->grid = (int)std::min<long long>(op->total_gran, want);
  if (aligned) {
    // The fewest CTAs that keep the same largest share of tiles: no CTA
    // waits on another that holds one tile more.
    const long long per = (op->total_gran + op->grid - 1) / op->grid;
    op->grid = (int)((op->total_gran + per - 1) / per);
  }
  // The kernels' partition arithmetic is 32-bit.
  if ((op->total_gran + 2) * (long long)op->grid >= (1LL << 31)) return B2G_ERR_UNSUPPORTED;
  plan_partition(op);
  if (op->n_slots > kMaxSlots) {
    *slots_full = true;
    return B2G_ERR_UNSUPPORTED;
  }
  LaunchPlan lp;
  if (!plan_launch(op, op->f.max_m, &lp)) return B2G_ERR_OOM;
  return B2G_OK;
}

b2g_status replan(b2g_op* op) {
  bool slots_full = false;
  if (op->grid_override > 0) return plan_at(op, op->grid_override, &slots_full);
  // One CTA per SM; or, when that hands a CTA more virtual tiles than its
  // shared slots hold (very wide outputs, e.g. a 3072 -> 128256 vocabulary
  // projection: 8016 tiles), the CTAs that keep each range within
  // kMaxSlots - 1 whole tiles (a split range touches one more), run as
  // successive waves.
  b2g_status st = plan_at(op, op->num_sms, &slots_full);
  const long long n_vt = (long long)op->ksplit * op->n_tiles;
  long long want = (n_vt + kMaxSlots - 2) / (kMaxSlots - 1);
  for (int i = 0; slots_full && i < 8; ++i, want += want / 4 + 1) st = plan_at(op, want, &slots_full);
  return st;
}

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// The plan-derived fields of one GEMV launch over `workspace` for m rows.
void fill_plan(const b2g_op* op, int m, const LaunchPlan& lp, void* workspace, int dev, GemvParams* p) {
  p->counters = static_cast<int*>(workspace);
  p->partials = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + kCounterRegionBytes);
  p->error = g_err_word[dev];
  p->total_units = op->total_units;
  p->gran = op->gran;
  p->div_gran = make_fast_div((uint32_t)op->gran);
  p->total_gran = (int)op->total_gran;
  p->div_tg = make_fast_div((uint32_t)op->total_gran);
  p->div_grid = make_fast_div((uint32_t)op->grid);
  p->grid = op->grid;
  p->n_tiles = op->n_tiles;
  p->kb_total = op->kb_total;
  p->ksplit = op->ksplit;
  p->kbpv = op->kbpv;
  p->div_kbpv = make_fast_div((uint32_t)op->kbpv);
  p->div_tiles = make_fast_div((uint32_t)op->n_tiles);
  p->M = m;
  p->K = op->K;
  p->N = op->N;
  p->scale_mode = op->f.scale_mode;
  p->rmsnorm = (op->f.fuse & B2G_FUSE_RMSNORM_INPUT) ? 1 : 0;
  p->residual_add = (op->f.fuse & B2G_FUSE_RESIDUAL_ADD) ? 1 : 0;
  p->max_contrib = op->max_contrib;
  p->n_slots = op->n_slots;
  p->off_epi = lp.off_epi;
  p->off_x = lp.off_x;
  p->x_rs = lp.x_rs;
}

}  // namespace

extern "C" {

const char* b2g_status_string(b2g_status s) {
  switch (s) {
    case B2G_OK: return "ok";
    case B2G_ERR_INVALID: return "invalid argument";
    case B2G_ERR_UNSUPPORTED: return "unsupported";
    case B2G_ERR_CUDA: return "CUDA error";
    case B2G_ERR_PEER_TIMEOUT: return "peer wait timed out";
    case B2G_ERR_OOM: return "out of shared memory or workspace";
    case B2G_ERR_DEVICE: return "device-side error";
    case B2G_ERR_SCRATCH_LIMIT: return "call needs more workspace than the static scratch (B2G_STATIC_SCRATCH_BYTES)";
  }
  return "unknown status";
}

int32_t b2g_version(void) { return 100; }

namespace {

// A new op with the fields checked and the derived sizes set (no device
// attributes yet, no plan).
b2g_status new_op(const b2g_fields* f, b2g_op** out) {
  *out = nullptr;
  if (f->in_features <= 0 || f->out_features <= 0) return B2G_ERR_INVALID;
  if (f->weight_dtype != B2G_DTYPE_FP16 && f->weight_dtype != B2G_DTYPE_FP8_E4M3) return B2G_ERR_INVALID;
  if (f->scale_mode < B2G_SCALE_NONE || f->scale_mode > B2G_SCALE_CHANNEL_FP32) return B2G_ERR_INVALID;
  if (f->weight_layout != B2G_LAYOUT_KN && f->weight_layout != B2G_LAYOUT_NK) return B2G_ERR_INVALID;
  if (f->max_m < 1 || f->max_m > kMaxM) return B2G_ERR_UNSUPPORTED;
  if (f->fuse & ~(B2G_FUSE_GATE_UP_SILU | B2G_FUSE_RMSNORM_INPUT | B2G_FUSE_RESIDUAL_ADD))
    return B2G_ERR_INVALID;
  if ((f->fuse & B2G_FUSE_GATE_UP_SILU) && (f->fuse & B2G_FUSE_RESIDUAL_ADD)) return B2G_ERR_UNSUPPORTED;
  if (f->tp_size < 0 || (f->tp_size > 0 && (f->tp_rank < 0 || f->tp_rank >= f->tp_size)))
    return B2G_ERR_INVALID;

  b2g_op* op = new (std::nothrow) b2g_op();
  if (!op) return B2G_ERR_OOM;
  op->f = *f;
  op->planes = (f->fuse & B2G_FUSE_GATE_UP_SILU) ? 2 : 1;
  op->wbytes = f->weight_dtype == B2G_DTYPE_FP8_E4M3 ? 1 : 2;
  op->kpb = op->wbytes == 1 ? 32 : 16;
  op->K = f->in_features;
  op->N = f->out_features;
  op->Kp = (op->K + 31) / 32 * 32;
  op->kb_total = op->Kp / op->kpb;
  op->n_tiles = (op->N + kTileCh - 1) / kTileCh;
  if (op->n_tiles > kMaxTiles || ((f->fuse & B2G_FUSE_RMSNORM_INPUT) && (op->K % 8) != 0)) {
    delete op;
    return B2G_ERR_UNSUPPORTED;
  }
  op->ksplit = choose_ksplit(op, 0);
  op->kbpv = op->kb_total / op->ksplit;
  op->total_units = (long long)op->n_tiles * op->kb_total;
  if (op->total_units >= (1LL << 30)) {
    delete op;
    return B2G_ERR_UNSUPPORTED;
  }
  op->unit_bytes = op->planes * kUnitPlaneBytes;
  op->packed_bytes = (size_t)op->total_units * op->unit_bytes;
  op->math = kMathMma;
  *out = op;
  return B2G_OK;
}

}  // namespace

b2g_status b2g_create(const b2g_fields* f, b2g_op** out) {
  if (!f || !out) return B2G_ERR_INVALID;
  b2g_op* op = nullptr;
  b2g_status st = new_op(f, &op);
  if (st != B2G_OK) {
    *out = nullptr;
    return st;
  }
  cudaError_t e = cudaGetDevice(&op->device);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&op->num_sms, cudaDevAttrMultiProcessorCount, op->device);
  if (e == cudaSuccess)
    e = cudaDeviceGetAttribute(&op->smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, op->device);
  if (e == cudaSuccess)
    e = cudaDeviceGetAttribute(&op->smem_per_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, op->device);
  if (e != cudaSuccess) {
    delete op;
    return B2G_ERR_CUDA;
  }
  st = replan(op);
  if (st != B2G_OK) {
    delete op;
    return st;
  }
  *out = op;
  return B2G_OK;
}

b2g_status b2g_plan_for_device(const b2g_fields* f, int32_t num_sms, int32_t smem_optin, int32_t m,
                               b2g_plan_info* info, size_t* packed_bytes, size_t* workspace_bytes) {
  if (!f || !info || num_sms < 1 || smem_optin < 1) return B2G_ERR_INVALID;
  b2g_op* op = nullptr;
  b2g_status st = new_op(f, &op);
  if (st != B2G_OK) return st;
  op->device = -1;
  op->num_sms = num_sms;
  op->smem_optin = smem_optin;
  op->smem_per_sm = smem_optin;
  st = replan(op);
  if (st == B2G_OK) st = b2g_op_query(op, m, info);
  if (st == B2G_OK && packed_bytes) st = b2g_prepack_size(op, packed_bytes);
  if (st == B2G_OK && workspace_bytes) st = b2g_workspace_size(op, m, workspace_bytes);
  delete op;
  return st;
}

b2g_status b2g_destroy(b2g_op* op) {
  delete op;
  return B2G_OK;
}

static b2g_status set_option_unchecked(b2g_op* op, int32_t key, int32_t value);

// An option that leaves no valid plan is refused and the op keeps its plan.
b2g_status b2g_op_set_option(b2g_op* op, int32_t key, int32_t value) {
  if (!op) return B2G_ERR_INVALID;
  const b2g_op saved = *op;
  const b2g_status st = set_option_unchecked(op, key, value);
  if (st != B2G_OK) *op = saved;
  return st;
}

static b2g_status set_option_unchecked(b2g_op* op, int32_t key, int32_t value) {
  switch (key) {
    case B2G_OPT_MATH:
      if (value != kMathMma && value != kMathFfma) return B2G_ERR_INVALID;
      op->math = value;
      return replan(op);
    case B2G_OPT_GRID:
      if (value < 0) return B2G_ERR_INVALID;
      op->grid_override = value;
      return replan(op);
    case B2G_OPT_PARTITION:
      if (value < B2G_PARTITION_AUTO || value > B2G_PARTITION_TILES) return B2G_ERR_INVALID;
      op->partition = value;
      return replan(op);
    case B2G_OPT_PIPE:
      if (value < B2G_PIPE_AUTO || value > B2G_PIPE_TMA) return B2G_ERR_INVALID;
      op->pipe = value;
      return replan(op);
    case B2G_OPT_KSPLIT: {
      const int ks = choose_ksplit(op, value);
      if (value < 0 || ks < 1) return B2G_ERR_INVALID;
      op->ksplit_override = value;
      op->ksplit = ks;
      op->kbpv = op->kb_total / ks;
      return replan(op);
    }
  }
  return B2G_ERR_INVALID;
}

b2g_status b2g_op_query(const b2g_op* op, int32_t m, b2g_plan_info* info) {
  if (!op || !info || m < 1 || m > op->f.max_m) return B2G_ERR_INVALID;
  LaunchPlan lp;
  if (!plan_launch(op, m, &lp)) return B2G_ERR_OOM;
  info->grid = op->grid;
  info->ksplit = op->ksplit;
  info->kblocks_per_vtile = op->kbpv;
  info->n_tiles = op->n_tiles;
  info->total_units = op->total_units;
  info->unit_bytes = op->unit_bytes;
  info->inflight_bytes_per_cta = (int64_t)kThreads * 16 * kRing;  // 16 B x kRing per thread, any plane count
  info->smem_bytes = (int64_t)lp.smem;
  info->max_contrib = op->max_contrib;
  info->partition = op->gran == 1 ? B2G_PARTITION_UNITS : B2G_PARTITION_TILES;
  info->n_slots = op->n_slots;
  info->x_kblocks = op->xk_cap;
  info->math = op->math;
  const bool tma = use_tma(op, lp);
  info->pipe = tma ? B2G_PIPE_TMA : B2G_PIPE_REGISTERS;
  info->n_stages = tma ? lp.n_stages : 0;
  info->stage_bytes = tma ? kStageBytes : 0;
  if (tma) {
    info->smem_bytes = (int64_t)lp.smem_tma;
    info->inflight_bytes_per_cta = (int64_t)lp.n_stages * kStageBytes;
  }
  return B2G_OK;
}

b2g_status b2g_prepack_size(const b2g_op* op, size_t* bytes) {
  if (!op || !bytes) return B2G_ERR_INVALID;
  *bytes = op->packed_bytes;
  return B2G_OK;
}

b2g_status b2g_prepack(const b2g_op* op, const void* w0, const void* w1, int64_t ld, void* packed,
                       b2g_stream_t stream) {
  if (!op || !w0 || !packed) return B2G_ERR_INVALID;
  if (op->planes == 2 && !w1) return B2G_ERR_INVALID;
  if (op->planes == 1 && w1) return B2G_ERR_INVALID;
  if (!aligned(packed, 16)) return B2G_ERR_INVALID;
  const long long dense = op->f.weight_layout == B2G_LAYOUT_KN ? op->N : op->K;
  if (ld == 0) ld = dense;
  if (ld < dense) return B2G_ERR_INVALID;
  const void* planes[2] = {w0, w1};
  for (int pl = 0; pl < op->planes; ++pl) {
    cudaError_t e = launch_prepack(planes[pl], ld, op->f.weight_layout, op->wbytes, op->K, op->N, pl,
                                   op->planes, op->ksplit, op->kbpv, op->n_tiles, op->kb_total,
                                   static_cast<uint8_t*>(packed), reinterpret_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return B2G_ERR_CUDA;
  }
  return B2G_OK;
}

b2g_status b2g_quantize_e4m3(const void* w16, int32_t K, int32_t N, int32_t layout, int32_t scale_mode,
                             void* w8, void* scales, b2g_stream_t stream) {
  if (!w16 || !w8 || K <= 0 || N <= 0) return B2G_ERR_INVALID;
  if (layout != B2G_LAYOUT_KN && layout != B2G_LAYOUT_NK) return B2G_ERR_INVALID;
  if (scale_mode < B2G_SCALE_NONE || scale_mode > B2G_SCALE_CHANNEL_FP32) return B2G_ERR_INVALID;
  if (scale_mode != B2G_SCALE_NONE && !scales) return B2G_ERR_INVALID;
  return cuda_status(launch_quantize(static_cast<const __half*>(w16), K, N, layout, scale_mode,
                                     static_cast<uint8_t*>(w8), scales,
                                     reinterpret_cast<cudaStream_t>(stream)));
}

static size_t ws_partials_bytes(const b2g_op* op) {
  return (size_t)op->ksplit * op->n_tiles * op->max_contrib * op->planes * kUnitPlaneBytes;
}

b2g_status b2g_workspace_size(const b2g_op* op, int32_t m, size_t* bytes) {
  if (!op || !bytes || m < 1 || m > op->f.max_m) return B2G_ERR_INVALID;
  *bytes = kCounterRegionBytes + ws_partials_bytes(op);
  return B2G_OK;
}

b2g_status b2g_workspace_init(const b2g_op* op, void* ws, b2g_stream_t stream) {
  if (!op || !ws) return B2G_ERR_INVALID;
  size_t bytes = 0;
  b2g_workspace_size(op, op->f.max_m, &bytes);
  return cuda_status(cudaMemsetAsync(ws, 0, bytes, reinterpret_cast<cudaStream_t>(stream)));
}

static b2g_status enqueue_impl(const b2g_op* op, const b2g_enqueue_args* a, const TpParams* tp,
                               b2g_stream_t stream);

b2g_status b2g_enqueue_ex(const b2g_op* op, const b2g_enqueue_args* a, b2g_stream_t stream) {
  return enqueue_impl(op, a, nullptr, stream);
}

// The checks of an enqueue's arguments that need no device (the workspace
// pointer is checked unless `own_workspace`: the static entry point supplies it).
static b2g_status check_args(const b2g_op* op, const b2g_enqueue_args* a, bool own_workspace) {
  if (!op || !a) return B2G_ERR_INVALID;
  if (a->m < 1 || a->m > op->f.max_m) return B2G_ERR_INVALID;
  if (!a->x || !a->packed_w || !a->y || (!own_workspace && !a->workspace)) return B2G_ERR_INVALID;
  if (op->f.scale_mode != B2G_SCALE_NONE && !a->scales) return B2G_ERR_INVALID;
  const bool resid = (op->f.fuse & B2G_FUSE_RESIDUAL_ADD) != 0;
  if (resid && !a->residual) return B2G_ERR_INVALID;
  if (a->ldx < op->K || a->ldy < op->N || (resid && a->ldr < op->N)) return B2G_ERR_INVALID;
  if (!aligned(a->packed_w, 16) || (!own_workspace && !aligned(a->workspace, 16))) return B2G_ERR_INVALID;
  if (!aligned(a->x, 2) || !aligned(a->y, 2)) return B2G_ERR_INVALID;
  if (op->f.scale_mode == B2G_SCALE_CHANNEL_FP32 && !aligned(a->scales, 4)) return B2G_ERR_INVALID;
  if (a->prefetch_op && a->prefetch_packed && !aligned(a->prefetch_packed, 16)) return B2G_ERR_INVALID;
  LaunchPlan lp;
  if (!plan_launch(op, a->m, &lp)) return B2G_ERR_OOM;
  return B2G_OK;
}

static b2g_status enqueue_impl(const b2g_op* op, const b2g_enqueue_args* a, const TpParams* tp,
                               b2g_stream_t stream) {
  b2g_status st = check_args(op, a, false);
  if (st != B2G_OK) return st;
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) return B2G_ERR_CUDA;
  if (dev != op->device) return B2G_ERR_INVALID;
  st = ensure_device_setup(dev, op->smem_optin);
  if (st != B2G_OK) return st;
  LaunchPlan lp;
  plan_launch(op, a->m, &lp);

  GemvParams p = {};
  fill_plan(op, a->m, lp, a->workspace, dev, &p);
  p.packed = static_cast<const uint8_t*>(a->packed_w);
  p.x = static_cast<const __half*>(a->x);
  p.ldx = a->ldx;
  p.scales = a->scales;
  p.residual = static_cast<const __half*>(a->residual);
  p.ldr = a->ldr;
  p.y = static_cast<__half*>(a->y);
  p.ldy = a->ldy;
  p.rms_eps = a->rms_eps;
  if (a->prefetch_op && a->prefetch_packed) {
    const b2g_op* nx = a->prefetch_op;
    p.pf_packed = static_cast<const uint8_t*>(a->prefetch_packed);
    p.pf_total_units = nx->total_units;
    p.pf_gran = nx->gran;
    p.pf_unit_bytes = nx->unit_bytes;
    p.pf_grid = nx->grid;
    p.pf_bytes = use_tma(op, lp)                  ? kPrefetchBytesTma
                 : (a->m <= 4 && nx->planes == 2) ? kPrefetchBytesSmallM
                                                  : kPrefetchBytesPerCta;
  }
  if (tp) p.tp = *tp;
  p.trace_slot = (int)(g_launch_count.fetch_add(1, std::memory_order_relaxed) & 0x3fffffff);
  // One contributor per output tile (no K split, no tile shared between
  // CTAs) and aligned rows: the lean kernel flavor.
  const bool resid = (op->f.fuse & B2G_FUSE_RESIDUAL_ADD) != 0;
  p.lean = op->ksplit == 1 && op->max_contrib == 1 && aligned(a->x, 16) && a->ldx % 8 == 0 && op->K % 32 == 0 &&
           (!resid || (aligned(a->residual, 16) && a->ldr % 8 == 0));
  if (tp && tp->mode == kTpReduce) {
    // The REDUCE flavor is the lean one: whole tiles, aligned rows; y takes
    // 4-byte pieces; one round count per CTA; register pipeline only.
    if (!p.lean || p.grid > kTpMaxCtas || !aligned(a->y, 4) || a->ldy % 2 != 0) return B2G_ERR_INVALID;
    if (use_tma(op, lp)) return B2G_ERR_UNSUPPORTED;
  }
  if (use_tma(op, lp)) {
    p.off_ring = lp.off_ring;
    p.n_stages = lp.n_stages;
    p.stage_bytes = kStageBytes;
    return cuda_status(launch_gemv_tma(p, op->planes, op->wbytes, lp.smem_tma, a->pdl != 0,
                                       reinterpret_cast<cudaStream_t>(stream)));
  }
  return cuda_status(launch_gemv(p, op->planes, op->wbytes, op->math, lp.smem, a->pdl != 0,
                                 reinterpret_cast<cudaStream_t>(stream)));
}

b2g_status b2g_enqueue(const b2g_op* op, int32_t m, const void* x, const void* packed_w, const void* scales,
                       void* y, void* workspace, b2g_stream_t stream) {
  if (!op) return B2G_ERR_INVALID;
  if (op->f.fuse & B2G_FUSE_RESIDUAL_ADD) return B2G_ERR_INVALID;  // needs b2g_enqueue_ex
  b2g_enqueue_args a = {};
  a.m = m;
  a.x = x;
  a.ldx = op->K;
  a.packed_w = packed_w;
  a.scales = scales;
  a.y = y;
  a.ldy = op->N;
  a.workspace = workspace;
  a.rms_eps = 1e-5f;
  a.pdl = 0;
  return b2g_enqueue_ex(op, &a, stream);
}

b2g_status b2g_device_error(int32_t* code, int32_t clear) {
  if (!code) return B2G_ERR_INVALID;
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) return B2G_ERR_CUDA;
  int* w = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (dev >= 0 && dev < 64) w = g_err_word[dev];
  }
  if (!w) {
    *code = 0;
    return B2G_OK;
  }
  if (cudaDeviceSynchronize() != cudaSuccess) return B2G_ERR_CUDA;
  int v = 0;
  if (cudaMemcpy(&v, w, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return B2G_ERR_CUDA;
  *code = v;
  if (clear && cudaMemset(w, 0, sizeof(int)) != cudaSuccess) return B2G_ERR_CUDA;
  return B2G_OK;
}

// ---------------------------------------------------------------------------
// No-allocation enqueue: b2g_enqueue_ex over the library's static scratch
// ---------------------------------------------------------------------------
static void* g_static_ws[64];  // scratch address per device, under g_mu

b2g_status b2g_enqueue_static(const b2g_op* op, const b2g_enqueue_args* args, b2g_stream_t stream) {
  if (!op || !args || args->workspace) return B2G_ERR_INVALID;
  size_t need = 0;
  b2g_status st = b2g_workspace_size(op, args->m, &need);
  if (st != B2G_OK) return st;
  if (need > B2G_STATIC_SCRATCH_BYTES) return B2G_ERR_SCRATCH_LIMIT;
  // Every argument is checked before anything is queued: a refused call
  // leaves the stream untouched.
  st = check_args(op, args, true);
  if (st != B2G_OK) return st;
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) return B2G_ERR_CUDA;
  if (dev != op->device || dev < 0 || dev >= 64) return B2G_ERR_INVALID;
  st = ensure_device_setup(dev, op->smem_optin);
  if (st != B2G_OK) return st;
  void* ws = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_static_ws[dev]) {
      void* p = nullptr;
      if (static_scratch_address(&p) != cudaSuccess || !p) return B2G_ERR_CUDA;
      g_static_ws[dev] = p;
    }
    ws = g_static_ws[dev];
  }
  // The tile counters must start at zero; nothing else in the scratch must.
  if (cudaMemsetAsync(ws, 0, (size_t)op->n_tiles * sizeof(int), reinterpret_cast<cudaStream_t>(stream)) !=
      cudaSuccess)
    return B2G_ERR_CUDA;
  b2g_enqueue_args a = *args;
  a.workspace = ws;
  a.pdl = 0;
  return b2g_enqueue_ex(op, &a, stream);
}

// ---------------------------------------------------------------------------
// Tensor-parallel exchange through peer memory
// ---------------------------------------------------------------------------
// The inbox holds either mode's buffers: PUSH / GATHER [2][world][max_m][width]
// fp16, REDUCE [2][world][max_m][width / 2] u64 (twice the bytes).
static size_t tp_inbox_bytes(int world, int max_m, int width) {
  return ((size_t)2 * world * max_m * (width / 2) * 8 + 255) / 256 * 256;
}

// After the inbox: the counter region (PUSH counters [world]), then the
// epoch region (epoch at word 0, REDUCE per-CTA rounds [kTpMaxCtas] at word
// kTpRoundsOffset).
static_assert(B2G_TP_MAX_CTAS == kTpMaxCtas, "REDUCE CTA limit");
constexpr size_t kTpCounterRegion = 256;
constexpr size_t kTpEpochRegion = ((size_t)(kTpRoundsOffset + kTpMaxCtas) * 4 + 255) / 256 * 256;

size_t b2g_tp_comm_bytes(int32_t world, int32_t max_m, int32_t width) {
  if (world < 1 || world > B2G_TP_MAX_RANKS || max_m < 1 || width < 8) return 0;
  return tp_inbox_bytes(world, max_m, width) + kTpCounterRegion + kTpEpochRegion;
}

b2g_status b2g_tp_comm_layout(void* base, int32_t world, int32_t max_m, int32_t width, void** inbox,
                              void** counters, void** epoch) {
  if (!base || !inbox || !counters || !epoch || b2g_tp_comm_bytes(world, max_m, width) == 0) return B2G_ERR_INVALID;
  uint8_t* b = static_cast<uint8_t*>(base);
  const size_t ib = tp_inbox_bytes(world, max_m, width);
  *inbox = b;
  *counters = b + ib;
  *epoch = b + ib + kTpCounterRegion;
  return B2G_OK;
}

// An IPC handle names a whole allocation; a caching allocator may hand out
// a buffer inside a larger one, so the record also carries the offset from
// the allocation's base (cuMemGetAddressRange, through the driver entry point).
using MemGetAddressRangeFn = int (*)(unsigned long long* base, size_t* size, unsigned long long ptr);

static MemGetAddressRangeFn get_address_range_fn() {
  static MemGetAddressRangeFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      p = nullptr;
    return reinterpret_cast<MemGetAddressRangeFn>(p);
  }();
  return fn;
}

static std::mutex g_ipc_mu;
static std::vector<std::pair<void*, void*>> g_ipc_open;  // (returned address, mapped base)

b2g_status b2g_ipc_handle(const void* dev_ptr, void* record) {
  if (!dev_ptr || !record) return B2G_ERR_INVALID;
  static_assert(sizeof(cudaIpcMemHandle_t) + 8 == B2G_IPC_RECORD_BYTES, "IPC record size");
  const MemGetAddressRangeFn range = get_address_range_fn();
  if (!range) return B2G_ERR_CUDA;
  unsigned long long base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<unsigned long long>(dev_ptr)) != 0) return B2G_ERR_CUDA;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)) != cudaSuccess) return B2G_ERR_CUDA;
  const uint64_t off = reinterpret_cast<unsigned long long>(dev_ptr) - base;
  std::memcpy(record, &h, sizeof(h));
  std::memcpy(static_cast<uint8_t*>(record) + sizeof(h), &off, 8);
  return B2G_OK;
}

b2g_status b2g_ipc_open(const void* record, void** dev_ptr) {
  if (!record || !dev_ptr) return B2G_ERR_INVALID;
  cudaIpcMemHandle_t h;
  uint64_t off = 0;
  std::memcpy(&h, record, sizeof(h));
  std::memcpy(&off, static_cast<const uint8_t*>(record) + sizeof(h), 8);
  void* base = nullptr;
  if (cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return B2G_ERR_CUDA;
  *dev_ptr = static_cast<uint8_t*>(base) + off;
  std::lock_guard<std::mutex> lk(g_ipc_mu);
  g_ipc_open.emplace_back(*dev_ptr, base);
  return B2G_OK;
}

b2g_status b2g_ipc_close(void* dev_ptr) {
  if (!dev_ptr) return B2G_ERR_INVALID;
  void* base = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_ipc_mu);
    for (size_t i = 0; i < g_ipc_open.size(); ++i)
      if (g_ipc_open[i].first == dev_ptr) {
        base = g_ipc_open[i].second;
        g_ipc_open.erase(g_ipc_open.begin() + i);
        break;
      }
  }
  if (!base) return B2G_ERR_INVALID;
  return cuda_status(cudaIpcCloseMemHandle(base));
}

static b2g_status fill_tp(const b2g_tp_comm* c, int mode, int buf, const b2g_op* push_op, void* h_out,
                          int64_t ldh, int m, TpParams* tp) {
  if (!c || !push_op || c->world < 1 || c->world > B2G_TP_MAX_RANKS || c->rank < 0 || c->rank >= c->world)
    return B2G_ERR_INVALID;
  if ((buf != 0 && buf != 1) || c->width % 8 != 0 || m > c->max_m || !c->epoch) return B2G_ERR_INVALID;
  for (int r = 0; r < c->world; ++r)
    if (!c->inbox[r] || !c->counters[r] || !aligned(c->inbox[r], 16) || !aligned(c->counters[r], 4))
      return B2G_ERR_INVALID;
  if (mode == B2G_TP_GATHER && (!h_out || !aligned(h_out, 16) || ldh < c->width || ldh % 8 != 0))
    return B2G_ERR_INVALID;
  *tp = TpParams{};
  tp->mode = mode;
  tp->world = c->world;
  tp->rank = c->rank;
  tp->buf = buf;
  tp->push_grid = push_op->grid;
  tp->inbox_m = c->max_m;
  tp->width = c->width;
  for (int r = 0; r < c->world; ++r) {
    tp->inbox[r] = static_cast<__half*>(c->inbox[r]);
    tp->counters[r] = static_cast<unsigned*>(c->counters[r]);
  }
  tp->epoch = static_cast<unsigned*>(c->epoch);
  tp->h_out = static_cast<__half*>(h_out);
  tp->ldh = ldh;
  tp->rounds = tp->epoch + kTpRoundsOffset;
  return B2G_OK;
}

b2g_status b2g_enqueue_tp(const b2g_op* op, const b2g_enqueue_args* a, const b2g_tp_comm* comm, int32_t mode,
                          int32_t buf, const b2g_op* push_op, void* h_out, int64_t ldh, b2g_stream_t stream) {
  if (!op || !a || !comm) return B2G_ERR_INVALID;
  if (mode == B2G_TP_PUSH || mode == B2G_TP_REDUCE) {
    if (op->planes != 1 || op->N != comm->width || op->N % kTileCh != 0) return B2G_ERR_INVALID;
    push_op = op;
  } else if (mode == B2G_TP_GATHER) {
    if (!push_op || op->ksplit != 1 || op->K != comm->width || op->K % 32 != 0) return B2G_ERR_INVALID;
  } else {
    return B2G_ERR_INVALID;
  }
  TpParams tp;
  b2g_status st = fill_tp(comm, mode, buf, push_op, h_out, ldh, a->m, &tp);
  if (st != B2G_OK) return st;
  return enqueue_impl(op, a, &tp, stream);
}

b2g_status b2g_tp_gather(const b2g_tp_comm* comm, int32_t buf, const b2g_op* push_op, int32_t m, void* h,
                         int64_t ldh, b2g_stream_t stream) {
  if (!comm || !push_op || m < 1) return B2G_ERR_INVALID;
  TpParams tp;
  b2g_status st = fill_tp(comm, B2G_TP_GATHER, buf, push_op, h, ldh, m, &tp);
  if (st != B2G_OK) return st;
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) return B2G_ERR_CUDA;
  st = ensure_device_setup(dev, push_op->smem_optin);
  if (st != B2G_OK) return st;
  return cuda_status(launch_tp_gather(tp, m, g_err_word[dev], reinterpret_cast<cudaStream_t>(stream)));
}

// ---------------------------------------------------------------------------
// Stack
// ---------------------------------------------------------------------------
b2g_status b2g_stack_create(const b2g_stack_fields* f, b2g_stack** out) {
  if (!f || !out) return B2G_ERR_INVALID;
  *out = nullptr;
  if (f->hidden <= 0 || f->intermediate <= 0 || f->n_layers <= 0) return B2G_ERR_INVALID;
  if (f->tp_size > 1) return B2G_ERR_UNSUPPORTED;
  b2g_fields g = {};
  g.in_features = f->hidden;
  g.out_features = f->intermediate;
  g.weight_dtype = f->weight_dtype;
  g.scale_mode = f->scale_mode;
  g.weight_layout = B2G_LAYOUT_KN;
  g.max_m = f->max_m;
  g.fuse = B2G_FUSE_GATE_UP_SILU | B2G_FUSE_RMSNORM_INPUT;
  g.tp_rank = f->tp_rank;
  g.tp_size = f->tp_size;
  b2g_fields d = g;
  d.in_features = f->intermediate;
  d.out_features = f->hidden;
  d.fuse = B2G_FUSE_RESIDUAL_ADD;
  auto* st = new (std::nothrow) b2g_stack();
  if (!st) return B2G_ERR_OOM;
  st->f = *f;
  st->mode = B2G_STACK_MODE_PER_LAYER;
  b2g_status s = b2g_create(&g, &st->gu);
  if (s == B2G_OK) s = b2g_create(&d, &st->dn);
  if (s != B2G_OK) {
    b2g_destroy(st->gu);
    b2g_destroy(st->dn);
    delete st;
    return s;
  }
  st->layers.assign(f->n_layers, b2g_stack::Layer{nullptr, nullptr, nullptr, nullptr});
  *out = st;
  return B2G_OK;
}

b2g_status b2g_stack_destroy(b2g_stack* st) {
  if (!st) return B2G_OK;
  b2g_destroy(st->gu);
  b2g_destroy(st->dn);
  delete st;
  return B2G_OK;
}

b2g_status b2g_stack_ops(const b2g_stack* st, const b2g_op** gu, const b2g_op** dn) {
  if (!st) return B2G_ERR_INVALID;
  if (gu) *gu = st->gu;
  if (dn) *dn = st->dn;
  return B2G_OK;
}

b2g_status b2g_stack_set_layer(b2g_stack* st, int32_t l, const void* pgu, const void* sgu, const void* pd,
                               const void* sd) {
  if (!st || l < 0 || l >= st->f.n_layers || !pgu || !pd) return B2G_ERR_INVALID;
  if (st->f.scale_mode != B2G_SCALE_NONE && (!sgu || !sd)) return B2G_ERR_INVALID;
  st->layers[l] = b2g_stack::Layer{pgu, sgu, pd, sd};
  return B2G_OK;
}

b2g_status b2g_stack_workspace_size(const b2g_stack* st, int32_t m, size_t* bytes) {
  if (!st || !bytes) return B2G_ERR_INVALID;
  size_t a = 0, b = 0;
  b2g_status s = b2g_workspace_size(st->gu, m, &a);
  if (s == B2G_OK) s = b2g_workspace_size(st->dn, m, &b);
  *bytes = std::max(a, b);
  return s;
}

b2g_status b2g_stack_workspace_init(const b2g_stack* st, void* ws, b2g_stream_t stream) {
  if (!st || !ws) return B2G_ERR_INVALID;
  size_t bytes = 0;
  b2g_status s = b2g_stack_workspace_size(st, st->f.max_m, &bytes);
  if (s != B2G_OK) return s;
  return cuda_status(cudaMemsetAsync(ws, 0, bytes, reinterpret_cast<cudaStream_t>(stream)));
}

b2g_status b2g_stack_set_option(b2g_stack* st, int32_t key, int32_t value) {
  if (!st) return B2G_ERR_INVALID;
  if (key != B2G_STACK_OPT_MODE) return B2G_ERR_INVALID;
  if (value != B2G_STACK_MODE_PERSISTENT && value != B2G_STACK_MODE_PER_LAYER &&
      value != B2G_STACK_MODE_PERSISTENT_TMA)
    return B2G_ERR_INVALID;
  st->mode = value;
  return B2G_OK;
}

// All layers in cooperative launches of up to kMaxStackLayers layers each.
static b2g_status stack_enqueue_persistent(const b2g_stack* st, int32_t m, void* h, void* act, void* ws,
                                           cudaStream_t stream) {
  const b2g_op* gu = st->gu;
  const b2g_op* dn = st->dn;
  if (gu->wbytes != dn->wbytes) return B2G_ERR_UNSUPPORTED;
  const int grid = std::max(gu->grid, dn->grid);
  if (!aligned(ws, 16) || !aligned(h, 2) || !aligned(act, 2)) return B2G_ERR_INVALID;
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) return B2G_ERR_CUDA;
  if (dev != gu->device) return B2G_ERR_INVALID;
  b2g_status s = ensure_device_setup(dev, gu->smem_optin);
  if (s != B2G_OK) return s;
  LaunchPlan lg, ld;
  if (!plan_launch(gu, m, &lg) || !plan_launch(dn, m, &ld)) return B2G_ERR_OOM;
  const size_t smem = std::max(lg.smem, ld.smem);
  int max_grid = 0;
  if (stack_max_coresident(gu->wbytes, smem, gu->num_sms, &max_grid) != cudaSuccess) return B2G_ERR_CUDA;
  if (grid > max_grid) return B2G_ERR_UNSUPPORTED;
  StackParams sp = {};
  fill_plan(gu, m, lg, ws, dev, &sp.gu);
  fill_plan(dn, m, ld, ws, dev, &sp.dn);
  sp.gu.rms_eps = st->f.rms_eps;
  sp.h = static_cast<__half*>(h);
  sp.ldh = st->f.hidden;
  sp.act = static_cast<__half*>(act);
  sp.ldact = st->f.intermediate;
  sp.barrier = reinterpret_cast<unsigned*>(static_cast<uint8_t*>(ws) + kBarrierWordOffset);
  for (int l0 = 0; l0 < st->f.n_layers; l0 += kMaxStackLayers) {
    sp.n_layers = std::min(kMaxStackLayers, st->f.n_layers - l0);
    for (int i = 0; i < sp.n_layers; ++i) {
      const auto& L = st->layers[l0 + i];
      sp.layers[i] = StackLayer{static_cast<const uint8_t*>(L.pgu), L.sgu, static_cast<const uint8_t*>(L.pd),
                                L.sd};
    }
    if (launch_stack(sp, grid, gu->wbytes, smem, stream) != cudaSuccess) return B2G_ERR_CUDA;
  }
  return B2G_OK;
}

// All layers in cooperative launches of the TMA-pipeline stack kernel: one
// ring after the larger of the two phases' shared-memory layouts.
static b2g_status stack_enqueue_tma(const b2g_stack* st, int32_t m, void* h, void* act, void* ws,
                                    cudaStream_t stream) {
  const b2g_op* gu = st->gu;
  const b2g_op* dn = st->dn;
  if (gu->wbytes != dn->wbytes || gu->math != kMathMma || dn->math != kMathMma) return B2G_ERR_UNSUPPORTED;
  const int grid = std::max(gu->grid, dn->grid);
  if (!aligned(ws, 16) || !aligned(h, 2) || !aligned(act, 2)) return B2G_ERR_INVALID;
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) return B2G_ERR_CUDA;
  if (dev != gu->device) return B2G_ERR_INVALID;
  b2g_status s = ensure_device_setup(dev, gu->smem_optin);
  if (s != B2G_OK) return s;
  LaunchPlan lg, ld;
  if (!plan_launch(gu, m, &lg) || !plan_launch(dn, m, &ld)) return B2G_ERR_OOM;
  const int off_ring = std::max(lg.off_ring, ld.off_ring);
  const long long room = (long long)gu->smem_optin - off_ring;
  const int n_stages = (int)std::min<long long>(kMaxStages, room / kStageBytes);
  if (n_stages < 2) return B2G_ERR_UNSUPPORTED;
  const size_t smem = (size_t)off_ring + (size_t)n_stages * kStageBytes;
  int max_grid = 0;
  if (stack_tma_max_coresident(gu->wbytes, smem, gu->num_sms, &max_grid) != cudaSuccess) return B2G_ERR_CUDA;
  if (grid > max_grid) return B2G_ERR_UNSUPPORTED;
  StackParams sp = {};
  fill_plan(gu, m, lg, ws, dev, &sp.gu);
  fill_plan(dn, m, ld, ws, dev, &sp.dn);
  for (GemvParams* p : {&sp.gu, &sp.dn}) {
    p->off_ring = off_ring;
    p->n_stages = n_stages;
    p->stage_bytes = kStageBytes;
  }
  sp.gu.rms_eps = st->f.rms_eps;
  sp.h = static_cast<__half*>(h);
  sp.ldh = st->f.hidden;
  sp.act = static_cast<__half*>(act);
  sp.ldact = st->f.intermediate;
  sp.barrier = reinterpret_cast<unsigned*>(static_cast<uint8_t*>(ws) + kBarrierWordOffset);
  for (int l0 = 0; l0 < st->f.n_layers; l0 += kMaxStackLayers) {
    sp.n_layers = std::min(kMaxStackLayers, st->f.n_layers - l0);
    for (int i = 0; i < sp.n_layers; ++i) {
      const auto& L = st->layers[l0 + i];
      sp.layers[i] = StackLayer{static_cast<const uint8_t*>(L.pgu), L.sgu, static_cast<const uint8_t*>(L.pd),
                                L.sd};
    }
    if (launch_stack_tma(sp, grid, gu->wbytes, smem, stream) != cudaSuccess) return B2G_ERR_CUDA;
  }
  return B2G_OK;
}

b2g_status b2g_stack_enqueue(const b2g_stack* st, int32_t m, void* h, void* act, void* ws, b2g_stream_t stream) {
  if (!st || !h || !act || !ws) return B2G_ERR_INVALID;
  if (m < 1 || m > st->f.max_m) return B2G_ERR_INVALID;
  for (int l = 0; l < st->f.n_layers; ++l) {
    const auto& L = st->layers[l];
    if (!L.pgu || !L.pd) return B2G_ERR_INVALID;
    if (!aligned(L.pgu, 16) || !aligned(L.pd, 16)) return B2G_ERR_INVALID;
    if (st->f.scale_mode == B2G_SCALE_CHANNEL_FP32 && (!aligned(L.sgu, 4) || !aligned(L.sd, 4)))
      return B2G_ERR_INVALID;
  }
  if (st->mode == B2G_STACK_MODE_PERSISTENT || st->mode == B2G_STACK_MODE_PERSISTENT_TMA) {
    // A grid that cannot be co-resident (or a ring that does not fit) runs
    // per layer instead.
    const b2g_status s =
        st->mode == B2G_STACK_MODE_PERSISTENT
            ? stack_enqueue_persistent(st, m, h, act, ws, reinterpret_cast<cudaStream_t>(stream))
            : stack_enqueue_tma(st, m, h, act, ws, reinterpret_cast<cudaStream_t>(stream));
    if (s != B2G_ERR_UNSUPPORTED) return s;
  }
  for (int l = 0; l < st->f.n_layers; ++l) {
    const auto& L = st->layers[l];
    if (!L.pgu || !L.pd) return B2G_ERR_INVALID;
    const auto& Ln = st->layers[(l + 1) % st->f.n_layers];
    b2g_enqueue_args a = {};
    a.m = m;
    a.x = h;
    a.ldx = st->f.hidden;
    a.packed_w = L.pgu;
    a.scales = L.sgu;
    a.y = act;
    a.ldy = st->f.intermediate;
    a.workspace = ws;
    a.rms_eps = st->f.rms_eps;
    a.pdl = 1;
    a.prefetch_packed = L.pd;
    a.prefetch_op = st->dn;
    b2g_status s = b2g_enqueue_ex(st->gu, &a, stream);
    if (s != B2G_OK) return s;
    b2g_enqueue_args d = {};
    d.m = m;
    d.x = act;
    d.ldx = st->f.intermediate;
    d.packed_w = L.pd;
    d.scales = L.sd;
    d.residual = h;
    d.ldr = st->f.hidden;
    d.y = h;
    d.ldy = st->f.hidden;
    d.workspace = ws;
    d.pdl = 1;
    d.prefetch_packed = Ln.pgu;
    d.prefetch_op = st->gu;
    s = b2g_enqueue_ex(st->dn, &d, stream);
    if (s != B2G_OK) return s;
  }
  return B2G_OK;
}

}  // extern "C"
