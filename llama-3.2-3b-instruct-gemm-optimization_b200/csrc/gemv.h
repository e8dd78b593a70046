// gemv.h -- internal interface between the host API (api.cpp) and the
// kernels (gemv.cu, pack.cu).  Not part of the public C ABI.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace b2g {

// Packed weight stream.
//   A "unit" is what one warp consumes per step: 32 lanes x 16 B = 512 B per
//   weight plane -- 16 output channels x 32 k (E4M3) or 16 x 16 k (FP16),
//   arranged so each lane's 16 B are its m16n8k16 A-fragment registers.
//   A "tile" is 16 output channels.  K is cut into `ksplit` equal k-ranges;
//   a "virtual tile" (vt) is one tile over one k-range.  The stream is ordered
//   [ks][tile][kb-in-range][plane][lane][16 B], so every CTA streams one
//   contiguous byte range: units [u0, u1) with u0 = cta * T / grid, which
//   its warps stream round-robin (warp w takes units u0 + w + j * kWarps).
constexpr int kUnitPlaneBytes = 512;
constexpr int kTileCh = 16;
constexpr int kWarps = 16;  // one CTA of 16 warps per SM
constexpr int kThreads = kWarps * 32;
constexpr int kMaxSlots = 8;  // virtual tiles one CTA may touch
constexpr int kRing = 16;     // uint4 registers per lane for in-flight weight units
// Shared memory: [64,68) barrier verdict, [68,72) REDUCE round, [128,640) RMSNorm sums of squares
// [16 warps][8 rows], then the per-warp partial slots
// [n_slots][warps][planes][32 lanes][16 B], then the per-slot epilogue inputs
// (scales [n_slots][planes][16], residual rows [n_slots][8][16], fp32), then
// the x rows.
constexpr int kOffMisc = 64;
constexpr int kOffRound = 68;  // REDUCE: this CTA's previous round (u32)
constexpr int kOffRed = 128;
constexpr int kOffBars = 640;  // TMA pipeline: full[kMaxStages] then empty[kMaxStages] mbarriers
constexpr int kMaxStages = 24;
constexpr int kOffSlots = 1024;
// TMA pipeline (gemv_tma_kernel): warps 0..15 compute, warp 16 streams the
// weights into a ring of n_stages stages of stage_bytes in shared memory.
constexpr int kTmaThreads = kThreads + 32;
constexpr int kStageBytes = 16384;
// Workspace: tile counters first (fixed size, so ops sharing one workspace
// agree on where they are), then the split-K partials.  The last 256 bytes of
// the counter region hold the stack kernel's grid-barrier counter.
constexpr int kCounterRegionBytes = 65536;
constexpr int kBarrierWordOffset = kCounterRegionBytes - 256;
constexpr int kMaxTiles = kBarrierWordOffset / 4;

enum MathKind : int { kMathMma = 0, kMathFfma = 1 };

// Tensor-parallel exchange through peer memory (one process per GPU).  Each
// rank owns an inbox [2 buffers][world][max_m][width] fp16 and arrival
// counters [world]; peers' inboxes and counters are mapped into this
// process.  PUSH: the epilogue stores this rank's output rows into slot
// `rank` of buffer `buf` of every rank's inbox, then every CTA releases one
// arrival on every rank's counter[rank] at system scope.  GATHER: the
// activation staging waits (bounded) until every counter reaches
// epoch * push_grid, then sums slots 0..world-1 of buffer `buf` in rank order
// (fp32, one fp16 rounding) and writes the sum to h_out as it stages it.
// REDUCE: flag-in-data words.  The epilogue stores each finished tile's rows
// into slot `rank` of buffer `buf` of every other rank's REDUCE inbox
// [2][world][max_m][width / 2] u64, each 8-byte word = (round << 32) | two
// fp16; then every CTA reads the words of its own tiles from the other
// ranks' slots (bounded polls until the round matches: the CTAs with the
// same index own the same tiles under the one plan), adds its own rows from
// shared memory in rank order and writes the sums to y.  Every rank ends the
// launch with the all-reduced rows, with no fence and no counters.  The round
// is the launch count kept per CTA index in this rank's memory (all
// kTpMaxCtas entries advance together, whatever the grid).
constexpr int kMaxTp = 8;
constexpr int kTpMaxCtas = 256;       // REDUCE: CTAs per launch
constexpr int kTpRoundsOffset = 64;   // u32 words from this rank's epoch to its per-CTA rounds
enum TpMode : int { kTpNone = 0, kTpPush = 1, kTpGather = 2, kTpReduce = 3 };
struct TpParams {
  int mode;
  int world, rank;
  int buf;
  int push_grid;      // CTAs of each rank's pushing launch (one plan on every rank)
  int inbox_m;        // max_m rows per slot
  int width;          // halves per row (the hidden size)
  __half* inbox[kMaxTp];     // every rank's inbox (this rank's entry is local)
  unsigned* counters[kMaxTp];  // every rank's arrival counters [world]
  unsigned* epoch;           // this rank's count of pushing launches
  __half* h_out;             // GATHER: the reduced rows [m, ldh] (this rank's memory)
  long long ldh;
  unsigned* rounds;          // REDUCE: this rank's per-CTA launch counts [kTpMaxCtas]
};

__host__ __device__ inline bool tp_pushes(int mode) { return mode == kTpPush || mode == kTpReduce; }

// Division of x < 2^31 by a divisor fixed per launch, as a multiply-high and
// a shift (Granlund & Montgomery, "Division by invariant integers using
// multiplication", 1994, fig. 4.1 with N = 32):
//   l = ceil(log2 d), mul = floor(2^32 (2^l - d) / d) + 1,
//   x / d = (umulhi(x, mul) + x) >> l   (the sum stays below 2^32 for x < 2^31).
struct FastDiv {
  uint32_t d, mul, shift;
};
inline FastDiv make_fast_div(uint32_t d) {
  uint32_t l = 0;
  while ((1ull << l) < d) ++l;
  const uint64_t m = ((1ull << 32) * ((1ull << l) - d)) / d + 1;
  return FastDiv{d, (uint32_t)m, l};
}

struct GemvParams {
  const uint8_t* packed;
  const __half* x;
  long long ldx;
  const void* scales;
  const __half* residual;
  long long ldr;
  __half* y;
  long long ldy;
  float* partials;  // [n_vt][max_contrib][planes][32 lanes][4]
  int* counters;    // [n_tiles], zero between calls
  int* error;
  long long total_units;
  // Partition: the stream is cut into `grid` ranges at granules of `gran`
  // units (1: stream-K, any unit; kbpv: whole virtual tiles).
  int gran;
  FastDiv div_gran;
  int total_gran;  // total_units / gran; (total_gran + 2) * grid < 2^31 (host-checked)
  FastDiv div_tg, div_grid;
  int grid;
  int n_tiles;
  int kb_total;  // k-blocks (32 k for E4M3, 16 k for FP16) over padded K
  int ksplit;
  int kbpv;  // k-blocks per virtual tile
  FastDiv div_kbpv, div_tiles;  // / kbpv and / n_tiles
  int M, K, N;
  int scale_mode;
  int rmsnorm;  // rows are RMS-normalised: the factor is applied to the accumulators
  int residual_add;
  float rms_eps;
  int max_contrib;
  int n_slots;    // max virtual tiles per CTA (<= kMaxSlots)
  int off_epi;    // shared-memory byte offset of the epilogue inputs
  int off_x;      // shared-memory byte offset of the x rows
  int x_rs;       // x row stride in shared memory (halves)
  int lean;       // one contributor per output tile (ksplit 1, max_contrib 1) and every
                  // x row piece 16-byte aligned and inside K: the lean kernel flavor applies
  int off_ring;   // TMA pipeline: shared-memory byte offset of the weight ring
  int n_stages;   // ring stages (<= kMaxStages)
  int stage_bytes;
  // L2 prefetch of the next kernel's stream (pf_packed null = off): the
  // first pf_bytes of every range the next launch's CTAs will stream (its
  // partition: pf_total_units units of pf_unit_bytes in granules of pf_gran
  // over pf_grid CTAs); this launch's CTA c takes the next CTAs c, c + grid, ...
  const uint8_t* pf_packed;
  long long pf_total_units;
  int pf_gran;
  int pf_unit_bytes;
  int pf_grid;
  int pf_bytes;
  TpParams tp;
  int trace_slot;  // trace builds: this launch's slot in the per-launch timeline
};

// Final gather of a tensor-parallel chain: h = sum of the inbox slots once
// every rank's last push has arrived (TpParams as for GATHER).
cudaError_t launch_tp_gather(const TpParams& tp, int m, int* error, cudaStream_t stream);

// Launch one GEMV (planes = 1 or 2, wbytes = 1 for E4M3 or 2 for FP16).
cudaError_t launch_gemv(const GemvParams& p, int planes, int wbytes, int math, size_t smem,
                        bool pdl, cudaStream_t stream);
// The same GEMV with the weights streamed through a shared-memory ring by
// 1-D bulk copies (gemv_tma_kernel; tensor-core math only).
cudaError_t launch_gemv_tma(const GemvParams& p, int planes, int wbytes, size_t smem, bool pdl,
                            cudaStream_t stream);

// The decode-MLP stack in one cooperative launch.  Per layer l: phase 1 =
// gu (RMSNorm(h) -> gate||up -> SiLU*up -> act), phase 2 = dn (act -> down ->
// h += .), grid barriers between phases.  gu / dn hold each phase's plan and
// workspace pointers; their packed / x / y / scales / residual fields are
// unused (taken from layers, h and act).
constexpr int kMaxStackLayers = 32;  // per launch; the host chunks longer stacks
struct StackLayer {
  const uint8_t* pgu;
  const void* sgu;
  const uint8_t* pd;
  const void* sd;
};
struct StackParams {
  GemvParams gu, dn;
  StackLayer layers[kMaxStackLayers];
  __half* h;
  long long ldh;
  __half* act;
  long long ldact;
  unsigned* barrier;  // zero at launch; the kernel leaves it zero
  int n_layers;
};
// grid >= both phases' planned grids; CTAs past a phase's grid idle in it.
cudaError_t launch_stack(const StackParams& sp, int grid, int wbytes, size_t smem, cudaStream_t stream);
// Largest grid of stack_kernel<wbytes> that can be co-resident with `smem` bytes per CTA.
cudaError_t stack_max_coresident(int wbytes, size_t smem, int num_sms, int* max_grid);
// The stack on the TMA pipeline (gu and dn carry the same ring: off_ring,
// n_stages, stage_bytes), and its co-residency limit.
cudaError_t launch_stack_tma(const StackParams& sp, int grid, int wbytes, size_t smem, cudaStream_t stream);
cudaError_t stack_tma_max_coresident(int wbytes, size_t smem, int num_sms, int* max_grid);
// Raises the dynamic shared-memory limit of every kernel variant.
cudaError_t gemv_set_smem_limit(int bytes);

// Pack / quantise kernels (pack.cu).
cudaError_t launch_prepack(const void* w, long long ld, int layout, int wbytes, int K, int N,
                           int plane, int planes, int ksplit, int kbpv, int n_tiles, int kb_total,
                           uint8_t* packed, cudaStream_t stream);
cudaError_t launch_quantize(const __half* w16, int K, int N, int layout, int scale_mode,
                            uint8_t* w8, void* scales, cudaStream_t stream);

int* device_error_word();  // address of the library's device error word (current device)
// Device address of the fixed scratch used by b2g_enqueue_static (current
// device; static_scratch.cu).
cudaError_t static_scratch_address(void** ptr);

}  // namespace b2g
