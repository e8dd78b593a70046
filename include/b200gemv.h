/*
 * b200gemv.h -- C ABI of the B200 (sm_100a) decode-GEMV library for the
 * Llama-3.2-3B MLP projections (gate/up 3072->8192, down 8192->3072, M=1..8).
 *
 * This is the drop-in boundary.  The reference project
 * (sudb97/Llama-3.2-3B-Instruct-gemm-optimization) has no plugin code yet --
 * plugin/ holds only .gitkeep and the IPluginV3 is an open TODO (TODO.md:69-70)
 * -- so its operator surface is the in-file host API of kernels/gemv_fp8.cu and
 * kernels/gemv_fp16.cu, plus the plugin-creator fields it planned
 * (tensorrt_custom_tactic_kernel_b07f17a4.plan.md:57-58).  Each entry point
 * below names the reference interface it replaces.
 *
 * Conventions (all entry points):
 *  - The caller owns every device buffer; ops own host metadata only.
 *  - Work is stream-ordered on the given cudaStream_t; no entry point that
 *    takes a stream synchronises the host.
 *  - Errors are returned as b2g_status, never by exit() (the reference calls
 *    exit(1) from CHECK_CUDA, kernels/gemv_fp8.cu:38-46, and on an
 *    unsupported N, :270-273).
 *  - Weights are [K, N] row-major ("KN", the reference layout,
 *    kernels/gemv_fp8.cu:93) or [N, K] ("NK", nn.Linear); activations x are
 *    [m, K] fp16 with a row stride; outputs y are [m, N] fp16.
 */
#ifndef B200GEMV_H_
#define B200GEMV_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* b2g_stream_t; /* == cudaStream_t */

typedef enum {
  B2G_OK = 0,
  B2G_ERR_INVALID = 1,      /* bad argument (null pointer, size, alignment) */
  B2G_ERR_UNSUPPORTED = 2,  /* valid request this build does not implement */
  B2G_ERR_CUDA = 3,         /* a CUDA runtime call failed */
  B2G_ERR_PEER_TIMEOUT = 4, /* a device-side wait on a peer gave up */
  B2G_ERR_OOM = 5,          /* shared memory or workspace too small */
  B2G_ERR_DEVICE = 6,       /* a kernel recorded an error (bounded wait expired) */
  B2G_ERR_SCRATCH_LIMIT = 7 /* b2g_enqueue_static: the call needs more than
                               B2G_STATIC_SCRATCH_BYTES of workspace */
} b2g_status;

/* Weight element type (reference: FP16 kernels/gemv_fp16.cu, E4M3 kernels/gemv_fp8.cu). */
enum { B2G_DTYPE_FP16 = 0, B2G_DTYPE_FP8_E4M3 = 1 };

/* Scale modes.  NONE, TENSOR_FP16 and CHANNEL_FP16 are the reference's
 * ScaleMode {kScaleNone, kScaleTensor, kScaleChannel} (kernels/gemv_fp8.cu:459)
 * with fp16 scales (:515-540); CHANNEL_FP32 is the per-output-channel FP32
 * absmax/448 rule.  Scales multiply the fp32 accumulator in the epilogue
 * (the reference's cast_scale_f32_to_f16_kernel, kernels/gemv_fp8.cu:164-173). */
enum {
  B2G_SCALE_NONE = 0,
  B2G_SCALE_TENSOR_FP16 = 1,  /* scales: 1 fp16 */
  B2G_SCALE_CHANNEL_FP16 = 2, /* scales: [N] fp16 */
  B2G_SCALE_CHANNEL_FP32 = 3  /* scales: [N] fp32 */
};

enum { B2G_LAYOUT_KN = 0, B2G_LAYOUT_NK = 1 };

/* Fusion flags (bit mask).  None of these exist in the reference, which runs
 * one GEMV per launch; they implement the decode-MLP dataflow of its ONNX
 * graph (kernels/opt_loop/fp8_accuracy/capture_real_activations.py:39-42). */
enum {
  B2G_FUSE_NONE = 0,
  B2G_FUSE_GATE_UP_SILU = 1, /* two weight planes (gate, up) of width N;
                                y = fp16(SiLU(fp16(g)) * fp16(u)) */
  B2G_FUSE_RMSNORM_INPUT = 2, /* x rows are RMS-normalised (gamma = 1) first */
  B2G_FUSE_RESIDUAL_ADD = 4   /* y = fp16(residual + fp16(x W s)) */
};

/* Plugin-creator fields (the planned IPluginV3 creator's PluginFields:
 * in_features / out_features / weight dtype / scale mode,
 * tensorrt_custom_tactic_kernel_b07f17a4.plan.md:57-58, plus what the
 * library adds: layout, max rows, fusion and the tensor-parallel slot). */
typedef struct {
  int32_t in_features;   /* K */
  int32_t out_features;  /* N (per weight plane) */
  int32_t weight_dtype;  /* B2G_DTYPE_* */
  int32_t scale_mode;    /* B2G_SCALE_* */
  int32_t weight_layout; /* B2G_LAYOUT_* of the unpacked weights given to prepack */
  int32_t max_m;         /* 1..8 rows (decode tokens) per call */
  int32_t fuse;          /* B2G_FUSE_* mask */
  int32_t tp_rank;       /* informational: this shard's rank */
  int32_t tp_size;       /* informational: number of shards (1 = unsharded) */
} b2g_fields;

typedef struct b2g_op b2g_op;

/* Per-call arguments of b2g_enqueue_ex. */
typedef struct {
  int32_t m;              /* rows of x, 1..max_m */
  const void* x;          /* [m, ldx] fp16 */
  int64_t ldx;
  const void* packed_w;   /* from b2g_prepack */
  const void* scales;     /* per scale_mode; GATE_UP_SILU: gate then up
                             ([2][N] per-channel, or 2 tensor scalars) */
  const void* residual;   /* [m, ldr] fp16, FUSE_RESIDUAL_ADD only (may alias y) */
  int64_t ldr;
  void* y;                /* [m, ldy] fp16 */
  int64_t ldy;
  void* workspace;        /* b2g_workspace_size bytes, zeroed once by b2g_workspace_init */
  float rms_eps;          /* FUSE_RMSNORM_INPUT epsilon (Llama: 1e-5) */
  int32_t pdl;            /* 1: programmatic dependent launch.  The kernel then
                             starts streaming packed_w before the preceding
                             kernel in the stream has finished, so that kernel
                             must not write packed_w (x, residual, scales,
                             y and workspace are safe: they are touched only
                             after the wait). */
  const void* prefetch_packed; /* optional: packed weights of the kernel that
                                  will follow this one in the stream; at its
                                  start CTA c asks L2 for the first 256 KB of
                                  the ranges that kernel's CTAs c, c + grid,
                                  ... will stream (NULL = off) */
  const struct b2g_op* prefetch_op; /* the op prefetch_packed belongs to */
} b2g_enqueue_args;

/* Status string. */
const char* b2g_status_string(b2g_status s);

/* Library version (major*10000 + minor*100 + patch). */
int32_t b2g_version(void);

/* Plugin creator: validates the fields and plans the launch for the current
 * device.  Replaces the reference's compile-time Tiling/variant tables
 * (kernels/gemv_fp8.cu:192-234), which only accept N in {8192, 3072}. */
b2g_status b2g_create(const b2g_fields* fields, b2g_op** out);
b2g_status b2g_destroy(b2g_op* op);

/* Tuning options (the reference's CLI knobs variant/grid/KU,
 * kernels/gemv_fp8.cu:820-901, become per-op options).
 *  B2G_OPT_MATH: 0 = tensor-core m16n8k16 tiles (default),
 *                1 = CUDA-core FFMA with the same data layout.
 *  B2G_OPT_GRID: CTA count, 0 = one per SM (default).
 *  B2G_OPT_PARTITION: how the weight stream is cut among the CTAs:
 *    UNITS = equal byte ranges (a 16-channel tile may be split between two
 *    CTAs, which then combine partial sums); TILES = whole tiles per CTA (no
 *    split, up to one tile of imbalance); AUTO (default) = TILES when K is
 *    not split and the imbalance is at most 20%, else UNITS.
 *  B2G_OPT_KSPLIT: number of K ranges (0 = automatic).  Changes the packed
 *    layout: set it before b2g_prepack.
 *  B2G_OPT_PIPE: how the weights reach the math: REGISTERS = each warp
 *    streams its units into a register ring with 16-byte loads; TMA = one
 *    warp streams the CTA's range into a shared-memory ring of 16 KB stages
 *    with 1-D bulk copies, 16 warps compute from it (tensor-core math only;
 *    ops whose x rows leave fewer than two stages of shared memory stay on
 *    REGISTERS).  AUTO (default) = REGISTERS, the faster of the two per
 *    decode layer on B200.  The packed layout is the same for both. */
enum { B2G_OPT_MATH = 1, B2G_OPT_GRID = 2, B2G_OPT_PARTITION = 3, B2G_OPT_KSPLIT = 4, B2G_OPT_PIPE = 5 };
enum { B2G_PARTITION_AUTO = 0, B2G_PARTITION_UNITS = 1, B2G_PARTITION_TILES = 2 };
enum { B2G_PIPE_AUTO = 0, B2G_PIPE_REGISTERS = 1, B2G_PIPE_TMA = 2 };
b2g_status b2g_op_set_option(b2g_op* op, int32_t key, int32_t value);

/* The launch plan chosen for calls with m rows. */
typedef struct {
  int32_t grid;             /* CTAs (one per SM) */
  int32_t ksplit;           /* K ranges */
  int32_t kblocks_per_vtile;
  int32_t n_tiles;          /* 16-channel output tiles */
  int64_t total_units;      /* stream units (512 B per weight plane) */
  int32_t unit_bytes;
  int64_t inflight_bytes_per_cta; /* weight bytes each CTA keeps in flight */
  int64_t smem_bytes;       /* dynamic shared memory per CTA */
  int32_t max_contrib;      /* max CTAs sharing one virtual tile */
  int32_t partition;        /* B2G_PARTITION_UNITS or _TILES, as planned */
  int32_t n_slots;          /* virtual tiles per CTA (max) */
  int32_t x_kblocks;        /* 32-wide k blocks of x staged per CTA */
  int32_t math;
  int32_t pipe;             /* B2G_PIPE_REGISTERS or _TMA, as planned for m */
  int32_t n_stages;         /* TMA pipeline: ring stages (0 otherwise) */
  int32_t stage_bytes;      /* TMA pipeline: bytes per stage (0 otherwise) */
} b2g_plan_info;
b2g_status b2g_op_query(const b2g_op* op, int32_t m, b2g_plan_info* info);
/* The plan b2g_create would make on a GPU with num_sms SMs and smem_optin
 * bytes of opt-in shared memory per block, made without touching a device
 * (build-time sizing, e.g. IPluginV3OneBuild::getWorkspaceSize on a machine
 * without the target GPU; planner tests).  Also returns the packed-weight and
 * workspace bytes for m rows (either pointer may be NULL).  B200: 148 SMs,
 * 232448 bytes. */
b2g_status b2g_plan_for_device(const b2g_fields* f, int32_t num_sms, int32_t smem_optin, int32_t m,
                               b2g_plan_info* info, size_t* packed_bytes, size_t* workspace_bytes);

/* Bytes of the pre-packed weight buffer.  (The reference streams the raw
 * [K, N] bytes, kernels/gemv_fp8.cu:93; the library streams a tile layout.) */
b2g_status b2g_prepack_size(const b2g_op* op, size_t* bytes);

/* Device-side repack of unpacked weights (op's dtype and layout, ld = row
 * stride in elements of the unpacked matrix, 0 = dense) into the streaming
 * tile layout.  GATE_UP_SILU takes the up plane in w_plane1, else NULL. */
b2g_status b2g_prepack(const b2g_op* op, const void* w_plane0, const void* w_plane1,
                       int64_t ld, void* packed, b2g_stream_t stream);

/* Device-side E4M3 quantisation of fp16 weights [K, N] (KN) or [N, K] (NK)
 * under a scale mode; writes E4M3 codes in the same layout and the scales.
 * NONE is pack_e4m3 (kernels/gemv_fp8.cu:297-304); TENSOR_FP16/CHANNEL_FP16
 * are check_real's scale + pre-divide (kernels/gemv_fp8.cu:515-543);
 * CHANNEL_FP32 is s = max(amax,1e-12)/448 in fp32, q = e4m3(w / s). */
b2g_status b2g_quantize_e4m3(const void* w16, int32_t K, int32_t N, int32_t layout,
                             int32_t scale_mode, void* w8, void* scales, b2g_stream_t stream);

/* Workspace bytes for calls with up to m rows, and its one-time zeroing
 * (the kernels leave it zeroed after every complete call).  Replaces the
 * reference's caller-provided y_acc that run_gemv memsets on every call
 * (kernels/gemv_fp8.cu:276-283). */
b2g_status b2g_workspace_size(const b2g_op* op, int32_t m, size_t* bytes);
b2g_status b2g_workspace_init(const b2g_op* op, void* workspace, b2g_stream_t stream);

/* enqueue(x, W, scales) -> y: the plugin's enqueue.  One kernel launch
 * replaces the reference's run_gemv (memset + gemv_chunk_kernel + cast,
 * kernels/gemv_fp8.cu:276-283; kernels/gemv_fp16.cu:262-271). */
b2g_status b2g_enqueue(const b2g_op* op, int32_t m, const void* x, const void* packed_w,
                       const void* scales, void* y, void* workspace, b2g_stream_t stream);
b2g_status b2g_enqueue_ex(const b2g_op* op, const b2g_enqueue_args* args, b2g_stream_t stream);

/* Reads (and optionally clears) the device error word that kernels set when
 * a bounded wait expires.  Synchronises the current device. */
b2g_status b2g_device_error(int32_t* code, int32_t clear);

/* ------------------------------------------------------------------------
 * No-allocation enqueue.  No counterpart in the reference (its run_gemv takes
 * a caller-allocated y_acc, kernels/gemv_fp8.cu:276-283).
 *
 * Same computation and arguments as b2g_enqueue_ex, except that
 * args->workspace must be NULL: the workspace is a fixed array of
 * B2G_STATIC_SCRATCH_BYTES compiled into the library (one per device), so
 * the call itself allocates nothing, on the device or the host.  It is for
 * callers that cannot allocate at enqueue time: a plugin whose engine
 * granted it no workspace, a process whose device memory is all handed to
 * another allocator's pool up front, or a latency-bound loop that must not
 * reach cudaFree (which synchronises the device).
 *  - Limit: a call whose b2g_workspace_size exceeds B2G_STATIC_SCRATCH_BYTES
 *    returns B2G_ERR_SCRATCH_LIMIT and launches nothing.  2 MiB covers every
 *    Llama-3.2-3B MLP op (the largest, fused gate||up, needs 1.06 MiB).
 *  - Zeroing: the tile counters at the start of the scratch must be zero
 *    when the kernel starts; this call clears them on `stream` before every
 *    launch (the split-K partials need no clearing).
 *  - Races: the scratch is shared by every call on the device.  Calls that
 *    can run at the same time -- on different streams, or from different
 *    host threads -- race on it and give wrong results.  Calls in one stream
 *    are ordered and safe.
 *  - args->pdl is ignored (launched without programmatic dependent launch,
 *    so the counter clearing is complete before the kernel starts).
 * ------------------------------------------------------------------------ */
#define B2G_STATIC_SCRATCH_BYTES (2u * 1024u * 1024u)
b2g_status b2g_enqueue_static(const b2g_op* op, const b2g_enqueue_args* args, b2g_stream_t stream);

/* ------------------------------------------------------------------------
 * Tensor-parallel exchange through peer memory (no reference counterpart:
 * the reference runs on one GPU).  One process per GPU.  Each rank allocates
 * a zero-filled communication buffer of b2g_tp_comm_bytes(), shares it with
 * b2g_ipc_handle / b2g_ipc_open, and fills a b2g_tp_comm with every rank's
 * mapped addresses (b2g_tp_comm_layout).  Then, per layer, either
 *   down op, mode REDUCE: the epilogue stores this rank's output rows into
 *     its slot of every other rank's inbox as 8-byte words that carry the
 *     launch's round number beside two fp16 values (so no fence and no
 *     counter is needed); each CTA then polls (bounded) the words of its own
 *     tiles from the other ranks -- the CTAs with the same index own the same
 *     output tiles under the one plan -- and writes y = the sum in rank order
 *     (fp32, one fp16 rounding; its own rows come from shared memory).  Every
 *     rank ends the launch with the all-reduced rows; the next gate||up op is
 *     a plain launch.  Needs whole tiles (K split 1, one CTA per tile),
 *     16-byte-aligned x rows (ldx a multiple of 8, K a multiple of 32),
 *     4-byte-aligned y rows, at most B2G_TP_MAX_CTAS CTAs and the register
 *     pipeline.  Or
 *   down op, mode PUSH: instead of writing y, the epilogue stores this rank's
 *     output rows straight into its slot of every rank's inbox (NVLink peer
 *     stores); each CTA then fences at system scope once and adds one
 *     arrival on every rank's counter;
 *   next gate||up op, mode GATHER: its activation staging waits (bounded)
 *     for all ranks' arrivals, sums the slots in rank order (fp32, one fp16
 *     rounding: every rank gets bitwise the same rows) and writes the sum to
 *     h_out (the residual input of the next down op).
 * and after the last layer b2g_tp_gather writes the final rows.  Consecutive
 * layers alternate between the inbox's two buffers (`buf`): a rank writes a
 * buffer again two exchanges later, after every rank has arrived in the
 * exchange between, which each rank does only after its reads of the
 * earlier one.  A wait that
 * expires sets the device error word (B2G_ERR_PEER_TIMEOUT class, code 4);
 * while the word is set, later waits give up at once (a lost peer costs one
 * 2 s wait, not one per layer).  A REDUCE CTA then writes none of its
 * rows of y, b2g_tp_gather leaves h as it was, and
 * a GATHER launch writes neither h_out nor its own output rows (its tiles'
 * split-K handshakes still complete, so the workspace stays consistent).
 * Every row produced since the error is invalid: read and clear the word
 * (b2g_device_error), then re-zero the exchange buffers and the ops'
 * workspaces (b2g_workspace_init) before the next step.
 * ------------------------------------------------------------------------ */
#define B2G_TP_MAX_RANKS 8
#define B2G_TP_MAX_CTAS 256 /* REDUCE: CTAs per launch */
enum { B2G_TP_NONE = 0, B2G_TP_PUSH = 1, B2G_TP_GATHER = 2, B2G_TP_REDUCE = 3 };
typedef struct {
  int32_t world, rank;
  int32_t max_m;   /* rows per inbox slot */
  int32_t width;   /* halves per row (the hidden size, a multiple of 8) */
  void* inbox[B2G_TP_MAX_RANKS];    /* every rank's inbox, mapped in this process */
  void* counters[B2G_TP_MAX_RANKS]; /* every rank's arrival counters */
  void* epoch;                      /* this rank's launch counter */
} b2g_tp_comm;
/* Bytes of one rank's communication buffer, and the addresses inside a
 * buffer at `base` (the same layout on every rank): the inbox (PUSH and
 * GATHER: [2][world][max_m][width] fp16; REDUCE: [2][world][max_m][width/2]
 * 8-byte words); the counter region (PUSH counters [world] u32); the epoch
 * region (epoch u32, then from byte 256 the REDUCE per-CTA launch counts
 * [B2G_TP_MAX_CTAS] u32).  `counters` and `epoch` point at the starts of the
 * two regions.  The buffer is zero-filled before first use and re-zeroed
 * after an expired wait (every region, the counts included). */
size_t b2g_tp_comm_bytes(int32_t world, int32_t max_m, int32_t width);
b2g_status b2g_tp_comm_layout(void* base, int32_t world, int32_t max_m, int32_t width, void** inbox,
                              void** counters, void** epoch);
/* CUDA IPC of a device buffer: a B2G_IPC_RECORD_BYTES record (the handle of
 * the allocation holding dev_ptr and dev_ptr's offset in it, so buffers from
 * a caching allocator work), opened in another process on its own device;
 * b2g_ipc_close takes the address b2g_ipc_open returned. */
#define B2G_IPC_RECORD_BYTES 72
b2g_status b2g_ipc_handle(const void* dev_ptr, void* record);
b2g_status b2g_ipc_open(const void* record, void** dev_ptr);
b2g_status b2g_ipc_close(void* dev_ptr);
/* b2g_enqueue_ex with an exchange mode.  REDUCE: as PUSH, and args->y
 * receives the all-reduced rows (requirements above; push_op is ignored).
 * PUSH: the op must not fuse gate||up; args->y is not written.  GATHER: the op's rows must be whole (K split 1),
 * K == comm->width; args->x is not read; push_op is the op whose launches push
 * (its CTA count is the arrival count per round); h_out [m, ldh] receives the
 * summed rows. */
b2g_status b2g_enqueue_tp(const b2g_op* op, const b2g_enqueue_args* args, const b2g_tp_comm* comm,
                          int32_t mode, int32_t buf, const b2g_op* push_op, void* h_out, int64_t ldh,
                          b2g_stream_t stream);
/* h [m, ldh] = sum of the inbox slots of buffer `buf` once every rank's
 * pushing launch of this round (push_op's) has arrived. */
b2g_status b2g_tp_gather(const b2g_tp_comm* comm, int32_t buf, const b2g_op* push_op, int32_t m, void* h,
                         int64_t ldh, b2g_stream_t stream);

/* ------------------------------------------------------------------------
 * Decode MLP stack: n_layers x [RMSNorm -> fused gate||up + SiLU*up -> down +
 * residual], hidden state updated in place.  No reference counterpart (the
 * reference runs single GEMVs); the layer dataflow is its ONNX graph's
 * (capture_real_activations.py:39-42).
 * ------------------------------------------------------------------------ */
typedef struct {
  int32_t hidden;        /* 3072 */
  int32_t intermediate;  /* 8192 (per tensor-parallel shard: 8192 / tp_size) */
  int32_t n_layers;      /* 28 */
  int32_t weight_dtype;
  int32_t scale_mode;
  int32_t max_m;
  float rms_eps;
  int32_t tp_rank;
  int32_t tp_size;
} b2g_stack_fields;

typedef struct b2g_stack b2g_stack;

b2g_status b2g_stack_create(const b2g_stack_fields* fields, b2g_stack** out);
b2g_status b2g_stack_destroy(b2g_stack* st);
/* The fused gate||up op and the down op the stack uses (owned by the stack),
 * for prepacking layer weights. */
b2g_status b2g_stack_ops(const b2g_stack* st, const b2g_op** gate_up, const b2g_op** down);
b2g_status b2g_stack_set_layer(b2g_stack* st, int32_t layer, const void* packed_gate_up,
                               const void* scales_gate_up, const void* packed_down,
                               const void* scales_down);
b2g_status b2g_stack_workspace_size(const b2g_stack* st, int32_t m, size_t* bytes);
b2g_status b2g_stack_workspace_init(const b2g_stack* st, void* workspace, b2g_stream_t stream);
/* Execution mode (key B2G_STACK_OPT_MODE):
 *  PER_LAYER (default): two launches per layer chained with programmatic
 *    dependent launch; each launch first loads its own leading weights, then
 *    asks L2 for the first 256 KB of each range the next launch's CTAs will
 *    stream.
 *  PERSISTENT: one cooperative launch runs every layer (up to 32 layers per
 *    launch), grid barriers between the gate||up and down phases; each
 *    phase's first weights are loaded while the barrier completes.
 *  PERSISTENT_TMA: one cooperative launch as PERSISTENT, the weights on the
 *    TMA pipeline (B2G_OPT_PIPE): in each CTA one warp streams every phase's
 *    range, layer after layer, through a shared-memory ring and asks L2 for
 *    the phase after it, while 16 warps compute; the grid barriers involve
 *    the computing warps only, so the weight stream runs through them.
 * All modes give bitwise-identical results (see the benchmark's detail
 * output for their speeds on B200). */
enum { B2G_STACK_OPT_MODE = 1 };
enum { B2G_STACK_MODE_PERSISTENT = 0, B2G_STACK_MODE_PER_LAYER = 1, B2G_STACK_MODE_PERSISTENT_TMA = 2 };
b2g_status b2g_stack_set_option(b2g_stack* st, int32_t key, int32_t value);
/* h [m, hidden] fp16 is read and overwritten; act is [m, intermediate] fp16
 * scratch.  The workspace must have been zeroed once by
 * b2g_stack_workspace_init (and again after a call that reported a device
 * error).  tp_size > 1 is not handled here (see the Python TP driver). */
b2g_status b2g_stack_enqueue(const b2g_stack* st, int32_t m, void* h, void* act,
                             void* workspace, b2g_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* B200GEMV_H_ */
