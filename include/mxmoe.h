/*
 * mxmoe.h -- C ABI of the B200 (sm_100a) MXFP4 mixture-of-experts layer.
 *
 * This is the drop-in boundary for burn-extended's `moe` / `quant` modules:
 * every entry point below replaces one reference item (cited file:line, paths
 * relative to the burn-extended crate root).  All functions return an
 * mxmoe_status; they never abort or throw across the boundary.  The message
 * of the last failure on the calling thread is available from
 * mxmoe_last_error().  `stream` arguments are cudaStream_t values passed as
 * plain pointers (NULL = legacy default stream).
 *
 * Threading: a layer handle serves one stream at a time; distinct handles are
 * independent.  Forward calls are stream-ordered and asynchronous.
 */
#ifndef MXMOE_H
#define MXMOE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MXMOE_ABI_VERSION 1

#if defined(__GNUC__)
#define MXMOE_API __attribute__((visibility("default")))
#else
#define MXMOE_API
#endif

typedef enum mxmoe_status {
  MXMOE_OK = 0,
  MXMOE_ERR_INVALID_ARG = 1,   /* null pointer, bad shape, bad flag */
  MXMOE_ERR_NOT_READY = 2,     /* forward before the weights were uploaded */
  MXMOE_ERR_CUDA = 3,          /* a CUDA runtime/driver call failed */
  MXMOE_ERR_OOM = 4,           /* device allocation failed */
  MXMOE_ERR_UNSUPPORTED = 5,   /* shape outside what the kernels handle */
  MXMOE_ERR_TIMEOUT = 6,       /* a bounded device-side wait gave up */
  MXMOE_ERR_TOO_LARGE = 7      /* request exceeds a fixed-size buffer */
} mxmoe_status;

/* Element types of activation / bias buffers. */
typedef enum mxmoe_dtype {
  MXMOE_F32 = 0,
  MXMOE_BF16 = 1
} mxmoe_dtype;

/* Behaviour flags (mxmoe_config.flags). */
#define MXMOE_FLAG_INTERLEAVED_GLU 0x1u /* W1 rows interleaved [glu0, lin0, ...]
                                           (src/activation/mod.rs:28-30);
                                           default split-half rows [glu; lin]
                                           as src/quant/gpu.rs:108-113 reads */
#define MXMOE_FLAG_BIAS_PER_FTILE  0x2u /* reproduce src/quant/gpu.rs:191: b2 is
                                           added once per 256-wide f tile */
#define MXMOE_FLAG_NO_RESIDUAL     0x4u /* y = moe(x) (no x + ... at
                                           src/moe/mod.rs:411) */
#define MXMOE_FLAG_DISABLED        0x8u /* MoeConfig.disabled: y = x
                                           (src/moe/mod.rs:106-108) */
#define MXMOE_FLAG_SIMT            0x10u /* run the expert FFN on the CUDA-core
                                            kernels instead of tcgen05 (a second,
                                            independent GPU implementation used to
                                            cross-check the tensor-core path) */
#define MXMOE_FLAG_NO_GRAPHS       0x20u /* never replay mxmoe_forward as a CUDA
                                            graph (by default the second call with
                                            the same x, y, n and dtypes is captured
                                            and later ones replay it) */
#define MXMOE_FLAG_NO_FP4          0x40u /* keep decode batches (at most 24 routed
                                            pairs per expert) on the E4M3
                                            tensor-core tiles instead of the
                                            kind::mxf4 tiles with a four-term
                                            E2M1 activation */
#define MXMOE_FLAG_NO_GEMV         0x80u /* never run tiny batches (at most 64
                                            routed pairs) on the CUDA-core
                                            dequant-GEMV; they take the
                                            tensor-core tiles like any other */

/* Mirrors moe::MoeConfig (src/moe/mod.rs:22-33).  `initializer` and `verbose`
 * have no device meaning; swiglu_alpha / swiglu_limit are honoured (the
 * reference kernel hardcodes 1.702 / 7.0 at src/quant/gpu.rs:140-141). */
typedef struct mxmoe_config {
  uint32_t d_model;
  uint32_t ffn_hidden;
  uint32_t num_experts;
  uint32_t experts_per_token;
  float swiglu_alpha;
  float swiglu_limit;
  float rms_eps;          /* RmsNorm epsilon (model.bin header stores 1e-5) */
  uint32_t flags;         /* MXMOE_FLAG_* */
  int32_t device;         /* CUDA device ordinal the layer lives on */
} mxmoe_config;

/* Field-for-field quant::QuantLinearMxFp4Desc (src/quant/mod.rs:3-11).
 * blocks: [experts][rows][bpr] bytes, two E2M1 codes per byte (low nibble =
 * even column); scales: [experts][rows][gpr] E8M0 bytes, one per 32 columns;
 * stored exponent = true exponent + 127 + ue8_offset (model.bin uses 14,
 * src/loader/modelbin.rs:452-453). */
typedef struct mxmoe_quant_desc {
  uint64_t experts;
  uint64_t rows;
  uint64_t cols;
  uint64_t bpr;
  uint64_t gpr;
  int32_t ue8_offset;
} mxmoe_quant_desc;

typedef struct mxmoe_layer mxmoe_layer;

/* ABI version and a short build description. */
MXMOE_API int mxmoe_abi_version(void);
MXMOE_API const char* mxmoe_build_info(void);

/* Thread-local message of the last failure (truncated to cap bytes). */
MXMOE_API int mxmoe_last_error(char* buf, size_t cap);

/* Replaces MoeConfig::init (src/moe/mod.rs:60-91): validates the config and
 * creates an empty layer on cfg->device. */
MXMOE_API int mxmoe_create(const mxmoe_config* cfg, mxmoe_layer** out);

/* Device buffers of the FP4 decode operands of the last forward that used
 * them (for inspection): ptrs[0] W1 input codes [4 * rows4][kp1 / 2],
 * ptrs[1] their scale atoms [rows4 / 32][kp1 / 128][512], ptrs[2] / ptrs[3]
 * the same for the W2 input (kp2 = f padded); pair pos, term t sits at
 * code row (pos / 32) * 128 + (pos % 32 / 8) * 32 + 8 t + pos % 8.  NULL and
 * rows4 = 0 before the first FP4 forward. */
MXMOE_API int mxmoe_fp4_operands(mxmoe_layer* layer, void** ptrs, uint32_t* rows4);

/* The layer's config as created (the loaders fill in the shapes and flags
 * from the file). */
MXMOE_API int mxmoe_get_config(const mxmoe_layer* layer, mxmoe_config* out);

/* Frees every device buffer the layer owns. */
MXMOE_API int mxmoe_destroy(mxmoe_layer* layer);

/* Router parameters: the MoE block's RmsNorm gain (`norm`, src/moe/mod.rs:37,
 * [d]) and the gate Linear (`gate`, :38) as weight [E][d] (output-major; Burn's
 * Linear keeps [d][E] -- the Rust shim transposes) and bias [E].  Host
 * pointers; dtype applies to all three.  Copies are made; the caller keeps its
 * buffers. */
MXMOE_API int mxmoe_set_router(mxmoe_layer* layer, const void* norm_gamma,
                     const void* gate_w, const void* gate_b, mxmoe_dtype dtype,
                     void* stream);

/* Replaces MoeQuantLayerResident::new (src/quant/gpu.rs:31-53) together with
 * set_resident (src/moe/mod.rs:95-97) and the bias params (:42, :45).
 * Host pointers; W1 is [E][2f][d] (split-half or interleaved rows per the
 * config flag), W2 is [E][d][f].  The library repacks into its tensor-core
 * operand layout (scale offset removed, rows/columns padded) and owns the
 * device copies; the caller keeps its buffers.  b1 [E][2f], b2 [E][d] in
 * bias_dtype. */
MXMOE_API int mxmoe_upload_experts(mxmoe_layer* layer, const mxmoe_quant_desc* w1_desc,
                         const uint8_t* w1_blocks, const uint8_t* w1_scales,
                         const mxmoe_quant_desc* w2_desc,
                         const uint8_t* w2_blocks, const uint8_t* w2_scales,
                         const void* b1, const void* b2, mxmoe_dtype bias_dtype,
                         void* stream);

/* Pre-sizes the per-forward workspace for up to max_tokens tokens so that
 * later forwards allocate nothing.  Optional. */
MXMOE_API int mxmoe_reserve(mxmoe_layer* layer, uint32_t max_tokens);

/* Replaces MoeGatedSwiGLU::forward (src/moe/mod.rs:99-115, forward_resident
 * :122-412): y = x + sum_k w_k * FFN_{e_k}(RmsNorm(x)).  x and y are DEVICE
 * pointers of n_tokens x d_model elements (row-major, batch and sequence
 * flattened), both starting on 16-byte boundaries (MXMOE_ERR_INVALID_ARG
 * otherwise).  Stream-ordered; returns before the work finishes. */
MXMOE_API int mxmoe_forward(mxmoe_layer* layer, const void* x, mxmoe_dtype x_dtype,
                  void* y, mxmoe_dtype y_dtype, uint32_t n_tokens, void* stream);

/* Same computation on HOST buffers: copies x to the device, runs the forward
 * and copies y back, then synchronizes `stream`.  Pinned host memory makes
 * the copies asynchronous with respect to other streams. */
MXMOE_API int mxmoe_forward_host(mxmoe_layer* layer, const void* x_host,
                       mxmoe_dtype x_dtype, void* y_host, mxmoe_dtype y_dtype,
                       uint32_t n_tokens, void* stream);

/* Routing results of the most recent forward on this layer (device
 * pointers owned by the layer, valid until the next forward):
 *   topk_idx [n][k] int32, topk_w [n][k] f32, offsets [E+1] int32 (unpadded
 *   prefix counts), perm [n*k] int32 (sorted position -> pair t*k+s),
 *   inv [n*k] int32 (pair -> sorted position), logits [n][E] f32.
 * Replaces the router tensors of src/moe/mod.rs:270-288 for parity checks. */
MXMOE_API int mxmoe_routing_results(mxmoe_layer* layer, const int32_t** topk_idx,
                          const float** topk_w, const int32_t** offsets,
                          const int32_t** perm, const int32_t** inv,
                          const float** logits);

/* Replaces loader::mxfp4::dequant_mxfp4_bytes (src/loader/mxfp4.rs:57-79) on
 * the device: blocks [rows_total][b] bytes, scales [rows_total] (one E8M0 per
 * row of b bytes), out [rows_total][2b] f32, bit-exact.  Device pointers. */
MXMOE_API int mxmoe_dequant_mxfp4_bytes(const uint8_t* blocks, uint64_t rows_total,
                              uint64_t b, const uint8_t* scales, float* out,
                              void* stream);

/* Dequantizes expert weights in the MoE layout described by `desc` (the
 * decode of src/quant/gpu.rs:124-134, with exact powers of two): out
 * [experts][rows][cols] f32.  Device pointers. */
MXMOE_API int mxmoe_dequant_rows(const mxmoe_quant_desc* desc, const uint8_t* blocks,
                       const uint8_t* scales, float* out, void* stream);

/* Top-k + softmax over given router logits [n][E] (the Burn ops of
 * src/moe/mod.rs:272-276), for bit-exact index checks on identical logits.
 * Device pointers. */
MXMOE_API int mxmoe_topk_softmax(const float* logits, uint32_t n_tokens,
                       uint32_t num_experts, uint32_t k, int32_t* topk_idx,
                       float* topk_w, void* stream);

/* Canonical permutation of given top-k indices (replaces the dense masks of
 * src/moe/mod.rs:279-288): stable counting sort of pairs p = t*k+s by expert.
 * offsets [E+1], perm [n*k], inv [n*k].  Device pointers.  Synchronizes
 * `stream`.  Ids outside [0, num_experts) are left out of the maps (their inv
 * entry is -1) and the call returns MXMOE_ERR_INVALID_ARG; n*k above INT32_MAX
 * returns MXMOE_ERR_TOO_LARGE. */
MXMOE_API int mxmoe_permute(const int32_t* topk_idx, uint32_t n_tokens, uint32_t k,
                  uint32_t num_experts, int32_t* offsets, int32_t* perm,
                  int32_t* inv, void* stream);

/* mxmoe_permute without any device allocation.  No counterpart in the
 * reference: it is for callers that cannot call cudaMalloc, for instance code
 * running under a caching or arena allocator that owns all device memory, or
 * an embedding runtime that forbids allocation after start-up.  Its scratch
 * (per-expert offsets and counts) is a fixed 8 KB array inside the library,
 * held on every GPU that loads it until the process exits; num_experts above
 * 1024 is rejected with MXMOE_ERR_TOO_LARGE.  The first call on a device
 * looks the array's device address up (cudaGetSymbolAddress) -- make that
 * first call before any stream capture.  All calls share the one array, so
 * calls that overlap on the GPU (different streams, different threads) race;
 * serialize them.  Unlike mxmoe_permute it does not synchronize `stream`, so
 * ids outside [0, num_experts) cannot be reported: they are left out of the
 * maps (inv entry -1, offsets[E] short of n*k).  It always runs the one-block
 * permutation (1024 threads), fine for decode and small prefill batches but
 * slow past tens of thousands of pairs, where mxmoe_permute's multi-block form
 * takes over.  Device pointers, same meaning as mxmoe_permute. */
MXMOE_API int mxmoe_permute_noalloc(const int32_t* topk_idx, uint32_t n_tokens,
                                    uint32_t k, uint32_t num_experts,
                                    int32_t* offsets, int32_t* perm,
                                    int32_t* inv, void* stream);

/* Synchronizes `stream` and reports a device-side failure of the layer's
 * kernels since the last forward (MXMOE_ERR_TIMEOUT when a bounded wait gave
 * up).  mxmoe_forward_host performs this check itself. */
MXMOE_API int mxmoe_sync_status(mxmoe_layer* layer, void* stream);

/* Per-stage timing of mxmoe_forward (no counterpart in the reference, whose
 * timing is eprintln! of wall clock, src/models/gpt_oss.rs:223-281).  When
 * enabled, every forward records CUDA events on its stream around the stages
 * router, permute, quantize, W1 GEMM, W2 GEMM, combine; mxmoe_last_profile
 * waits for the last forward and writes up to `cap` stage times in
 * milliseconds (returns the stage count through *count). */
MXMOE_API int mxmoe_set_profiling(mxmoe_layer* layer, int enable);

/* Test hook for the failure path; no counterpart in the reference, whose
 * errors are panics (src/moe/mod.rs:112).  MXMOE_FAULT_SKIP_SIGNAL makes the
 * next mxmoe_forward of this layer withhold one device-side signal: the
 * tensor-core GEMM leaves one pipeline stage unarmed (its consumer's wait
 * runs out), the dequant-GEMV's block 0 never reports its W1 columns (its
 * expert's other blocks stop waiting).  The waits of that forward give up
 * after 1 ms instead of 2 s, record MXMOE_ERR_TIMEOUT in the layer's status
 * (mxmoe_sync_status reports it), drain their copies and MMAs, free TMEM and
 * return; the output of that forward is undefined.  Nothing faults, traps or
 * hangs, and the next forward runs normally.  The injected forward is never
 * captured as a CUDA graph.  MXMOE_FAULT_NONE clears a pending injection. */
#define MXMOE_FAULT_NONE 0u
#define MXMOE_FAULT_SKIP_SIGNAL 1u
MXMOE_API int mxmoe_set_fault_injection(mxmoe_layer* layer, uint32_t mode);
MXMOE_API int mxmoe_last_profile(mxmoe_layer* layer, float* ms, int cap,
                                 int* count);

/* ---------------------------------------------------------------------------
 * Expert parallelism (no counterpart in the single-rank reference, whose
 * docs/gpt-oss-architecture.md:22 leaves sharding out): experts are split into
 * contiguous shards, one per GPU; a host runtime moves routed pairs with an
 * NCCL all-to-all and uses the entry points below on either side.
 * ------------------------------------------------------------------------- */

/* This layer holds experts [expert_begin, expert_begin + expert_count) of the
 * global num_experts.  Must precede mxmoe_upload_experts, whose descriptors
 * then cover only the local experts.  The router stays global. */
MXMOE_API int mxmoe_set_expert_shard(mxmoe_layer* layer, uint32_t expert_begin,
                           uint32_t expert_count);

/* Router + canonical permutation on device x [n][d] (source side):
 * rscale [n] (1 / rms), topk_idx [n][k], topk_w [n][k], offsets [E+1],
 * perm [n*k], inv [n*k] (global expert ids; pairs sorted by expert are sorted
 * by destination rank).  Device pointers owned by the caller; x may start
 * at any element boundary. */
MXMOE_API int mxmoe_route(mxmoe_layer* layer, const void* x, mxmoe_dtype x_dtype,
                uint32_t n_tokens, float* rscale, int32_t* topk_idx,
                float* topk_w, int32_t* offsets, int32_t* perm, int32_t* inv,
                void* stream);

/* Packs routed pairs in permuted order for dispatch: for every position q,
 * pair p = perm[q], token t = p / k: out_x[q] = x[t] (x's dtype, rows must
 * start on 16-byte boundaries), and out_meta[q] = three 32-bit words
 * {bits of rscale[t], topk_idx[p], bits of topk_w[p]}.  Device pointers. */
MXMOE_API int mxmoe_gather_pairs(const void* x, mxmoe_dtype x_dtype, uint32_t n_tokens,
                       uint32_t d_model, uint32_t k, const int32_t* perm,
                       const float* rscale, const int32_t* topk_idx,
                       const float* topk_w, void* out_x, uint32_t* out_meta,
                       void* stream);

/* Receive side: expert FFN of this layer's shard for dispatched pairs.
 * xr [n_pairs][d] raw token rows (x's dtype), rscale [n_pairs], expert
 * [n_pairs] GLOBAL ids inside the shard, weight [n_pairs];
 * out [n_pairs][d] (out_dtype) = weight * (W2 act + b2).  Device pointers;
 * xr and out start on 16-byte boundaries. */
MXMOE_API int mxmoe_forward_local(mxmoe_layer* layer, const void* xr, mxmoe_dtype xr_dtype,
                        const float* rscale, const int32_t* expert,
                        const float* weight, uint32_t n_pairs, void* out,
                        mxmoe_dtype out_dtype, void* stream);

/* ---- expert parallelism over peer memory (NVLink / NVSwitch) -------------
 * Instead of a gather and two NCCL all-to-alls, the source GPU's dispatch
 * kernel writes each routed pair straight into the owning GPU's receive
 * buffers, and the owner's W2 epilogue writes each pair's output straight
 * into the source GPU's return buffer.  Buffers are shared with CUDA IPC:
 * every rank allocates with mxmoe_ipc_alloc, exchanges the handles on the
 * host, and opens its peers' handles with mxmoe_ipc_open.  Ordering between
 * the writes and their readers is the caller's (a collective barrier on the
 * stream after mxmoe_dispatch_pairs and after mxmoe_forward_local_meta). */
#define MXMOE_IPC_HANDLE_BYTES 64
MXMOE_API int mxmoe_ipc_alloc(size_t bytes, int device, void** ptr, void* handle);
MXMOE_API int mxmoe_ipc_free(void* ptr, int device);
MXMOE_API int mxmoe_ipc_open(const void* handle, int device, void** peer_ptr);
MXMOE_API int mxmoe_ipc_close(void* peer_ptr, int device);

/* Source side.  perm / offsets: the canonical permutation of mxmoe_route;
 * experts of rank g are [g * experts_per_rank, (g + 1) * experts_per_rank).
 * counts [world][world] (device): pairs rank s sends to rank g at
 * counts[s * world + g].  For every pair, writes the token row (x's dtype)
 * to peer_x[g] and four 32-bit words {bits of rscale[t], expert, bits of
 * topk_w[p], rank << 24 | canonical position} to peer_meta[g], at row
 * (pairs lower ranks send to g) + (position within the pairs for g).
 * peer_x / peer_meta: device arrays of world pointers; every receive buffer
 * holds recv_cap rows.  A row at or past recv_cap is not written and sets
 * *err (device int, may be null) to 8.  n_tokens * k < 2^24. */
MXMOE_API int mxmoe_dispatch_pairs(const void* x, mxmoe_dtype x_dtype, uint32_t n_tokens, uint32_t d_model,
                         uint32_t k, const int32_t* perm, const float* rscale,
                         const int32_t* topk_idx, const float* topk_w, const int32_t* offsets,
                         uint32_t experts_per_rank, uint32_t world, uint32_t rank,
                         const int32_t* counts, void* const* peer_x, uint32_t* const* peer_meta,
                         uint32_t recv_cap, int* err, void* stream);

/* Owner side: expert FFN of this layer's shard over n_pairs received rows
 * xr [n_pairs][d] with metadata [n_pairs][4] as written by
 * mxmoe_dispatch_pairs.  The bf16 output weight * (W2 act + b2) of each pair
 * goes to row (slot & 0xFFFFFF) of ret_ptrs[slot >> 24] (device array of the
 * world ranks' return buffers, ret_rows x d bf16 each, canonical order).
 * flags: MXMOE_RETURN_FROM_EPILOGUE makes the W2 epilogue store to the peers
 * directly; by default W2 writes locally and a copy pass pushes whole rows.
 * A slot outside (world, ret_rows) is not written and sets status 8. */
#define MXMOE_RETURN_FROM_EPILOGUE 0x1u
MXMOE_API int mxmoe_forward_local_meta(mxmoe_layer* layer, const void* xr, mxmoe_dtype xr_dtype,
                             const uint32_t* meta, uint32_t n_pairs, void* const* ret_ptrs,
                             uint32_t world, uint32_t ret_rows, uint32_t flags, void* stream);

/* ---- expert parallelism, quantized dispatch into the owners' layouts ----
 * The source rank quantizes its own tokens once and writes each pair's E4M3
 * codes, scale words and row metadata straight into the owning rank's GEMM
 * operand buffers, at the pair's row in the owner's expert-sorted layout,
 * which every rank derives from the all-gathered pair counts.  The owner
 * then runs W1/W2 with no permutation or quantization of its own and pushes
 * each output row back to the source's return buffer.  No host
 * synchronisation is needed within a step.
 *
 * mxmoe_ep_reserve: sizes this layer's workspace for world ranks of up to
 * max_tokens tokens each (it cannot grow afterwards) and returns 3 IPC
 * handles (3 x MXMOE_IPC_HANDLE_BYTES): activation codes, row-major scale
 * bytes, row metadata.  Ranks exchange them and open the peers' with
 * mxmoe_ipc_open.  The layer's shard must be E / world experts. */
MXMOE_API int mxmoe_ep_reserve(mxmoe_layer* layer, uint32_t max_tokens, uint32_t world, void* handles);
/* The same 3 buffers as device pointers of this process (ranks emulated on
 * one GPU use them in place of opened handles). */
MXMOE_API int mxmoe_ep_buffers(mxmoe_layer* layer, void** ptrs);

/* Source side, after mxmoe_route: counts [world][E] (device) = every rank's
 * pairs per expert (offsets[e + 1] - offsets[e], all-gathered); inv and
 * offsets are this rank's canonical maps.  peer_bufs: device array of
 * 3 x world pointers, grouped by buffer in the mxmoe_ep_reserve order
 * ([codes of ranks 0..world-1][scales ...][metadata ...]).  Also records, for this
 * rank's own experts, the layout mxmoe_ep_experts runs on.  Every rank must
 * pass the same counts and x dtype. */
MXMOE_API int mxmoe_ep_dispatch(mxmoe_layer* layer, const void* x, mxmoe_dtype x_dtype, uint32_t n_tokens,
                      const float* rscale, const int32_t* topk_idx, const float* topk_w,
                      const int32_t* inv, const int32_t* offsets, const int32_t* counts,
                      uint32_t rank, void* const* peer_bufs, void* stream);

/* Owner side, once every rank's dispatch has completed: the expert FFN over
 * the rows the sources wrote, each output weight * (W2 act + b2) pushed to
 * row (slot & 0xFFFFFF) of peer_ret[slot >> 24] (bf16 return buffers of
 * ret_rows rows, canonical order at the source). */
MXMOE_API int mxmoe_ep_experts(mxmoe_layer* layer, mxmoe_dtype x_dtype, void* const* peer_ret, uint32_t ret_rows,
                     void* stream);

/* ---- expert-parallel step behind the C ABI ----
 * One call per rank and step runs the whole expert-parallel layer: route ->
 * count exchange -> quantized dispatch -> expert FFN -> return -> combine
 * (the QuantizedPeerMoe step of the Python host, without Python).  Between
 * the phases the ranks meet three times through the caller's barrier:
 *   barrier(ctx, stream) must return once every rank of the group has called
 *   it for this phase, with each rank's work enqueued on its stream before the
 *   call complete before any rank's work enqueued after it starts (a stream
 *   synchronize plus a host barrier, or a collective enqueued on `stream`).
 *   Non-zero means failure; mxmoe_ep_forward then returns MXMOE_ERR_CUDA.
 * The library never waits on another rank inside a kernel, so ranks may also
 * share one GPU (each on its own stream and thread).
 *
 * mxmoe_ep_attach (after mxmoe_ep_reserve on every rank): peer_bufs is a host
 * array of 3 x world device pointers grouped by buffer ([codes of ranks
 * 0..world-1][scales ...][metadata ...], mxmoe_ep_buffers of each rank, opened
 * with mxmoe_ipc_open); peer_ret[r] is rank r's bf16 return buffer of
 * max_tokens * k x d_model values, peer_counts[r] rank r's int32 count table
 * of world x num_experts values (both caller-allocated, mxmoe_ipc_alloc for
 * ranks on other GPUs), each as this process sees it. */
typedef int (*mxmoe_ep_barrier_fn)(void* ctx, void* stream);
MXMOE_API int mxmoe_ep_attach(mxmoe_layer* layer, uint32_t rank, uint32_t world, void* const* peer_bufs,
                              void* const* peer_ret, int32_t* const* peer_counts, mxmoe_ep_barrier_fn barrier,
                              void* barrier_ctx);
/* One expert-parallel step of this rank: x [n_tokens][d_model] device (f32 or
 * bf16, n_tokens <= the reserved max_tokens, may be 0), y likewise; y = x +
 * MoE(x) over all ranks' experts.  Every rank of the group must call it for
 * every step with the same x dtype.  16-byte aligned buffers. */
MXMOE_API int mxmoe_ep_forward(mxmoe_layer* layer, const void* x, mxmoe_dtype x_dtype, uint32_t n_tokens,
                               void* y, mxmoe_dtype y_dtype, void* stream);

/* ---- expert placement for skewed routing (host only, no device work) ----
 * New surface: the reference is single-rank (docs/gpt-oss-architecture.md:22).
 * mxmoe_ep_plan_replicas: `extra` copy slots handed out greedily to the
 * expert with the largest load per copy (lowest id on ties); src[0 .. E +
 * extra) receives the original expert of every slot (src[e] = e for e < E).
 * mxmoe_ep_balanced_placement: expert order for contiguous shards of
 * E / world experts: experts in decreasing load (ties to the lower id) go to
 * the rank with the least load that has a free slot (ties to the lower rank);
 * order[r * E / world ..] lists rank r's experts in increasing id.  The caller
 * permutes the gate rows, gate bias, weights, scales and biases by `order`
 * before mxmoe_set_router / mxmoe_upload_experts.  Both give the results of
 * mxmoe.ep.plan_replicas / balanced_placement in the Python mirror. */
MXMOE_API int mxmoe_ep_plan_replicas(const double* loads, uint32_t num_experts, uint32_t extra, int32_t* src);
MXMOE_API int mxmoe_ep_balanced_placement(const double* loads, uint32_t num_experts, uint32_t world,
                                          int32_t* order);

/* Combine (src/moe/mod.rs:405-411): y[t] = x[t] + sum over the token's k
 * pairs in increasing expert index of pair_out[inv[t*k+s]] (pair_out in
 * permuted order, pair_dtype).  residual = 0 omits x.  Device pointers, each
 * starting on a 16-byte boundary; d_model a multiple of 4. */
MXMOE_API int mxmoe_combine(const void* x, mxmoe_dtype x_dtype, uint32_t n_tokens,
                  uint32_t d_model, uint32_t k, const int32_t* topk_idx,
                  const int32_t* inv, const void* pair_out,
                  mxmoe_dtype pair_dtype, int residual, void* y,
                  mxmoe_dtype y_dtype, void* stream);

/* ---------------------------------------------------------------------------
 * model.bin reader (src/loader/modelbin.rs).  The file is the GPT-OSS v1.0
 * container that src/bin/gptoss_export.rs writes: a header, a tokenizer
 * section padded to 16 KiB, the bf16 dense tensors (embedding, per-layer
 * attention / MoE norm / gate, final norm, unembedding, each segment 16-byte
 * aligned), then one 16 KiB-aligned MXFP4 expert payload per layer.  Only the
 * MoE part is loaded here; the reader checks the magic and that every section
 * it touches lies inside the file (MXMOE_ERR_INVALID_ARG otherwise).
 * ------------------------------------------------------------------------- */

/* Header fields parse_headers reads (src/loader/modelbin.rs:75-151), plus the
 * byte offsets this reader derives. */
typedef struct mxmoe_modelbin_header {
  uint32_t context_length;
  uint32_t num_blocks;          /* layers */
  uint32_t num_experts;
  uint32_t num_active_experts;  /* experts per token */
  uint32_t embedding_dim;       /* d_model */
  uint32_t mlp_dim;             /* ffn_hidden */
  float swiglu_limit;
  uint32_t head_dim;
  uint32_t num_heads;
  uint32_t num_kv_heads;
  uint32_t attention_window;
  float rms_eps;
  uint32_t num_text_tokens;
  uint32_t num_special_tokens;
  uint64_t dense_offset;        /* first byte of the embedding table (16 KiB aligned) */
  uint64_t moe_offset;          /* first byte of layer 0's expert payload */
  uint64_t moe_layer_stride;    /* bytes from one layer's expert payload to the next */
  uint64_t file_bytes;
} mxmoe_modelbin_header;

/* Parses the header of the model.bin at `path` (a host file). */
MXMOE_API int mxmoe_modelbin_info(const char* path, mxmoe_modelbin_header* out);

/* Creates the MoE layer `layer` of the model.bin at `path` on `device`, the
 * part of load_modelbin_into (src/loader/modelbin.rs:158-462) that feeds
 * MoeGatedSwiGLU: config from the header (d_model, ffn_hidden, num_experts,
 * num_active_experts, swiglu_limit, rms_eps; alpha 1.702), the router from
 * layers.{layer}.mlp.norm.scale and mlp.gate (bf16, :273-291), the experts
 * from the layer's MXFP4 payload with ue8_offset 14 (:452-453) and the bf16
 * mlp1/mlp2 biases (:362-406).  flags are MXMOE_FLAG_*.  expert_count == 0
 * loads every expert; otherwise only [expert_begin, expert_begin +
 * expert_count) is read and uploaded (mxmoe_set_expert_shard), so each
 * expert-parallel rank reads its own share of the file. */
MXMOE_API int mxmoe_modelbin_load_layer(const char* path, uint32_t layer, int32_t device, uint32_t flags,
                              uint32_t expert_begin, uint32_t expert_count, void* stream,
                              mxmoe_layer** out);

/* Replaces load_gptoss_moe (src/loader/gpt_oss.rs:369-423) for one layer:
 * creates MoE layer `layer` from a GPT-OSS safetensors checkpoint split over
 * paths[0..n_paths) (tensors block.{layer}.mlp.{norm.scale, gate.weight,
 * gate.bias, mlp1_weight.blocks, mlp1_weight.scales, mlp1_bias,
 * mlp2_weight.blocks, mlp2_weight.scales, mlp2_bias}).  The MXFP4 bytes are
 * uploaded packed (scales E8M0 with bias 127, ue8_offset 0), not dequantized
 * on the host as src/loader/mxfp4.rs:82-125 does, and land in the layer
 * itself rather than the stale `layers.{l}.mlp.mlp1_weight` path.  cfg gives
 * experts_per_token, swiglu_alpha / limit, rms_eps, flags and device;
 * d_model / ffn_hidden / num_experts are taken from the tensor shapes (a
 * non-zero value in cfg must agree).  MXMOE_FLAG_INTERLEAVED_GLU is always
 * set: checkpoint W1 rows are [glu0, lin0, glu1, lin1, ...]
 * (src/activation/mod.rs:8-13).  expert_count == 0 loads every expert,
 * otherwise [expert_begin, expert_begin + expert_count) only. */
MXMOE_API int mxmoe_safetensors_load_layer(const char* const* paths, uint32_t n_paths, uint32_t layer,
                                 const mxmoe_config* cfg, uint32_t expert_begin, uint32_t expert_count,
                                 void* stream, mxmoe_layer** out);

/* ===================== streaming multi-query attention =====================
 * The attention half of a GPT-OSS decoder block:
 * StreamingMultiQueryAttention::forward_streaming
 * (src/attention/streaming_mqa.rs:239-435) with its rolling KV cache
 * StreamingMqaCache (:132-203), window policy AttnWindow
 * (src/attention/streaming.rs:14-19), sinks and quiet softmax
 * (src/attention/core.rs:7-55), cache eviction evict_and_roll_mqa
 * (src/attention/cache_ops.rs:74-117) and RoPE with NTK/YaRN scaling
 * (burn RotaryEncoding, src/rope/mod.rs:11-50).  Dropout is inference-off. */

#define MXMQA_FLAG_QUIET_SOFTMAX 0x1u /* quiet_softmax: 1 joins the normalizer */
#define MXMQA_FLAG_PRE_SCALED_QK 0x2u /* skip the 1/sqrt(d_k) score scale */
#define MXMQA_FLAG_ROPE_BY_HEAD  0x4u /* reproduce the reference's RoPE call
                                         exactly: it applies burn's rotation
                                         (which rotates along dim -2) to a
                                         [B, T, heads, d_k] tensor, so the
                                         angle index is start_pos + head, not
                                         start_pos + token.  Default off: the
                                         angle index is the token position */

/* Mirrors StreamingMultiQueryAttentionConfig (src/attention/streaming_mqa.rs:12-42)
 * without the initializer (weights are always loaded). */
typedef struct mxmqa_config {
  uint32_t d_model;
  uint32_t n_heads;
  uint32_t kv_heads;   /* num_key_value_heads; n_heads % kv_heads == 0 */
  uint32_t head_dim;   /* multiple of 4, at most 256 */
  uint32_t flags;      /* MXMQA_FLAG_* */
  int32_t device;
} mxmqa_config;

/* burn RotaryEncodingConfig + the NTK/YaRN scaling of init_ntk_yarn. */
typedef struct mxmqa_rope {
  uint32_t max_seq_len;    /* informational (positions are not table-limited) */
  float theta;             /* base, 10000 by default */
  float scaling_factor;    /* <= 1: plain RoPE */
  float initial_context;   /* YaRN: original context length */
  float ntk_alpha;
  float ntk_beta;
} mxmqa_rope;

typedef struct mxmqa_layer mxmqa_layer;
typedef struct mxmqa_cache mxmqa_cache;

/* Replaces StreamingMultiQueryAttentionConfig::init (:94-131). */
MXMOE_API int mxmqa_create(const mxmqa_config* cfg, mxmqa_layer** out);
MXMOE_API int mxmqa_destroy(mxmqa_layer* layer);

/* The query / key / value / output Linear layers as Burn stores them:
 * weight [d_in][d_out], bias [d_out] (NULL = zero).  q: d_model -> n_heads *
 * head_dim, k and v: d_model -> kv_heads * head_dim, o: n_heads * head_dim ->
 * d_model.  Host pointers; copies are made. */
MXMOE_API int mxmqa_set_weights(mxmqa_layer* layer, const void* wq, const void* bq, const void* wk,
                                const void* bk, const void* wv, const void* bv, const void* wo,
                                const void* bo, mxmoe_dtype dtype, void* stream);

/* The module's learned sinks (learned_sinks, :117-124): [kv_heads][groups]
 * logits, host f32; NULL removes them. */
MXMOE_API int mxmqa_set_sinks(mxmqa_layer* layer, const float* sinks);

/* RoPE for every forward of this layer (StreamingMqaParams::rope); NULL = none. */
MXMOE_API int mxmqa_set_rope(mxmqa_layer* layer, const mxmqa_rope* rope);

/* StreamingMqaCache::new (:146-167): batch x cache_len tokens of kv_heads x
 * head_dim keys and values (f32) on the layer's device, of which the first
 * sink_tokens written are never evicted. */
MXMOE_API int mxmqa_cache_create(const mxmqa_layer* layer, uint32_t batch, uint32_t cache_len,
                                 uint32_t sink_tokens, mxmqa_cache** out);
/* StreamingMqaCache::reset (:169-173). */
MXMOE_API int mxmqa_cache_reset(mxmqa_cache* cache);
/* global_end_index and local_end_index (len()) of the cache. */
MXMOE_API int mxmqa_cache_state(const mxmqa_cache* cache, uint64_t* global_end, uint64_t* local_end);
MXMOE_API int mxmqa_cache_destroy(mxmqa_cache* cache);

/* forward_streaming (:239-435): x [batch][seq_len][d_model] device (f32 or
 * bf16), written to the cache at absolute positions start_pos ..; window 0 =
 * AttnWindow::Full, w > 0 = AttnWindow::Window(w) (sink tokens + the w most
 * recent); sinks: device [n_heads] logits for this call (NULL: the module's);
 * attn_bias: device [batch][n_heads][seq_len][active window] f32 or NULL.
 * Like the reference, no causal mask is applied inside a chunk.  y
 * [batch][seq_len][d_model] device.  Stream-ordered; the cache bookkeeping
 * is host state, so calls on one cache must be issued in order. */
MXMOE_API int mxmqa_forward_streaming(mxmqa_layer* layer, mxmqa_cache* cache, const void* x,
                                      mxmoe_dtype x_dtype, uint32_t batch, uint32_t seq_len,
                                      uint64_t start_pos, uint32_t window, const float* sinks,
                                      const float* attn_bias, void* y, mxmoe_dtype y_dtype,
                                      void* stream);

#ifdef __cplusplus
}
#endif
#endif /* MXMOE_H */
