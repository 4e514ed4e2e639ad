// api.cu -- host runtime behind include/mxmoe.h: layer state, one-time weight
// repack into the tensor-core operand layout, workspace management, TMA
// descriptor creation and the forward orchestration
//   router -> permute -> quantize -> W1 GEMM -> W2 GEMM -> combine.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <climits>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <new>
#include <string>
#include <vector>

#include "../../include/mxmoe.h"
#include "kernels.h"
#include "layout.cuh"
#include "tc_gemm.h"
#include "launch_util.h"

using namespace mxmoe;

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

}  // namespace

namespace mxmoe {
// Lets the other translation units of the library (the model.bin reader)
// report through mxmoe_last_error().
int set_last_error(int code, const char* msg) {
  g_last_error = msg;
  return code;
}
}  // namespace mxmoe

namespace {

#define CUDA_TRY(expr)                                                                        \
  do {                                                                                        \
    cudaError_t _e = (expr);                                                                  \
    if (_e != cudaSuccess)                                                                    \
      return fail(_e == cudaErrorMemoryAllocation ? MXMOE_ERR_OOM : MXMOE_ERR_CUDA, "%s: %s (%s:%d)", #expr, \
                  cudaGetErrorString(_e), __FILE__, __LINE__);                                \
  } while (0)

#define TRY(expr)                  \
  do {                             \
    int _r = (expr);               \
    if (_r != MXMOE_OK) return _r; \
  } while (0)

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// 3-D tiled map: dims {inner, rows, outer}, byte strides {row, outer}, box {128, box_rows, 1}, 128-byte swizzle.
int make_tmap(CUtensorMap* m, CUtensorMapDataType dt, void* base, uint64_t inner, uint64_t rows, uint64_t outer,
              uint64_t row_stride, uint64_t outer_stride, uint32_t box_rows) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return fail(MXMOE_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  const cuuint64_t gdim[3] = {inner, rows, outer};
  const cuuint64_t gstr[2] = {row_stride, outer_stride};
  const cuuint32_t box[3] = {static_cast<cuuint32_t>(kTileK), box_rows, 1};
  const cuuint32_t es[3] = {1, 1, 1};
  CUresult r = enc(m, dt, 3, base, gdim, gstr, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(MXMOE_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d): inner=%llu rows=%llu outer=%llu box_rows=%u",
                static_cast<int>(r), (unsigned long long)inner, (unsigned long long)rows,
                (unsigned long long)outer, box_rows);
  return MXMOE_OK;
}

template <typename T>
int dalloc(T** p, size_t count) {
  *p = nullptr;
  if (count == 0) return MXMOE_OK;
  cudaError_t e = cudaMalloc(reinterpret_cast<void**>(p), count * sizeof(T));
  if (e != cudaSuccess) {
    *p = nullptr;
    return fail(MXMOE_ERR_OOM, "cudaMalloc(%zu bytes): %s", count * sizeof(T), cudaGetErrorString(e));
  }
  return MXMOE_OK;
}
template <typename T>
void dfree(T*& p) {
  if (p) cudaFree(p);
  p = nullptr;
}

// Row-major weight scale rows for the dequant-GEMV: kp / 32 bytes rounded up
// to 16, so that a row range is one bulk copy.
uint32_t dq_scale_row_bytes(uint32_t kp) { return round_up(kp / 32u, 16u); }

// Status block: word 0 is the status code, words 2-4 where the dequant-GEMV's
// W1 -> W2 grid wait gave up (-1, arrivals seen, arrivals expected), word
// kStatusSyncOffset that wait's arrival counter; the words after it are
// spare (one per local expert).  Zeroed before every forward.
constexpr int kStatusSyncOffset = 16;
// Wait limit of a forward run under mxmoe_set_fault_injection.
constexpr unsigned long long kFaultWaitNs = 1000ull * 1000ull;  // 1 ms

// mxmoe_forward_host splits large batches into up to this many chunks so
// that the copies of one chunk overlap the forward of another.
constexpr int kReturnParts = 2;  // W2 expert ranges of the expert-parallel return overlap (4 measured slower: launch tails)
constexpr int kHostChunksMax = 4;
constexpr uint32_t kHostChunkMinTokens = 1024;

// The dequant-GEMV takes forwards of at most this many routed pairs (so at
// most this many tokens); the router then also writes their normalized f16
// rows for it.
constexpr uint32_t kGemvMaxTokens = 64;

float bf16_to_f32(uint16_t h) {
  uint32_t u = static_cast<uint32_t>(h) << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

void to_f32(const void* src, mxmoe_dtype dt, size_t n, float* dst) {
  if (dt == MXMOE_F32) {
    std::memcpy(dst, src, n * sizeof(float));
  } else {
    const uint16_t* s = static_cast<const uint16_t*>(src);
    for (size_t i = 0; i < n; ++i) dst[i] = bf16_to_f32(s[i]);
  }
}

cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

// Box rows of the activation tensor maps; 16-row boxes feed the stacked tiles.
constexpr int kNumTileWidths = 4;
constexpr int kTileWidths[kNumTileWidths] = {32, 64, 128, 256};

}  // namespace

// Per-forward scratch sized for `cap_tokens` tokens x k pairs.
struct Workspace {
  uint32_t cap_tokens = 0;  // tokens
  uint32_t cap_pairs = 0;   // n * k
  uint32_t rows = 0;        // padded activation rows
  uint32_t row_blocks = 0;  // scale-atom row blocks (rows / 16 + slack)
  float* logits = nullptr;
  int32_t* topk_idx = nullptr;
  float* topk_w = nullptr;
  float* rscale = nullptr;
  int32_t* offsets = nullptr;
  int32_t* perm_c = nullptr;
  int32_t* inv_c = nullptr;
  int32_t* poff = nullptr;
  int32_t* counts = nullptr;
  int32_t* ntile_prefix = nullptr;
  int32_t* perm_p = nullptr;
  int32_t* inv_p = nullptr;
  uint8_t* xq = nullptr;   // [3][rows][kp1]
  uint8_t* xsf = nullptr;  // [3][row_blocks][kp1/128][512]
  uint8_t* aq = nullptr;   // [2][rows][kp2]
  uint8_t* asf = nullptr;  // [2][row_blocks][kp2/128][512]
  float* y_pair = nullptr; // [rows][d]
  float* act_f32 = nullptr;// [rows][fp] (SIMT path only)
  int32_t* local_idx = nullptr; // [cap_pairs] local expert ids (expert-parallel receive side)
  int32_t* perm_scratch = nullptr; // multi-block permutation (permute_scratch_ints)
  uint32_t* ret_slot = nullptr;    // [cap_pairs] expert-parallel return slots of received pairs
  // expert-parallel rows written by the source ranks (mxmoe_ep_dispatch), per layout row
  float* pos_rscale = nullptr;     // [rows]
  float* pos_weight = nullptr;     // [rows]
  uint32_t* pos_slot = nullptr;    // [rows]
  int32_t* iota = nullptr;         // [rows] identity permutation
  int32_t* ep_src_base = nullptr;  // [E_total]
  uint8_t* ep_sf_rows = nullptr;   // [rows][kMaxTerms][ep_sf_row_bytes] scale bytes written by the sources
  uint32_t* ep_meta = nullptr;     // [rows][4] {1/rms, route weight, return slot, 0} written by the sources
  uint32_t ep_sf_row_bytes = 0;
  int pair_dtype = MXMOE_F32;   // element type the last run_experts wrote y_pair in
  CUtensorMap tmap_x[kNumTileWidths];
  CUtensorMap tmap_act[kNumTileWidths];
  // stacked tiles of 16 / 32 / 64 pairs: boxes of 32 / 64 / 128 rows over 2 x rows code rows
  CUtensorMap tmap_x_stk[3], tmap_act_stk[3];
  // FP4 decode tiles (allocated on first use, sized for the at most
  // kF4MaxAvgPairs pairs per expert that select them): four E2M1 terms per
  // pair, rows4 pair rows, packed codes [4 * rows4][kp / 2], scale atoms
  // [rows4 / 32][kp / 128][512]
  uint32_t rows4 = 0;
  uint8_t* xq4 = nullptr;
  uint8_t* xsf4 = nullptr;
  uint8_t* aq4 = nullptr;
  uint8_t* asf4 = nullptr;
  float* act4_f32 = nullptr;  // [rows4][fp] W1 output before quantization
  __half* xh = nullptr;       // [kGemvMaxTokens][d] router-normalized f16 token rows (dequant-GEMV input)
  int* tok_ctr = nullptr;     // [8] per-token block counters of the small-batch router (kept zero)
  CUtensorMap tmap_x4[2], tmap_act4[2];  // boxes of 4 x 16 and 4 x 32 rows
};

struct mxmoe_layer {
  mxmoe_config cfg{};
  uint32_t d = 0, f = 0, fp = 0, E_total = 0, k = 0;
  uint32_t e_begin = 0, e_count = 0;  // local expert shard
  uint32_t kp1 = 0, kp2 = 0, m_tiles1 = 0, m_tiles2 = 0;
  int num_sms = 148;
  size_t smem_limit = 227 * 1024;
  bool router_ready = false, experts_ready = false;
  bool gamma_is_one = true;
  // powers of two that keep the dequant-GEMV's f16 operands in range:
  // normalized rows |x * gamma / rms| <= sqrt(d) * max|gamma|, and SwiGLU
  // outputs |act| <= max(limit, 0.28 / alpha) * (limit + 1)
  float dq_x_scale = 1.0f, dq_act_scale = 1.0f;
  float* gamma = nullptr;
  float* gate_w = nullptr;  // packed for the router kernel (pack_router_gate)
  float* gate_b = nullptr;
  uint8_t* w1q = nullptr;
  uint8_t* w1sf = nullptr;
  float* b1 = nullptr;
  uint8_t* w2q = nullptr;
  uint8_t* w2sf = nullptr;
  float* b2 = nullptr;
  uint8_t* w1sr = nullptr;  // row-major scale copies for the dequant-GEMV (dq_scale_row_bytes per row)
  uint8_t* w2sr = nullptr;
  int* err = nullptr;       // status block (kStatusSyncOffset + E_total words)
  CUtensorMap tmap_w1[2] = {}, tmap_w2[2] = {};  // box rows 128 (weights-as-A) / 256 (tokens-as-A)
  CUtensorMap tmap_w1_f4 = {}, tmap_w2_f4 = {};  // packed bytes, 256-row boxes of K 256 (FP4 tiles)
  Workspace ws;
  uint32_t last_n = 0;
  bool profiling = false;
  bool profile_valid = false;
  uint32_t fault = 0;  // mxmoe_set_fault_injection: applies to the next forward, then clears
  // CUDA-graph replay of mxmoe_forward: bumped by anything that moves a buffer
  // or changes a launch (uploads, workspace growth, shard changes)
  uint64_t generation = 0;
  struct FwdGraph {
    const void* x = nullptr;
    void* y = nullptr;
    uint32_t n = 0;
    int xd = -1, yd = -1;
    uint64_t gen = ~0ull;
    cudaGraphExec_t exec = nullptr;
    bool failed = false;  // capture failed for this key: run directly
  } graph;
  cudaStream_t cap_stream = nullptr;  // capture happens here; replays go to the caller's stream
  // mxmoe_forward_host: device copies of the host rows, copy streams and
  // per-chunk events and status words (this layer's device only)
  struct HostStaging {
    void* dx = nullptr;
    void* dy = nullptr;
    size_t cx = 0, cy = 0;
    cudaStream_t s_in = nullptr, s_out = nullptr;
    cudaEvent_t ev_in[kHostChunksMax] = {}, ev_done[kHostChunksMax] = {};
    int* status = nullptr;  // pinned host, one word per chunk
  } hs;
  // expert parallelism over peer memory: the workspace is shared with peers and must not move
  bool ep_reserved = false;
  uint32_t ep_world = 0, ep_max_tokens = 0;
  // mxmoe_ep_attach: this rank's place and the peers' buffers, as device tables
  struct EpAttach {
    bool on = false;
    uint32_t rank = 0;
    void** bufs = nullptr;        // [3][world] layout buffers (device table)
    void** ret = nullptr;         // [world] return buffers (device table)
    int32_t** counts = nullptr;   // [world] count tables (device table)
    void* own_ret = nullptr;
    int32_t* own_counts = nullptr;
    mxmoe_ep_barrier_fn barrier = nullptr;
    void* ctx = nullptr;
  } epa;
  cudaEvent_t ev[8] = {};
  // expert-parallel return of W2's first expert half (run_experts with a ReturnSplit)
  cudaStream_t ret_stream = nullptr;
  cudaEvent_t ret_ev[kReturnParts + 1] = {};
};

namespace {

void free_workspace(Workspace& w) {
  dfree(w.logits); dfree(w.topk_idx); dfree(w.topk_w); dfree(w.rscale);
  dfree(w.offsets); dfree(w.perm_c); dfree(w.inv_c); dfree(w.poff); dfree(w.counts);
  dfree(w.ntile_prefix); dfree(w.perm_p); dfree(w.inv_p);
  dfree(w.xq); dfree(w.xsf); dfree(w.aq); dfree(w.asf); dfree(w.y_pair); dfree(w.act_f32);
  dfree(w.xq4); dfree(w.xsf4); dfree(w.aq4); dfree(w.asf4); dfree(w.act4_f32); dfree(w.xh); dfree(w.tok_ctr);
  w.rows4 = 0;
  dfree(w.local_idx);
  dfree(w.ret_slot);
  dfree(w.pos_rscale);
  dfree(w.pos_weight);
  dfree(w.pos_slot);
  dfree(w.iota);
  dfree(w.ep_src_base);
  dfree(w.ep_sf_rows);
  dfree(w.ep_meta);
  dfree(w.perm_scratch);
  w.cap_tokens = w.cap_pairs = w.rows = w.row_blocks = 0;
}

// Sizes the workspace for n tokens with k pairs each (k = 1 for the
// expert-parallel receive side).
int ensure_workspace(mxmoe_layer* L, uint32_t n_tokens, uint32_t k) {
  Workspace& w = L->ws;
  const uint64_t pairs = static_cast<uint64_t>(n_tokens) * k;
  if (n_tokens <= w.cap_tokens && pairs <= w.cap_pairs && w.cap_tokens > 0) return MXMOE_OK;
  if (pairs > (1u << 28)) return fail(MXMOE_ERR_TOO_LARGE, "too many pairs: %llu", (unsigned long long)pairs);
  if (L->ep_reserved)
    return fail(MXMOE_ERR_TOO_LARGE, "workspace is shared with peer ranks and cannot grow to %llu pairs",
                (unsigned long long)pairs);
  // Capacities only grow (the expert-parallel receive side alternates sizes
  // from step to step), with an eighth of headroom on the requested growth.
  const uint32_t old_t = w.cap_tokens, old_p = w.cap_pairs;
  CUDA_TRY(cudaDeviceSynchronize());
  free_workspace(w);
  ++L->generation;
  const uint32_t E = L->e_count, Et = L->E_total;
  auto grow = [](uint32_t old, uint64_t want) -> uint32_t {
    if (want <= old) return old;
    const uint64_t g = old ? want + want / 8 : want;
    return static_cast<uint32_t>(std::max<uint64_t>(std::min<uint64_t>(g, 1u << 28), 1));
  };
  const uint32_t cap_t = grow(old_t, n_tokens);
  const uint32_t cap_p = grow(old_p, pairs);
  w.rows = round_up(cap_p, kRowBlock) + E * kRowBlock + 256;
  w.row_blocks = w.rows / 16 + 2;  // enough atoms for the smallest (16-pair stacked) tile
  const uint64_t kc1 = L->kp1 / kTileK, kc2 = L->kp2 / kTileK;
  TRY(dalloc(&w.logits, static_cast<size_t>(cap_t) * Et));
  TRY(dalloc(&w.topk_idx, cap_p));
  TRY(dalloc(&w.topk_w, cap_p));
  TRY(dalloc(&w.rscale, std::max(cap_t, cap_p)));
  TRY(dalloc(&w.offsets, Et + 1));
  TRY(dalloc(&w.perm_c, cap_p));
  TRY(dalloc(&w.inv_c, cap_p));
  TRY(dalloc(&w.poff, Et + 1));
  TRY(dalloc(&w.counts, Et + 1));
  TRY(dalloc(&w.ntile_prefix, Et + 1));
  TRY(dalloc(&w.perm_p, w.rows));
  TRY(dalloc(&w.inv_p, cap_p));
  TRY(dalloc(&w.local_idx, cap_p));
  TRY(dalloc(&w.ret_slot, cap_p));
  TRY(dalloc(&w.pos_rscale, w.rows));
  TRY(dalloc(&w.pos_weight, w.rows));
  TRY(dalloc(&w.pos_slot, w.rows));
  TRY(dalloc(&w.iota, w.rows));
  TRY(dalloc(&w.ep_src_base, Et));
  w.ep_sf_row_bytes = round_up(L->d / 32, 16);
  TRY(dalloc(&w.ep_sf_rows, static_cast<size_t>(w.rows) * 3 * w.ep_sf_row_bytes));  // up to 3 terms
  TRY(dalloc(&w.ep_meta, static_cast<size_t>(w.rows) * 4));
  CUDA_TRY(launch_iota(w.iota, static_cast<int>(w.rows), 0));
  const size_t pscr = permute_scratch_ints(static_cast<int>(cap_p), static_cast<int>(Et));
  TRY(dalloc(&w.perm_scratch, pscr));
  CUDA_TRY(cudaMemset(w.perm_scratch, 0, pscr * sizeof(int32_t)));
  TRY(dalloc(&w.xq, 3ull * w.rows * L->kp1));
  TRY(dalloc(&w.xsf, 3ull * w.row_blocks * kc1 * kSfAtomBytes));
  TRY(dalloc(&w.aq, 2ull * w.rows * L->kp2));
  TRY(dalloc(&w.asf, 2ull * w.row_blocks * kc2 * kSfAtomBytes));
  TRY(dalloc(&w.y_pair, static_cast<size_t>(w.rows) * L->d));
  TRY(dalloc(&w.xh, static_cast<size_t>(std::min<uint32_t>(cap_t, kGemvMaxTokens)) * L->d));
  TRY(dalloc(&w.tok_ctr, 8));
  CUDA_TRY(cudaMemset(w.tok_ctr, 0, 8 * sizeof(int)));
  // Padding columns (K beyond d or f) and never-written scale bytes must read
  // as zero codes / finite scales for every later forward.
  CUDA_TRY(cudaMemset(w.xq, 0, 3ull * w.rows * L->kp1));
  CUDA_TRY(cudaMemset(w.xsf, 0, 3ull * w.row_blocks * kc1 * kSfAtomBytes));
  CUDA_TRY(cudaMemset(w.aq, 0, 2ull * w.rows * L->kp2));
  CUDA_TRY(cudaMemset(w.asf, 0, 2ull * w.row_blocks * kc2 * kSfAtomBytes));
  CUDA_TRY(cudaMemset(w.perm_p, 0, sizeof(int32_t) * w.rows));
  for (int i = 0; i < 3; ++i) {
    const uint32_t box = 32u << i;
    TRY(make_tmap(&w.tmap_x_stk[i], CU_TENSOR_MAP_DATA_TYPE_UINT8, w.xq, L->kp1, 2ull * w.rows, 1, L->kp1,
                  2ull * w.rows * L->kp1, box));
    TRY(make_tmap(&w.tmap_act_stk[i], CU_TENSOR_MAP_DATA_TYPE_UINT8, w.aq, L->kp2, 2ull * w.rows, 1, L->kp2,
                  2ull * w.rows * L->kp2, box));
  }
  for (int i = 0; i < kNumTileWidths; ++i) {
    TRY(make_tmap(&w.tmap_x[i], CU_TENSOR_MAP_DATA_TYPE_UINT8, w.xq, L->kp1, w.rows, 3, L->kp1,
                  static_cast<uint64_t>(w.rows) * L->kp1, kTileWidths[i]));
    TRY(make_tmap(&w.tmap_act[i], CU_TENSOR_MAP_DATA_TYPE_UINT8, w.aq, L->kp2, w.rows, 2, L->kp2,
                  static_cast<uint64_t>(w.rows) * L->kp2, kTileWidths[i]));
  }
  w.cap_tokens = cap_t;
  w.cap_pairs = cap_p;
  return MXMOE_OK;
}

// FP4 decode tiles serve up to this many routed pairs per expert on average
// (beyond it the E4M3 64-pair stacked tiles issue no more MMAs per weight
// byte and read each weight tile once).
constexpr int kF4MaxAvgPairs = 24;

// FP4 decode buffers: fp4 plans keep at most kF4MaxAvgPairs * E pairs, and
// their expert segments are padded to the pair tile (at most kF4PairTile).
int ensure_f4(mxmoe_layer* L) {
  Workspace& w = L->ws;
  if (w.xq4) return MXMOE_OK;
  const uint32_t E = L->e_count;
  const uint32_t rows4 = round_up((kF4MaxAvgPairs + kF4PairTile) * E + 64, kF4PairTile);
  const uint64_t kc1 = L->kp1 / kTileK, kc2 = L->kp2 / kTileK;
  const uint64_t tiles = rows4 / kF4PairTileSmall;  // scale atoms per 128-K chunk, smallest tile
  const size_t xq_bytes = static_cast<size_t>(kF4Terms) * rows4 * (L->kp1 / 2);
  const size_t aq_bytes = static_cast<size_t>(kF4Terms) * rows4 * (L->kp2 / 2);
  TRY(dalloc(&w.xq4, xq_bytes));
  TRY(dalloc(&w.aq4, aq_bytes));
  TRY(dalloc(&w.xsf4, tiles * kc1 * kSfAtomBytes));
  TRY(dalloc(&w.asf4, tiles * kc2 * kSfAtomBytes));
  TRY(dalloc(&w.act4_f32, static_cast<size_t>(rows4) * L->fp));
  // K padding and rows of absent pairs read as zero codes and finite scales
  CUDA_TRY(cudaMemset(w.xq4, 0, xq_bytes));
  CUDA_TRY(cudaMemset(w.aq4, 0, aq_bytes));
  CUDA_TRY(cudaMemset(w.xsf4, 0, tiles * kc1 * kSfAtomBytes));
  CUDA_TRY(cudaMemset(w.asf4, 0, tiles * kc2 * kSfAtomBytes));
  for (int i = 0; i < 2; ++i) {
    const uint32_t box = kF4Terms * (i ? kF4PairTile : kF4PairTileSmall);
    TRY(make_tmap(&w.tmap_x4[i], CU_TENSOR_MAP_DATA_TYPE_UINT8, w.xq4, L->kp1 / 2, uint64_t(kF4Terms) * rows4, 1,
                  L->kp1 / 2, xq_bytes, box));
    TRY(make_tmap(&w.tmap_act4[i], CU_TENSOR_MAP_DATA_TYPE_UINT8, w.aq4, L->kp2 / 2, uint64_t(kF4Terms) * rows4, 1,
                  L->kp2 / 2, aq_bytes, box));
  }
  w.rows4 = rows4;
  return MXMOE_OK;
}

// Power of two p with bound * p <= 2^14 (f16 keeps 11 significant bits up to
// 65504, so the scaled operand stays normal and well inside the range).
// Power of two that maps |v| <= bound to at most 512: the dequant-GEMV sums
// 16 products of an E2M1 value (|code| <= 6) and a scaled activation in f16,
// 16 * 6 * 512 = 49152 < 65504.
float f16_range_scale(float bound) {
  if (!(bound > 0.0f) || !std::isfinite(bound)) return 1.0f;
  const int ex = static_cast<int>(std::floor(std::log2(512.0f / bound)));
  return std::ldexp(1.0f, std::max(-60, std::min(60, ex)));
}

// The dequant-GEMV stores SwiGLU outputs as f16, which needs the clamp to
// bound them: a finite limit of at most 128 and a positive alpha.
bool gemv_ok(const mxmoe_layer* L) {
  const float lim = L->cfg.swiglu_limit, al = L->cfg.swiglu_alpha;
  return !(L->cfg.flags & MXMOE_FLAG_NO_GEMV) && L->d <= static_cast<uint32_t>(kDqMaxK) && L->fp <= static_cast<uint32_t>(kDqMaxK) &&
         std::isfinite(lim) && lim > 0.0f && lim <= 128.0f && al > 0.0f && std::isfinite(al);
}

// Tile plan from the average routed pairs per expert:
//   few pairs  -> weights-as-A, pair tiles of 32 / 64 / 128 (HBM-bound decode);
//   many pairs -> tokens-as-A, pair tiles of 128 x weight tiles of 256 rows.
// tw indexes the activation tensor maps (box rows 32, 64, 128, 256).
// Few pairs per expert (decode) with two-term activations: stacked 64-pair
// tiles, both terms in one MMA operand, so the tensor work per weight byte is
// halved.
// W2 in launches over up to kReturnParts ranges of the layer's experts; once
// a range is done, its rows go back to their sources on a side stream while
// the next range computes (expert-parallel step).
struct ReturnSplit {
  void* const* peer_ret;
  uint32_t ret_rows;
};

struct TilePlan {
  bool tok;
  int pair_tile;
  int tw;
  bool stacked;
  bool gemv = false;  // fused dequant-GEMV on CUDA cores instead of tensor-core tiles
  bool fp4 = false;   // kind::mxf4 stacked tiles of 16 / 32 pairs (tw 0 / 1), four E2M1 activation terms
};


// Tiny batches (at most kGemvMaxPairs routed pairs in all) go to the fused
// dequant-GEMV kernel, which spreads the weights over every SM; tensor-core
// tiles would leave most SMs idle there.
// Measured on B200 (GPT-OSS-20B layer forward): batch 1 at top-4 38 us, batch
// 2 (8 pairs) 58 us against 69 us on the kind::mxf4 tiles; the kernel takes
// at most 8 pairs.
constexpr uint64_t kGemvMaxPairs = 8;

TilePlan pick_tiles(uint64_t pairs, uint32_t experts, int x_terms, bool allow_gemv = false, bool allow_fp4 = false) {
  if (allow_gemv && pairs <= kGemvMaxPairs) return {true, 8, 0, false, true};  // callers check kGemvMaxK
  const double avg = experts ? static_cast<double>(pairs) / experts : 0.0;
  // FP4: 32-pair tiles.  16-pair tiles (half the activation bytes per
  // stage, five stages instead of four) measured no faster, and their extra
  // tiles for experts past 16 pairs break the even waves of 148 CTAs (GPT-OSS
  // decode: 23 x 32 = 736 W1 tiles, 5 per CTA, against 759).  They stay
  // selectable through the tile table for experiments.
  if (allow_fp4 && avg <= kF4MaxAvgPairs) return {true, kF4PairTile, 1, true, false, true};
  // two-term activations: stacked tiles (tw indexes tmap_x_stk / tmap_act_stk)
  if (x_terms == 2 && avg <= 12) return {true, 16, 0, true};
  if (x_terms == 2 && avg <= 24) return {true, 32, 1, true};
  if (x_terms == 2 && avg <= 48) return {true, 64, 2, true};
  if (avg <= 24) return {true, 32, 0, false};
  if (avg <= 48) return {true, 64, 1, false};
  return {true, 128, 2, false};
}

// Two E4M3 terms represent bf16 activations exactly when the RmsNorm gain is
// one (the gain is then applied nowhere and 1/rms goes to the epilogue);
// otherwise three terms keep the operand error near 2^-13.
int x_terms_for(const mxmoe_layer* L, int x_dtype) {
  return (x_dtype == MXMOE_BF16 && L->gamma_is_one) ? 2 : 3;
}

// The FP4 decode variant of run_experts: four-term E2M1 quantization into
// the stacked 32-pair layout, then W1 and W2 on kind::mxf4 tiles (K = 256
// per stage; the last stage issues only the MMAs that reach real K).
int run_experts_f4(mxmoe_layer* L, const void* x, int x_dtype, uint32_t n_tok, uint32_t k, const float* rscale,
                   const float* route_w, const TilePlan& tp, cudaStream_t st, void* const* ret_ptrs,
                   const uint32_t* ret_slot, bool y_by_pair, const int32_t* perm) {
  Workspace& w = L->ws;
  if (!w.xq4) return fail(MXMOE_ERR_INVALID_ARG, "FP4 decode buffers were not reserved");
  const uint64_t P = static_cast<uint64_t>(n_tok) * k;
  const int PT = tp.pair_tile;
  const uint64_t kc1 = L->kp1 / kTileK, kc2 = L->kp2 / kTileK;
  const float bias_mult = (L->cfg.flags & MXMOE_FLAG_BIAS_PER_FTILE) ? static_cast<float>((L->f + 255) / 256) : 1.0f;
  CUDA_TRY(launch_quantize_f4_pairs(x, x_dtype, n_tok, L->d, k, L->gamma, L->gamma_is_one ? 1 : 0, w.inv_p, w.xq4,
                                    static_cast<int>(L->kp1 / 2), w.xsf4, static_cast<int>(kc1), PT, 0, st));
  if (L->profiling) CUDA_TRY(cudaEventRecord(L->ev[3], st));
  const uint64_t max_pair_tiles = (P + PT - 1) / PT + L->e_count;
  TcParams p{};
  p.N = 256;
  p.sf_rows = PT;
  p.stacked = 1;
  p.fp4 = 1;
  p.b_terms = 1;
  p.E = L->e_count;
  p.poff = w.poff;
  p.counts = w.counts;
  p.ntile_prefix = w.ntile_prefix;
  p.alpha = L->cfg.swiglu_alpha;
  p.limit = L->cfg.swiglu_limit;
  p.rscale = rscale;
  p.perm = perm ? perm : w.perm_p;
  p.k = static_cast<int>(k);
  p.topk_w = route_w;
  p.err = L->err;
  if (L->fault == MXMOE_FAULT_SKIP_SIGNAL) {
    p.skip_stage = 1;
    p.wait_ns = kFaultWaitNs;
  }
  p.d = L->d;
  p.units = static_cast<int>(L->fp);
  p.stages = tc_gemm_max_stages(true, 256, 1, L->smem_limit, PT, true, true);
  auto stage_plan = [&](uint64_t kc, uint32_t k_real) {
    p.k_chunks = static_cast<int>(kc);
    p.k_tiles = static_cast<int>((kc + 1) / 2);
    p.last_mmas = static_cast<int>((k_real - static_cast<uint32_t>(p.k_tiles - 1) * 256u + 63u) / 64u);
  };
  // W1 + SwiGLU
  p.mode = 1;
  stage_plan(kc1, L->d);
  p.m_tiles = static_cast<int>((2 * L->fp + 255) / 256);
  p.w_row_pairs = static_cast<int>(w_sf_row_pairs(2 * L->fp));
  p.a_sf = L->w1sf;
  p.b_sf = w.xsf4;
  p.bias = L->b1;
  p.bias_stride = static_cast<int>(2 * L->fp);
  p.rows_valid = static_cast<int>(2 * L->fp);
  p.bias_mult = 1.0f;
  p.act_f32 = w.act4_f32;
  int grid = static_cast<int>(std::min<uint64_t>(L->num_sms, p.m_tiles * max_pair_tiles));
  CUDA_TRY(tc_gemm_launch(true, L->tmap_w1_f4, w.tmap_x4[tp.tw], p, grid, st));
  // the f32 activation rows of the routed pairs -> four-term E2M1 operand of W2
  CUDA_TRY(launch_quantize_f4_pairs(w.act4_f32, MXMOE_F32, static_cast<int>(P), static_cast<int>(L->fp), 1, nullptr, 1,
                                    w.inv_p, w.aq4, static_cast<int>(L->kp2 / 2), w.asf4, static_cast<int>(kc2), PT,
                                    1, st));
  if (L->profiling) CUDA_TRY(cudaEventRecord(L->ev[4], st));
  // W2 + bias + route weight
  p.mode = 2;
  stage_plan(kc2, L->fp);
  p.m_tiles = static_cast<int>((L->d + 255) / 256);
  p.w_row_pairs = static_cast<int>(w_sf_row_pairs(L->d));
  p.a_sf = L->w2sf;
  p.b_sf = w.asf4;
  p.bias = L->b2;
  p.bias_stride = static_cast<int>(L->d);
  p.rows_valid = static_cast<int>(L->d);
  p.bias_mult = bias_mult;
  p.y_pair = w.y_pair;
  p.y_pair_bf16 = reinterpret_cast<__nv_bfloat16*>(w.y_pair);
  p.ret_ptrs = ret_ptrs;
  p.ret_slot = ret_slot;
  p.y_by_pair = y_by_pair ? 1 : 0;
  w.pair_dtype = MXMOE_BF16;
  grid = static_cast<int>(std::min<uint64_t>(L->num_sms, p.m_tiles * max_pair_tiles));
  CUDA_TRY(tc_gemm_launch(true, L->tmap_w2_f4, w.tmap_act4[tp.tw], p, grid, st));
  if (L->profiling) CUDA_TRY(cudaEventRecord(L->ev[5], st));
  return MXMOE_OK;
}

// The dequant-GEMV expert FFN (dqgemv.cu) for at most kGemvMaxPairs routed
// pairs.  With y (fused mode, mxmoe_forward) it also combines into y and
// writes the canonical routing maps, and needs no permutation kernel before
// it: its pairs come from the top-k ids and the router's f16 rows xh.
// Without y it takes each pair's local expert (pair_expert) and writes pair
// row inv[pair] of y_pair for mxmoe_combine.
int run_dqgemv(mxmoe_layer* L, const void* x, int x_dtype, uint32_t n_tok, uint32_t k, const float* rscale,
               const float* route_w, const int32_t* pair_expert, const int32_t* inv, cudaStream_t st,
               const __half* xh = nullptr, void* y = nullptr, int y_dtype = MXMOE_F32) {
  Workspace& w = L->ws;
  const uint64_t P = static_cast<uint64_t>(n_tok) * k;
  // SwiGLU rows as f16 in the f32 activation buffer (half its bytes)
  if (!w.act_f32) TRY(dalloc(&w.act_f32, static_cast<size_t>(w.rows) * L->fp));
  w.pair_dtype = MXMOE_F32;
  if (L->profiling) CUDA_TRY(cudaEventRecord(L->ev[3], st));
  DqParams a{};
  a.d = static_cast<int>(L->d);
  a.fp = static_cast<int>(L->fp);
  a.kp1 = static_cast<int>(L->kp1);
  a.kp2 = static_cast<int>(L->kp2);
  a.w1q = L->w1q;
  a.w1sr = L->w1sr;
  a.sr1 = dq_scale_row_bytes(L->kp1);
  a.b1 = L->b1;
  a.w2q = L->w2q;
  a.w2sr = L->w2sr;
  a.sr2 = dq_scale_row_bytes(L->kp2);
  a.b2 = L->b2;
  a.bias_mult = (L->cfg.flags & MXMOE_FLAG_BIAS_PER_FTILE) ? static_cast<float>((L->f + 255) / 256) : 1.0f;
  a.E = static_cast<int>(L->e_count);
  a.topk_idx = pair_expert;
  a.P = static_cast<int>(P);
  a.pair_k = static_cast<int>(k);
  a.xh = xh;
  a.x = x;
  a.x_dtype = x_dtype == MXMOE_F32 ? kDqSrcF32 : kDqSrcBf16;
  a.gamma = L->gamma;
  a.rscale = rscale;
  a.x_scale = L->dq_x_scale;
  a.inv_x_scale = 1.0f / L->dq_x_scale;
  a.alpha = L->cfg.swiglu_alpha;
  a.limit = L->cfg.swiglu_limit;
  a.act_scale = L->dq_act_scale;
  a.inv_act_scale = 1.0f / L->dq_act_scale;
  a.act = reinterpret_cast<__half*>(w.act_f32);
  a.y_pair = w.y_pair;
  a.inv = inv;
  a.topk_w = route_w;
  a.err = L->err;
  a.sync = L->err + kStatusSyncOffset;
  if (L->fault == MXMOE_FAULT_SKIP_SIGNAL) {
    a.skip_arrival = 1;
    a.wait_ns = kFaultWaitNs;
  }
  if (y) {
    a.fused = 1;
    a.n_tok = static_cast<int>(n_tok);
    a.residual = (L->cfg.flags & MXMOE_FLAG_NO_RESIDUAL) ? 0 : 1;
    a.y = y;
    a.y_dtype = y_dtype == MXMOE_F32 ? kDqSrcF32 : kDqSrcBf16;
    a.offsets = w.offsets;
    a.perm_c = w.perm_c;
    a.inv_c = w.inv_c;
  }
  CUDA_TRY(launch_dqgemv_ffn(a, L->num_sms, L->smem_limit, st));
  if (L->profiling) {
    CUDA_TRY(cudaEventRecord(L->ev[4], st));  // W1, W2 (and in fused mode the combine) are one launch
    CUDA_TRY(cudaEventRecord(L->ev[5], st));
  }
  return MXMOE_OK;
}

// Expert FFN over already-routed pairs: quantize -> W1 -> W2 (or the SIMT
// pair) -> y_pair.  Uses ws.poff / counts / ntile_prefix / perm_p / inv_p.
int run_experts(mxmoe_layer* L, const void* x, int x_dtype, uint32_t n_tok, uint32_t k, const float* rscale,
                const float* route_w, const TilePlan& tp, int x_terms, cudaStream_t st,
                void* const* ret_ptrs = nullptr, const uint32_t* ret_slot = nullptr, bool y_by_pair = false,
                bool input_quantized = false, const int32_t* perm = nullptr, const ReturnSplit* split = nullptr) {
  Workspace& w = L->ws;
  const uint64_t P = static_cast<uint64_t>(n_tok) * k;
  const int N = tp.pair_tile;
  const float bias_mult = (L->cfg.flags & MXMOE_FLAG_BIAS_PER_FTILE) ? static_cast<float>((L->f + 255) / 256) : 1.0f;
  if (L->cfg.flags & MXMOE_FLAG_SIMT) {
    if (!w.act_f32) TRY(dalloc(&w.act_f32, static_cast<size_t>(w.rows) * L->fp));
    w.pair_dtype = MXMOE_F32;
    if (L->profiling) CUDA_TRY(cudaEventRecord(L->ev[3], st));
    CUDA_TRY(launch_simt_w1(x, x_dtype, L->d, k, L->gamma, rscale, L->w1q, L->w1sf, L->b1, L->fp, L->kp1, L->e_count,
                            w.poff, w.counts, w.perm_p, L->cfg.swiglu_alpha, L->cfg.swiglu_limit, w.act_f32, st));
    if (L->profiling) CUDA_TRY(cudaEventRecord(L->ev[4], st));
    CUDA_TRY(launch_simt_w2(w.act_f32, L->fp, L->d, k, L->w2q, L->w2sf, L->b2, bias_mult, L->kp2, L->e_count, w.poff,
                            w.counts, w.perm_p, route_w, w.y_pair, st));
    if (L->profiling) CUDA_TRY(cudaEventRecord(L->ev[5], st));
    return MXMOE_OK;
  }
  // (the dequant-GEMV plan comes only from mxmoe_forward_local, whose pairs'
  // local experts are ws.local_idx)
  if (tp.gemv) return run_dqgemv(L, x, x_dtype, n_tok, k, rscale, route_w, w.local_idx, w.inv_p, st);
  const uint64_t kc1 = L->kp1 / kTileK, kc2 = L->kp2 / kTileK;
  if (tp.fp4)
    return run_experts_f4(L, x, x_dtype, n_tok, k, rscale, route_w, tp, st, ret_ptrs, ret_slot, y_by_pair, perm);
  if (!input_quantized)
    CUDA_TRY(launch_quantize_pairs(x, x_dtype, n_tok, L->d, k, L->gamma, L->gamma_is_one ? 1 : 0, w.inv_p, x_terms,
                                   w.xq, static_cast<uint64_t>(w.rows) * L->kp1, L->kp1, w.xsf,
                                   static_cast<uint64_t>(w.row_blocks) * kc1 * kSfAtomBytes, static_cast<int>(kc1),
                                   N, tp.stacked ? 1 : 0, st));
  if (L->profiling) CUDA_TRY(cudaEventRecord(L->ev[3], st));
  const uint64_t max_pair_tiles = (P + N - 1) / N + L->e_count;
  const bool tok = tp.tok;
  const int wrows = tok ? 256 : 128;  // weight rows per tile
  TcParams p{};
  p.N = tok ? 256 : N;
  p.sf_rows = N;
  p.stacked = tp.stacked ? 1 : 0;
  p.E = L->e_count;
  p.poff = w.poff;
  p.counts = w.counts;
  p.ntile_prefix = w.ntile_prefix;
  p.alpha = L->cfg.swiglu_alpha;
  p.limit = L->cfg.swiglu_limit;
  p.rscale = rscale;
  p.perm = perm ? perm : w.perm_p;
  p.k = static_cast<int>(k);
  p.topk_w = route_w;
  p.err = L->err;
  if (L->fault == MXMOE_FAULT_SKIP_SIGNAL) {
    p.skip_stage = 1;
    p.wait_ns = kFaultWaitNs;
  }
  p.d = L->d;
  p.units = static_cast<int>(L->fp);
  // W1 + SwiGLU: weights W1, activations x terms; writes act terms.
  p.mode = 1;
  p.b_terms = x_terms;
  p.stages = tc_gemm_max_stages(tok, p.N, x_terms, L->smem_limit, N, tp.stacked);
  p.m_tiles = static_cast<int>((2 * L->fp + wrows - 1) / wrows);
  p.w_row_pairs = static_cast<int>(w_sf_row_pairs(2 * L->fp));
  p.k_tiles = static_cast<int>(kc1);
  p.a_sf = L->w1sf;
  p.b_sf = w.xsf;
  p.b_sf_term_stride = static_cast<uint64_t>(w.row_blocks) * kc1 * kSfAtomBytes;
  p.bias = L->b1;
  p.bias_stride = static_cast<int>(2 * L->fp);
  p.rows_valid = static_cast<int>(2 * L->fp);
  p.bias_mult = 1.0f;
  p.act_codes = w.aq;
  p.act_term_stride = static_cast<uint64_t>(w.rows) * L->kp2;
  p.act_kp = static_cast<int>(L->kp2);
  p.act_sf = w.asf;
  p.act_sf_term_stride = static_cast<uint64_t>(w.row_blocks) * kc2 * kSfAtomBytes;
  p.act_kchunks = static_cast<int>(kc2);
  int grid = static_cast<int>(std::min<uint64_t>(L->num_sms, p.m_tiles * max_pair_tiles));
  CUDA_TRY(tc_gemm_launch(tok, L->tmap_w1[tok ? 1 : 0], tp.stacked ? w.tmap_x_stk[tp.tw] : w.tmap_x[tp.tw], p, grid, st));
  if (L->profiling) CUDA_TRY(cudaEventRecord(L->ev[4], st));
  // W2 + bias + route weight: weights W2, activations act terms; writes y_pair.
  p.mode = 2;
  p.b_terms = 2;
  p.stages = tc_gemm_max_stages(tok, p.N, 2, L->smem_limit, N, tp.stacked);
  p.m_tiles = static_cast<int>((L->d + wrows - 1) / wrows);
  p.w_row_pairs = static_cast<int>(w_sf_row_pairs(L->d));
  p.k_tiles = static_cast<int>(kc2);
  p.a_sf = L->w2sf;
  p.b_sf = w.asf;
  p.b_sf_term_stride = static_cast<uint64_t>(w.row_blocks) * kc2 * kSfAtomBytes;
  p.bias = L->b2;
  p.bias_stride = static_cast<int>(L->d);
  p.rows_valid = static_cast<int>(L->d);
  p.bias_mult = bias_mult;
  p.y_pair = w.y_pair;
  p.y_pair_bf16 = reinterpret_cast<__nv_bfloat16*>(w.y_pair);
  p.ret_ptrs = ret_ptrs;
  p.ret_slot = ret_slot;
  p.y_by_pair = y_by_pair ? 1 : 0;
  w.pair_dtype = MXMOE_BF16;
  grid = static_cast<int>(std::min<uint64_t>(L->num_sms, p.m_tiles * max_pair_tiles));
  const CUtensorMap& tm_act = tp.stacked ? w.tmap_act_stk[tp.tw] : w.tmap_act[tp.tw];
  if (split == nullptr || L->e_count < 2) {
    CUDA_TRY(tc_gemm_launch(tok, L->tmap_w2[tok ? 1 : 0], tm_act, p, grid, st));
    if (split != nullptr)
      CUDA_TRY(launch_ep_return(w.y_pair, static_cast<int>(L->d), static_cast<int>(w.rows), w.poff, w.counts,
                                static_cast<int>(L->e_count), w.pos_slot, static_cast<int>(L->ep_world),
                                split->peer_ret, split->ret_rows, L->err, st));
  } else {
    if (!L->ret_stream) {
      CUDA_TRY(cudaStreamCreateWithFlags(&L->ret_stream, cudaStreamNonBlocking));
      for (cudaEvent_t& e : L->ret_ev) CUDA_TRY(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    }
    // up to kReturnParts expert ranges; each range's rows go back on the side
    // stream while the next range's W2 runs, only the last range's push is exposed
    const int E = static_cast<int>(L->e_count), parts = std::min(kReturnParts, E);
    for (int i = 0; i < parts; ++i) {
      const int e0 = E * i / parts, e1 = E * (i + 1) / parts;
      p.e_lo = e0;
      p.e_hi = e1;
      CUDA_TRY(tc_gemm_launch(tok, L->tmap_w2[tok ? 1 : 0], tm_act, p, grid, st));
      const bool last = i == parts - 1;
      if (!last) {
        CUDA_TRY(cudaEventRecord(L->ret_ev[i], st));
        CUDA_TRY(cudaStreamWaitEvent(L->ret_stream, L->ret_ev[i], 0));
      }
      CUDA_TRY(launch_ep_return(w.y_pair, static_cast<int>(L->d), static_cast<int>(w.rows), w.poff + e0,
                                w.counts + e0, e1 - e0, w.pos_slot, static_cast<int>(L->ep_world), split->peer_ret,
                                split->ret_rows, L->err, last ? st : L->ret_stream, last ? 256 : 64));
    }
    CUDA_TRY(cudaEventRecord(L->ret_ev[kReturnParts], L->ret_stream));
    CUDA_TRY(cudaStreamWaitEvent(st, L->ret_ev[kReturnParts], 0));
  }
  if (L->profiling) CUDA_TRY(cudaEventRecord(L->ev[5], st));
  return MXMOE_OK;
}

int check_layer(const mxmoe_layer* L) {
  if (!L) return fail(MXMOE_ERR_INVALID_ARG, "null layer");
  return MXMOE_OK;
}

// Device status word -> ABI status.
int device_status(int code) {
  if (code == 0) return MXMOE_OK;
  if (code == 7) return fail(MXMOE_ERR_INVALID_ARG, "a dispatched pair names an expert outside this layer's shard");
  return fail(MXMOE_ERR_TIMEOUT, "a bounded device-side wait gave up (code %d)", code);
}

}  // namespace

// The vectorized token-row kernels (activation quantization, gather,
// combine) move 16 bytes per access; the router takes any alignment.
static bool aligned16(const void* p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; }

extern "C" {

int mxmoe_abi_version(void) { return MXMOE_ABI_VERSION; }

const char* mxmoe_build_info(void) {
  return "mxmoe sm_100a: tcgen05 kind::mxf8f6f4.block_scale grouped GEMM (E2M1 weights x E4M3 hi/lo activations), "
         "CUDA-core router/permute/combine";
}

int mxmoe_last_error(char* buf, size_t cap) {
  if (!buf || cap == 0) return MXMOE_ERR_INVALID_ARG;
  std::snprintf(buf, cap, "%s", g_last_error.c_str());
  return MXMOE_OK;
}

int mxmoe_create(const mxmoe_config* cfg, mxmoe_layer** out) {
  if (!cfg || !out) return fail(MXMOE_ERR_INVALID_ARG, "null argument");
  *out = nullptr;
  if (cfg->d_model == 0 || cfg->ffn_hidden == 0 || cfg->num_experts == 0 || cfg->experts_per_token == 0)
    return fail(MXMOE_ERR_INVALID_ARG, "zero dimension in config");
  if (cfg->d_model % 32 != 0 || cfg->ffn_hidden % 32 != 0)
    return fail(MXMOE_ERR_UNSUPPORTED, "d_model (%u) and ffn_hidden (%u) must be multiples of 32", cfg->d_model,
                cfg->ffn_hidden);
  if (cfg->experts_per_token > static_cast<uint32_t>(kMaxTopK) || cfg->experts_per_token > cfg->num_experts)
    return fail(MXMOE_ERR_UNSUPPORTED, "experts_per_token %u unsupported (max %d, <= num_experts)",
                cfg->experts_per_token, kMaxTopK);
  if (cfg->num_experts > 1024) return fail(MXMOE_ERR_UNSUPPORTED, "num_experts %u > 1024", cfg->num_experts);
  int ndev = 0;
  CUDA_TRY(cudaGetDeviceCount(&ndev));
  if (cfg->device < 0 || cfg->device >= ndev) return fail(MXMOE_ERR_INVALID_ARG, "bad device %d", cfg->device);
  DeviceGuard g(cfg->device);
  mxmoe_layer* L = new (std::nothrow) mxmoe_layer();
  if (!L) return fail(MXMOE_ERR_OOM, "host allocation failed");
  L->cfg = *cfg;
  L->d = cfg->d_model;
  L->f = cfg->ffn_hidden;
  L->fp = round_up(L->f, kGluBlock);
  L->E_total = cfg->num_experts;
  L->k = cfg->experts_per_token;
  L->e_begin = 0;
  L->e_count = cfg->num_experts;
  L->kp1 = round_up(L->d, kTileK);
  L->kp2 = round_up(L->fp, kTileK);
  L->m_tiles1 = 2 * L->fp / 128;
  L->m_tiles2 = (L->d + 127) / 128;
  if (gemv_ok(L))
    L->dq_act_scale = f16_range_scale(std::max(cfg->swiglu_limit, 0.28f / cfg->swiglu_alpha) *
                                      (cfg->swiglu_limit + 1.0f));
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, cfg->device) == cudaSuccess) {
    L->num_sms = prop.multiProcessorCount;
    L->smem_limit = prop.sharedMemPerBlockOptin;
  }
  const size_t status_words = kStatusSyncOffset + static_cast<size_t>(L->E_total);
  int rc = dalloc(&L->err, status_words);
  if (rc == MXMOE_OK && cudaMemset(L->err, 0, status_words * sizeof(int)) != cudaSuccess) rc = MXMOE_ERR_CUDA;
  if (rc != MXMOE_OK) {
    delete L;
    return rc;
  }
  *out = L;
  return MXMOE_OK;
}

int mxmoe_fp4_operands(mxmoe_layer* L, void** ptrs, uint32_t* rows4) {
  if (!L || !ptrs || !rows4) return fail(MXMOE_ERR_INVALID_ARG, "mxmoe_fp4_operands: null argument");
  const Workspace& w = L->ws;
  ptrs[0] = w.xq4;
  ptrs[1] = w.xsf4;
  ptrs[2] = w.aq4;
  ptrs[3] = w.asf4;
  *rows4 = w.rows4;
  return MXMOE_OK;
}

int mxmoe_get_config(const mxmoe_layer* L, mxmoe_config* out) {
  if (!L || !out) return fail(MXMOE_ERR_INVALID_ARG, "mxmoe_get_config: null argument");
  *out = L->cfg;
  return MXMOE_OK;
}

int mxmoe_destroy(mxmoe_layer* L) {
  if (!L) return MXMOE_OK;
  DeviceGuard g(L->cfg.device);
  cudaDeviceSynchronize();
  free_workspace(L->ws);
  dfree(L->gamma); dfree(L->gate_w); dfree(L->gate_b);
  dfree(L->w1q); dfree(L->w1sf); dfree(L->b1); dfree(L->w2q); dfree(L->w2sf); dfree(L->b2);
  dfree(L->w1sr); dfree(L->w2sr);
  dfree(L->err);
  if (L->epa.bufs) cudaFree(L->epa.bufs);
  if (L->epa.ret) cudaFree(L->epa.ret);
  if (L->epa.counts) cudaFree(L->epa.counts);
  for (auto& e : L->ev)
    if (e) cudaEventDestroy(e);
  if (L->graph.exec) cudaGraphExecDestroy(L->graph.exec);
  if (L->cap_stream) cudaStreamDestroy(L->cap_stream);
  if (L->ret_stream) cudaStreamDestroy(L->ret_stream);
  for (cudaEvent_t e : L->ret_ev)
    if (e) cudaEventDestroy(e);
  {
    auto& h = L->hs;
    if (h.dx) cudaFree(h.dx);
    if (h.dy) cudaFree(h.dy);
    if (h.s_in) cudaStreamDestroy(h.s_in);
    if (h.s_out) cudaStreamDestroy(h.s_out);
    for (int i = 0; i < kHostChunksMax; ++i) {
      if (h.ev_in[i]) cudaEventDestroy(h.ev_in[i]);
      if (h.ev_done[i]) cudaEventDestroy(h.ev_done[i]);
    }
    if (h.status) cudaFreeHost(h.status);
  }
  delete L;
  return MXMOE_OK;
}

int mxmoe_set_router(mxmoe_layer* L, const void* norm_gamma, const void* gate_w, const void* gate_b,
                     mxmoe_dtype dtype, void* stream) {
  TRY(check_layer(L));
  if (!norm_gamma || !gate_w || !gate_b) return fail(MXMOE_ERR_INVALID_ARG, "null router parameter");
  if (dtype != MXMOE_F32 && dtype != MXMOE_BF16) return fail(MXMOE_ERR_INVALID_ARG, "bad dtype");
  DeviceGuard g(L->cfg.device);
  const size_t d = L->d, E = L->E_total;
  std::vector<float> gm(d), w(E * d), b(E);
  to_f32(norm_gamma, dtype, d, gm.data());
  to_f32(gate_w, dtype, E * d, w.data());
  to_f32(gate_b, dtype, E, b.data());
  L->gamma_is_one = std::all_of(gm.begin(), gm.end(), [](float v) { return v == 1.0f; });
  float gmax = 0.0f;
  for (float v : gm) gmax = std::max(gmax, std::fabs(v));
  L->dq_x_scale = f16_range_scale(std::sqrt(static_cast<float>(d)) * gmax);
  ++L->generation;
  if (!L->gamma) TRY(dalloc(&L->gamma, d));
  std::vector<float> wp(router_gate_packed_floats(static_cast<int>(E), static_cast<int>(d)));
  pack_router_gate(w.data(), static_cast<int>(E), static_cast<int>(d), wp.data());
  if (!L->gate_w) TRY(dalloc(&L->gate_w, wp.size()));
  if (!L->gate_b) TRY(dalloc(&L->gate_b, E));
  cudaStream_t st = as_stream(stream);
  CUDA_TRY(cudaMemcpyAsync(L->gamma, gm.data(), d * 4, cudaMemcpyHostToDevice, st));
  CUDA_TRY(cudaMemcpyAsync(L->gate_w, wp.data(), wp.size() * 4, cudaMemcpyHostToDevice, st));
  CUDA_TRY(cudaMemcpyAsync(L->gate_b, b.data(), E * 4, cudaMemcpyHostToDevice, st));
  CUDA_TRY(cudaStreamSynchronize(st));
  L->router_ready = true;
  return MXMOE_OK;
}

int mxmoe_set_expert_shard(mxmoe_layer* L, uint32_t expert_begin, uint32_t expert_count) {
  TRY(check_layer(L));
  if (expert_count == 0 || expert_begin + expert_count > L->E_total)
    return fail(MXMOE_ERR_INVALID_ARG, "bad shard [%u, %u) of %u experts", expert_begin, expert_begin + expert_count,
                L->E_total);
  if (L->experts_ready) return fail(MXMOE_ERR_INVALID_ARG, "shard must be set before uploading experts");
  DeviceGuard g(L->cfg.device);
  free_workspace(L->ws);
  L->e_begin = expert_begin;
  L->e_count = expert_count;
  ++L->generation;
  return MXMOE_OK;
}

int mxmoe_upload_experts(mxmoe_layer* L, const mxmoe_quant_desc* w1d, const uint8_t* w1_blocks,
                         const uint8_t* w1_scales, const mxmoe_quant_desc* w2d, const uint8_t* w2_blocks,
                         const uint8_t* w2_scales, const void* b1, const void* b2, mxmoe_dtype bias_dtype,
                         void* stream) {
  TRY(check_layer(L));
  if (!w1d || !w2d || !w1_blocks || !w1_scales || !w2_blocks || !w2_scales || !b1 || !b2)
    return fail(MXMOE_ERR_INVALID_ARG, "null expert parameter");
  const uint64_t E = L->e_count, d = L->d, f = L->f, fp = L->fp;
  if (w1d->experts != E || w1d->rows != 2 * f || w1d->cols != d || w1d->bpr != (d + 1) / 2 ||
      w1d->gpr != (d + 31) / 32)
    return fail(MXMOE_ERR_INVALID_ARG,
                "W1 desc mismatch: got experts=%llu rows=%llu cols=%llu bpr=%llu gpr=%llu, want %llu/%llu/%llu/%llu/%llu",
                (unsigned long long)w1d->experts, (unsigned long long)w1d->rows, (unsigned long long)w1d->cols,
                (unsigned long long)w1d->bpr, (unsigned long long)w1d->gpr, (unsigned long long)E,
                (unsigned long long)(2 * f), (unsigned long long)d, (unsigned long long)((d + 1) / 2),
                (unsigned long long)((d + 31) / 32));
  if (w2d->experts != E || w2d->rows != d || w2d->cols != f || w2d->bpr != (f + 1) / 2 || w2d->gpr != (f + 31) / 32)
    return fail(MXMOE_ERR_INVALID_ARG, "W2 desc mismatch");
  DeviceGuard g(L->cfg.device);
  const bool inter = (L->cfg.flags & MXMOE_FLAG_INTERLEAVED_GLU) != 0;
  const uint64_t kp1 = L->kp1, kp2 = L->kp2, kc1 = kp1 / kTileK, kc2 = kp2 / kTileK;
  const uint64_t rows1 = 2 * fp;
  const uint64_t bpr1 = w1d->bpr, gpr1 = w1d->gpr, bpr2 = w2d->bpr, gpr2 = w2d->gpr;

  auto sf_byte = [](uint8_t s, int ue8) -> uint8_t {
    const int v = static_cast<int>(s) - ue8;
    return static_cast<uint8_t>(v < 0 ? 0 : (v > 255 ? 255 : v));
  };

  const uint64_t rp1 = w_sf_row_pairs(static_cast<uint32_t>(rows1)), rp2 = w_sf_row_pairs(static_cast<uint32_t>(d));
  std::vector<uint8_t> q1(E * rows1 * (kp1 / 2), 0), s1(E * rp1 * kc1 * kWSfPairBytes, 0);
  const uint64_t sr1 = dq_scale_row_bytes(static_cast<uint32_t>(kp1)), sr2 = dq_scale_row_bytes(static_cast<uint32_t>(kp2));
  std::vector<uint8_t> r1(E * rows1 * sr1, 0), r2(E * d * sr2, 0);  // row-major scales (dequant-GEMV)
  std::vector<float> bb1(E * rows1, 0.0f), src_b1(E * 2 * f);
  to_f32(b1, bias_dtype, E * 2 * f, src_b1.data());
  for (uint64_t e = 0; e < E; ++e)
    for (uint64_t j = 0; j < f; ++j)
      for (uint32_t half = 0; half < 2; ++half) {
        const uint64_t src = inter ? 2 * j + half : half * f + j;
        const uint64_t dst = w1_packed_row(static_cast<uint32_t>(j), half);
        std::memcpy(&q1[(e * rows1 + dst) * (kp1 / 2)], &w1_blocks[(e * 2 * f + src) * bpr1], bpr1);
        uint8_t* atoms = &s1[e * rp1 * kc1 * kWSfPairBytes];
        for (uint64_t gi = 0; gi < gpr1; ++gi) {
          const uint8_t v = sf_byte(w1_scales[(e * 2 * f + src) * gpr1 + gi], w1d->ue8_offset);
          atoms[w_sf_offset(static_cast<uint32_t>(dst), static_cast<uint32_t>(gi), static_cast<uint32_t>(kc1))] = v;
          r1[(e * rows1 + dst) * sr1 + gi] = v;
        }
        bb1[e * rows1 + dst] = src_b1[e * 2 * f + src];
      }
  std::vector<uint8_t> q2(E * d * (kp2 / 2), 0), s2(E * rp2 * kc2 * kWSfPairBytes, 0);
  std::vector<float> bb2(E * d);
  to_f32(b2, bias_dtype, E * d, bb2.data());
  for (uint64_t e = 0; e < E; ++e)
    for (uint64_t c = 0; c < d; ++c) {
      std::memcpy(&q2[(e * d + c) * (kp2 / 2)], &w2_blocks[(e * d + c) * bpr2], bpr2);
      uint8_t* atoms = &s2[e * rp2 * kc2 * kWSfPairBytes];
      for (uint64_t gi = 0; gi < gpr2; ++gi) {
        const uint8_t v = sf_byte(w2_scales[(e * d + c) * gpr2 + gi], w2d->ue8_offset);
        atoms[w_sf_offset(static_cast<uint32_t>(c), static_cast<uint32_t>(gi), static_cast<uint32_t>(kc2))] = v;
        r2[(e * d + c) * sr2 + gi] = v;
      }
    }

  dfree(L->w1q); dfree(L->w1sf); dfree(L->b1); dfree(L->w2q); dfree(L->w2sf); dfree(L->b2);
  dfree(L->w1sr); dfree(L->w2sr);
  ++L->generation;
  TRY(dalloc(&L->w1sr, r1.size()));
  TRY(dalloc(&L->w2sr, r2.size()));
  TRY(dalloc(&L->w1q, q1.size()));
  TRY(dalloc(&L->w1sf, s1.size()));
  TRY(dalloc(&L->b1, bb1.size()));
  TRY(dalloc(&L->w2q, q2.size()));
  TRY(dalloc(&L->w2sf, s2.size()));
  TRY(dalloc(&L->b2, bb2.size()));
  cudaStream_t st = as_stream(stream);
  CUDA_TRY(cudaMemcpyAsync(L->w1q, q1.data(), q1.size(), cudaMemcpyHostToDevice, st));
  CUDA_TRY(cudaMemcpyAsync(L->w1sf, s1.data(), s1.size(), cudaMemcpyHostToDevice, st));
  CUDA_TRY(cudaMemcpyAsync(L->b1, bb1.data(), bb1.size() * 4, cudaMemcpyHostToDevice, st));
  CUDA_TRY(cudaMemcpyAsync(L->w2q, q2.data(), q2.size(), cudaMemcpyHostToDevice, st));
  CUDA_TRY(cudaMemcpyAsync(L->w2sf, s2.data(), s2.size(), cudaMemcpyHostToDevice, st));
  CUDA_TRY(cudaMemcpyAsync(L->b2, bb2.data(), bb2.size() * 4, cudaMemcpyHostToDevice, st));
  CUDA_TRY(cudaMemcpyAsync(L->w1sr, r1.data(), r1.size(), cudaMemcpyHostToDevice, st));
  CUDA_TRY(cudaMemcpyAsync(L->w2sr, r2.data(), r2.size(), cudaMemcpyHostToDevice, st));
  CUDA_TRY(cudaStreamSynchronize(st));
  for (int i = 0; i < 2; ++i) {
    const uint32_t box = i == 0 ? 128 : 256;
    TRY(make_tmap(&L->tmap_w1[i], CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, L->w1q, kp1, rows1, E, kp1 / 2,
                  rows1 * (kp1 / 2), box));
    TRY(make_tmap(&L->tmap_w2[i], CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, L->w2q, kp2, d, E, kp2 / 2, d * (kp2 / 2),
                  box));
  }
  // the same codes as packed bytes for the kind::mxf4 tiles (128-byte rows = K 256)
  TRY(make_tmap(&L->tmap_w1_f4, CU_TENSOR_MAP_DATA_TYPE_UINT8, L->w1q, kp1 / 2, rows1, E, kp1 / 2, rows1 * (kp1 / 2),
                256));
  TRY(make_tmap(&L->tmap_w2_f4, CU_TENSOR_MAP_DATA_TYPE_UINT8, L->w2q, kp2 / 2, d, E, kp2 / 2, d * (kp2 / 2), 256));
  L->experts_ready = true;
  return MXMOE_OK;
}

int mxmoe_reserve(mxmoe_layer* L, uint32_t max_tokens) {
  TRY(check_layer(L));
  DeviceGuard g(L->cfg.device);
  return ensure_workspace(L, max_tokens, L->k);
}

// Tile plan of mxmoe_forward for P routed pairs.
static TilePlan forward_plan(const mxmoe_layer* L, uint64_t P, int x_terms) {
  const bool simt = (L->cfg.flags & MXMOE_FLAG_SIMT) != 0;
  return pick_tiles(P, L->e_count, x_terms, gemv_ok(L),
                    !simt && !(L->cfg.flags & MXMOE_FLAG_NO_FP4));
}

// The kernel chain of mxmoe_forward (router, permutation, experts, combine)
// on stream st; everything that can allocate or resize ran before.
static int forward_chain(mxmoe_layer* L, const void* x, mxmoe_dtype x_dtype, void* y, mxmoe_dtype y_dtype,
                         uint32_t n_tokens, cudaStream_t st) {
  // kernels of the chain start while their predecessor finishes (the event
  // records of profiling mode break that overlap, so it stays off there)
  PdlScope pdl(!L->profiling);
  Workspace& w = L->ws;
  const uint32_t k = L->k, E = L->e_count;
  const uint64_t P = static_cast<uint64_t>(n_tokens) * k;
  const int xt = x_terms_for(L, x_dtype);
  const TilePlan tp = forward_plan(L, P, xt);
  const int status_words = static_cast<int>(kStatusSyncOffset + L->E_total);
  // the small-batch router zeroes the status words itself (one graph node less)
  if (!tp.gemv) CUDA_TRY(cudaMemsetAsync(L->err, 0, status_words * sizeof(int), st));
  if (L->profiling) CUDA_TRY(cudaEventRecord(L->ev[0], st));
  // the dequant-GEMV stages the router's normalized f16 token rows
  __half* xh = tp.gemv ? w.xh : nullptr;
  // small batches on tensor-core tiles: the router's last block also runs the
  // permutation (its ticket is a status word the memset above cleared)
  const int pad = tp.fp4 ? tp.pair_tile : kRowBlock;
  const bool fold = !tp.gemv && router_folds_permute(static_cast<int>(n_tokens), static_cast<int>(L->d),
                                                     static_cast<int>(L->E_total), static_cast<int>(k));
  const PermFold pf{L->err + kStatusSyncOffset, pad, tp.pair_tile, w.offsets, w.perm_c, w.inv_c, w.poff, w.counts,
                    w.ntile_prefix, w.perm_p, w.inv_p};
  CUDA_TRY(launch_router(x, x_dtype, n_tokens, L->d, L->E_total, k, L->gamma, L->gate_w, L->gate_b, L->cfg.rms_eps,
                         w.logits, w.topk_idx, w.topk_w, w.rscale, st, xh, L->dq_x_scale, w.tok_ctr,
                         tp.gemv ? L->err : nullptr, status_words, fold ? &pf : nullptr));
  if (L->profiling) CUDA_TRY(cudaEventRecord(L->ev[1], st));
  if (tp.gemv) {
    // router -> one fused kernel (expert FFN, combine, routing maps)
    if (L->profiling) CUDA_TRY(cudaEventRecord(L->ev[2], st));
    TRY(run_dqgemv(L, x, x_dtype, n_tokens, k, w.rscale, w.topk_w, w.topk_idx, nullptr, st, xh, y, y_dtype));
    return MXMOE_OK;
  }
  if (!fold)
    CUDA_TRY(launch_permute(w.topk_idx, static_cast<int>(P), E, pad, tp.pair_tile, w.offsets, w.perm_c, w.inv_c,
                            w.poff, w.counts, w.ntile_prefix, w.perm_p, w.inv_p, st, w.perm_scratch));
  if (L->profiling) CUDA_TRY(cudaEventRecord(L->ev[2], st));
  TRY(run_experts(L, x, x_dtype, n_tokens, k, w.rscale, w.topk_w, tp, xt, st));
  const int residual = (L->cfg.flags & MXMOE_FLAG_NO_RESIDUAL) ? 0 : 1;
  CUDA_TRY(launch_combine(x, x_dtype, w.y_pair, w.pair_dtype, w.topk_idx, w.inv_p, n_tokens, L->d, k, residual, y,
                          y_dtype, st));
  return MXMOE_OK;
}

// Capture the chain for this key into L->graph (on the layer's capture stream).
static int capture_forward(mxmoe_layer* L, const void* x, mxmoe_dtype x_dtype, void* y, mxmoe_dtype y_dtype,
                           uint32_t n_tokens) {
  if (!L->cap_stream) CUDA_TRY(cudaStreamCreateWithFlags(&L->cap_stream, cudaStreamNonBlocking));
  CUDA_TRY(cudaStreamBeginCapture(L->cap_stream, cudaStreamCaptureModeThreadLocal));
  const int rc = forward_chain(L, x, x_dtype, y, y_dtype, n_tokens, L->cap_stream);
  cudaGraph_t graph = nullptr;
  const cudaError_t ce = cudaStreamEndCapture(L->cap_stream, &graph);
  if (rc != MXMOE_OK || ce != cudaSuccess || !graph) {
    if (graph) cudaGraphDestroy(graph);
    cudaGetLastError();
    return rc != MXMOE_OK ? rc : fail(MXMOE_ERR_CUDA, "forward capture failed: %s", cudaGetErrorString(ce));
  }
  cudaGraphExec_t exec = nullptr;
  const cudaError_t ie = cudaGraphInstantiate(&exec, graph, 0);
  cudaGraphDestroy(graph);
  if (ie != cudaSuccess) return fail(MXMOE_ERR_CUDA, "graph instantiate failed: %s", cudaGetErrorString(ie));
  L->graph.exec = exec;
  return MXMOE_OK;
}

int mxmoe_forward(mxmoe_layer* L, const void* x, mxmoe_dtype x_dtype, void* y, mxmoe_dtype y_dtype,
                  uint32_t n_tokens, void* stream) {
  TRY(check_layer(L));
  if ((!x || !y) && n_tokens > 0) return fail(MXMOE_ERR_INVALID_ARG, "null x or y");
  if (!aligned16(x) || !aligned16(y)) return fail(MXMOE_ERR_INVALID_ARG, "x and y must be 16-byte aligned");
  if ((x_dtype != MXMOE_F32 && x_dtype != MXMOE_BF16) || (y_dtype != MXMOE_F32 && y_dtype != MXMOE_BF16))
    return fail(MXMOE_ERR_INVALID_ARG, "bad dtype");
  DeviceGuard g(L->cfg.device);
  cudaStream_t st = as_stream(stream);
  L->last_n = n_tokens;
  if (n_tokens == 0) return MXMOE_OK;
  const size_t xbytes = static_cast<size_t>(n_tokens) * L->d * (x_dtype == MXMOE_F32 ? 4 : 2);
  if (L->cfg.flags & MXMOE_FLAG_DISABLED) {
    // MoeConfig.disabled (src/moe/mod.rs:106-108): y = x.
    if (x_dtype == y_dtype) {
      CUDA_TRY(cudaMemcpyAsync(y, x, xbytes, cudaMemcpyDeviceToDevice, st));
    } else {
      CUDA_TRY(launch_combine(x, x_dtype, nullptr, 0, nullptr, nullptr, n_tokens, L->d, 0, 1, y, y_dtype, st));
    }
    return MXMOE_OK;
  }
  if (!L->router_ready || !L->experts_ready) return fail(MXMOE_ERR_NOT_READY, "router or experts not uploaded");
  if (L->e_count != L->E_total)
    return fail(MXMOE_ERR_INVALID_ARG, "layer holds an expert shard; use the expert-parallel entry points");
  TRY(ensure_workspace(L, n_tokens, L->k));
  if (forward_plan(L, static_cast<uint64_t>(n_tokens) * L->k, x_terms_for(L, x_dtype)).fp4) TRY(ensure_f4(L));
  L->profile_valid = false;
  if (L->fault) {
    // a fault-injected forward runs once, directly, and is not cached as a graph
    const int rc = forward_chain(L, x, x_dtype, y, y_dtype, n_tokens, st);
    L->fault = 0;
    return rc;
  }
  if (!L->profiling && !(L->cfg.flags & MXMOE_FLAG_NO_GRAPHS)) {
    auto& gr = L->graph;
    const bool same = gr.x == x && gr.y == y && gr.n == n_tokens && gr.xd == x_dtype && gr.yd == y_dtype &&
                      gr.gen == L->generation;
    if (same && !gr.exec && !gr.failed)  // second call with this key: capture
      gr.failed = capture_forward(L, x, x_dtype, y, y_dtype, n_tokens) != MXMOE_OK;
    if (same && gr.exec) {
      CUDA_TRY(cudaGraphLaunch(gr.exec, st));
      return MXMOE_OK;
    }
    if (!same) {  // a new key: run directly and remember it
      if (gr.exec) cudaGraphExecDestroy(gr.exec);
      gr = mxmoe_layer::FwdGraph{};
      gr.x = x;
      gr.y = y;
      gr.n = n_tokens;
      gr.xd = x_dtype;
      gr.yd = y_dtype;
      gr.gen = L->generation;
    }
  }
  TRY(forward_chain(L, x, x_dtype, y, y_dtype, n_tokens, st));
  if (L->profiling) {
    CUDA_TRY(cudaEventRecord(L->ev[6], st));
    L->profile_valid = true;
  }
  return MXMOE_OK;
}

int mxmoe_forward_host(mxmoe_layer* L, const void* x_host, mxmoe_dtype x_dtype, void* y_host, mxmoe_dtype y_dtype,
                       uint32_t n_tokens, void* stream) {
  TRY(check_layer(L));
  if (n_tokens == 0) return MXMOE_OK;
  if (!x_host || !y_host) return fail(MXMOE_ERR_INVALID_ARG, "null host buffer");
  if ((x_dtype != MXMOE_F32 && x_dtype != MXMOE_BF16) || (y_dtype != MXMOE_F32 && y_dtype != MXMOE_BF16))
    return fail(MXMOE_ERR_INVALID_ARG, "bad dtype");
  DeviceGuard g(L->cfg.device);
  cudaStream_t st = as_stream(stream);
  const size_t xrow = static_cast<size_t>(L->d) * (x_dtype == MXMOE_F32 ? 4 : 2);
  const size_t yrow = static_cast<size_t>(L->d) * (y_dtype == MXMOE_F32 ? 4 : 2);
  const size_t xb = n_tokens * xrow, yb = n_tokens * yrow;
  TRY(ensure_workspace(L, n_tokens, L->k));
  auto& h = L->hs;
  if (!h.s_in) {
    CUDA_TRY(cudaStreamCreateWithFlags(&h.s_in, cudaStreamNonBlocking));
    CUDA_TRY(cudaStreamCreateWithFlags(&h.s_out, cudaStreamNonBlocking));
    for (int i = 0; i < kHostChunksMax; ++i) {
      CUDA_TRY(cudaEventCreateWithFlags(&h.ev_in[i], cudaEventDisableTiming));
      CUDA_TRY(cudaEventCreateWithFlags(&h.ev_done[i], cudaEventDisableTiming));
    }
    CUDA_TRY(cudaMallocHost(&h.status, kHostChunksMax * sizeof(int)));
  }
  if (h.cx < xb) {
    if (h.dx) cudaFree(h.dx);
    h.dx = nullptr;
    h.cx = 0;
    CUDA_TRY(cudaMalloc(&h.dx, xb));
    h.cx = xb;
  }
  if (h.cy < yb) {
    if (h.dy) cudaFree(h.dy);
    h.dy = nullptr;
    h.cy = 0;
    CUDA_TRY(cudaMalloc(&h.dy, yb));
    h.cy = yb;
  }
  // Chunks of whole 128-token blocks: chunk i's host->device copy runs on
  // s_in, its forward on the caller's stream, its device->host copy on s_out,
  // so the copies of neighbouring chunks overlap each forward.  The first
  // and last chunks are small, since nothing overlaps the first copy in or
  // the last copy out; the middle two carry the rest.  Each chunk streams
  // every expert's weights once more, so more, smaller chunks lose.
  uint32_t bounds[kHostChunksMax + 1] = {0};
  uint32_t chunks = 1;
  bounds[1] = n_tokens;
  if (n_tokens >= 4 * kHostChunkMinTokens) {
    // first chunk 3/32 of the batch (nothing overlaps its copy in), last 1/8
    // (nothing overlaps its copy out); measured at 8192 tokens 2.37 ms
    // against 2.46 for 1/8 + 3/8 + 3/8 + 1/8 and 3.27 unchunked
    const uint32_t first = round_up(n_tokens * 3 / 32, 128), last = round_up(n_tokens / 8, 128);
    const uint32_t mid = round_up((n_tokens - first - last) / 2, 128);
    chunks = 4;
    bounds[1] = first;
    bounds[2] = first + mid;
    bounds[3] = n_tokens - last;
    bounds[4] = n_tokens;
  } else if (n_tokens >= 2 * kHostChunkMinTokens) {
    chunks = 2;
    bounds[1] = round_up(n_tokens / 2, 128);
    bounds[2] = n_tokens;
  }
  for (uint32_t i = 0; i < chunks; ++i) h.status[i] = 0;
  uint32_t used = 0;
  for (uint32_t i = 0; i < chunks && bounds[i] < bounds[i + 1]; ++i, ++used) {
    const uint32_t t0 = bounds[i], nt = bounds[i + 1] - bounds[i];
    char* dxi = static_cast<char*>(h.dx) + t0 * xrow;
    char* dyi = static_cast<char*>(h.dy) + t0 * yrow;
    CUDA_TRY(cudaMemcpyAsync(dxi, static_cast<const char*>(x_host) + t0 * xrow, nt * xrow, cudaMemcpyHostToDevice,
                             h.s_in));
    CUDA_TRY(cudaEventRecord(h.ev_in[i], h.s_in));
    CUDA_TRY(cudaStreamWaitEvent(st, h.ev_in[i], 0));
    TRY(mxmoe_forward(L, dxi, x_dtype, dyi, y_dtype, nt, st));
    // each forward resets the status word: keep this chunk's
    CUDA_TRY(cudaMemcpyAsync(&h.status[i], L->err, sizeof(int), cudaMemcpyDeviceToHost, st));
    CUDA_TRY(cudaEventRecord(h.ev_done[i], st));
    CUDA_TRY(cudaStreamWaitEvent(h.s_out, h.ev_done[i], 0));
    CUDA_TRY(cudaMemcpyAsync(static_cast<char*>(y_host) + t0 * yrow, dyi, nt * yrow, cudaMemcpyDeviceToHost, h.s_out));
  }
  CUDA_TRY(cudaStreamSynchronize(h.s_out));
  CUDA_TRY(cudaStreamSynchronize(st));
  for (uint32_t i = 0; i < used; ++i)
    if (h.status[i] != 0) return device_status(h.status[i]);
  return MXMOE_OK;
}

int mxmoe_sync_status(mxmoe_layer* L, void* stream) {
  TRY(check_layer(L));
  DeviceGuard g(L->cfg.device);
  CUDA_TRY(cudaStreamSynchronize(as_stream(stream)));
  CUDA_TRY(cudaGetLastError());
  int herr[5] = {0, 0, 0, 0, 0};
  CUDA_TRY(cudaMemcpy(herr, L->err, sizeof(herr), cudaMemcpyDeviceToHost));
  if (herr[0] == 8)
    return fail(MXMOE_ERR_TIMEOUT, "dequant-GEMV W1->W2 grid wait gave up: saw %d of %d block arrivals", herr[3],
                herr[4]);
  return device_status(herr[0]);
}

int mxmoe_routing_results(mxmoe_layer* L, const int32_t** topk_idx, const float** topk_w, const int32_t** offsets,
                          const int32_t** perm, const int32_t** inv, const float** logits) {
  TRY(check_layer(L));
  if (!L->ws.cap_tokens) return fail(MXMOE_ERR_NOT_READY, "no forward has run");
  if (topk_idx) *topk_idx = L->ws.topk_idx;
  if (topk_w) *topk_w = L->ws.topk_w;
  if (offsets) *offsets = L->ws.offsets;
  if (perm) *perm = L->ws.perm_c;
  if (inv) *inv = L->ws.inv_c;
  if (logits) *logits = L->ws.logits;
  return MXMOE_OK;
}

int mxmoe_dequant_mxfp4_bytes(const uint8_t* blocks, uint64_t rows_total, uint64_t b, const uint8_t* scales,
                              float* out, void* stream) {
  if (rows_total * b > 0 && (!blocks || !scales || !out)) return fail(MXMOE_ERR_INVALID_ARG, "null pointer");
  CUDA_TRY(launch_dequant_bytes(blocks, rows_total, b, scales, out, as_stream(stream)));
  return MXMOE_OK;
}

int mxmoe_dequant_rows(const mxmoe_quant_desc* desc, const uint8_t* blocks, const uint8_t* scales, float* out,
                       void* stream) {
  if (!desc) return fail(MXMOE_ERR_INVALID_ARG, "null desc");
  const uint64_t rows = desc->experts * desc->rows;
  if (rows * desc->cols > 0 && (!blocks || !scales || !out)) return fail(MXMOE_ERR_INVALID_ARG, "null pointer");
  if (desc->bpr < (desc->cols + 1) / 2 || desc->gpr < (desc->cols + 31) / 32)
    return fail(MXMOE_ERR_INVALID_ARG, "bpr/gpr too small for cols");
  CUDA_TRY(launch_dequant_rows(blocks, scales, rows, desc->cols, desc->bpr, desc->gpr, desc->ue8_offset, out,
                               as_stream(stream)));
  return MXMOE_OK;
}

int mxmoe_topk_softmax(const float* logits, uint32_t n_tokens, uint32_t num_experts, uint32_t k, int32_t* topk_idx,
                       float* topk_w, void* stream) {
  if (k == 0 || k > static_cast<uint32_t>(kMaxTopK) || k > num_experts)
    return fail(MXMOE_ERR_UNSUPPORTED, "k=%u unsupported", k);
  if (n_tokens > 0 && (!logits || !topk_idx || !topk_w)) return fail(MXMOE_ERR_INVALID_ARG, "null pointer");
  CUDA_TRY(launch_topk_softmax(logits, n_tokens, num_experts, k, topk_idx, topk_w, as_stream(stream)));
  return MXMOE_OK;
}

int mxmoe_permute(const int32_t* topk_idx, uint32_t n_tokens, uint32_t k, uint32_t num_experts, int32_t* offsets,
                  int32_t* perm, int32_t* inv, void* stream) {
  if (num_experts == 0 || num_experts > 1024) return fail(MXMOE_ERR_UNSUPPORTED, "num_experts %u", num_experts);
  const uint64_t P = static_cast<uint64_t>(n_tokens) * k;
  if (P > static_cast<uint64_t>(INT32_MAX)) return fail(MXMOE_ERR_TOO_LARGE, "n_tokens * k = %llu pairs", (unsigned long long)P);
  if (!offsets || (P > 0 && (!topk_idx || !perm || !inv))) return fail(MXMOE_ERR_INVALID_ARG, "null pointer");
  // pad = 1 makes the padded maps equal to the canonical ones; the scratch
  // outputs (poff, counts) are written to the tail of `offsets`' companion
  // buffers allocated here.
  int32_t* tmp = nullptr;
  TRY(dalloc(&tmp, 2 * (num_experts + 1)));
  cudaStream_t st = as_stream(stream);
  const cudaError_t le = launch_permute(topk_idx, static_cast<int>(P), num_experts, 1, 1, offsets, nullptr, nullptr,
                                        tmp, tmp + num_experts + 1, nullptr, perm, inv, st);
  const cudaError_t se = le == cudaSuccess ? cudaStreamSynchronize(st) : le;
  dfree(tmp);
  CUDA_TRY(se);
  // ids outside [0, num_experts) are left out of the maps: the total falls short
  int32_t total = 0;
  CUDA_TRY(cudaMemcpy(&total, offsets + num_experts, sizeof(int32_t), cudaMemcpyDeviceToHost));
  if (static_cast<uint64_t>(total) != P)
    return fail(MXMOE_ERR_INVALID_ARG, "%llu of %llu expert ids lie outside [0, %u)",
                (unsigned long long)(P - static_cast<uint64_t>(total)), (unsigned long long)P, num_experts);
  return MXMOE_OK;
}

}  // extern "C"

// Scratch of mxmoe_permute_noalloc: per-expert padded offsets and counts
// (2 x (kNoAllocMaxExperts + 1) int32 = 8 KB).  It lives in the library's own
// device memory on every GPU that loads it, for the life of the process.
namespace {
constexpr uint32_t kNoAllocMaxExperts = 1024;
static __device__ __align__(256) int32_t g_permute_scratch[2 * (kNoAllocMaxExperts + 1)];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
int32_t* g_scratch_ptr[kMaxDevices] = {};

// Device address of the scratch array for the current device, looked up once
// per device.  Host code cannot pass g_permute_scratch itself: on the host
// that name is only a stand-in, not a device address.
int scratch_for_current_device(int32_t** out) {
  int dev = -1;
  CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return fail(MXMOE_ERR_UNSUPPORTED, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    CUDA_TRY(cudaGetSymbolAddress(&p, g_permute_scratch));
    g_scratch_ptr[dev] = static_cast<int32_t*>(p);
  }
  *out = g_scratch_ptr[dev];
  return MXMOE_OK;
}
}  // namespace

extern "C" {

int mxmoe_permute_noalloc(const int32_t* topk_idx, uint32_t n_tokens, uint32_t k, uint32_t num_experts,
                          int32_t* offsets, int32_t* perm, int32_t* inv, void* stream) {
  if (num_experts == 0)
    return fail(MXMOE_ERR_UNSUPPORTED, "num_experts must be at least 1");
  if (num_experts > kNoAllocMaxExperts)
    return fail(MXMOE_ERR_TOO_LARGE, "mxmoe_permute_noalloc handles at most %u experts (got %u)",
                kNoAllocMaxExperts, num_experts);
  const uint64_t P = static_cast<uint64_t>(n_tokens) * k;
  if (P > static_cast<uint64_t>(INT32_MAX)) return fail(MXMOE_ERR_TOO_LARGE, "n_tokens * k = %llu pairs", (unsigned long long)P);
  if (!offsets || (P > 0 && (!topk_idx || !perm || !inv))) return fail(MXMOE_ERR_INVALID_ARG, "null pointer");
  int32_t* scratch = nullptr;
  TRY(scratch_for_current_device(&scratch));
  // The kernel writes every scratch entry it reads, so nothing needs clearing.
  CUDA_TRY(launch_permute(topk_idx, static_cast<int>(P), num_experts, 1, 1, offsets, nullptr, nullptr, scratch,
                          scratch + num_experts + 1, nullptr, perm, inv, as_stream(stream)));
  return MXMOE_OK;
}

int mxmoe_set_fault_injection(mxmoe_layer* L, uint32_t mode) {
  TRY(check_layer(L));
  if (mode > MXMOE_FAULT_SKIP_SIGNAL) return fail(MXMOE_ERR_INVALID_ARG, "unknown fault mode %u", mode);
  L->fault = mode;
  return MXMOE_OK;
}

int mxmoe_set_profiling(mxmoe_layer* L, int enable) {
  TRY(check_layer(L));
  DeviceGuard g(L->cfg.device);
  if (enable && !L->ev[0])
    for (auto& e : L->ev) CUDA_TRY(cudaEventCreate(&e));
  L->profiling = enable != 0;
  L->profile_valid = false;
  return MXMOE_OK;
}

int mxmoe_last_profile(mxmoe_layer* L, float* ms, int cap, int* count) {
  TRY(check_layer(L));
  if (!L->profiling || !L->profile_valid) return fail(MXMOE_ERR_NOT_READY, "no profiled forward");
  DeviceGuard g(L->cfg.device);
  CUDA_TRY(cudaEventSynchronize(L->ev[6]));
  const int n = 6;
  for (int i = 0; i < n && i < cap; ++i) CUDA_TRY(cudaEventElapsedTime(&ms[i], L->ev[i], L->ev[i + 1]));
  if (count) *count = n;
  return MXMOE_OK;
}

int mxmoe_route(mxmoe_layer* L, const void* x, mxmoe_dtype x_dtype, uint32_t n_tokens, float* rscale,
                int32_t* topk_idx, float* topk_w, int32_t* offsets, int32_t* perm, int32_t* inv, void* stream) {
  TRY(check_layer(L));
  if (!L->router_ready) return fail(MXMOE_ERR_NOT_READY, "router not uploaded");
  if (n_tokens == 0) return MXMOE_OK;
  if (!x || !rscale || !topk_idx || !topk_w) return fail(MXMOE_ERR_INVALID_ARG, "null pointer");
  DeviceGuard g(L->cfg.device);
  TRY(ensure_workspace(L, n_tokens, L->k));
  Workspace& w = L->ws;
  cudaStream_t st = as_stream(stream);
  const uint32_t k = L->k;
  CUDA_TRY(launch_router(x, x_dtype, n_tokens, L->d, L->E_total, k, L->gamma, L->gate_w, L->gate_b, L->cfg.rms_eps,
                         w.logits, topk_idx, topk_w, rscale, st));
  if (offsets || perm || inv) {
    if (!offsets || !perm || !inv) return fail(MXMOE_ERR_INVALID_ARG, "offsets, perm and inv go together");
    CUDA_TRY(launch_permute(topk_idx, static_cast<int>(n_tokens * k), L->E_total, 1, 1, offsets, nullptr, nullptr,
                            w.poff, w.counts, nullptr, perm, inv, st, w.perm_scratch));
  }
  return MXMOE_OK;
}

int mxmoe_gather_pairs(const void* x, mxmoe_dtype x_dtype, uint32_t n_tokens, uint32_t d_model, uint32_t k,
                       const int32_t* perm, const float* rscale, const int32_t* topk_idx, const float* topk_w,
                       void* out_x, uint32_t* out_meta, void* stream) {
  const uint64_t P = static_cast<uint64_t>(n_tokens) * k;
  if (P == 0) return MXMOE_OK;
  if (!x || !perm || !rscale || !topk_idx || !topk_w || !out_x || !out_meta)
    return fail(MXMOE_ERR_INVALID_ARG, "null pointer");
  if (d_model % 32 != 0) return fail(MXMOE_ERR_UNSUPPORTED, "d_model must be a multiple of 32");
  if (!aligned16(x) || !aligned16(out_x)) return fail(MXMOE_ERR_INVALID_ARG, "x and out_x must be 16-byte aligned");
  CUDA_TRY(launch_gather_pairs(x, x_dtype, d_model, k, static_cast<int>(P), perm, rscale, topk_idx, topk_w, out_x,
                               out_meta, as_stream(stream)));
  return MXMOE_OK;
}

int mxmoe_forward_local(mxmoe_layer* L, const void* xr, mxmoe_dtype xr_dtype, const float* rscale,
                        const int32_t* expert, const float* weight, uint32_t n_pairs, void* out,
                        mxmoe_dtype out_dtype, void* stream) {
  TRY(check_layer(L));
  if (!L->experts_ready) return fail(MXMOE_ERR_NOT_READY, "experts not uploaded");
  if (n_pairs == 0) return MXMOE_OK;
  if (!xr || !rscale || !expert || !weight || !out) return fail(MXMOE_ERR_INVALID_ARG, "null pointer");
  if (!aligned16(xr) || !aligned16(out)) return fail(MXMOE_ERR_INVALID_ARG, "xr and out must be 16-byte aligned");
  DeviceGuard g(L->cfg.device);
  TRY(ensure_workspace(L, n_pairs, 1));
  Workspace& w = L->ws;
  cudaStream_t st = as_stream(stream);
  const int xt = x_terms_for(L, xr_dtype);
  const TilePlan tp = pick_tiles(n_pairs, L->e_count, xt, gemv_ok(L));
  CUDA_TRY(cudaMemsetAsync(L->err, 0, (kStatusSyncOffset + L->E_total) * sizeof(int), st));
  CUDA_TRY(launch_localize(expert, static_cast<int>(n_pairs), static_cast<int>(L->e_begin),
                           static_cast<int>(L->e_count), w.local_idx, L->err, st));
  CUDA_TRY(launch_permute(w.local_idx, static_cast<int>(n_pairs), L->e_count, kRowBlock, tp.pair_tile, nullptr,
                          nullptr, nullptr, w.poff, w.counts, w.ntile_prefix, w.perm_p, w.inv_p, st,
                          w.perm_scratch));
  TRY(run_experts(L, xr, xr_dtype, n_pairs, 1, rscale, weight, tp, xt, st));
  CUDA_TRY(launch_combine(nullptr, 0, w.y_pair, w.pair_dtype, w.local_idx, w.inv_p, n_pairs, L->d, 1, 0, out, out_dtype, st));
  return MXMOE_OK;
}

int mxmoe_combine(const void* x, mxmoe_dtype x_dtype, uint32_t n_tokens, uint32_t d_model, uint32_t k,
                  const int32_t* topk_idx, const int32_t* inv, const void* pair_out, mxmoe_dtype pair_dtype,
                  int residual, void* y, mxmoe_dtype y_dtype, void* stream) {
  if (n_tokens == 0) return MXMOE_OK;
  if (!y || (residual && !x) || (k > 0 && (!topk_idx || !inv || !pair_out)))
    return fail(MXMOE_ERR_INVALID_ARG, "null pointer");
  if (k > static_cast<uint32_t>(kMaxTopK)) return fail(MXMOE_ERR_UNSUPPORTED, "k=%u", k);
  if (d_model % 4 != 0) return fail(MXMOE_ERR_UNSUPPORTED, "d_model must be a multiple of 4");
  if (!aligned16(x) || !aligned16(pair_out) || !aligned16(y))
    return fail(MXMOE_ERR_INVALID_ARG, "x, pair_out and y must be 16-byte aligned");
  CUDA_TRY(launch_combine(x, x_dtype, pair_out, pair_dtype, topk_idx, inv, n_tokens, d_model, k, residual, y, y_dtype,
                          as_stream(stream)));
  return MXMOE_OK;
}

// ------------------------------------------------------------------ expert-parallel over peer memory
int mxmoe_ipc_alloc(size_t bytes, int device, void** ptr, void* handle) {
  if (!ptr || !handle || bytes == 0) return fail(MXMOE_ERR_INVALID_ARG, "bad ipc allocation request");
  DeviceGuard g(device);
  *ptr = nullptr;
  CUDA_TRY(cudaMalloc(ptr, bytes));
  CUDA_TRY(cudaMemset(*ptr, 0, bytes));
  cudaIpcMemHandle_t h;
  CUDA_TRY(cudaIpcGetMemHandle(&h, *ptr));
  static_assert(sizeof(cudaIpcMemHandle_t) == MXMOE_IPC_HANDLE_BYTES, "IPC handle size");
  std::memcpy(handle, &h, sizeof(h));
  return MXMOE_OK;
}

int mxmoe_ipc_free(void* ptr, int device) {
  if (!ptr) return MXMOE_OK;
  DeviceGuard g(device);
  CUDA_TRY(cudaFree(ptr));
  return MXMOE_OK;
}

int mxmoe_ipc_open(const void* handle, int device, void** peer_ptr) {
  if (!handle || !peer_ptr) return fail(MXMOE_ERR_INVALID_ARG, "null ipc handle");
  DeviceGuard g(device);
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  CUDA_TRY(cudaIpcOpenMemHandle(peer_ptr, h, cudaIpcMemLazyEnablePeerAccess));
  return MXMOE_OK;
}

int mxmoe_ipc_close(void* peer_ptr, int device) {
  if (!peer_ptr) return MXMOE_OK;
  DeviceGuard g(device);
  CUDA_TRY(cudaIpcCloseMemHandle(peer_ptr));
  return MXMOE_OK;
}

int mxmoe_dispatch_pairs(const void* x, mxmoe_dtype x_dtype, uint32_t n_tokens, uint32_t d_model, uint32_t k,
                         const int32_t* perm, const float* rscale, const int32_t* topk_idx, const float* topk_w,
                         const int32_t* offsets, uint32_t experts_per_rank, uint32_t world, uint32_t rank,
                         const int32_t* counts, void* const* peer_x, uint32_t* const* peer_meta,
                         uint32_t recv_cap, int* err, void* stream) {
  const uint64_t P = static_cast<uint64_t>(n_tokens) * k;
  if (P == 0) return MXMOE_OK;
  if (!x || !perm || !rscale || !topk_idx || !topk_w || !offsets || !counts || !peer_x || !peer_meta)
    return fail(MXMOE_ERR_INVALID_ARG, "null pointer");
  if (world == 0 || rank >= world || world > 256 || experts_per_rank == 0)
    return fail(MXMOE_ERR_INVALID_ARG, "bad world %u / rank %u", world, rank);
  if (P >= (1u << 24)) return fail(MXMOE_ERR_TOO_LARGE, "too many pairs for return slots: %llu", (unsigned long long)P);
  if (d_model % 32 != 0) return fail(MXMOE_ERR_UNSUPPORTED, "d_model must be a multiple of 32");
  if (!aligned16(x)) return fail(MXMOE_ERR_INVALID_ARG, "x must be 16-byte aligned");
  CUDA_TRY(launch_dispatch_pairs(x, x_dtype, d_model, k, static_cast<int>(P), perm, rscale, topk_idx, topk_w, offsets,
                                 experts_per_rank, world, rank, counts, peer_x, peer_meta, recv_cap, err,
                                 as_stream(stream)));
  return MXMOE_OK;
}

int mxmoe_forward_local_meta(mxmoe_layer* L, const void* xr, mxmoe_dtype xr_dtype, const uint32_t* meta,
                             uint32_t n_pairs, void* const* ret_ptrs, uint32_t world, uint32_t ret_rows,
                             uint32_t flags, void* stream) {
  TRY(check_layer(L));
  if (!L->experts_ready) return fail(MXMOE_ERR_NOT_READY, "experts not uploaded");
  if (n_pairs == 0) return MXMOE_OK;
  if (!xr || !meta || !ret_ptrs) return fail(MXMOE_ERR_INVALID_ARG, "null pointer");
  if (!aligned16(xr) || !aligned16(meta)) return fail(MXMOE_ERR_INVALID_ARG, "xr and meta must be 16-byte aligned");
  if (L->cfg.flags & MXMOE_FLAG_SIMT) return fail(MXMOE_ERR_UNSUPPORTED, "peer return needs the tensor-core path");
  DeviceGuard g(L->cfg.device);
  TRY(ensure_workspace(L, n_pairs, 1));
  Workspace& w = L->ws;
  cudaStream_t st = as_stream(stream);
  const int xt = x_terms_for(L, xr_dtype);
  const TilePlan tp = pick_tiles(n_pairs, L->e_count, xt);
  CUDA_TRY(cudaMemsetAsync(L->err, 0, (kStatusSyncOffset + L->E_total) * sizeof(int), st));
  // profiled stages: split + localize in the "router" slot, no combine
  L->profile_valid = false;
  if (L->profiling) CUDA_TRY(cudaEventRecord(L->ev[0], st));
  CUDA_TRY(launch_split_meta(meta, static_cast<int>(n_pairs), w.rscale, w.topk_idx, w.topk_w, w.ret_slot, st));
  CUDA_TRY(launch_localize(w.topk_idx, static_cast<int>(n_pairs), static_cast<int>(L->e_begin),
                           static_cast<int>(L->e_count), w.local_idx, L->err, st));
  if (L->profiling) CUDA_TRY(cudaEventRecord(L->ev[1], st));
  CUDA_TRY(launch_permute(w.local_idx, static_cast<int>(n_pairs), L->e_count, kRowBlock, tp.pair_tile, nullptr,
                          nullptr, nullptr, w.poff, w.counts, w.ntile_prefix, w.perm_p, w.inv_p, st,
                          w.perm_scratch));
  if (L->profiling) CUDA_TRY(cudaEventRecord(L->ev[2], st));
  if (flags & MXMOE_RETURN_FROM_EPILOGUE) {
    TRY(run_experts(L, xr, xr_dtype, n_pairs, 1, w.rscale, w.topk_w, tp, xt, st, ret_ptrs, w.ret_slot));
  } else {
    // W2 writes this GPU's rows in received order, then one pass pushes each
    // row to its source in 512-byte warp stores
    TRY(run_experts(L, xr, xr_dtype, n_pairs, 1, w.rscale, w.topk_w, tp, xt, st, nullptr, nullptr, true));
    CUDA_TRY(launch_return_pairs(w.y_pair, static_cast<int>(L->d), static_cast<int>(n_pairs), w.ret_slot,
                                 static_cast<int>(world), ret_ptrs, ret_rows, L->err, st));
  }
  if (L->profiling) {
    CUDA_TRY(cudaEventRecord(L->ev[6], st));
    L->profile_valid = true;
  }
  return MXMOE_OK;
}

// ---- expert parallelism: quantized dispatch into the owners' layouts
constexpr int kEpBuffers = 3;  // codes, row-major scales, row metadata (mxmoe_ep_reserve order)

int mxmoe_ep_reserve(mxmoe_layer* L, uint32_t max_tokens, uint32_t world, void* handles) {
  TRY(check_layer(L));
  if (!handles || max_tokens == 0 || world == 0) return fail(MXMOE_ERR_INVALID_ARG, "bad ep reservation");
  if (L->ep_reserved) return fail(MXMOE_ERR_INVALID_ARG, "ep workspace already reserved");
  if (L->e_count * world != L->E_total)
    return fail(MXMOE_ERR_INVALID_ARG, "shard of %u experts x %u ranks != %u experts", L->e_count, world, L->E_total);
  if (static_cast<uint64_t>(max_tokens) * L->k >= (1u << 24))
    return fail(MXMOE_ERR_TOO_LARGE, "max_tokens * k must stay below 2^24 (return slots)");
  DeviceGuard g(L->cfg.device);
  TRY(ensure_workspace(L, world * max_tokens, L->k));
  CUDA_TRY(cudaDeviceSynchronize());
  Workspace& w = L->ws;
  void* bufs[kEpBuffers] = {w.xq, w.ep_sf_rows, w.ep_meta};
  for (int i = 0; i < kEpBuffers; ++i) {
    cudaIpcMemHandle_t h;
    CUDA_TRY(cudaIpcGetMemHandle(&h, bufs[i]));
    std::memcpy(static_cast<uint8_t*>(handles) + i * MXMOE_IPC_HANDLE_BYTES, &h, sizeof(h));
  }
  L->ep_reserved = true;
  L->ep_world = world;
  L->ep_max_tokens = max_tokens;
  return MXMOE_OK;
}

static TilePlan ep_tiles(const mxmoe_layer* L, int xt) {
  // every rank derives the owners' tile plan from the same numbers
  return pick_tiles(static_cast<uint64_t>(L->ep_max_tokens) * L->k, L->e_count, xt);
}

int mxmoe_ep_dispatch(mxmoe_layer* L, const void* x, mxmoe_dtype x_dtype, uint32_t n_tokens, const float* rscale,
                      const int32_t* topk_idx, const float* topk_w, const int32_t* inv, const int32_t* offsets,
                      const int32_t* counts, uint32_t rank, void* const* peer_bufs, void* stream) {
  TRY(check_layer(L));
  if (!L->ep_reserved) return fail(MXMOE_ERR_NOT_READY, "mxmoe_ep_reserve first");
  if (n_tokens > L->ep_max_tokens) return fail(MXMOE_ERR_TOO_LARGE, "%u tokens > reserved %u", n_tokens, L->ep_max_tokens);
  if (rank >= L->ep_world) return fail(MXMOE_ERR_INVALID_ARG, "rank %u of %u", rank, L->ep_world);
  if (!counts || !peer_bufs || (n_tokens > 0 && (!x || !rscale || !topk_idx || !topk_w || !inv || !offsets)))
    return fail(MXMOE_ERR_INVALID_ARG, "null pointer");
  if (!aligned16(x)) return fail(MXMOE_ERR_INVALID_ARG, "x must be 16-byte aligned");
  if (L->cfg.flags & MXMOE_FLAG_SIMT) return fail(MXMOE_ERR_UNSUPPORTED, "ep dispatch needs the tensor-core path");
  DeviceGuard g(L->cfg.device);
  Workspace& w = L->ws;
  cudaStream_t st = as_stream(stream);
  const int xt = x_terms_for(L, x_dtype);
  const TilePlan tp = ep_tiles(L, xt);
  const int world = static_cast<int>(L->ep_world);
  CUDA_TRY(cudaMemsetAsync(L->err, 0, (kStatusSyncOffset + L->E_total) * sizeof(int), st));
  CUDA_TRY(launch_ep_layout(counts, world, static_cast<int>(rank), static_cast<int>(L->E_total),
                            static_cast<int>(L->e_count), kRowBlock, tp.pair_tile, w.ep_src_base, w.poff, w.counts,
                            w.ntile_prefix, st));
  if (n_tokens == 0) return MXMOE_OK;
  void* const* pb = peer_bufs;
  CUDA_TRY(launch_ep_quantize_dispatch(
      x, x_dtype, static_cast<int>(n_tokens), static_cast<int>(L->d), static_cast<int>(L->k), L->gamma,
      L->gamma_is_one ? 1 : 0, inv, xt, static_cast<uint64_t>(w.rows) * L->kp1, static_cast<int>(L->kp1),
      tp.pair_tile, tp.stacked ? 1 : 0, w.ep_src_base, offsets, topk_idx, topk_w, rscale,
      static_cast<int>(L->e_count), static_cast<int>(rank), w.rows, w.ep_sf_row_bytes,
      reinterpret_cast<uint8_t* const*>(pb), reinterpret_cast<uint8_t* const*>(pb + world), pb + 2 * world, L->err,
      st));
  return MXMOE_OK;
}

int mxmoe_ep_experts(mxmoe_layer* L, mxmoe_dtype x_dtype, void* const* peer_ret, uint32_t ret_rows, void* stream) {
  TRY(check_layer(L));
  if (!L->ep_reserved) return fail(MXMOE_ERR_NOT_READY, "mxmoe_ep_reserve first");
  if (!L->experts_ready) return fail(MXMOE_ERR_NOT_READY, "experts not uploaded");
  if (!peer_ret) return fail(MXMOE_ERR_INVALID_ARG, "null pointer");
  DeviceGuard g(L->cfg.device);
  Workspace& w = L->ws;
  cudaStream_t st = as_stream(stream);
  const int xt = x_terms_for(L, x_dtype);
  const TilePlan tp = ep_tiles(L, xt);
  L->profile_valid = false;
  const uint64_t kc1 = L->kp1 / kTileK;
  CUDA_TRY(launch_ep_unpack(w.ep_meta, w.ep_sf_rows, w.ep_sf_row_bytes, xt, static_cast<int>(L->d / 32),
                            static_cast<int>(w.rows), w.poff, w.counts, static_cast<int>(L->e_count), w.pos_rscale,
                            w.pos_weight, w.pos_slot, w.xsf, static_cast<uint64_t>(w.row_blocks) * kc1 * kSfAtomBytes,
                            static_cast<int>(kc1), tp.pair_tile, tp.stacked ? 1 : 0, st));
  // rows are their own pairs (identity permutation, one pair per row); W2
  // runs in two halves and the first half's rows return while the second computes
  const ReturnSplit split{peer_ret, ret_rows};
  TRY(run_experts(L, nullptr, x_dtype, L->ep_world * L->ep_max_tokens * L->k, 1, w.pos_rscale, w.pos_weight, tp, xt,
                  st, nullptr, nullptr, false, true, w.iota, &split));
  return MXMOE_OK;
}

int mxmoe_ep_attach(mxmoe_layer* L, uint32_t rank, uint32_t world, void* const* peer_bufs, void* const* peer_ret,
                    int32_t* const* peer_counts, mxmoe_ep_barrier_fn barrier, void* barrier_ctx) {
  TRY(check_layer(L));
  if (!L->ep_reserved) return fail(MXMOE_ERR_NOT_READY, "mxmoe_ep_reserve first");
  if (world != L->ep_world || rank >= world)
    return fail(MXMOE_ERR_INVALID_ARG, "rank %u of %u does not match the reservation for %u ranks", rank, world,
                L->ep_world);
  if (!peer_bufs || !peer_ret || !peer_counts || !barrier) return fail(MXMOE_ERR_INVALID_ARG, "null pointer");
  for (uint32_t i = 0; i < world; ++i) {
    if (!peer_ret[i] || !peer_counts[i]) return fail(MXMOE_ERR_INVALID_ARG, "null peer buffer for rank %u", i);
    for (int b = 0; b < kEpBuffers; ++b)
      if (!peer_bufs[b * world + i]) return fail(MXMOE_ERR_INVALID_ARG, "null peer buffer for rank %u", i);
  }
  DeviceGuard g(L->cfg.device);
  auto& a = L->epa;
  if (!a.bufs) {
    CUDA_TRY(cudaMalloc(reinterpret_cast<void**>(&a.bufs), kEpBuffers * world * sizeof(void*)));
    CUDA_TRY(cudaMalloc(reinterpret_cast<void**>(&a.ret), world * sizeof(void*)));
    CUDA_TRY(cudaMalloc(reinterpret_cast<void**>(&a.counts), world * sizeof(int32_t*)));
  }
  CUDA_TRY(cudaMemcpy(a.bufs, peer_bufs, kEpBuffers * world * sizeof(void*), cudaMemcpyHostToDevice));
  CUDA_TRY(cudaMemcpy(a.ret, peer_ret, world * sizeof(void*), cudaMemcpyHostToDevice));
  CUDA_TRY(cudaMemcpy(a.counts, peer_counts, world * sizeof(int32_t*), cudaMemcpyHostToDevice));
  a.own_ret = peer_ret[rank];
  a.own_counts = peer_counts[rank];
  a.rank = rank;
  a.barrier = barrier;
  a.ctx = barrier_ctx;
  a.on = true;
  return MXMOE_OK;
}

int mxmoe_ep_forward(mxmoe_layer* L, const void* x, mxmoe_dtype x_dtype, uint32_t n_tokens, void* y,
                     mxmoe_dtype y_dtype, void* stream) {
  TRY(check_layer(L));
  auto& a = L->epa;
  if (!a.on) return fail(MXMOE_ERR_NOT_READY, "mxmoe_ep_attach first");
  if (n_tokens > L->ep_max_tokens) return fail(MXMOE_ERR_TOO_LARGE, "%u tokens > reserved %u", n_tokens, L->ep_max_tokens);
  if (n_tokens > 0 && (!x || !y)) return fail(MXMOE_ERR_INVALID_ARG, "null pointer");
  if (!aligned16(x) || !aligned16(y)) return fail(MXMOE_ERR_INVALID_ARG, "x and y must be 16-byte aligned");
  DeviceGuard g(L->cfg.device);
  Workspace& w = L->ws;
  cudaStream_t st = as_stream(stream);
  const int world = static_cast<int>(L->ep_world), rank = static_cast<int>(a.rank);
  // 1. route this rank's tokens (full router) and sort its pairs by expert
  if (n_tokens > 0)
    TRY(mxmoe_route(L, x, x_dtype, n_tokens, w.rscale, w.topk_idx, w.topk_w, w.offsets, w.perm_c, w.inv_c, stream));
  // 2. this rank's pairs per expert into every rank's count table
  CUDA_TRY(launch_ep_push_counts(n_tokens > 0 ? w.offsets : nullptr, static_cast<int>(L->E_total), rank, world,
                                 a.counts, st));
  if (a.barrier(a.ctx, stream) != 0) return fail(MXMOE_ERR_CUDA, "ep barrier failed after the count exchange");
  // 3. quantize and write every pair into its owner's layout
  TRY(mxmoe_ep_dispatch(L, x, x_dtype, n_tokens, w.rscale, w.topk_idx, w.topk_w, w.inv_c, w.offsets, a.own_counts,
                        a.rank, a.bufs, stream));
  if (a.barrier(a.ctx, stream) != 0) return fail(MXMOE_ERR_CUDA, "ep barrier failed after the dispatch");
  // 4. this rank's experts over every source's pairs, outputs pushed back to the sources
  TRY(mxmoe_ep_experts(L, x_dtype, a.ret, L->ep_max_tokens * L->k, stream));
  if (a.barrier(a.ctx, stream) != 0) return fail(MXMOE_ERR_CUDA, "ep barrier failed after the expert FFN");
  // 5. combine in expert order (+ residual)
  if (n_tokens > 0)
    TRY(mxmoe_combine(x, x_dtype, n_tokens, L->d, L->k, w.topk_idx, w.inv_c, a.own_ret, MXMOE_BF16,
                      (L->cfg.flags & MXMOE_FLAG_NO_RESIDUAL) ? 0 : 1, y, y_dtype, stream));
  return MXMOE_OK;
}

int mxmoe_ep_buffers(mxmoe_layer* L, void** ptrs) {
  TRY(check_layer(L));
  if (!L->ep_reserved) return fail(MXMOE_ERR_NOT_READY, "mxmoe_ep_reserve first");
  if (!ptrs) return fail(MXMOE_ERR_INVALID_ARG, "null pointer");
  Workspace& w = L->ws;
  ptrs[0] = w.xq;
  ptrs[1] = w.ep_sf_rows;
  ptrs[2] = w.ep_meta;
  return MXMOE_OK;
}

// Hot-expert copies: each extra slot goes to the expert with the largest load
// per copy (lowest id on ties).
int mxmoe_ep_plan_replicas(const double* loads, uint32_t num_experts, uint32_t extra, int32_t* src) {
  if (num_experts == 0 || !loads || !src) return fail(MXMOE_ERR_INVALID_ARG, "bad replica plan arguments");
  if (static_cast<uint64_t>(num_experts) + extra > INT32_MAX) return fail(MXMOE_ERR_TOO_LARGE, "too many slots");
  std::vector<int64_t> copies(num_experts, 1);
  for (uint32_t e = 0; e < num_experts; ++e) src[e] = static_cast<int32_t>(e);
  for (uint32_t i = 0; i < extra; ++i) {
    uint32_t best = 0;
    double best_v = loads[0] / static_cast<double>(copies[0]);
    for (uint32_t e = 1; e < num_experts; ++e) {
      const double v = loads[e] / static_cast<double>(copies[e]);
      if (v > best_v) {
        best_v = v;
        best = e;
      }
    }
    ++copies[best];
    src[num_experts + i] = static_cast<int32_t>(best);
  }
  return MXMOE_OK;
}

// Greedy longest-first placement into world ranks of num_experts / world slots.
int mxmoe_ep_balanced_placement(const double* loads, uint32_t num_experts, uint32_t world, int32_t* order) {
  if (num_experts == 0 || world == 0 || !loads || !order) return fail(MXMOE_ERR_INVALID_ARG, "bad placement arguments");
  if (num_experts % world != 0)
    return fail(MXMOE_ERR_INVALID_ARG, "%u experts do not split over %u ranks", num_experts, world);
  const uint32_t per = num_experts / world;
  std::vector<uint32_t> ids(num_experts);
  for (uint32_t e = 0; e < num_experts; ++e) ids[e] = e;
  std::stable_sort(ids.begin(), ids.end(), [&](uint32_t a, uint32_t b) { return loads[a] > loads[b]; });
  std::vector<double> total(world, 0.0);
  std::vector<std::vector<uint32_t>> slots(world);
  for (uint32_t e : ids) {
    uint32_t best = world;
    for (uint32_t r = 0; r < world; ++r) {
      if (slots[r].size() >= per) continue;
      if (best == world || total[r] < total[best]) best = r;
    }
    slots[best].push_back(e);
    total[best] += loads[e];
  }
  uint32_t o = 0;
  for (uint32_t r = 0; r < world; ++r) {
    std::sort(slots[r].begin(), slots[r].end());
    for (uint32_t e : slots[r]) order[o++] = static_cast<int32_t>(e);
  }
  return MXMOE_OK;
}

}  // extern "C"
