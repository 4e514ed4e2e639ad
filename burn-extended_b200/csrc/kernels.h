// kernels.h -- launchers of the CUDA-core kernels (kernels.cu).
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace mxmoe {

constexpr int kMaxTopK = 8;

cudaError_t launch_dequant_bytes(const uint8_t* blocks, uint64_t rows, uint64_t b, const uint8_t* scales, float* out,
                                 cudaStream_t st);
cudaError_t launch_dequant_rows(const uint8_t* blocks, const uint8_t* scales, uint64_t rows, uint64_t cols,
                                uint64_t bpr, uint64_t gpr, int ue8, float* out, cudaStream_t st);
cudaError_t launch_topk_softmax(const float* logits, int n, int E, int k, int32_t* idx, float* w, cudaStream_t st);
// Router gate weights in the router kernel's chunk order: expert groups of
// kRouterGroup rows, column chunks of kRouterChunk; inside a chunk, row r's
// column c = l + 32*j (l = c % 32) sits at r*kRouterChunk + (j/4)*128 + l*4 +
// j%4, zero past d and past E.  One chunk of a group is one contiguous copy.
constexpr int kRouterGroup = 32;
constexpr int kRouterChunk = 128;
inline size_t router_gate_packed_floats(int E, int d) {
  const size_t groups = (E + kRouterGroup - 1) / kRouterGroup, chunks = (d + kRouterChunk - 1) / kRouterChunk;
  return groups * chunks * kRouterGroup * kRouterChunk;
}
inline void pack_router_gate(const float* w, int E, int d, float* out) {
  const int chunks = (d + kRouterChunk - 1) / kRouterChunk;
  for (size_t i = 0; i < router_gate_packed_floats(E, d); ++i) out[i] = 0.0f;
  for (int e = 0; e < E; ++e)
    for (int c = 0; c < d; ++c) {
      const int g = e / kRouterGroup, r = e % kRouterGroup, ch = c / kRouterChunk, cc = c % kRouterChunk;
      const int l = cc % 32, j = cc / 32;
      const size_t base = (static_cast<size_t>(g) * chunks + ch) * kRouterGroup * kRouterChunk;
      out[base + r * kRouterChunk + (j / 4) * 128 + l * 4 + j % 4] = w[static_cast<size_t>(e) * d + c];
    }
}

// gate_packed: pack_router_gate layout.  Small batches (n <= 512, E <= 32)
// run as one launch (RmsNorm + logits + top-k), larger ones as two or three.
// With tok_ctr ([n] ints, zero; the kernel leaves them zero) batches of at
// most 8 tokens run on many blocks per token (router_tiny_kernel), which
// also zeroes status[0 .. status_words) when status is given.
// The permutation folded into the small-batch router (router_folds_permute):
// the router block that finishes last, by an atomic ticket on *ticket (zero
// before the launch), runs launch_permute's one-block counting sort over all
// n * k pairs with these outputs and arguments.
struct PermFold {
  int* ticket;
  int pad, N;
  int32_t *offsets, *perm_c, *inv_c, *poff, *counts, *ntile_prefix, *perm_p, *inv_p;
};
// Whether launch_router with a PermFold runs the permutation for this shape
// (the small-batch router without token rows for the dequant-GEMV, and a
// one-block permutation).
bool router_folds_permute(int n, int d, int E, int k);
cudaError_t launch_router(const void* x, int x_dtype, int n, int d, int E, int k, const float* gamma,
                          const float* gate_packed, const float* gate_b, float eps, float* logits, int32_t* topk_idx,
                          float* topk_w, float* rscale, cudaStream_t st, __half* xh = nullptr, float xh_scale = 1.0f,
                          int* tok_ctr = nullptr, int* status = nullptr, int status_words = 0,
                          const PermFold* fold = nullptr);
// Canonical permutation.  With scratch (permute_scratch_ints(P, E) int32,
// zeroed once before first use) and P >= kPermMultiBlockMin it runs on many
// blocks; otherwise on one block with no scratch.
constexpr int kPermMultiBlockMin = 2048;
size_t permute_scratch_ints(int P, int E);
cudaError_t launch_permute(const int32_t* topk_idx, int P, int E, int pad, int N, int32_t* offsets, int32_t* perm_c,
                           int32_t* inv_c, int32_t* poff, int32_t* counts, int32_t* ntile_prefix, int32_t* perm_p,
                           int32_t* inv_p, cudaStream_t st, int32_t* scratch = nullptr);
// Four-term E2M1 stacked decode operand (kind::mxf4 tiles of pt <= 32 pairs).
// src_by_pos: x holds one row per padded pair position (k = 1, row
// inv_p[t]) instead of one row per token.
cudaError_t launch_quantize_f4_pairs(const void* x, int x_dtype, int n, int d, int k, const float* gamma,
                                     int gamma_is_one, const int32_t* inv_p, uint8_t* codes, int row_bytes,
                                     uint8_t* sf, int kchunks, int pt, int src_by_pos, cudaStream_t st);
cudaError_t launch_quantize_pairs(const void* x, int x_dtype, int n, int d, int k, const float* gamma,
                                  int gamma_is_one, const int32_t* inv_p, int terms, uint8_t* codes,
                                  uint64_t term_stride, int kp, uint8_t* sf, uint64_t sf_term_stride, int kchunks,
                                  int sf_rows, int stacked, cudaStream_t st);
cudaError_t launch_combine(const void* x, int x_dtype, const void* y_pair, int pair_dtype, const int32_t* topk_idx,
                           const int32_t* inv_p, int n, int d, int k, int residual, void* y, int y_dtype,
                           cudaStream_t st);
cudaError_t launch_localize(const int32_t* expert, int P, int begin, int count, int32_t* local, int* err,
                            cudaStream_t st);
cudaError_t launch_gather_pairs(const void* x, int x_dtype, int d, int k, int P, const int32_t* perm,
                                const float* rscale, const int32_t* topk_idx, const float* topk_w, void* out_x,
                                uint32_t* out_meta, cudaStream_t st);
cudaError_t launch_dispatch_pairs(const void* x, int x_dtype, int d, int k, int P, const int32_t* perm,
                                  const float* rscale, const int32_t* topk_idx, const float* topk_w,
                                  const int32_t* offsets, int experts_per_rank, int world, int rank,
                                  const int32_t* counts, void* const* peer_x, uint32_t* const* peer_meta,
                                  uint32_t recv_cap, int* err, cudaStream_t st);
cudaError_t launch_return_pairs(const void* y_bf16, int d, int R, const uint32_t* slot, int world,
                                void* const* peer_ret, uint32_t ret_rows, int* err, cudaStream_t st);
// Source side of the count exchange: this rank's pairs per expert
// (offsets[e + 1] - offsets[e], or zeros when offsets is null) into row
// `rank` of every rank's [world][E] count table (peer memory).
cudaError_t launch_ep_push_counts(const int32_t* offsets, int E, int rank, int world, int32_t* const* peer_counts,
                                  cudaStream_t st);
cudaError_t launch_ep_layout(const int32_t* counts, int world, int rank, int E, int epr, int pad, int n_tile,
                             int32_t* src_base, int32_t* poff, int32_t* seg_counts, int32_t* ntile_prefix,
                             cudaStream_t st);
cudaError_t launch_ep_quantize_dispatch(const void* x, int x_dtype, int n, int d, int k, const float* gamma,
                                        int gamma_is_one, const int32_t* inv_c, int terms, uint64_t term_stride,
                                        int kp, int sf_rows_n, int stacked, const int32_t* src_base,
                                        const int32_t* offsets, const int32_t* topk_idx, const float* topk_w,
                                        const float* rscale, int epr, int rank, uint32_t dst_rows,
                                        uint32_t sf_row_bytes, uint8_t* const* xq, uint8_t* const* sf_rows,
                                        void* const* meta, int* err, cudaStream_t st);
cudaError_t launch_ep_unpack(const void* meta, const uint8_t* sf_rows, uint32_t sf_row_bytes, int terms, int nb,
                             int rows, const int32_t* poff, const int32_t* seg_counts, int epr, float* rs, float* wt,
                             uint32_t* slot, uint8_t* xsf, uint64_t sf_term_stride, int kchunks, int pt, int stacked,
                             cudaStream_t st);
// threads: block size (a warp per row); 64-thread blocks fit beside a
// tensor-core GEMM CTA on every SM, so a return can run while a GEMM does.
cudaError_t launch_ep_return(const void* y_bf16, int d, int rows, const int32_t* poff, const int32_t* seg_counts,
                             int epr, const uint32_t* slot, int world, void* const* peer_ret, uint32_t ret_rows,
                             int* err, cudaStream_t st, int threads = 256);
cudaError_t launch_iota(int32_t* a, int n, cudaStream_t st);
cudaError_t launch_split_meta(const uint32_t* meta, int R, float* rscale, int32_t* expert, float* weight,
                              uint32_t* slot, cudaStream_t st);
// Fused dequant-GEMV expert FFN for a few pairs per expert (dqgemv.cu):
// W1 + SwiGLU-clamp + W2 + bias + route weight in one launch.  d is a
// multiple of 32, fp of 64, both at most kDqMaxK.
constexpr int kDqMaxK = 4096;
constexpr int kDqSrcF32 = 0, kDqSrcBf16 = 1, kDqSrcF16 = 2;
struct DqParams {
  int d, fp, kp1, kp2;     // kp: padded row length (codes kp / 2 bytes per row)
  const uint8_t* w1q;      // [E][2 fp][kp1 / 2], GLU / linear rows in 64-row blocks
  const uint8_t* w1sr;     // [E][2 fp][sr1] E8M0 scales, row-major copy
  uint32_t sr1;            // scale row stride (kp1 / 32 rounded up to 16)
  const float* b1;         // [E][2 fp] packed row order
  const uint8_t* w2q;      // [E][d][kp2 / 2]
  const uint8_t* w2sr;     // [E][d][sr2]
  uint32_t sr2;
  const float* b2;         // [E][d]
  float bias_mult;
  int E;                   // local experts
  const int32_t* topk_idx; // [P] local expert of each pair (canonical order); out of range: no expert
  int P;                   // routed pairs (at most 8)
  int pair_k;              // pairs per token
  const __half* xh;        // [n][d] normalized token rows * x_scale as f16 (router output), or null
  const void* x;           // [n][d] token rows (staged from here when xh is null)
  int x_dtype;             // kDqSrcF32 / kDqSrcBf16
  const float* gamma;      // [d] RmsNorm gain
  const float* rscale;     // [n] 1 / rms
  float x_scale, inv_x_scale;      // power of two on the staged f16 token rows
  float alpha, limit;
  float act_scale, inv_act_scale;  // power of two on the f16 SwiGLU rows
  __half* act;             // [P][fp] SwiGLU rows by canonical pair (W1 -> W2)
  float* y_pair;           // not fused: [rows][d] f32, row inv[pair]
  const int32_t* inv;      // not fused: [P] pair -> y_pair row
  const float* topk_w;     // [P] canonical route weights
  int fused;               // write y (expert-order sum + residual) and the canonical maps
  int n_tok;               // fused: tokens
  int residual;            // fused: y = x + moe(x)
  void* y;                 // fused: [n][d] layer output
  int y_dtype;             // fused: kDqSrcF32 / kDqSrcBf16
  int32_t* offsets;        // fused: canonical maps written for the caller ([E + 1], [P], [P])
  int32_t* perm_c;
  int32_t* inv_c;
  int* err;                // status block (word 0 code, words 2-4 where the grid wait gave up)
  int* sync;               // grid arrival counter, zero at launch
  int skip_arrival;        // test hook: block 0 never signals its W1 completion
  unsigned long long wait_ns;  // limit of the device-side waits (0: the default 2 s)
  // set by the launcher
  int cu, cr;              // W1 units / W2 rows per chunk
  int slots;               // shared-memory ring slots
  int ahead;               // chunks in flight at most
  uint32_t slot_bytes;
  int xs_rows;             // staged activation rows (pairs rounded up to a power of two)
};
// One block per SM; pairs P <= 8, d and fp <= kDqMaxK, d <= 64 * num_sms,
// 8 * fp <= 256 * num_sms.
cudaError_t launch_dqgemv_ffn(DqParams a, int num_sms, size_t smem_limit, cudaStream_t st);
cudaError_t launch_simt_w1(const void* x, int x_dtype, int d, int k, const float* gamma, const float* rscale,
                           const uint8_t* w1q, const uint8_t* w1sf, const float* b1, int fp, int kp1, int E,
                           const int32_t* poff, const int32_t* counts, const int32_t* perm_p, float alpha, float limit,
                           float* act, cudaStream_t st);
cudaError_t launch_simt_w2(const float* act, int fp, int d, int k, const uint8_t* w2q, const uint8_t* w2sf,
                           const float* b2, float bias_mult, int kp2, int E, const int32_t* poff,
                           const int32_t* counts, const int32_t* perm_p, const float* topk_w, float* y_pair,
                           cudaStream_t st);

}  // namespace mxmoe
