/*
 * mxmoe_oracle.h -- CPU restatement of burn-extended's MXFP4 mixture-of-experts
 * hot path.  TEST INFRASTRUCTURE ONLY: it is the checker that the CUDA path is
 * compared against (tests/, __graft_entry__.smoke(), bench.py's cpu_baseline
 * and --impl reference legs).  Nothing in the shipped library links or calls it.
 *
 * Parity status:
 *   - MXFP4 dequant is pinned by the reference's own known-answer test
 *     (tests/mxfp4_dequant_tests.rs:4-25), checked in tests/test_oracle.py.
 *   - Router, permutation, expert FFN and combine: parity unpinned against the
 *     reference binary (the Rust crate cannot be built here and its MoE forward
 *     only runs on wgpu/Metal).  The algorithm restates src/moe/mod.rs and
 *     src/quant/gpu.rs line by line; the points the reference leaves to
 *     third-party code (Burn's RmsNorm epsilon, top-k tie order, summation
 *     order) are fixed by the definitions documented on each function.
 */
#ifndef MXMOE_ORACLE_H
#define MXMOE_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Flags mirror the library's MXMOE_FLAG_* values (include/mxmoe.h). */
#define ORC_FLAG_INTERLEAVED_GLU 0x1u  /* W1 rows [glu0, lin0, glu1, ...] */
#define ORC_FLAG_BIAS_PER_FTILE  0x2u  /* add b2 once per 256-wide f tile */
#define ORC_FLAG_NO_RESIDUAL     0x4u  /* y = moe(x) instead of x + moe(x) */

typedef struct orc_cfg {
  uint32_t d_model;          /* d */
  uint32_t ffn_hidden;       /* f */
  uint32_t num_experts;      /* E */
  uint32_t experts_per_token;/* k */
  float swiglu_alpha;
  float swiglu_limit;
  float rms_eps;
  uint32_t flags;
  int32_t ue8_offset;        /* subtracted from every stored scale byte */
} orc_cfg;

/* Reference src/loader/mxfp4.rs:57-79 (dequant_mxfp4_bytes): one E8M0 scale
 * per row of b packed bytes; out[r, 2i] = LUT[lo], out[r, 2i+1] = LUT[hi]. */
void orc_dequant_mxfp4_bytes(const uint8_t* blocks, size_t rows_total, size_t b,
                             const uint8_t* scales, float* out);

/* MoE weight layout (src/quant/gpu.rs:124-134): blocks [rows][bpr],
 * scales [rows][gpr], one scale per 32 columns, exponent s - 127 - ue8_offset. */
void orc_dequant_rows(const uint8_t* blocks, const uint8_t* scales, size_t rows,
                      size_t cols, size_t bpr, size_t gpr, int ue8_offset,
                      float* out);

/* Router (src/moe/mod.rs:109-110, :270-276): RMSNorm then Linear then
 * top-k then softmax over the k selected logits.  Any output may be NULL. */
void orc_route(const orc_cfg* cfg, size_t n, const float* x, const float* gamma,
               const float* gate_w, const float* gate_b, float* normed,
               float* rscale, float* logits, int32_t* topk_idx, float* topk_w);

/* Top-k + softmax on given logits [n][E] (src/moe/mod.rs:272-276). */
void orc_topk_softmax(size_t n, uint32_t E, uint32_t k, const float* logits,
                      int32_t* topk_idx, float* topk_w);

/* Canonical permutation: stable counting sort of pairs p = t*k + s by expert. */
void orc_permute(size_t n, uint32_t k, uint32_t E, const int32_t* topk_idx,
                 int32_t* offsets, int32_t* perm, int32_t* inv);

/* SwiGLU with clamp (src/quant/gpu.rs:140-145). */
float orc_swiglu(float g, float l, float alpha, float limit);

/* Whole MoE block forward (src/moe/mod.rs:99-115, :122-412), f32 throughout.
 * x [n][d]; gamma [d]; gate_w [E][d]; gate_b [E]; w1 blocks [E][2f][d/2],
 * scales [E][2f][d/32]; b1 [E][2f]; w2 blocks [E][d][f/2], scales [E][d][f/32];
 * b2 [E][d]; y [n][d].  Routing outputs may be NULL.  nthreads <= 0 uses all. */
void orc_moe_forward(const orc_cfg* cfg, size_t n, const float* x,
                     const float* gamma, const float* gate_w, const float* gate_b,
                     const uint8_t* w1_blocks, const uint8_t* w1_scales,
                     const float* b1, const uint8_t* w2_blocks,
                     const uint8_t* w2_scales, const float* b2, float* y,
                     int32_t* topk_idx, float* topk_w, int nthreads);

/* Expert FFN for externally supplied routing (same math as orc_moe_forward
 * after the router); used to check the CUDA expert path on identical routes. */
void orc_moe_experts(const orc_cfg* cfg, size_t n, const float* x,
                     const float* normed, const int32_t* topk_idx,
                     const float* topk_w, const uint8_t* w1_blocks,
                     const uint8_t* w1_scales, const float* b1,
                     const uint8_t* w2_blocks, const uint8_t* w2_scales,
                     const float* b2, float* y, int nthreads);

int orc_num_threads(void);

#ifdef __cplusplus
}
#endif
#endif
