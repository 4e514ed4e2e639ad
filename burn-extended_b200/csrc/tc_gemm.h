// tc_gemm.h -- host-side interface of the tcgen05 grouped expert GEMM.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstddef>
#include <cstdint>

namespace mxmoe {

struct TcParams {
  int mode;      // 1 = W1 + SwiGLU (writes act codes), 2 = W2 + bias + route weight (writes y_pair)
  int N;         // weights-as-A: routed pairs per tile (32, 64, 128); tokens-as-A: 256 weight rows
  int m_tiles;   // weight tiles per expert (128 rows weights-as-A, 256 rows tokens-as-A)
  int w_row_pairs;   // 256-row scale-atom pairs per expert of the weight operand (w_sf_offset)
  int units;     // W1: GLU units written to the activation operand (f padded to 64)
  int k_tiles;   // K / 128
  int E;         // experts held by this layer
  int stages;    // smem pipeline depth
  int b_terms;   // E4M3 terms of the activation operand (2 or 3)
  int sf_rows;   // rows per activation scale atom (= pairs per tile, <= 128)
  int stacked;   // tokens-as-A tiles of 64 pairs with both activation terms in one 128-row operand
  int fp4;       // kind::mxf4 stacked tiles: four E2M1 activation terms, K = 256 per stage
  int k_chunks;  // 128-K scale chunks of the operands (= k_tiles except in fp4 tiles)
  int last_mmas; // fp4: MMAs of K = 64 issued in the last stage (the rest is K padding)
  const int* poff;          // [E+1] padded segment starts (multiples of 128)
  const int* counts;        // [E] pairs per expert
  const int* ntile_prefix;  // [E+1] prefix sums of ceil(count / N)
  const uint8_t* a_sf;      // weight scale atoms [E][m_tiles][k_tiles][512]
  const uint8_t* b_sf;      // activation scale atoms [terms][row_blocks][k_tiles][512]
  uint64_t b_sf_term_stride;
  const float* bias;        // W1: [E][2fp] packed rows; W2: [E][d]
  int bias_stride;
  int rows_valid;           // W2: d
  float alpha, limit, bias_mult;
  const float* rscale;      // [n] 1 / rms per token
  const int* perm;          // padded position -> pair t*k+s
  int k;
  const float* topk_w;      // [n*k]
  uint8_t* act_codes;       // W1 output [2][rows][act_kp]
  uint64_t act_term_stride;
  int act_kp;    // bytes per activation code row
  uint8_t* act_sf;          // W1 output atoms [2][row_blocks][act_kchunks][512]
  float* act_f32;           // fp4 W1 output [rows][units] f32 (SwiGLU, before quantization)
  uint64_t act_sf_term_stride;
  int act_kchunks;
  float* y_pair;            // W2 output [rows][d] f32 (weights-as-A)
  __nv_bfloat16* y_pair_bf16;  // W2 output [rows][d] bf16 (tokens-as-A)
  // Expert-parallel return (tokens-as-A W2): when set, the output of pair
  // `pair` goes to row (ret_slot[pair] & 0xFFFFFF) of the bf16 buffer
  // ret_ptrs[ret_slot[pair] >> 24] (a peer GPU's return buffer) instead of
  // y_pair_bf16.
  void* const* ret_ptrs;
  const uint32_t* ret_slot;
  int y_by_pair;  // W2 output row = the pair's own index (received row) instead of its sorted position
  // Expert range [e_lo, e_hi) of this launch (e_hi = 0: all E): its tiles are
  // m_tiles * ntile_prefix[e_lo] .. m_tiles * ntile_prefix[e_hi], read on the device.
  int e_lo, e_hi;
  int d;
  int* err;                 // device status word (0 = ok)
  // Test hook (mxmoe_set_fault_injection): with skip_stage set, CTA 0's
  // producer never arms its first pipeline stage, so the MMA issuer's wait
  // for it runs out; wait_ns limits the waits that record a status.
  int skip_stage;
  unsigned long long wait_ns;
};

size_t tc_gemm_smem_bytes(bool tokens_as_a, int N, int terms, int stages, int pair_tile, bool stacked,
                          bool fp4 = false);
int tc_gemm_max_stages(bool tokens_as_a, int N, int terms, size_t smem_limit, int pair_tile, bool stacked,
                       bool fp4 = false);
// tmap_w: weight codes (box 128 rows weights-as-A, 256 rows tokens-as-A);
// tmap_x: activation terms (box = pairs per tile rows).
cudaError_t tc_gemm_launch(bool tokens_as_a, const CUtensorMap& tmap_w, const CUtensorMap& tmap_x,
                           const TcParams& p, int grid, cudaStream_t stream);

}  // namespace mxmoe
