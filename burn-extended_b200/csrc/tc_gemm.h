// tc_gemm.h -- host-side interface of the tcgen05 grouped expert GEMM.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cstddef>
#include <cstdint>

namespace mxmoe {

struct TcParams {
  int mode;      // 1 = W1 + SwiGLU (writes act codes), 2 = W2 + bias + route weight (writes y_pair)
  int N;         // routed pairs per tile: 32, 64, 128 or 256
  int m_tiles;   // 128-row weight tiles per expert
  int k_tiles;   // K / 128
  int E;         // experts held by this layer
  int stages;    // smem pipeline depth
  int b_terms;   // E4M3 terms of the activation operand (2 or 3)
  int sf_rows;   // rows per activation scale atom: min(N, 128)
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
  int act_kp;
  uint8_t* act_sf;          // W1 output atoms [2][row_blocks][act_kchunks][512]
  uint64_t act_sf_term_stride;
  int act_kchunks;
  float* y_pair;            // W2 output [rows][d]
  int d;
  int* err;                 // device status word (0 = ok)
};

size_t tc_gemm_smem_bytes(int N, int terms, int stages);
int tc_gemm_max_stages(int N, int terms, size_t smem_limit);
cudaError_t tc_gemm_launch(const CUtensorMap& tmap_a, const CUtensorMap& tmap_b, const TcParams& p, int grid,
                           cudaStream_t stream);

}  // namespace mxmoe
