// kernels.cu -- the CUDA-core kernels of the MoE hot path: MXFP4 dequant,
// router (RmsNorm + gate + top-k + softmax), canonical permutation, activation
// quantization into block-scaled E4M3 terms, combine, and the SIMT expert FFN
// (an independent GPU implementation used to cross-check the tensor-core one).
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <type_traits>

#include "kernels.h"
#include "launch_util.h"
#include "layout.cuh"
#include "quant.cuh"

namespace mxmoe {

namespace {

// E2M1 code -> value (src/loader/mxfp4.rs:11-13); codes 8..15 are negatives
// of 0..7, with -0.0 for code 8.
__constant__ float kFp4Lut[16] = {0.0f,  0.5f,  1.0f,  1.5f,  2.0f,  3.0f,  4.0f,  6.0f,
                                  -0.0f, -0.5f, -1.0f, -1.5f, -2.0f, -3.0f, -4.0f, -6.0f};

template <typename T>
__device__ __forceinline__ float load_f32(const T* p, uint64_t i);
template <>
__device__ __forceinline__ float load_f32<float>(const float* p, uint64_t i) { return p[i]; }
template <>
__device__ __forceinline__ float load_f32<__nv_bfloat16>(const __nv_bfloat16* p, uint64_t i) {
  return __bfloat162float(p[i]);
}

__device__ __forceinline__ float load_any(const void* p, int dtype, uint64_t i) {
  return dtype == 0 ? static_cast<const float*>(p)[i]
                    : __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
}

// Butterfly sum over the warp: offsets 16, 8, 4, 2, 1.  Every lane ends with
// the same value (IEEE addition is commutative).
__device__ __forceinline__ float warp_sum_butterfly(float v) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
  return v;
}

// ------------------------------------------------------------------ dequant
// src/loader/mxfp4.rs:57-79: out[r, 2i + {0,1}] = LUT[lo/hi] * 2^(s_r - 127).
__global__ void dequant_bytes_kernel(const uint8_t* __restrict__ blocks, uint64_t rows, uint64_t b,
                                     const uint8_t* __restrict__ scales, float* __restrict__ out) {
  const uint64_t total = rows * b;
  for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
    const uint64_t r = i / b;
    const float scale = ldexpf(1.0f, static_cast<int>(scales[r]) - 127);
    const uint8_t byte = blocks[i];
    out[2 * i] = kFp4Lut[byte & 0x0F] * scale;
    out[2 * i + 1] = kFp4Lut[byte >> 4] * scale;
  }
}

// MoE layout (src/quant/gpu.rs:124-134): blocks [rows][bpr], scales [rows][gpr].
__global__ void dequant_rows_kernel(const uint8_t* __restrict__ blocks, const uint8_t* __restrict__ scales,
                                    uint64_t rows, uint64_t cols, uint64_t bpr, uint64_t gpr, int ue8,
                                    float* __restrict__ out) {
  const uint64_t total = rows * cols;
  for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
    const uint64_t r = i / cols, c = i % cols;
    const uint8_t byte = blocks[r * bpr + (c >> 1)];
    const uint8_t nib = (c & 1) ? (byte >> 4) : (byte & 0x0F);
    const int e = static_cast<int>(scales[r * gpr + (c >> 5)]) - 127 - ue8;
    out[i] = kFp4Lut[nib] * ldexpf(1.0f, e);
  }
}

// ------------------------------------------------------------------ router
// Top-k (ties to the lower expert index) + softmax over the k selected values
// (src/moe/mod.rs:272-276) for one token, by one warp: lane l holds logits
// l, l + 32, ... (PL per lane, E <= 32*PL); each of the k rounds is a
// warp-wide argmax, then lane 0 forms the softmax over the k values.
template <int PL>
__device__ __forceinline__ void warp_topk_softmax(const float (&v)[PL], int E, int k, int lane, int32_t* idx_out,
                                                  float* w_out) {
  uint32_t taken = 0;
  float my_v = 0.0f;  // lane s < k keeps the s-th selection
  int my_i = 0;
  for (int s = 0; s < k; ++s) {
    float bv = 0.0f;
    int bi = -1;
#pragma unroll
    for (int i = 0; i < PL; ++i) {
      const int e = lane + 32 * i;
      if (e < E && !((taken >> i) & 1u) && (bi < 0 || v[i] > bv)) {
        bv = v[i];
        bi = e;
      }
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
      const float ov = __shfl_xor_sync(0xFFFFFFFFu, bv, o);
      const int oi = __shfl_xor_sync(0xFFFFFFFFu, bi, o);
      if (oi >= 0 && (bi < 0 || ov > bv || (ov == bv && oi < bi))) {
        bv = ov;
        bi = oi;
      }
    }
    if ((bi & 31) == lane) taken |= 1u << (bi >> 5);
    if (lane == s) {
      my_v = bv;
      my_i = bi;
    }
  }
  // softmax: exp(v_s - v_0), summed in increasing s
  const float v0 = __shfl_sync(0xFFFFFFFFu, my_v, 0);
  const float ex = lane < k ? expf(__fsub_rn(my_v, v0)) : 0.0f;
  float sum = 0.0f;
  for (int s = 0; s < k; ++s) sum = __fadd_rn(sum, __shfl_sync(0xFFFFFFFFu, ex, s));
  if (lane < k) {
    idx_out[lane] = my_i;
    w_out[lane] = __fdiv_rn(ex, sum);
  }
}

// One warp per token over a logits matrix [n][E].
template <int PL>
__global__ void topk_softmax_kernel(const float* __restrict__ logits, int n, int E, int k, int32_t* topk_idx,
                                    float* topk_w) {
  griddep_wait();
  const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (t >= n) return;
  const float* lg = logits + static_cast<uint64_t>(t) * E;
  float v[PL];
#pragma unroll
  for (int i = 0; i < PL; ++i) v[i] = lane + 32 * i < E ? lg[lane + 32 * i] : 0.0f;
  warp_topk_softmax<PL>(v, E, k, lane, topk_idx + static_cast<uint64_t>(t) * k, topk_w + static_cast<uint64_t>(t) * k);
}

// RmsNorm (src/moe/mod.rs:109) + gate Linear (:110): router logits, as two
// kernels -- rms_kernel (1 / rms per token) and router_logits_kernel.
constexpr int kRouterThreads = 256;
constexpr int kRouterWarps = kRouterThreads / 32;

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, int src_bytes) {
  const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(s), "l"(gmem), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// 1 / rms per token (src/moe/mod.rs:109), one warp per token: the lane chain
// of fused multiply-adds over c = lane, lane + 32, ... in increasing order,
// then a butterfly.  With 16-byte aligned rows the warp moves its row in
// segments of 512 bytes per load round (four 16-byte vectors per lane, the
// next segment's loads in flight while the current one is summed) through a
// shared-memory buffer from which each lane reads its own chain values.
constexpr int kRmsVec = 4;  // 16-byte vectors per lane per segment

// The normalized token row ((x * 1/rms) * gamma, times a power of two) as
// f16, for the decode dequant-GEMV to stage without recomputing it; d is a
// multiple of 32; xr and gamma are shared-memory copies.  Threads tid,
// tid + nthreads, ... each write two columns.
template <typename XT>
__device__ __forceinline__ void write_xh_row(const XT* xr, int d, float r, const float* gamma, float scale,
                                             __half* dst, int tid, int nthreads) {
  for (int c = 2 * tid; c < d; c += 2 * nthreads) {
    const float v0 = __fmul_rn(__fmul_rn(load_f32(xr, c), r), gamma[c]);
    const float v1 = __fmul_rn(__fmul_rn(load_f32(xr, c + 1), r), gamma[c + 1]);
    *reinterpret_cast<__half2*>(dst + c) = __floats2half2_rn(v0 * scale, v1 * scale);
  }
}
template <typename XT>
__global__ void __launch_bounds__(256) rms_kernel(const XT* __restrict__ x, int n, int d, float eps,
                                                  float* __restrict__ rscale, int aligned) {
  griddep_wait();
  constexpr int kEpv = 16 / static_cast<int>(sizeof(XT));  // elements per vector
  constexpr int kSeg = 32 * kRmsVec * kEpv;                  // elements per segment
  __shared__ __align__(16) XT buf[8][kSeg];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x * 8 + warp;
  if (t >= n) return;
  const XT* xr = x + static_cast<uint64_t>(t) * d;
  float acc = 0.0f;
  if (aligned) {
    const uint4* xv = reinterpret_cast<const uint4*>(xr);
    const int nvec = d / kEpv;
    uint4 cur[kRmsVec];
#pragma unroll
    for (int v = 0; v < kRmsVec; ++v) {
      const int vi = lane + 32 * v;
      cur[v] = vi < nvec ? __ldg(xv + vi) : make_uint4(0, 0, 0, 0);
    }
    for (int s0 = 0; s0 < d; s0 += kSeg) {
      __syncwarp();
#pragma unroll
      for (int v = 0; v < kRmsVec; ++v) reinterpret_cast<uint4*>(buf[warp])[lane + 32 * v] = cur[v];
      __syncwarp();
      const int nv0 = (s0 + kSeg) / kEpv;
#pragma unroll
      for (int v = 0; v < kRmsVec; ++v) {
        const int vi = nv0 + lane + 32 * v;
        cur[v] = vi < nvec ? __ldg(xv + vi) : make_uint4(0, 0, 0, 0);
      }
      const int len = min(kSeg, d - s0);
#pragma unroll 8
      for (int c = lane; c < len; c += 32) {
        const float f = load_f32(buf[warp], c);
        acc = __fmaf_rn(f, f, acc);
      }
    }
  } else {
    for (int c0 = lane; c0 < d; c0 += 32 * 32) {
      float v[32];
#pragma unroll
      for (int u = 0; u < 32; ++u) v[u] = c0 + 32 * u < d ? load_f32(xr, c0 + 32 * u) : 0.0f;
#pragma unroll
      for (int u = 0; u < 32; ++u)
        if (c0 + 32 * u < d) acc = __fmaf_rn(v[u], v[u], acc);
    }
  }
  const float ss = warp_sum_butterfly(acc);
  if (lane == 0) rscale[t] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, static_cast<float>(d)), eps)));
}

template <typename XT, int BT>
__host__ __device__ constexpr int router_x_bytes() {
  return ((BT * kRouterChunk * static_cast<int>(sizeof(XT)) + 15) / 16) * 16;
}
template <typename XT, int BT>
__host__ __device__ constexpr int router_stage_bytes() {
  return router_x_bytes<XT, BT>() + kRouterChunk * 4 + kRouterGroup * kRouterChunk * 4;
}
template <int BT>
__host__ __device__ constexpr int router_stages() {
  return BT <= 2 ? 8 : 4;  // small token tiles: deeper pipeline, one block per SM
}

// Gate logits for a block of BT = WT*TT tokens and the 32 experts of group
// blockIdx.y.  Per column chunk of kRouterChunk, a stage holds the raw token
// rows, the gamma slice and the packed gate weights (pack_router_gate); the
// stages stream through a cp.async pipeline.  One chunk ahead of the FMAs,
// the block normalizes the chunk's token values, (x * 1/rms) * gamma rounded
// exactly as the CPU restatement rounds them, into a float buffer laid out
// like the packed gate (column c = l + 32*j at (j/4)*128 + l*4 + j%4).  Each
// thread owns one lane chain (c = lane, lane + 32, ...) of a TT x TE register
// tile of (token, expert) accumulators and reads four chain values of a token
// or an expert as one float4.  Summation order is fixed -- 32 lane chains of
// fused multiply-adds over c in increasing order, then a butterfly -- so the
// logits are reproducible bit for bit whatever the tiling.
template <typename XT, int TT, int TE>
__global__ void __launch_bounds__(kRouterThreads)
    router_logits_kernel(const XT* __restrict__ x, int n, int d, int E, const float* __restrict__ gamma,
                         const float* __restrict__ gate_packed, const float* __restrict__ gate_b,
                         const float* __restrict__ rscale, float* __restrict__ logits_out, int x_aligned,
                         int k, int32_t* __restrict__ topk_idx, float* __restrict__ topk_w) {
  griddep_wait();
  constexpr int WE = kRouterGroup / TE;       // warps along experts
  constexpr int WT = kRouterWarps / WE;       // warps along tokens
  constexpr int BT = WT * TT;                 // tokens per block
  constexpr int C = kRouterChunk;
  constexpr int kXBytes = router_x_bytes<XT, BT>();
  constexpr int kStage = router_stage_bytes<XT, BT>();
  constexpr int kStages = router_stages<BT>();
  constexpr int kXPieces = C * static_cast<int>(sizeof(XT)) / 16;  // 16-byte pieces per token row
  static_assert(WE * TE == kRouterGroup && WT * WE == kRouterWarps, "router tile");
  static_assert(kStages >= 3, "normalization runs one chunk ahead");
  extern __shared__ __align__(16) uint8_t router_smem[];
  float* nbuf = reinterpret_cast<float*>(router_smem + kStages * kStage);  // [2][BT][C] normalized chunks
  __shared__ float rs_s[BT];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t0 = blockIdx.x * BT;
  const int e_base = blockIdx.y * kRouterGroup;
  const int nt = min(BT, n - t0);
  const int nch = (d + C - 1) / C;
  const float* gsrc = gate_packed + static_cast<uint64_t>(blockIdx.y) * nch * kRouterGroup * C;

  auto issue = [&](int ch) {
    if (ch < nch) {
      uint8_t* st = router_smem + (ch % kStages) * kStage;
      const int cb = ch * C;
      for (int pc = threadIdx.x; pc < BT * kXPieces; pc += kRouterThreads) {
        const int row = pc / kXPieces, col = (pc % kXPieces) * (16 / static_cast<int>(sizeof(XT)));
        XT* dst = reinterpret_cast<XT*>(st) + row * C + col;
        const int valid = row < nt ? min(max(d - (cb + col), 0), 16 / static_cast<int>(sizeof(XT))) : 0;
        const XT* src = x + static_cast<uint64_t>(t0 + (row < nt ? row : 0)) * d + (valid ? cb + col : 0);
        if (x_aligned) {
          cp_async16(dst, src, valid * static_cast<int>(sizeof(XT)));
        } else {
          for (int q = 0; q < 16 / static_cast<int>(sizeof(XT)); ++q) dst[q] = q < valid ? src[q] : XT(0.0f);
        }
      }
      float* gdst = reinterpret_cast<float*>(st + kXBytes);
      for (int pc = threadIdx.x; pc < C / 4; pc += kRouterThreads) {
        const int valid = min(max(d - (cb + 4 * pc), 0), 4);
        cp_async16(gdst + 4 * pc, gamma + (valid ? cb + 4 * pc : 0), valid * 4);
      }
      const float* wsrc = gsrc + static_cast<uint64_t>(ch) * kRouterGroup * C;
      float* wdst = gdst + C;
      for (int pc = threadIdx.x; pc < kRouterGroup * C / 4; pc += kRouterThreads) cp_async16(wdst + pc * 4, wsrc + pc * 4, 16);
    }
    cp_async_commit();  // an empty group past the last chunk keeps the wait count uniform
  };
  // chunk ch's raw rows and gamma (landed) -> nbuf[ch % 2]
  auto normalize = [&](int ch) {
    if (ch >= nch) return;
    const uint8_t* st = router_smem + (ch % kStages) * kStage;
    const XT* xs = reinterpret_cast<const XT*>(st);
    const float* gs = reinterpret_cast<const float*>(st + kXBytes);
    float* nb = nbuf + (ch & 1) * BT * C;
    for (int pc = threadIdx.x; pc < BT * (C / 4); pc += kRouterThreads) {
      const int row = pc / (C / 4), p = pc % (C / 4), j4 = p >> 5, l = p & 31;
      const float r = rs_s[row];
      float4 v;
      float* vp = reinterpret_cast<float*>(&v);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int c = l + 32 * (4 * j4 + q);
        vp[q] = __fmul_rn(__fmul_rn(load_f32(xs, row * C + c), r), gs[c]);
      }
      *reinterpret_cast<float4*>(nb + row * C + j4 * 128 + l * 4) = v;
    }
  };

  for (int s = 0; s < kStages - 1; ++s) issue(s);
  if (threadIdx.x < BT) rs_s[threadIdx.x] = threadIdx.x < nt ? __ldg(rscale + t0 + threadIdx.x) : 0.0f;
  cp_async_wait<kStages - 2>();  // chunk 0 landed
  __syncthreads();
  normalize(0);

  const int tw = warp / WE, ew = warp % WE;  // this warp's token group and expert group
  float acc[TT][TE];
#pragma unroll
  for (int t = 0; t < TT; ++t)
#pragma unroll
    for (int e = 0; e < TE; ++e) acc[t][e] = 0.0f;

  for (int ch = 0; ch < nch; ++ch) {
    cp_async_wait<kStages - 3>();  // chunk ch + 1 landed
    __syncthreads();  // nbuf[ch % 2] complete; stage (ch - 1) and nbuf[(ch + 1) % 2] fully consumed
    issue(ch + kStages - 1);
    normalize(ch + 1);
    const float* ws = reinterpret_cast<const float*>(router_smem + (ch % kStages) * kStage + kXBytes) + C;
    const float* nb = nbuf + (ch & 1) * BT * C;
    const int cw = min(C, d - ch * C);
    if (cw == C) {
#pragma unroll
      for (int j4 = 0; j4 < C / 128; ++j4) {
        float4 wv[TE];
#pragma unroll
        for (int e = 0; e < TE; ++e)
          wv[e] = *reinterpret_cast<const float4*>(ws + (ew * TE + e) * C + j4 * 128 + lane * 4);
#pragma unroll
        for (int t = 0; t < TT; ++t) {
          const float4 xv = *reinterpret_cast<const float4*>(nb + (tw * TT + t) * C + j4 * 128 + lane * 4);
#pragma unroll
          for (int e = 0; e < TE; ++e) {
            acc[t][e] = __fmaf_rn(xv.x, wv[e].x, acc[t][e]);
            acc[t][e] = __fmaf_rn(xv.y, wv[e].y, acc[t][e]);
            acc[t][e] = __fmaf_rn(xv.z, wv[e].z, acc[t][e]);
            acc[t][e] = __fmaf_rn(xv.w, wv[e].w, acc[t][e]);
          }
        }
      }
    } else {
      // ragged last chunk: only the lane's columns below d join its chain
      const int jmax = (cw - lane + 31) / 32;
      for (int j = 0; j < jmax; ++j) {
        const int pos = (j >> 2) * 128 + lane * 4 + (j & 3);
#pragma unroll
        for (int t = 0; t < TT; ++t) {
          const float xv = nb[(tw * TT + t) * C + pos];
#pragma unroll
          for (int e = 0; e < TE; ++e) acc[t][e] = __fmaf_rn(xv, ws[(ew * TE + e) * C + pos], acc[t][e]);
        }
      }
    }
  }
  cp_async_wait<0>();
  // all experts in this block (E <= 32): the block also does top-k + softmax
  const bool fused = topk_idx != nullptr;
  float* lg_s = nbuf;  // [BT][33]; nbuf is free once every warp passed the barrier below
  if (fused) __syncthreads();
#pragma unroll
  for (int t = 0; t < TT; ++t) {
#pragma unroll
    for (int e = 0; e < TE; ++e) {
      const float s = warp_sum_butterfly(acc[t][e]);
      const int tok = tw * TT + t, ex = e_base + ew * TE + e;
      if (lane == 0 && tok < nt && ex < E) {
        const float l = __fadd_rn(s, gate_b[ex]);
        logits_out[static_cast<uint64_t>(t0 + tok) * E + ex] = l;
        if (fused) lg_s[tok * 33 + ex] = l;
      }
    }
  }
  if (!fused) return;
  __syncthreads();
  for (int tok = warp; tok < nt; tok += kRouterWarps) {
    const float v[1] = {lane < E ? lg_s[tok * 33 + lane] : 0.0f};
    warp_topk_softmax<1>(v, E, k, lane, topk_idx + static_cast<uint64_t>(t0 + tok) * k,
                         topk_w + static_cast<uint64_t>(t0 + tok) * k);
  }
}

// Small batches (decode): RmsNorm, gate logits and top-k + softmax of one
// token per block in one launch (E <= 32, one packed gate group, one warp
// per expert).  The block stages the token row in shared memory with
// 16-byte loads; every warp computes 1/rms from it with the lane chain c =
// lane, lane + 32, ... and a butterfly, as rms_kernel does; the block writes
// the normalized token, (x * 1/rms) * gamma, in the packed gate's order, and
// warp e accumulates expert e: per 128-column chunk one float4 of the token
// and one of the expert's packed row hold a lane's four chain values in
// increasing column order.  The fused multiply-adds therefore run in the
// order of router_logits_kernel and the logits are bit-identical to it.
// Everything a warp reads from global memory is issued in a few rounds of
// independent loads: the step is latency-bound at these sizes.
constexpr int kRouterSmallMaxN = 512;
constexpr int kRouterSmallMaxD = 8192;
__device__ void permute_block(const int32_t* __restrict__ topk_idx, int P, int E, int pad, int N, int32_t* offsets,
                              int32_t* perm_c, int32_t* inv_c, int32_t* poff, int32_t* counts, int32_t* ntile_prefix,
                              int32_t* perm_p, int32_t* inv_p, int32_t* cnt);
template <typename XT>
__global__ void __launch_bounds__(1024)
    router_small_kernel(const XT* __restrict__ x, int n, int d, int E, int k, const float* __restrict__ gamma,
                        const float* __restrict__ gate_packed, const float* __restrict__ gate_b, float eps,
                        float* __restrict__ logits_out, int32_t* __restrict__ topk_idx, float* __restrict__ topk_w,
                        float* __restrict__ rscale, int x_aligned, PermFold pf) {
  const int C = kRouterChunk;
  const int nch = (d + C - 1) / C;
  extern __shared__ __align__(16) float router_small_smem[];
  float* g_s = router_small_smem + nch * C + (d * static_cast<int>(sizeof(XT)) + 15) / 16 * 4;  // [d] gamma
  // gamma is a constant: copied in while the previous kernel finishes (d % 32 == 0)
  for (int i = threadIdx.x; i < d / 4; i += blockDim.x) cp_async16(g_s + 4 * i, gamma + 4 * i, 16);
  cp_async_commit();
  {
    // the gate rows do not depend on earlier kernels: pull this warp's
    // expert row into L2 while the previous kernel finishes
    const int e = threadIdx.x >> 5, l = threadIdx.x & 31;
    if (e < E)
      for (int ch = l; ch < nch; ch += 32) {
        const float* p = gate_packed + (static_cast<uint64_t>(ch) * kRouterGroup + e) * C;
#pragma unroll
        for (int q = 0; q < 4; ++q) asm volatile("prefetch.global.L2 [%0];" ::"l"(p + 32 * q));
      }
  }
  griddep_wait();
  float* xn_s = router_small_smem;                                           // [nch][128] packed order
  XT* xr_s = reinterpret_cast<XT*>(router_small_smem + nch * C);             // [d] raw row
  __shared__ float lg_s[32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x;
  const XT* xr = x + static_cast<uint64_t>(t) * d;
  constexpr int kEpv = 16 / static_cast<int>(sizeof(XT));
  if (x_aligned) {
    for (int i = threadIdx.x; i < d / kEpv; i += blockDim.x)
      reinterpret_cast<uint4*>(xr_s)[i] = __ldg(reinterpret_cast<const uint4*>(xr) + i);
  } else {
    for (int i = threadIdx.x; i < d; i += blockDim.x) xr_s[i] = xr[i];
  }
  cp_async_wait<0>();
  __syncthreads();
  float ss = 0.0f;
#pragma unroll 8
  for (int c = lane; c < d; c += 32) {
    const float f = load_f32(xr_s, c);
    ss = __fmaf_rn(f, f, ss);
  }
  ss = warp_sum_butterfly(ss);
  const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, static_cast<float>(d)), eps)));
#pragma unroll 4
  for (int i = threadIdx.x; i < nch * C; i += blockDim.x) {
    const int ch = i / C, cc = i % C, l = cc % 32, j = cc / 32;
    const int c = ch * C + cc;
    xn_s[ch * C + l * 4 + j] = c < d ? __fmul_rn(__fmul_rn(load_f32(xr_s, c), r), g_s[c]) : 0.0f;
  }
  __syncthreads();
  const int e = warp;
  if (e < E) {
    float acc = 0.0f;
    const int full = d / C;  // chunks with all 128 columns
    const float* wrow = gate_packed + static_cast<uint64_t>(e) * C + lane * 4;
#pragma unroll 8
    for (int ch = 0; ch < full; ++ch) {
      const float4 xv = *reinterpret_cast<const float4*>(xn_s + ch * C + lane * 4);
      const float4 wv = __ldg(reinterpret_cast<const float4*>(wrow + static_cast<uint64_t>(ch) * kRouterGroup * C));
      acc = __fmaf_rn(xv.x, wv.x, acc);
      acc = __fmaf_rn(xv.y, wv.y, acc);
      acc = __fmaf_rn(xv.z, wv.z, acc);
      acc = __fmaf_rn(xv.w, wv.w, acc);
    }
    if (full < nch) {
      // ragged last chunk: only the lane's columns below d join its chain
      const float* wl = wrow + static_cast<uint64_t>(full) * kRouterGroup * C;
      for (int j = 0; j < 4; ++j) {
        if (full * C + lane + 32 * j >= d) break;
        acc = __fmaf_rn(xn_s[full * C + lane * 4 + j], __ldg(wl + j), acc);
      }
    }
    const float sum = warp_sum_butterfly(acc);
    if (lane == 0) {
      const float l = __fadd_rn(sum, __ldg(gate_b + e));
      logits_out[static_cast<uint64_t>(t) * E + e] = l;
      lg_s[e] = l;
    }
  }
  __syncthreads();
  if (warp == 0) {
    if (lane == 0) rscale[t] = r;
    const float v[1] = {lane < E ? lg_s[lane] : 0.0f};
    warp_topk_softmax<1>(v, E, k, lane, topk_idx + static_cast<uint64_t>(t) * k, topk_w + static_cast<uint64_t>(t) * k);
  }
  if (pf.ticket == nullptr) return;
  // Folded permutation: the block that takes the last ticket sorts all pairs
  // (every block's top-k row is visible by then: its writers fence before the
  // block's ticket, the last block fences after it).
  __shared__ int last;
  if (warp == 0) __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) last = atomicAdd(pf.ticket, 1) == static_cast<int>(gridDim.x) - 1 ? 1 : 0;
  __syncthreads();
  if (!last) return;
  __threadfence();
  permute_block(topk_idx, n * k, E, pf.pad, pf.N, pf.offsets, pf.perm_c, pf.inv_c, pf.poff, pf.counts,
                pf.ntile_prefix, pf.perm_p, pf.inv_p, reinterpret_cast<int32_t*>(router_small_smem));
  if (threadIdx.x == 0) *pf.ticket = 0;
}

// Tiny batches (decode, at most kRouterTinyMaxN tokens, d <= 4096): the
// gate GEMV is spread over blocks of kRouterTinyExperts experts per token
// instead of one block per token, so the gate rows stream through many SMs.
// Each warp holds its expert's packed gate row in registers, loaded before
// griddepcontrol.wait (the weights depend on no earlier kernel), and runs
// the lane chains of router_small_kernel in the same order (bit-identical
// logits).  The last block of a token to finish (a per-token counter, reset
// by that block) does the top-k + softmax.  Block (t, 0) also writes 1/rms
// and the normalized f16 row, and block (0, 0) zeroes the layer's status
// words for the kernels after it (after its wait).
constexpr int kRouterTinyMaxN = 8;
constexpr int kRouterTinyExperts = 8;
template <typename XT, int NCH>
__global__ void __launch_bounds__(32 * kRouterTinyExperts)
    router_tiny_kernel(const XT* __restrict__ x, int n, int d, int E, int k, const float* __restrict__ gamma,
                       const float* __restrict__ gate_packed, const float* __restrict__ gate_b, float eps,
                       float* __restrict__ logits_out, int32_t* __restrict__ topk_idx, float* __restrict__ topk_w,
                       float* __restrict__ rscale, int x_aligned, __half* __restrict__ xh, float xh_scale,
                       int* __restrict__ tok_ctr, int* __restrict__ status, int status_words) {
  const int C = kRouterChunk;
  const int nch = (d + C - 1) / C, full = d / C;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x, e = blockIdx.y * kRouterTinyExperts + warp;
  extern __shared__ __align__(16) float router_tiny_smem[];
  float* g_s = router_tiny_smem;                           // [d] gamma
  XT* x_s = reinterpret_cast<XT*>(router_tiny_smem + d);   // [d] raw token row
  __shared__ int last;
  // the gate row and gamma are constants: fetched while the previous kernel finishes
  float4 wv[NCH];
  if (e < E) {
    const float* wrow = gate_packed + (static_cast<uint64_t>(e / kRouterGroup) * nch) * kRouterGroup * C +
                        (e % kRouterGroup) * C + lane * 4;
#pragma unroll
    for (int ch = 0; ch < NCH; ++ch)
      if (ch < nch) wv[ch] = __ldg(reinterpret_cast<const float4*>(wrow + static_cast<uint64_t>(ch) * kRouterGroup * C));
  }
  for (int i = threadIdx.x; i < d / 4; i += blockDim.x) cp_async16(g_s + 4 * i, gamma + 4 * i, 16);  // d % 32 == 0
  cp_async_commit();
  // from here on the previous kernel in the stream has completed (it may be
  // the last forward's expert kernel, which still uses the status words)
  griddep_wait();
  if (status != nullptr && t == 0 && blockIdx.y == 0)
    for (int i = threadIdx.x; i < status_words; i += blockDim.x) status[i] = 0;
  const XT* xr = x + static_cast<uint64_t>(t) * d;
  constexpr int kEpv = 16 / static_cast<int>(sizeof(XT));
  if (x_aligned) {
    for (int i = threadIdx.x; i < d / kEpv; i += blockDim.x) cp_async16(x_s + kEpv * i, xr + kEpv * i, 16);
    cp_async_commit();
  } else {
    for (int i = threadIdx.x; i < d; i += blockDim.x) x_s[i] = xr[i];
  }
  cp_async_wait<0>();
  __syncthreads();
  float ss = 0.0f;
#pragma unroll 8
  for (int c = lane; c < d; c += 32) {
    const float f = load_f32(x_s, c);
    ss = __fmaf_rn(f, f, ss);
  }
  ss = warp_sum_butterfly(ss);
  const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, static_cast<float>(d)), eps)));
  if (e < E) {
    float acc = 0.0f;
#pragma unroll
    for (int ch = 0; ch < NCH; ++ch) {
      if (ch < full) {
        const float* wf = reinterpret_cast<const float*>(&wv[ch]);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int c = ch * C + lane + 32 * q;
          acc = __fmaf_rn(__fmul_rn(__fmul_rn(load_f32(x_s, c), r), g_s[c]), wf[q], acc);
        }
      } else if (ch < nch) {
        // ragged last chunk: only the lane's columns below d join its chain
        const float* wf = reinterpret_cast<const float*>(&wv[ch]);
        for (int q = 0; q < 4; ++q) {
          const int c = ch * C + lane + 32 * q;
          if (c >= d) break;
          acc = __fmaf_rn(__fmul_rn(__fmul_rn(load_f32(x_s, c), r), g_s[c]), wf[q], acc);
        }
      }
    }
    const float sum = warp_sum_butterfly(acc);
    if (lane == 0) logits_out[static_cast<uint64_t>(t) * E + e] = __fadd_rn(sum, __ldg(gate_b + e));
  }
  if (blockIdx.y == 0) {
    if (threadIdx.x == 0) rscale[t] = r;
    if (xh) write_xh_row(x_s, d, r, g_s, xh_scale, xh + static_cast<uint64_t>(t) * d, threadIdx.x, blockDim.x);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    last = atomicAdd(tok_ctr + t, 1) == static_cast<int>(gridDim.y) - 1;
  }
  __syncthreads();
  if (!last || warp != 0) return;
  __threadfence();
  const float* lg = logits_out + static_cast<uint64_t>(t) * E;
  int32_t* io = topk_idx + static_cast<uint64_t>(t) * k;
  float* wo = topk_w + static_cast<uint64_t>(t) * k;
  auto run = [&](auto pl) {
    constexpr int PL = decltype(pl)::value;
    float v[PL];
#pragma unroll
    for (int i = 0; i < PL; ++i) v[i] = lane + 32 * i < E ? __ldcg(lg + lane + 32 * i) : 0.0f;
    warp_topk_softmax<PL>(v, E, k, lane, io, wo);
  };
  if (E <= 32) run(std::integral_constant<int, 1>());
  else if (E <= 64) run(std::integral_constant<int, 2>());
  else if (E <= 128) run(std::integral_constant<int, 4>());
  else if (E <= 256) run(std::integral_constant<int, 8>());
  else if (E <= 512) run(std::integral_constant<int, 16>());
  else run(std::integral_constant<int, 32>());
  if (lane == 0) tok_ctr[t] = 0;  // ready for the next forward
}

// ------------------------------------------------------------------ permute
// Canonical permutation (replaces src/moe/mod.rs:279-288): pairs p = t*k+s are
// stably sorted by expert id.  One block of 1024 threads; warp w owns a
// contiguous segment of pairs, so the order within an expert is (t, s).
// Writes the unpadded canonical maps (offsets / perm_c / inv_c, optional)
// and the padded maps used by the GEMMs, where every expert segment starts
// at a multiple of `pad` rows.
constexpr int kPermThreads = 1024;
constexpr int kPermBatch = 16;  // rows of 32 pairs whose expert ids are loaded together

// Lanes of the warp holding the same expert id (ex = -1 for none), from one
// ballot per bit of ex + 1 -- cheaper than a match instruction.
__device__ __forceinline__ unsigned same_expert_lanes(int ex, int nbits) {
  const unsigned v = static_cast<unsigned>(ex + 1);
  unsigned m = 0xFFFFFFFFu;
  for (int i = 0; i < nbits; ++i) {
    const unsigned bit = (v >> i) & 1u;
    const unsigned bal = __ballot_sync(0xFFFFFFFFu, bit);
    m &= bit ? bal : ~bal;
  }
  return m;
}

// Expert ids of pairs [base0, base0 + 32*kPermBatch) (-1 past p_end) into a
// warp's staging buffer; all loads in flight together.
__device__ __forceinline__ void stage_expert_ids(const int32_t* __restrict__ topk_idx, int E, int base0, int p_end,
                                                 int lane,
                                                 int32_t* stg) {
  int v[kPermBatch];
#pragma unroll
  for (int b = 0; b < kPermBatch; ++b) {
    const int p = base0 + 32 * b + lane;
    // (coherent loads: the router that folds the permutation in wrote the ids in the same launch)
    const int id = p < p_end ? __ldcg(topk_idx + p) : -1;
    v[b] = id >= 0 && id < E ? id : -1;  // ids outside [0, E) are absent from the maps
  }
  __syncwarp();  // the previous batch is consumed
#pragma unroll
  for (int b = 0; b < kPermBatch; ++b) stg[32 * b + lane] = v[b];
  __syncwarp();
}

// The counting sort of one block of kPermThreads threads; cnt: shared
// memory of permute_smem_ints(E) ints.
__device__ void permute_block(const int32_t* __restrict__ topk_idx, int P, int E, int pad, int N, int32_t* offsets,
                              int32_t* perm_c, int32_t* inv_c, int32_t* poff, int32_t* counts, int32_t* ntile_prefix,
                              int32_t* perm_p, int32_t* inv_p, int32_t* cnt) {
  // cnt: [32 warps][E], canonical and padded starts [E] each, staging
  int32_t* cstart = cnt + 32 * E;
  int32_t* pstart = cstart + E;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int32_t* stg = pstart + E + warp * 32 * kPermBatch;  // this warp's staged expert ids
  const int seg = (P + 31) / 32;
  const int p_begin = warp * seg, p_end = min(P, p_begin + seg);
  const int nbits = 32 - __clz(E);  // bits of the largest ex + 1
  for (int i = threadIdx.x; i < 32 * E; i += blockDim.x) cnt[i] = 0;
  __syncthreads();
  // pass 1: per-warp expert histogram of the warp's contiguous segment.  The
  // expert ids of kPermBatch rows of 32 pairs are loaded together into the
  // warp's staging buffer, then consumed by a rolled loop (a one-block kernel
  // runs each instruction once, so the loop body is kept small).
  for (int base0 = p_begin; base0 < p_end; base0 += 32 * kPermBatch) {
    stage_expert_ids(topk_idx, E, base0, p_end, lane, stg);
    for (int b = 0; b < kPermBatch && base0 + 32 * b < p_end; ++b) {
      const int ex = stg[32 * b + lane];
      const unsigned grp = same_expert_lanes(ex, nbits);
      if (ex >= 0 && lane == __ffs(grp) - 1) cnt[warp * E + ex] += __popc(grp);
      __syncwarp();
    }
  }
  __syncthreads();
  if (E <= 32) {
    // warp e scans expert e's per-warp counts across its lanes; then warp 0
    // scans the expert totals (exclusive scans by shuffles, no serial loops)
    if (warp < E) {
      const int c = cnt[lane * E + warp];
      int inc = c;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int u = __shfl_up_sync(0xFFFFFFFFu, inc, o);
        if (lane >= o) inc += u;
      }
      cnt[lane * E + warp] = inc - c;
      if (lane == 31) cstart[warp] = inc;  // total
    }
    __syncthreads();
    if (warp == 0) {
      const int tot = lane < E ? cstart[lane] : 0;
      int a = tot, b2 = (tot + pad - 1) / pad * pad, c = (tot + N - 1) / N;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int ua = __shfl_up_sync(0xFFFFFFFFu, a, o);
        const int ub = __shfl_up_sync(0xFFFFFFFFu, b2, o);
        const int uc = __shfl_up_sync(0xFFFFFFFFu, c, o);
        if (lane >= o) {
          a += ua;
          b2 += ub;
          c += uc;
        }
      }
      const int run = a - tot, prun = b2 - (tot + pad - 1) / pad * pad, trun = c - (tot + N - 1) / N;
      if (lane < E) {
        cstart[lane] = run;
        pstart[lane] = prun;
        if (offsets) offsets[lane] = run;
        poff[lane] = prun;
        counts[lane] = tot;
        if (ntile_prefix) ntile_prefix[lane] = trun;
      }
      if (lane == 31) {
        if (offsets) offsets[E] = a;
        poff[E] = b2;
        if (ntile_prefix) ntile_prefix[E] = c;
      }
    }
  } else {
    // per expert: totals, and each warp's base within the expert
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
      int run = 0;
      for (int w = 0; w < 32; ++w) {
        const int c = cnt[w * E + e];
        cnt[w * E + e] = run;
        run += c;
      }
      cstart[e] = run;  // total, turned into the start below
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      int run = 0, prun = 0, trun = 0;
      for (int e = 0; e < E; ++e) {
        const int tot = cstart[e];
        cstart[e] = run;
        pstart[e] = prun;
        if (offsets) offsets[e] = run;
        poff[e] = prun;
        counts[e] = tot;
        if (ntile_prefix) ntile_prefix[e] = trun;
        run += tot;
        prun += (tot + pad - 1) / pad * pad;
        trun += (tot + N - 1) / N;
      }
      if (offsets) offsets[E] = run;
      poff[E] = prun;
      if (ntile_prefix) ntile_prefix[E] = trun;
    }
  }
  __syncthreads();
  // pass 2: stable ranks within each expert, (token, slot) order
  for (int base0 = p_begin; base0 < p_end; base0 += 32 * kPermBatch) {
    stage_expert_ids(topk_idx, E, base0, p_end, lane, stg);
    for (int b = 0; b < kPermBatch && base0 + 32 * b < p_end; ++b) {
      const int p = base0 + 32 * b + lane;
      const int ex = stg[32 * b + lane];
      const unsigned grp = same_expert_lanes(ex, nbits);
      if (ex < 0 && p < p_end) {  // an id outside [0, E): no position
        inv_p[p] = -1;
        if (inv_c) inv_c[p] = -1;
      }
      if (ex >= 0) {
        const int rank = cnt[warp * E + ex] + __popc(grp & ((1u << lane) - 1u));
        const int pos_p = pstart[ex] + rank;
        perm_p[pos_p] = p;
        inv_p[p] = pos_p;
        if (perm_c) {
          perm_c[cstart[ex] + rank] = p;
          inv_c[p] = cstart[ex] + rank;
        }
      }
      __syncwarp();
      if (ex >= 0 && lane == __ffs(grp) - 1) cnt[warp * E + ex] += __popc(grp);
      __syncwarp();
    }
  }
}

__global__ void __launch_bounds__(kPermThreads)
    permute_kernel(const int32_t* __restrict__ topk_idx, int P, int E, int pad, int N, int32_t* offsets,
                   int32_t* perm_c, int32_t* inv_c, int32_t* poff, int32_t* counts, int32_t* ntile_prefix,
                   int32_t* perm_p, int32_t* inv_p) {
  griddep_wait();
  extern __shared__ int32_t perm_smem[];
  permute_block(topk_idx, P, E, pad, N, offsets, perm_c, inv_c, poff, counts, ntile_prefix, perm_p, inv_p, perm_smem);
}

// Multi-block form of the same permutation for large pair counts: chunks of
// kPermChunk pairs, one block each.  perm_hist_kernel counts each chunk's
// experts; the last block to finish (atomic ticket after a fence -- no block
// waits on another) turns the chunk counts into per-expert exclusive bases
// and scans the expert totals into the offsets.  perm_scatter_kernel then
// ranks each chunk's pairs stably: chunk base + earlier warps of the chunk +
// earlier lanes of the warp.  Scratch (int32): [0] ticket, [32, 32+E) canonical
// starts, [32+E, 32+2E) padded starts, then counts [chunks][E].
constexpr int kPermChunk = 512;
constexpr int kPermChunkThreads = 256;  // 8 warps x 2 rows of 32 pairs

// In-place exclusive scan of a[0, len) in shared memory by the whole block
// (len <= 4 * blockDim.x); returns the total.  Every thread must call it.
__device__ int block_exclusive_scan(int* a, int len, int* warp_tot) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  const int i0 = 4 * threadIdx.x;
  int v[4], s = 0;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    v[j] = i0 + j < len ? a[i0 + j] : 0;
    s += v[j];
  }
  int inc = s;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int u = __shfl_up_sync(0xFFFFFFFFu, inc, o);
    if (lane >= o) inc += u;
  }
  if (lane == 31) warp_tot[warp] = inc;
  __syncthreads();
  if (threadIdx.x == 0) {
    int run = 0;
    for (int w = 0; w < nw; ++w) {
      const int t = warp_tot[w];
      warp_tot[w] = run;
      run += t;
    }
    warp_tot[nw] = run;
  }
  __syncthreads();
  int run = warp_tot[warp] + inc - s;
#pragma unroll
  for (int j = 0; j < 4; ++j)
    if (i0 + j < len) {
      a[i0 + j] = run;
      run += v[j];
    }
  const int total = warp_tot[nw];
  __syncthreads();
  return total;
}

__global__ void __launch_bounds__(kPermChunkThreads)
    perm_hist_kernel(const int32_t* __restrict__ topk_idx, int P, int E, int pad, int N, int32_t* scratch,
                     int32_t* offsets, int32_t* poff, int32_t* counts, int32_t* ntile_prefix) {
  griddep_wait();
  extern __shared__ int32_t sh[];  // [E] counts, then 3 x [E] scan arrays
  __shared__ int warp_tot[kPermChunkThreads / 32 + 1];
  __shared__ bool last;
  const int nch = (P + kPermChunk - 1) / kPermChunk;
  int32_t* hist = scratch + 32 + 2 * E;
  for (int e = threadIdx.x; e < E; e += blockDim.x) sh[e] = 0;
  __syncthreads();
  const int p0 = blockIdx.x * kPermChunk;
  for (int p = p0 + threadIdx.x; p < min(P, p0 + kPermChunk); p += blockDim.x) {
    const int id = __ldg(topk_idx + p);
    if (id >= 0 && id < E) atomicAdd(&sh[id], 1);  // ids outside [0, E) are absent from the maps
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) hist[static_cast<uint64_t>(blockIdx.x) * E + e] = sh[e];
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) last = atomicAdd(scratch, 1) == nch - 1;
  __syncthreads();
  if (!last) return;
  __threadfence();
  // per expert: exclusive bases over chunks, and the totals
  int* tot = sh;
  int* pc = sh + E;   // padded sizes -> padded starts
  int* tc = sh + 2 * E;  // tiles -> tile prefix
  int* cs = sh + 3 * E;  // totals -> canonical starts
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int base = 0;
    for (int c = 0; c < nch; ++c) {
      int32_t* h = hist + static_cast<uint64_t>(c) * E + e;
      const int v = __ldcg(h);
      *h = base;
      base += v;
    }
    tot[e] = base;
    cs[e] = base;
    pc[e] = (base + pad - 1) / pad * pad;
    tc[e] = (base + N - 1) / N;
  }
  __syncthreads();
  const int run = block_exclusive_scan(cs, E, warp_tot);
  const int prun = block_exclusive_scan(pc, E, warp_tot);
  const int trun = block_exclusive_scan(tc, E, warp_tot);
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    if (offsets) offsets[e] = cs[e];
    poff[e] = pc[e];
    counts[e] = tot[e];
    if (ntile_prefix) ntile_prefix[e] = tc[e];
    scratch[32 + e] = cs[e];
    scratch[32 + E + e] = pc[e];
  }
  if (threadIdx.x == 0) {
    if (offsets) offsets[E] = run;
    poff[E] = prun;
    if (ntile_prefix) ntile_prefix[E] = trun;
    scratch[0] = 0;  // ticket for the next launch
  }
}

__global__ void __launch_bounds__(kPermChunkThreads)
    perm_scatter_kernel(const int32_t* __restrict__ topk_idx, int P, int E, const int32_t* __restrict__ scratch,
                        int32_t* perm_c, int32_t* inv_c, int32_t* perm_p, int32_t* inv_p) {
  griddep_wait();
  constexpr int kWarps = kPermChunkThreads / 32;
  constexpr int kRows = kPermChunk / kPermChunkThreads;
  extern __shared__ int32_t wcnt[];  // [kWarps][E]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nbits = 32 - __clz(E);
  const int32_t* cstart = scratch + 32;
  const int32_t* pstart = scratch + 32 + E;
  const int32_t* hist = scratch + 32 + 2 * E + static_cast<uint64_t>(blockIdx.x) * E;
  for (int i = threadIdx.x; i < kWarps * E; i += blockDim.x) wcnt[i] = 0;
  const int pw = blockIdx.x * kPermChunk + warp * 32 * kRows;  // this warp's first pair
  int exv[kRows];
  unsigned grp[kRows];
#pragma unroll
  for (int r = 0; r < kRows; ++r) {
    const int p = pw + 32 * r + lane;
    const int id = p < P ? __ldg(topk_idx + p) : -1;
    exv[r] = id >= 0 && id < E ? id : -1;
  }
  __syncthreads();
#pragma unroll
  for (int r = 0; r < kRows; ++r) {
    grp[r] = same_expert_lanes(exv[r], nbits);
    if (exv[r] >= 0 && lane == __ffs(grp[r]) - 1) wcnt[warp * E + exv[r]] += __popc(grp[r]);
    __syncwarp();
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int base = hist[e];
    for (int w = 0; w < kWarps; ++w) {
      const int c = wcnt[w * E + e];
      wcnt[w * E + e] = base;
      base += c;
    }
  }
  __syncthreads();
#pragma unroll
  for (int r = 0; r < kRows; ++r) {
    const int ex = exv[r];
    if (ex < 0 && pw + 32 * r + lane < P) {  // an id outside [0, E): no position
      inv_p[pw + 32 * r + lane] = -1;
      if (inv_c) inv_c[pw + 32 * r + lane] = -1;
    }
    if (ex >= 0) {
      const int p = pw + 32 * r + lane;
      const int rank = wcnt[warp * E + ex] + __popc(grp[r] & ((1u << lane) - 1u));
      const int pos_p = pstart[ex] + rank;
      perm_p[pos_p] = p;
      inv_p[p] = pos_p;
      if (perm_c) {
        perm_c[cstart[ex] + rank] = p;
        inv_c[p] = cstart[ex] + rank;
      }
    }
    __syncwarp();
    if (ex >= 0 && lane == __ffs(grp[r]) - 1) wcnt[warp * E + ex] += __popc(grp[r]);
    __syncwarp();
  }
}

// Expert-parallel dispatch of quantized pairs (quantize_pairs_kernel<true>):
// the codes, scale words and per-row metadata of a pair go to its owner
// rank g's buffers (peer pointers) at row src_base[e] + (canonical position -
// offsets[e]), the pair's row in g's expert-sorted, padded layout.
struct EpDispatch {
  const int32_t* src_base;  // [E] this rank's first row per expert at the owner
  const int32_t* offsets;   // [E + 1] canonical offsets of this rank's pairs
  const int32_t* topk_idx;
  const float* topk_w;
  const float* rscale;
  int epr, rank;
  uint32_t dst_rows;        // rows of every owner's layout
  uint32_t sf_row_bytes;    // scale bytes per row and term in sf_rows (a multiple of 16)
  uint8_t* const* xq;       // [world] code buffers
  uint8_t* const* sf_rows;  // [world] row-major scale bytes [rows][terms][sf_row_bytes]
  uint4* const* meta;       // [world] per-row {bits of 1/rms, bits of route weight, return slot, 0}
  int* err;
};

// ------------------------------------------------------------------ quantize
// Gathers each routed pair's token row into its padded expert-sorted position
// and writes it as `terms` block-scaled E4M3 terms (two reproduce bf16 input
// with unit gain exactly; three are used for f32 input or a non-unit gain).
// Each token block is quantized once and written to the positions of all k
// pairs of the token.
// Warp per (token, group of sixteen 32-column blocks); the two lanes of a
// lane pair share one block, sixteen columns (32 bytes of bf16) each, so a
// warp's loads and 16-byte code stores cover 1 KB / 512 B contiguous.  The
// block's per-term scale comes from a max over the lane pair; the arithmetic
// per element is quantize_block32's.  Lanes of blocks past d / 32 store no
// codes and add zero scale bytes (the K padding).
constexpr int kQBlocksPerWarp = 16;
template <bool kDispatch>
__global__ void __launch_bounds__(256)
    quantize_pairs_kernel(const void* __restrict__ x, int x_dtype, int n, int d, int k,
                          const float* __restrict__ gamma, int gamma_is_one, const int32_t* __restrict__ inv_p,
                          int terms, uint8_t* codes, uint64_t term_stride, int kp, uint8_t* sf,
                          uint64_t sf_term_stride, int kchunks, int sf_rows, int stacked, const EpDispatch ep) {
  griddep_wait();
  const int nb = d / 32;
  const int ngrp = (nb + kQBlocksPerWarp - 1) / kQBlocksPerWarp;
  const uint64_t items = static_cast<uint64_t>(n) * ngrp;
  const int lane = threadIdx.x & 31;
  const int hf = lane & 1, lb = lane >> 1;  // half of the block, block within the group
  const uint64_t wstride = static_cast<uint64_t>(gridDim.x) * (blockDim.x >> 5);
  for (uint64_t it = static_cast<uint64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); it < items;
       it += wstride) {
    const int t = static_cast<int>(it / ngrp);
    const int grp = static_cast<int>(it - static_cast<uint64_t>(t) * ngrp);
    const int b = grp * kQBlocksPerWarp + lb;
    const bool active = b < nb;
    const int c0 = b * 32 + hf * 16;
    float v[16];
    if (!active) {
#pragma unroll
      for (int i = 0; i < 16; ++i) v[i] = 0.0f;
    } else if (x_dtype == 1) {
      const uint4* xs = reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(x) +
                                                        static_cast<uint64_t>(t) * d + c0);
      const uint4 u0 = __ldg(xs), u1 = __ldg(xs + 1);
      const uint32_t w8[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
#pragma unroll
      for (int h = 0; h < 8; ++h) {
        v[2 * h] = __uint_as_float(w8[h] << 16);
        v[2 * h + 1] = __uint_as_float(w8[h] & 0xFFFF0000u);
      }
    } else {
      const float4* xs = reinterpret_cast<const float4*>(static_cast<const float*>(x) + static_cast<uint64_t>(t) * d + c0);
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const float4 a = __ldg(xs + h);
        v[4 * h] = a.x; v[4 * h + 1] = a.y; v[4 * h + 2] = a.z; v[4 * h + 3] = a.w;
      }
    }
    if (!gamma_is_one && active) {
#pragma unroll
      for (int i = 0; i < 16; ++i) v[i] = __fmul_rn(v[i], __ldg(gamma + c0 + i));
    }
    uint32_t words[kMaxTerms][4];
    uint32_t sword[kMaxTerms];
#pragma unroll
    for (int q = 0; q < kMaxTerms; ++q) {
      words[q][0] = words[q][1] = words[q][2] = words[q][3] = 0;
      sword[q] = 0;
      if (q < terms) {
        float amax = 0.0f;
#pragma unroll
        for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(v[i]));
        amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, 1));
        const int s = e4m3_block_exp(amax);
        // a finite block has s <= 120; s = -127 (amax below 2^-118) is written as zero codes
        const bool live = s > -127;
        const float inv = live ? __int_as_float((127 - s) << 23) : 0.0f;
        const float back = live ? __int_as_float((127 + s) << 23) : 0.0f;
#pragma unroll
        for (int w = 0; w < 4; ++w) {
          uint32_t word = 0;
#pragma unroll
          for (int hp = 0; hp < 2; ++hp) {
            const int i = w * 4 + hp * 2;
            const uint32_t c = cvt_e4m3x2(v[i] * inv, v[i + 1] * inv);
            float da, db;
            dec_e4m3x2(c, da, db);
            v[i] = fmaf(-da, back, v[i]);
            v[i + 1] = fmaf(-db, back, v[i + 1]);
            word |= c << (16 * hp);
          }
          words[q][w] = word;
        }
        // the scale word of four consecutive blocks (lane pairs lb & ~3 .. +3)
        uint32_t sw = active ? static_cast<uint32_t>(s + 127) << (8 * (lb & 3)) : 0u;
        sw |= __shfl_xor_sync(0xFFFFFFFFu, sw, 2);
        sw |= __shfl_xor_sync(0xFFFFFFFFu, sw, 4);
        sword[q] = sw;
      }
    }
    // one lane per group of four blocks stores the group's scale word; a group
    // wholly past d / 32 would land in the next row block's atom and stores nothing
    const bool sf_lane = hf == 0 && (lb & 3) == 0 && active;
#pragma unroll
    for (int s = 0; s < kMaxTopK; ++s) {
      if (s >= k) break;
      int pos = __ldg(inv_p + static_cast<uint64_t>(t) * k + s);
      uint8_t* codes_d = codes;
      uint8_t* sf_d = sf;
      if constexpr (kDispatch) {
        // pos is the pair's canonical position; its row at the owner follows
        // from the owner's segment layout (ep.src_base)
        const int p = t * k + s;
        const int e = __ldg(ep.topk_idx + p);
        const int g = e / ep.epr;
        const int q0 = pos;
        pos = __ldg(ep.src_base + e) + (q0 - __ldg(ep.offsets + e));
        if (pos < 0 || static_cast<uint32_t>(pos) >= ep.dst_rows) {  // inconsistent counts: write nothing
          if (lane == 0 && ep.err != nullptr) atomicCAS(ep.err, 0, 8);
          continue;
        }
        codes_d = ep.xq[g];
        if (lane == 0 && grp == 0)
          ep.meta[g][pos] = make_uint4(__float_as_uint(__ldg(ep.rscale + t)), __float_as_uint(__ldg(ep.topk_w + p)),
                                       (static_cast<uint32_t>(ep.rank) << 24) | static_cast<uint32_t>(q0), 0u);
        // the warp's 16 scale bytes per term go out as one 16-byte store
        // (row-major; the owner moves them into its atom layout)
#pragma unroll
        for (int q = 0; q < kMaxTerms; ++q) {
          if (q >= terms) break;
          const uint32_t s0 = __shfl_sync(0xFFFFFFFFu, sword[q], 0), s1 = __shfl_sync(0xFFFFFFFFu, sword[q], 8);
          const uint32_t s2 = __shfl_sync(0xFFFFFFFFu, sword[q], 16), s3 = __shfl_sync(0xFFFFFFFFu, sword[q], 24);
          if (lane == 0)
            *reinterpret_cast<uint4*>(ep.sf_rows[g] + (static_cast<uint64_t>(pos) * terms + q) * ep.sf_row_bytes +
                                      grp * kQBlocksPerWarp) = make_uint4(s0, s1, s2, s3);
        }
      }
#pragma unroll
      for (int q = 0; q < kMaxTerms; ++q) {
        if (q >= terms) break;
        if (active) {
          const uint64_t row = stacked ? static_cast<uint64_t>(stacked_code_row(static_cast<uint32_t>(pos),
                                                                                static_cast<uint32_t>(q),
                                                                                static_cast<uint32_t>(sf_rows)))
                                       : static_cast<uint64_t>(pos);
          uint8_t* dst = codes_d + (stacked ? 0 : q * term_stride) + row * kp + c0;
          *reinterpret_cast<uint4*>(dst) = make_uint4(words[q][0], words[q][1], words[q][2], words[q][3]);
        }
        if (!kDispatch && sf_lane) {
          const uint64_t o = stacked ? stacked_sf_offset(static_cast<uint32_t>(pos), static_cast<uint32_t>(q),
                                                         static_cast<uint32_t>(b), static_cast<uint32_t>(kchunks),
                                                         static_cast<uint32_t>(sf_rows))
                                     : q * sf_term_stride + sf_offset(static_cast<uint32_t>(pos),
                                                                      static_cast<uint32_t>(b),
                                                                      static_cast<uint32_t>(kchunks),
                                                                      static_cast<uint32_t>(sf_rows));
          *reinterpret_cast<uint32_t*>(sf_d + o) = sword[q];
        }
      }
    }
  }
  if constexpr (kDispatch) __threadfence_system();  // peer writes ordered before this GPU's later work
}

// FP4 decode operand (kind::mxf4 tiles): each routed pair's token row as four
// block-scaled E2M1 terms in the stacked layout (stacked4_code_row,
// stacked4_sf_offset).  Warp per (row, group of eight 32-column blocks), a
// lane quad per block, eight columns per lane: the step is latency-bound at
// decode sizes, so the work is spread over many short warps.  Each lane
// stores one code word per term and pair position; the first lane of each
// quad's group of four blocks stores the 4-byte scale word.
constexpr int kQ4BlocksPerWarp = 8;
__global__ void __launch_bounds__(256)
    quantize_f4_pairs_kernel(const void* __restrict__ x, int x_dtype, int n, int d, int k,
                             const float* __restrict__ gamma, int gamma_is_one, const int32_t* __restrict__ inv_p,
                             uint8_t* codes, int row_bytes, uint8_t* sf, int kchunks, int pt, int src_by_pos) {
  griddep_wait();
  const int nb = d / 32;
  const int ngrp = (nb + kQ4BlocksPerWarp - 1) / kQ4BlocksPerWarp;
  const uint64_t items = static_cast<uint64_t>(n) * ngrp;
  const int lane = threadIdx.x & 31;
  const int qd = lane & 3, lb = lane >> 2;  // eighth of the block, block within the group
  const uint64_t wstride = static_cast<uint64_t>(gridDim.x) * (blockDim.x >> 5);
  for (uint64_t it = static_cast<uint64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); it < items;
       it += wstride) {
    const int t = static_cast<int>(it / ngrp);
    const int grp = static_cast<int>(it - static_cast<uint64_t>(t) * ngrp);
    const int b = grp * kQ4BlocksPerWarp + lb;
    const bool active = b < nb;
    const int c0 = b * 32 + qd * 8;
    // source row: token t, or (activation rows, k = 1) the pair's own position
    const uint64_t src = src_by_pos ? static_cast<uint64_t>(__ldg(inv_p + t)) : static_cast<uint64_t>(t);
    uint32_t pos_k[kMaxTopK];
#pragma unroll
    for (int q = 0; q < kMaxTopK; ++q)
      pos_k[q] = q < k ? static_cast<uint32_t>(__ldg(inv_p + static_cast<uint64_t>(t) * k + q)) : 0u;
    float v[8];
    if (!active) {
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = 0.0f;
    } else if (x_dtype == 1) {
      const uint4 u = __ldg(reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(x) + src * d + c0));
      const uint32_t w4[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        v[2 * h] = __uint_as_float(w4[h] << 16);
        v[2 * h + 1] = __uint_as_float(w4[h] & 0xFFFF0000u);
      }
    } else {
      const float4* xs = reinterpret_cast<const float4*>(static_cast<const float*>(x) + src * d + c0);
      const float4 a0 = __ldg(xs), a1 = __ldg(xs + 1);
      v[0] = a0.x; v[1] = a0.y; v[2] = a0.z; v[3] = a0.w; v[4] = a1.x; v[5] = a1.y; v[6] = a1.z; v[7] = a1.w;
    }
    if (!gamma_is_one && active) {
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = __fmul_rn(v[i], __ldg(gamma + c0 + i));
    }
    uint32_t words[kF4Terms];
    uint8_t sbyte[kF4Terms];
    quantize8_e2m1_terms(v, words, sbyte);
    uint32_t sword[kF4Terms];
#pragma unroll
    for (int q = 0; q < kF4Terms; ++q) {
      // blocks lb & ~3 .. +3 are lanes 16 * (lb >> 2) .. + 15 (quads 4 apart)
      uint32_t sw = active ? static_cast<uint32_t>(sbyte[q]) << (8 * (lb & 3)) : 0u;
      sw |= __shfl_xor_sync(0xFFFFFFFFu, sw, 4);
      sw |= __shfl_xor_sync(0xFFFFFFFFu, sw, 8);
      sword[q] = sw;
    }
    const bool sf_lane = qd == 0 && (lb & 3) == 0 && active;
#pragma unroll
    for (int s = 0; s < kMaxTopK; ++s) {
      if (s >= k) break;
      const uint32_t pos = pos_k[s];
#pragma unroll
      for (int q = 0; q < kF4Terms; ++q) {
        if (active) {
          const uint64_t row = stacked4_code_row(pos, static_cast<uint32_t>(q), static_cast<uint32_t>(pt));
          *reinterpret_cast<uint32_t*>(codes + row * row_bytes + c0 / 2) = words[q];
        }
        if (sf_lane)
          *reinterpret_cast<uint32_t*>(sf + stacked4_sf_offset(pos, static_cast<uint32_t>(q), static_cast<uint32_t>(b),
                                                               static_cast<uint32_t>(kchunks),
                                                               static_cast<uint32_t>(pt))) = sword[q];
      }
    }
  }
}

// ------------------------------------------------------------------ combine
// y[t] = x[t] + sum over the token's experts in increasing expert index of
// y_pair (src/moe/mod.rs:279, :405, :411).  One block per token, four
// consecutive columns per thread (d is a multiple of 32).  k == 0 copies x.
__device__ __forceinline__ float4 load4(const void* p, int dtype, uint64_t i) {
  if (dtype == 0) return *reinterpret_cast<const float4*>(static_cast<const float*>(p) + i);
  const uint2 u = *reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(p) + i);
  return make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xFFFF0000u), __uint_as_float(u.y << 16),
                     __uint_as_float(u.y & 0xFFFF0000u));
}
__device__ __forceinline__ void store4(void* p, int dtype, uint64_t i, float4 v) {
  if (dtype == 0) {
    *reinterpret_cast<float4*>(static_cast<float*>(p) + i) = v;
  } else {
    const __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y), b = __floats2bfloat162_rn(v.z, v.w);
    *reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(p) + i) =
        make_uint2(*reinterpret_cast<const uint32_t*>(&a), *reinterpret_cast<const uint32_t*>(&b));
  }
}

__global__ void combine_kernel(const void* __restrict__ x, int x_dtype, const void* __restrict__ y_pair,
                               int pair_dtype, const int32_t* __restrict__ topk_idx,
                               const int32_t* __restrict__ inv_p, int n, int d, int k, int residual, void* y,
                               int y_dtype) {
  griddep_wait();
  const int t = blockIdx.x;
  if (t >= n) return;
  int ord[kMaxTopK];
  int ex[kMaxTopK];
  for (int s = 0; s < k; ++s) {
    ord[s] = inv_p[t * k + s];
    ex[s] = topk_idx[t * k + s];
  }
  for (int a = 1; a < k; ++a)
    for (int b = a; b > 0 && ex[b - 1] > ex[b]; --b) {
      int tmp = ex[b]; ex[b] = ex[b - 1]; ex[b - 1] = tmp;
      tmp = ord[b]; ord[b] = ord[b - 1]; ord[b - 1] = tmp;
    }
  // kCombineVec column groups per thread per round, all their loads in
  // flight together; the sums keep the order of the expert ids, then x
  constexpr int kCombineVec = 4;
  const int stride = 4 * blockDim.x;
  for (int c0 = 4 * threadIdx.x; c0 < d; c0 += stride * kCombineVec) {
    float4 acc[kCombineVec];
    float4 xv[kCombineVec];
#pragma unroll
    for (int v = 0; v < kCombineVec; ++v) {
      const int c = c0 + v * stride;
      acc[v] = make_float4(0.f, 0.f, 0.f, 0.f);
      xv[v] = (c < d && (residual || k == 0)) ? load4(x, x_dtype, static_cast<uint64_t>(t) * d + c)
                                              : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int s = 0; s < kMaxTopK; ++s) {
      if (s < k) {
#pragma unroll
        for (int v = 0; v < kCombineVec; ++v) {
          const int c = c0 + v * stride;
          if (c < d) {
            const float4 q = load4(y_pair, pair_dtype, static_cast<uint64_t>(ord[s]) * d + c);
            acc[v].x = __fadd_rn(acc[v].x, q.x); acc[v].y = __fadd_rn(acc[v].y, q.y);
            acc[v].z = __fadd_rn(acc[v].z, q.z); acc[v].w = __fadd_rn(acc[v].w, q.w);
          }
        }
      }
    }
#pragma unroll
    for (int v = 0; v < kCombineVec; ++v) {
      const int c = c0 + v * stride;
      if (c >= d) continue;
      float4 o;
      if (k == 0) {
        o = xv[v];
      } else if (residual) {
        o.x = __fadd_rn(xv[v].x, acc[v].x); o.y = __fadd_rn(xv[v].y, acc[v].y);
        o.z = __fadd_rn(xv[v].z, acc[v].z); o.w = __fadd_rn(xv[v].w, acc[v].w);
      } else {
        o = acc[v];
      }
      store4(y, y_dtype, static_cast<uint64_t>(t) * d + c, o);
    }
  }
}

// The same sum for bf16 pair rows, one warp per (token, column strip): the
// token's pairs are put in increasing expert order once (ranks by
// comparison, no sorting loop), then each lane takes 8-column groups with
// 16-byte loads, U groups' k rows and residuals in flight at once.  Small
// batches spread a token's row over `slices` warps.  Needs d % 8 == 0 and
// 16-byte aligned rows.
__device__ __forceinline__ void bf16x8_to_f32(uint4 u, float (&v)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int h = 0; h < 4; ++h) {
    v[2 * h] = __uint_as_float(w[h] << 16);
    v[2 * h + 1] = __uint_as_float(w[h] & 0xFFFF0000u);
  }
}

template <int KM, int U>
__global__ void __launch_bounds__(256, KM <= 4 ? 3 : 2) combine_rows_kernel(const void* __restrict__ x, int x_dtype,
                                                           const __nv_bfloat16* __restrict__ y_pair,
                                                           const int32_t* __restrict__ topk_idx,
                                                           const int32_t* __restrict__ inv_p, int n, int d, int k,
                                                           int residual, void* y, int y_dtype, int slices) {
  griddep_wait();
  const int wg = static_cast<int>((blockIdx.x * blockDim.x + threadIdx.x) >> 5);
  const int t = wg / slices, strip = wg - t * slices;
  const int lane = threadIdx.x & 31;
  if (t >= n) return;
  int ex[KM], ord[KM];
#pragma unroll
  for (int s = 0; s < KM; ++s) {
    ex[s] = s < k ? __ldg(topk_idx + static_cast<uint64_t>(t) * k + s) : 0x7FFFFFFF;
    ord[s] = s < k ? __ldg(inv_p + static_cast<uint64_t>(t) * k + s) : 0;
  }
  // row of rank r = the pair with r smaller expert ids (ties by slot keep the
  // insertion sort's stable order)
  uint64_t row[KM];
#pragma unroll
  for (int r = 0; r < KM; ++r) row[r] = 0;
#pragma unroll
  for (int s = 0; s < KM; ++s) {
    int rank = 0;
#pragma unroll
    for (int u = 0; u < KM; ++u) rank += (ex[u] < ex[s] || (ex[u] == ex[s] && u < s)) ? 1 : 0;
#pragma unroll
    for (int r = 0; r < KM; ++r)
      if (rank == r && s < k) row[r] = static_cast<uint64_t>(ord[s]) * d;
  }
  const int ng = d / 8;
  const uint64_t xo = static_cast<uint64_t>(t) * d;
  const int gs = 32 * slices;  // group stride of a warp
  for (int g0 = lane + 32 * strip; g0 < ng; g0 += gs * U) {
    uint4 q[U][KM];
    float xv[U][8];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int g = g0 + gs * u;
#pragma unroll
      for (int i = 0; i < 8; ++i) xv[u][i] = 0.0f;
      if (g >= ng) continue;
#pragma unroll
      for (int r = 0; r < KM; ++r)
        if (r < k) q[u][r] = __ldcg(reinterpret_cast<const uint4*>(y_pair + row[r] + g * 8));
      if (residual || k == 0) {
        if (x_dtype == 0) {
          const float4* xp = reinterpret_cast<const float4*>(static_cast<const float*>(x) + xo + g * 8);
          const float4 a = __ldg(xp), b = __ldg(xp + 1);
          xv[u][0] = a.x; xv[u][1] = a.y; xv[u][2] = a.z; xv[u][3] = a.w;
          xv[u][4] = b.x; xv[u][5] = b.y; xv[u][6] = b.z; xv[u][7] = b.w;
        } else {
          bf16x8_to_f32(__ldg(reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(x) + xo + g * 8)),
                        xv[u]);
        }
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int g = g0 + gs * u;
      if (g >= ng) continue;
      float acc[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = 0.0f;
#pragma unroll
      for (int r = 0; r < KM; ++r) {
        if (r < k) {
          float v[8];
          bf16x8_to_f32(q[u][r], v);
#pragma unroll
          for (int i = 0; i < 8; ++i) acc[i] = __fadd_rn(acc[i], v[i]);
        }
      }
      float o[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = k == 0 ? xv[u][i] : residual ? __fadd_rn(xv[u][i], acc[i]) : acc[i];
      if (y_dtype == 0) {
        float4* yp = reinterpret_cast<float4*>(static_cast<float*>(y) + xo + g * 8);
        yp[0] = make_float4(o[0], o[1], o[2], o[3]);
        yp[1] = make_float4(o[4], o[5], o[6], o[7]);
      } else {
        uint32_t w[4];
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          const __nv_bfloat162 b2 = __floats2bfloat162_rn(o[2 * h], o[2 * h + 1]);
          w[h] = *reinterpret_cast<const uint32_t*>(&b2);
        }
        *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(y) + xo + g * 8) = make_uint4(w[0], w[1], w[2], w[3]);
      }
    }
  }
}

// ------------------------------------------------------------------ expert-parallel helpers
// Global -> local expert ids for the receive side; ids outside the shard are
// reported through *err (code 7) and mapped to expert 0 so indexing stays safe.
__global__ void localize_kernel(const int32_t* __restrict__ expert, int P, int begin, int count, int32_t* local,
                                int* err) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= P) return;
  int v = expert[i] - begin;
  if (v < 0 || v >= count) {
    atomicCAS(err, 0, 7);
    v = 0;
  }
  local[i] = v;
}

// Dispatch packing: one warp per permuted position q copies the token row
// with 16-byte moves (rows are multiples of 64 bytes) and writes the pair's
// metadata as three 32-bit words (1/rms bits, expert id, route weight bits).
__global__ void gather_pairs_kernel(const void* __restrict__ x, uint32_t row_bytes, int k, int P,
                                    const int32_t* __restrict__ perm, const float* __restrict__ rscale,
                                    const int32_t* __restrict__ topk_idx, const float* __restrict__ topk_w,
                                    void* out_x, uint32_t* out_meta) {
  const int q = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (q >= P) return;
  const int p = __ldg(perm + q);
  const int t = p / k;
  if (lane == 0) {
    out_meta[3 * static_cast<uint64_t>(q) + 0] = __float_as_uint(__ldg(rscale + t));
    out_meta[3 * static_cast<uint64_t>(q) + 1] = static_cast<uint32_t>(__ldg(topk_idx + p));
    out_meta[3 * static_cast<uint64_t>(q) + 2] = __float_as_uint(__ldg(topk_w + p));
  }
  const uint4* src = reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(x) + static_cast<uint64_t>(t) * row_bytes);
  uint4* dst = reinterpret_cast<uint4*>(static_cast<uint8_t*>(out_x) + static_cast<uint64_t>(q) * row_bytes);
  for (uint32_t i = lane; i < row_bytes / 16; i += 32) dst[i] = __ldg(src + i);
}

// Expert-parallel dispatch over peer memory (replaces gather + all-to-all):
// warp per canonical position q (pairs sorted by expert, hence by owning
// rank g = expert / experts_per_rank).  The pair's token row and its metadata
// {bits of 1/rms, expert, bits of the route weight, return slot} go straight
// into rank g's receive buffers at row base_g + (q - offsets[g * Epr]), where
// base_g = pairs that lower ranks send to g (counts [src][dst]).  The return
// slot (rank << 24 | q) tells the owner where to write the pair's output.
__global__ void dispatch_pairs_kernel(const void* __restrict__ x, uint32_t row_bytes, int k, int P,
                                      const int32_t* __restrict__ perm, const float* __restrict__ rscale,
                                      const int32_t* __restrict__ topk_idx, const float* __restrict__ topk_w,
                                      const int32_t* __restrict__ offsets, int epr, int world, int rank,
                                      const int32_t* __restrict__ counts, void* const* __restrict__ peer_x,
                                      uint32_t* const* __restrict__ peer_meta, uint32_t recv_cap, int* err) {
  const int q = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (q >= P) return;
  const int p = __ldg(perm + q);
  const int t = p / k;
  const int e = __ldg(topk_idx + p);
  const int g = e / epr;
  int base = 0;
  for (int s = 0; s < rank; ++s) base += __ldg(counts + s * world + g);
  const int row = base + (q - __ldg(offsets + g * epr));
  if (g >= world || row < 0 || static_cast<uint32_t>(row) >= recv_cap) {  // inconsistent counts: write nothing
    if (lane == 0 && err != nullptr) atomicCAS(err, 0, 8);
    return;
  }
  const uint4* src = reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(x) + static_cast<uint64_t>(t) * row_bytes);
  uint4* dst = reinterpret_cast<uint4*>(static_cast<uint8_t*>(peer_x[g]) + static_cast<uint64_t>(row) * row_bytes);
  for (uint32_t i = lane; i < row_bytes / 16; i += 32) dst[i] = __ldg(src + i);
  if (lane == 0)
    reinterpret_cast<uint4*>(peer_meta[g])[row] =
        make_uint4(__float_as_uint(__ldg(rscale + t)), static_cast<uint32_t>(e), __float_as_uint(__ldg(topk_w + p)),
                   (static_cast<uint32_t>(rank) << 24) | static_cast<uint32_t>(q));
  __threadfence_system();  // peer writes ordered before anything this thread's GPU does later
}

// Expert-parallel return: warp per received row r; its bf16 output row goes
// to row (slot & 0xFFFFFF) of the source rank's return buffer
// peer_ret[slot >> 24] in 16-byte lanes (512 contiguous bytes per store).
__global__ void return_pairs_kernel(const __nv_bfloat16* __restrict__ y, uint32_t row_bytes, int R,
                                    const uint32_t* __restrict__ slot, int world, void* const* __restrict__ peer_ret,
                                    uint32_t ret_rows, int* err) {
  const int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= R) return;
  const uint32_t s = __ldg(slot + r);
  const int src = static_cast<int>(s >> 24);
  const uint32_t row = s & 0xFFFFFFu;
  if (src >= world || row >= ret_rows) {  // corrupt slot: write nothing
    if (lane == 0 && err != nullptr) atomicCAS(err, 0, 8);
    return;
  }
  const uint4* from = reinterpret_cast<const uint4*>(reinterpret_cast<const uint8_t*>(y) + static_cast<uint64_t>(r) * row_bytes);
  uint4* to = reinterpret_cast<uint4*>(static_cast<uint8_t*>(peer_ret[src]) + static_cast<uint64_t>(row) * row_bytes);
  for (uint32_t i = lane; i < row_bytes / 16; i += 32) to[i] = __ldg(from + i);
  __threadfence_system();
}

// Expert-parallel layout from the all-gathered pair counts [world][E]
// (counts[s * E + e] = pairs rank s routes to expert e).  Every owner g lays
// its experts [g * epr, (g + 1) * epr) out as consecutive segments, each
// padded to `pad` rows, pairs in (source rank, canonical position) order.
// Outputs: src_base[e] = this rank's first row for expert e at its owner;
// for the experts this rank owns, the padded starts poff[epr + 1], counts
// [epr] and the tile prefix (tiles of n_tile pairs) [epr + 1].
__global__ void ep_layout_kernel(const int32_t* __restrict__ counts, int world, int rank, int E, int epr, int pad,
                                 int n_tile, int32_t* src_base, int32_t* poff, int32_t* seg_counts,
                                 int32_t* ntile_prefix) {
  extern __shared__ int32_t lay[];  // tot[E], below[E], start[E]
  int32_t* tot = lay;
  int32_t* below = lay + E;
  int32_t* start = lay + 2 * E;
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int t = 0, b = 0;
    for (int s = 0; s < world; ++s) {
      const int c = counts[s * E + e];
      t += c;
      if (s < rank) b += c;
    }
    tot[e] = t;
    below[e] = b;
  }
  __syncthreads();
  for (int g = threadIdx.x; g < world; g += blockDim.x) {
    int run = 0;
    for (int el = 0; el < epr; ++el) {
      start[g * epr + el] = run;
      run += (tot[g * epr + el] + pad - 1) / pad * pad;
    }
    if (g == rank) poff[epr] = run;
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) src_base[e] = start[e] + below[e];
  if (threadIdx.x == 0) {
    int tiles = 0;
    for (int el = 0; el < epr; ++el) {
      const int e = rank * epr + el;
      poff[el] = start[e];
      seg_counts[el] = tot[e];
      ntile_prefix[el] = tiles;
      tiles += (tot[e] + n_tile - 1) / n_tile;
    }
    ntile_prefix[epr] = tiles;
  }
}

// Expert-parallel return from the owner's layout: warp per row pos of the
// segments (poff / seg_counts); a row holding a pair sends its bf16 output
// y[pos] to row (slot & 0xFFFFFF) of peer_ret[slot >> 24] in 16-byte lanes.
__global__ void ep_return_kernel(const __nv_bfloat16* __restrict__ y, uint32_t row_bytes, int rows,
                                 const int32_t* __restrict__ poff, const int32_t* __restrict__ seg_counts, int epr,
                                 const uint32_t* __restrict__ slot, int world, void* const* __restrict__ peer_ret,
                                 uint32_t ret_rows, int* err) {
  extern __shared__ int32_t seg[];  // poff[epr + 1], counts[epr]
  for (int i = threadIdx.x; i <= epr; i += blockDim.x) seg[i] = poff[i];
  for (int i = threadIdx.x; i < epr; i += blockDim.x) seg[epr + 1 + i] = seg_counts[i];
  __syncthreads();
  const int pos = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (pos >= rows || pos < seg[0] || pos >= seg[epr]) return;  // rows of this launch's experts only
  int el = 0;
  while (el + 1 < epr && seg[el + 1] <= pos) ++el;
  if (pos - seg[el] >= seg[epr + 1 + el]) return;  // padding row
  const uint32_t s = __ldg(slot + pos);
  const int src = static_cast<int>(s >> 24);
  const uint32_t row = s & 0xFFFFFFu;
  if (src >= world || row >= ret_rows) {
    if (lane == 0 && err != nullptr) atomicCAS(err, 0, 8);
    return;
  }
  const uint4* from = reinterpret_cast<const uint4*>(reinterpret_cast<const uint8_t*>(y) + static_cast<uint64_t>(pos) * row_bytes);
  uint4* to = reinterpret_cast<uint4*>(static_cast<uint8_t*>(peer_ret[src]) + static_cast<uint64_t>(row) * row_bytes);
  for (uint32_t i = lane; i < row_bytes / 16; i += 32) to[i] = __ldg(from + i);
  __threadfence_system();
}

// Owner side of the quantized dispatch, before W1: warp per row pos of the
// segments (poff / seg_counts); the row's metadata record becomes the per-row
// 1/rms, route weight and return slot, and its row-major scale bytes move
// into the scale-atom layout the MMA reads (plain or stacked tiles of pt).
__global__ void ep_unpack_kernel(const uint4* __restrict__ meta, const uint8_t* __restrict__ sf_rows,
                                 uint32_t sf_row_bytes, int terms, int nb, int rows, const int32_t* __restrict__ poff,
                                 const int32_t* __restrict__ seg_counts, int epr, float* rs, float* wt,
                                 uint32_t* slot, uint8_t* xsf, uint64_t sf_term_stride, int kchunks, int pt,
                                 int stacked) {
  extern __shared__ int32_t useg[];  // poff[epr + 1], counts[epr]
  for (int i = threadIdx.x; i <= epr; i += blockDim.x) useg[i] = poff[i];
  for (int i = threadIdx.x; i < epr; i += blockDim.x) useg[epr + 1 + i] = seg_counts[i];
  __syncthreads();
  const int pos = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (pos >= rows || pos >= useg[epr]) return;
  int el = 0;
  while (el + 1 < epr && useg[el + 1] <= pos) ++el;
  if (pos - useg[el] >= useg[epr + 1 + el]) return;  // padding row
  if (lane == 0) {
    const uint4 m = __ldg(meta + pos);
    rs[pos] = __uint_as_float(m.x);
    wt[pos] = __uint_as_float(m.y);
    slot[pos] = m.z;
  }
  const int ngroups = (nb + 3) / 4;  // 4-block scale words per term
  for (int i = lane; i < terms * ngroups; i += 32) {
    const int q = i / ngroups, g4 = i - q * ngroups;
    const uint32_t word = __ldg(reinterpret_cast<const uint32_t*>(
        sf_rows + (static_cast<uint64_t>(pos) * terms + q) * sf_row_bytes + 4 * g4));
    const uint64_t o = stacked ? stacked_sf_offset(static_cast<uint32_t>(pos), static_cast<uint32_t>(q),
                                                   static_cast<uint32_t>(4 * g4), static_cast<uint32_t>(kchunks),
                                                   static_cast<uint32_t>(pt))
                               : q * sf_term_stride + sf_offset(static_cast<uint32_t>(pos), static_cast<uint32_t>(4 * g4),
                                                                static_cast<uint32_t>(kchunks), static_cast<uint32_t>(pt));
    *reinterpret_cast<uint32_t*>(xsf + o) = word;
  }
}

__global__ void iota_kernel(int32_t* a, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) a[i] = i;
}

// Received metadata [R][4] -> per-pair arrays for the expert pipeline.
__global__ void split_meta_kernel(const uint4* __restrict__ meta, int R, float* rscale, int32_t* expert,
                                  float* weight, uint32_t* slot) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= R) return;
  const uint4 m = __ldg(meta + i);
  rscale[i] = __uint_as_float(m.x);
  expert[i] = static_cast<int32_t>(m.y);
  weight[i] = __uint_as_float(m.z);
  slot[i] = m.w;
}

// ------------------------------------------------------------------ SIMT FFN
__device__ __forceinline__ float w_value(const uint8_t* codes, const uint8_t* sfa, uint64_t row_bytes, int kchunks,
                                         uint32_t row, uint32_t col) {
  const uint8_t byte = codes[row * row_bytes + (col >> 1)];
  const uint8_t nib = (col & 1) ? (byte >> 4) : (byte & 0x0F);
  const int s = static_cast<int>(sfa[w_sf_offset(row, col / 32, kchunks)]) - 127;
  return kFp4Lut[nib] * ldexpf(1.0f, s);
}

// W1 + SwiGLU on CUDA cores: one warp per (expert, GLU unit j), looping over
// the expert's pairs.  act [rows][fp] f32.
__global__ void simt_w1_kernel(const void* __restrict__ x, int x_dtype, int d, int k, const float* __restrict__ gamma,
                               const float* __restrict__ rscale, const uint8_t* __restrict__ w1q,
                               const uint8_t* __restrict__ w1sf, const float* __restrict__ b1, int fp, int kp1,
                               const int32_t* __restrict__ poff, const int32_t* __restrict__ counts,
                               const int32_t* __restrict__ perm_p, float alpha, float limit, float* act) {
  const int e = blockIdx.y;
  const int j = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (j >= fp) return;
  const uint64_t rows = 2ull * fp;
  const uint8_t* codes = w1q + static_cast<uint64_t>(e) * rows * (kp1 / 2);
  const uint8_t* sfa = w1sf + static_cast<uint64_t>(e) * w_sf_row_pairs(static_cast<uint32_t>(rows)) * (kp1 / kTileK) * kWSfPairBytes;
  const uint32_t rg = w1_packed_row(j, 0), rl = w1_packed_row(j, 1);
  const float bg = b1[static_cast<uint64_t>(e) * rows + rg];
  const float bl = b1[static_cast<uint64_t>(e) * rows + rl];
  const int p0 = poff[e], cnt = counts[e];
  for (int i = 0; i < cnt; ++i) {
    const int pos = p0 + i;
    const int t = perm_p[pos] / k;
    const float r = rscale[t];
    float sg = 0.f, sl = 0.f;
    for (int c = lane; c < d; c += 32) {
      const float u = __fmul_rn(__fmul_rn(load_any(x, x_dtype, static_cast<uint64_t>(t) * d + c), r), gamma[c]);
      sg = fmaf(u, w_value(codes, sfa, kp1 / 2, kp1 / kTileK, rg, c), sg);
      sl = fmaf(u, w_value(codes, sfa, kp1 / 2, kp1 / kTileK, rl, c), sl);
    }
    sg = warp_sum_butterfly(sg);
    sl = warp_sum_butterfly(sl);
    if (lane == 0) {
      const float xg = fminf(sg + bg, limit);
      const float xl = fmaxf(-limit, fminf(sl + bl, limit));
      act[static_cast<uint64_t>(pos) * fp + j] = (xg / (1.0f + expf(-alpha * xg))) * (xl + 1.0f);
    }
  }
}

// W2 + bias + routing weight on CUDA cores: one warp per (expert, output c).
__global__ void simt_w2_kernel(const float* __restrict__ act, int fp, int d, int k, const uint8_t* __restrict__ w2q,
                               const uint8_t* __restrict__ w2sf, const float* __restrict__ b2, float bias_mult,
                               int kp2, const int32_t* __restrict__ poff, const int32_t* __restrict__ counts,
                               const int32_t* __restrict__ perm_p, const float* __restrict__ topk_w,
                               float* y_pair) {
  const int e = blockIdx.y;
  const int c = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (c >= d) return;
  const uint8_t* codes = w2q + static_cast<uint64_t>(e) * d * (kp2 / 2);
  const uint8_t* sfa = w2sf + static_cast<uint64_t>(e) * w_sf_row_pairs(static_cast<uint32_t>(d)) * (kp2 / kTileK) * kWSfPairBytes;
  const float bb = b2[static_cast<uint64_t>(e) * d + c] * bias_mult;
  const int p0 = poff[e], cnt = counts[e];
  for (int i = 0; i < cnt; ++i) {
    const int pos = p0 + i;
    const float* a = act + static_cast<uint64_t>(pos) * fp;
    float s = 0.f;
    for (int j = lane; j < fp; j += 32) s = fmaf(a[j], w_value(codes, sfa, kp2 / 2, kp2 / kTileK, c, j), s);
    s = warp_sum_butterfly(s);
    if (lane == 0) y_pair[static_cast<uint64_t>(pos) * d + c] = (s + bb) * topk_w[perm_p[pos]];
  }
}

}  // namespace

// ------------------------------------------------------------------ launchers
cudaError_t launch_dequant_bytes(const uint8_t* blocks, uint64_t rows, uint64_t b, const uint8_t* scales, float* out,
                                 cudaStream_t st) {
  const uint64_t total = rows * b;
  if (total == 0) return cudaSuccess;
  const int grid = static_cast<int>(total / 256 + 1 < 148 * 16 ? total / 256 + 1 : 148 * 16);
  dequant_bytes_kernel<<<grid, 256, 0, st>>>(blocks, rows, b, scales, out);
  return cudaGetLastError();
}

cudaError_t launch_dequant_rows(const uint8_t* blocks, const uint8_t* scales, uint64_t rows, uint64_t cols,
                                uint64_t bpr, uint64_t gpr, int ue8, float* out, cudaStream_t st) {
  const uint64_t total = rows * cols;
  if (total == 0) return cudaSuccess;
  const int grid = static_cast<int>(total / 256 + 1 < 148 * 16 ? total / 256 + 1 : 148 * 16);
  dequant_rows_kernel<<<grid, 256, 0, st>>>(blocks, scales, rows, cols, bpr, gpr, ue8, out);
  return cudaGetLastError();
}

cudaError_t launch_topk_softmax(const float* logits, int n, int E, int k, int32_t* idx, float* w, cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  const dim3 grid((n + 7) / 8);
  if (E <= 32) topk_softmax_kernel<1><<<grid, 256, 0, st>>>(logits, n, E, k, idx, w);
  else if (E <= 64) topk_softmax_kernel<2><<<grid, 256, 0, st>>>(logits, n, E, k, idx, w);
  else if (E <= 128) topk_softmax_kernel<4><<<grid, 256, 0, st>>>(logits, n, E, k, idx, w);
  else if (E <= 256) topk_softmax_kernel<8><<<grid, 256, 0, st>>>(logits, n, E, k, idx, w);
  else if (E <= 512) topk_softmax_kernel<16><<<grid, 256, 0, st>>>(logits, n, E, k, idx, w);
  else topk_softmax_kernel<32><<<grid, 256, 0, st>>>(logits, n, E, k, idx, w);
  return cudaGetLastError();
}

template <typename XT, int TT, int TE>
static cudaError_t launch_router_tile(const XT* x, int n, int d, int E, int k, const float* gamma,
                                      const float* gate_packed, const float* gate_b, const float* rscale,
                                      float* logits, int aligned, int32_t* topk_idx, float* topk_w, cudaStream_t st) {
  constexpr int BT = (kRouterWarps / (kRouterGroup / TE)) * TT;
  const dim3 grid((n + BT - 1) / BT, (E + kRouterGroup - 1) / kRouterGroup);
  const size_t smem = static_cast<size_t>(router_stages<BT>()) * router_stage_bytes<XT, BT>() +
                      2 * static_cast<size_t>(BT) * kRouterChunk * sizeof(float);
  const auto fn = router_logits_kernel<XT, TT, TE>;
  {
    const cudaError_t ce = ensure_dynamic_smem(reinterpret_cast<const void*>(fn), smem);
    if (ce != cudaSuccess) return ce;
  }
  return launch_kernel(fn, grid, dim3(kRouterThreads), smem, st, x, n, d, E, gamma, gate_packed, gate_b, rscale, logits,
                       aligned, k, topk_idx, topk_w);
}

size_t permute_smem_ints(int E) { return static_cast<size_t>(34) * E + 32 * 32 * kPermBatch; }

bool router_folds_permute(int n, int d, int E, int k) {
  return n > kRouterTinyMaxN && n <= kRouterSmallMaxN && E <= kRouterGroup && d <= kRouterSmallMaxD &&
         static_cast<int64_t>(n) * k < kPermMultiBlockMin;
}

// rms_kernel, then the logits; with E <= 32 the logits blocks hold every
// expert of their tokens and also write top-k + softmax, else a separate
// top-k kernel follows.
template <typename XT>
static cudaError_t launch_router_x(const XT* x, int n, int d, int E, int k, const float* gamma,
                                   const float* gate_packed, const float* gate_b, float eps, float* logits,
                                   int32_t* topk_idx, float* topk_w, float* rscale, __half* xh, float xh_scale,
                                   int* tok_ctr, int* status, int status_words, cudaStream_t st,
                                   const PermFold* fold) {
  const int aligned = (reinterpret_cast<uintptr_t>(x) % 16 == 0) && ((static_cast<size_t>(d) * sizeof(XT)) % 16 == 0);
  if (tok_ctr != nullptr && n <= kRouterTinyMaxN && d <= 32 * kRouterChunk) {
    const size_t smem = static_cast<size_t>(d) * sizeof(float) + (static_cast<size_t>(d) * sizeof(XT) + 15) / 16 * 16;
    const dim3 grid(n, (E + kRouterTinyExperts - 1) / kRouterTinyExperts), block(32 * kRouterTinyExperts);
    const int nch = (d + kRouterChunk - 1) / kRouterChunk;
    auto go = [&](auto fn) -> cudaError_t {
      const cudaError_t ce = ensure_dynamic_smem(reinterpret_cast<const void*>(fn), smem);
      if (ce != cudaSuccess) return ce;
      return launch_kernel(fn, grid, block, smem, st, x, n, d, E, k, gamma, gate_packed, gate_b, eps, logits, topk_idx,
                           topk_w, rscale, aligned, xh, xh_scale, tok_ctr, status, status_words);
    };
    if (nch <= 8) return go(router_tiny_kernel<XT, 8>);
    if (nch <= 16) return go(router_tiny_kernel<XT, 16>);
    if (nch <= 24) return go(router_tiny_kernel<XT, 24>);
    return go(router_tiny_kernel<XT, 32>);
  }
  if (n <= kRouterSmallMaxN && E <= kRouterGroup && d <= kRouterSmallMaxD) {
    size_t smem = static_cast<size_t>((d + kRouterChunk - 1) / kRouterChunk) * kRouterChunk * sizeof(float) +
                  (static_cast<size_t>(d) * sizeof(XT) + 15) / 16 * 16 + static_cast<size_t>(d) * sizeof(float);
    PermFold pf{};
    if (fold != nullptr && router_folds_permute(n, d, E, k)) {
      pf = *fold;
      smem = std::max(smem, permute_smem_ints(E) * sizeof(int32_t));
    }
    const cudaError_t ce = ensure_dynamic_smem(reinterpret_cast<const void*>(router_small_kernel<XT>), smem);
    if (ce != cudaSuccess) return ce;
    // one warp per expert, and at least 8 warps to stage and normalize the
    // row; a block that may run the permutation has the sort's 1024 threads
    const int threads = pf.ticket != nullptr ? kPermThreads : 32 * (E < 8 ? 8 : E);
    return launch_kernel(router_small_kernel<XT>, dim3(n), dim3(threads), smem, st, x, n, d, E, k, gamma, gate_packed,
                         gate_b, eps, logits, topk_idx, topk_w, rscale, aligned, pf);
  }
  {
    const cudaError_t re = launch_kernel(rms_kernel<XT>, dim3((n + 7) / 8), dim3(256), 0, st, x, n, d, eps, rscale,
                                         aligned);
    if (re != cudaSuccess) return re;
  }
  const bool fuse = E <= kRouterGroup;
  // large batches with the gate resident in shared memory (two or more chunks
  // per row: the kernel's 1/rms double buffer assumes it)
  int32_t* fi = fuse ? topk_idx : nullptr;
  float* fw = fuse ? topk_w : nullptr;
  // large batches: 16 tokens x 32 experts per block (8x8 per thread);
  // small ones: one token per block so that enough blocks run
  const cudaError_t e =
      n >= 2048 ? launch_router_tile<XT, 8, 8>(x, n, d, E, k, gamma, gate_packed, gate_b, rscale, logits, aligned, fi,
                                               fw, st)
                : launch_router_tile<XT, 1, 4>(x, n, d, E, k, gamma, gate_packed, gate_b, rscale, logits, aligned, fi,
                                               fw, st);
  if (e != cudaSuccess || fuse) return e;
  return launch_topk_softmax(logits, n, E, k, topk_idx, topk_w, st);
}

cudaError_t launch_router(const void* x, int x_dtype, int n, int d, int E, int k, const float* gamma,
                          const float* gate_packed, const float* gate_b, float eps, float* logits, int32_t* topk_idx,
                          float* topk_w, float* rscale, cudaStream_t st, __half* xh, float xh_scale, int* tok_ctr,
                          int* status, int status_words, const PermFold* fold) {
  if (n == 0) return cudaSuccess;
  return x_dtype == 0 ? launch_router_x(static_cast<const float*>(x), n, d, E, k, gamma, gate_packed, gate_b, eps,
                                        logits, topk_idx, topk_w, rscale, xh, xh_scale, tok_ctr, status, status_words,
                                        st, fold)
                      : launch_router_x(static_cast<const __nv_bfloat16*>(x), n, d, E, k, gamma, gate_packed, gate_b,
                                        eps, logits, topk_idx, topk_w, rscale, xh, xh_scale, tok_ctr, status,
                                        status_words, st, fold);
}

size_t permute_scratch_ints(int P, int E) {
  return 32 + 2 * static_cast<size_t>(E) + static_cast<size_t>((P + kPermChunk - 1) / kPermChunk) * E;
}

cudaError_t launch_permute(const int32_t* topk_idx, int P, int E, int pad, int N, int32_t* offsets, int32_t* perm_c,
                           int32_t* inv_c, int32_t* poff, int32_t* counts, int32_t* ntile_prefix, int32_t* perm_p,
                           int32_t* inv_p, cudaStream_t st, int32_t* scratch) {
  if (scratch && P >= kPermMultiBlockMin) {
    const int nch = (P + kPermChunk - 1) / kPermChunk;
    const size_t hsmem = 4 * static_cast<size_t>(E) * sizeof(int32_t);
    {
      const cudaError_t ce = ensure_dynamic_smem(reinterpret_cast<const void*>(perm_hist_kernel), hsmem);
      if (ce != cudaSuccess) return ce;
    }
    cudaError_t pe = launch_kernel(perm_hist_kernel, dim3(nch), dim3(kPermChunkThreads), hsmem, st, topk_idx, P, E, pad,
                                   N, scratch, offsets, poff, counts, ntile_prefix);
    if (pe != cudaSuccess) return pe;
    const size_t ssmem = (kPermChunkThreads / 32) * static_cast<size_t>(E) * sizeof(int32_t);
    {
      const cudaError_t ce = ensure_dynamic_smem(reinterpret_cast<const void*>(perm_scatter_kernel), ssmem);
      if (ce != cudaSuccess) return ce;
    }
    return launch_kernel(perm_scatter_kernel, dim3(nch), dim3(kPermChunkThreads), ssmem, st, topk_idx, P, E, scratch,
                         perm_c, inv_c, perm_p, inv_p);
  }
  const size_t smem = permute_smem_ints(E) * sizeof(int32_t);
  {
    const cudaError_t ce = ensure_dynamic_smem(reinterpret_cast<const void*>(permute_kernel), smem);
    if (ce != cudaSuccess) return ce;
  }
  return launch_kernel(permute_kernel, dim3(1), dim3(kPermThreads), smem, st, topk_idx, P, E, pad, N, offsets, perm_c,
                       inv_c, poff, counts, ntile_prefix, perm_p, inv_p);
}

cudaError_t launch_quantize_pairs(const void* x, int x_dtype, int n, int d, int k, const float* gamma,
                                  int gamma_is_one, const int32_t* inv_p, int terms, uint8_t* codes,
                                  uint64_t term_stride, int kp, uint8_t* sf, uint64_t sf_term_stride, int kchunks,
                                  int sf_rows, int stacked, cudaStream_t st) {
  const uint64_t items = static_cast<uint64_t>(n) * ((d / 32 + kQBlocksPerWarp - 1) / kQBlocksPerWarp);  // warps
  if (items == 0 || k == 0) return cudaSuccess;
  const uint64_t blocks = (items + 7) / 8;
  const int grid = static_cast<int>(blocks < 148 * 64 ? blocks : 148 * 64);
  return launch_kernel(quantize_pairs_kernel<false>, dim3(grid), dim3(256), 0, st, x, x_dtype, n, d, k, gamma,
                       gamma_is_one, inv_p, terms, codes, term_stride, kp, sf, sf_term_stride, kchunks, sf_rows, stacked,
                       EpDispatch{});
}

cudaError_t launch_quantize_f4_pairs(const void* x, int x_dtype, int n, int d, int k, const float* gamma,
                                     int gamma_is_one, const int32_t* inv_p, uint8_t* codes, int row_bytes,
                                     uint8_t* sf, int kchunks, int pt, int src_by_pos, cudaStream_t st) {
  const uint64_t items = static_cast<uint64_t>(n) * ((d / 32 + kQ4BlocksPerWarp - 1) / kQ4BlocksPerWarp);  // warps
  if (items == 0 || k == 0) return cudaSuccess;
  const uint64_t blocks = (items + 7) / 8;
  const int grid = static_cast<int>(blocks < 148 * 64 ? blocks : 148 * 64);
  return launch_kernel(quantize_f4_pairs_kernel, dim3(grid), dim3(256), 0, st, x, x_dtype, n, d, k, gamma,
                       gamma_is_one, inv_p, codes, row_bytes, sf, kchunks, pt, src_by_pos);
}

cudaError_t launch_combine(const void* x, int x_dtype, const void* y_pair, int pair_dtype, const int32_t* topk_idx,
                           const int32_t* inv_p, int n, int d, int k, int residual, void* y, int y_dtype,
                           cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  const auto a16 = [](const void* p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; };
  if (pair_dtype == 1 && d % 8 == 0 && k <= kMaxTopK && a16(y_pair) && a16(y) && (x == nullptr || a16(x))) {
    // about 2400 warps (16 per SM) in flight, at most one 32-group strip per warp
    const int max_slices = std::max(1, (d / 8 + 31) / 32);
    const int slices = std::min(max_slices, std::max(1, 2400 / std::max(n, 1)));
    const uint64_t warps = static_cast<uint64_t>(n) * slices;
    // top-k <= 4 (GPT-OSS): smaller rank arrays, three blocks per SM
    const auto fn = k <= 4 ? combine_rows_kernel<4, 2> : combine_rows_kernel<kMaxTopK, 2>;
    return launch_kernel(fn, dim3(static_cast<unsigned>((warps + 7) / 8)), dim3(256), 0, st, x, x_dtype,
                         static_cast<const __nv_bfloat16*>(y_pair), topk_idx, inv_p, n, d, k, residual, y, y_dtype,
                         slices);
  }
  return launch_kernel(combine_kernel, dim3(n), dim3(256), 0, st, x, x_dtype, y_pair, pair_dtype, topk_idx, inv_p, n, d,
                       k, residual, y, y_dtype);
}

cudaError_t launch_localize(const int32_t* expert, int P, int begin, int count, int32_t* local, int* err,
                            cudaStream_t st) {
  if (P == 0) return cudaSuccess;
  localize_kernel<<<(P + 255) / 256, 256, 0, st>>>(expert, P, begin, count, local, err);
  return cudaGetLastError();
}

cudaError_t launch_gather_pairs(const void* x, int x_dtype, int d, int k, int P, const int32_t* perm,
                                const float* rscale, const int32_t* topk_idx, const float* topk_w, void* out_x,
                                uint32_t* out_meta, cudaStream_t st) {
  if (P == 0) return cudaSuccess;
  const uint32_t row_bytes = static_cast<uint32_t>(d) * (x_dtype == 0 ? 4u : 2u);
  gather_pairs_kernel<<<(P + 7) / 8, 256, 0, st>>>(x, row_bytes, k, P, perm, rscale, topk_idx, topk_w, out_x,
                                                   out_meta);
  return cudaGetLastError();
}

cudaError_t launch_dispatch_pairs(const void* x, int x_dtype, int d, int k, int P, const int32_t* perm,
                                  const float* rscale, const int32_t* topk_idx, const float* topk_w,
                                  const int32_t* offsets, int experts_per_rank, int world, int rank,
                                  const int32_t* counts, void* const* peer_x, uint32_t* const* peer_meta,
                                  uint32_t recv_cap, int* err, cudaStream_t st) {
  if (P == 0) return cudaSuccess;
  const uint32_t row_bytes = static_cast<uint32_t>(d) * (x_dtype == 0 ? 4u : 2u);
  dispatch_pairs_kernel<<<(P + 7) / 8, 256, 0, st>>>(x, row_bytes, k, P, perm, rscale, topk_idx, topk_w, offsets,
                                                      experts_per_rank, world, rank, counts, peer_x, peer_meta,
                                                      recv_cap, err);
  return cudaGetLastError();
}

cudaError_t launch_return_pairs(const void* y_bf16, int d, int R, const uint32_t* slot, int world,
                                void* const* peer_ret, uint32_t ret_rows, int* err, cudaStream_t st) {
  if (R == 0) return cudaSuccess;
  return_pairs_kernel<<<(R + 7) / 8, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(y_bf16),
                                                    static_cast<uint32_t>(d) * 2u, R, slot, world, peer_ret, ret_rows,
                                                    err);
  return cudaGetLastError();
}

__global__ void ep_push_counts_kernel(const int32_t* __restrict__ offsets, int E, int rank, int world,
                                      int32_t* const* __restrict__ peer_counts) {
  griddep_wait();
  for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < E; e += gridDim.x * blockDim.x) {
    const int c = offsets ? offsets[e + 1] - offsets[e] : 0;
    for (int r = 0; r < world; ++r) peer_counts[r][static_cast<size_t>(rank) * E + e] = c;
  }
}

cudaError_t launch_ep_push_counts(const int32_t* offsets, int E, int rank, int world, int32_t* const* peer_counts,
                                  cudaStream_t st) {
  return launch_kernel(ep_push_counts_kernel, dim3((E + 255) / 256), dim3(256), 0, st, offsets, E, rank, world,
                       peer_counts);
}

cudaError_t launch_ep_layout(const int32_t* counts, int world, int rank, int E, int epr, int pad, int n_tile,
                             int32_t* src_base, int32_t* poff, int32_t* seg_counts, int32_t* ntile_prefix,
                             cudaStream_t st) {
  const size_t smem = 3ull * E * sizeof(int32_t);
  {
    const cudaError_t ce = ensure_dynamic_smem(reinterpret_cast<const void*>(ep_layout_kernel), smem);
    if (ce != cudaSuccess) return ce;
  }
  ep_layout_kernel<<<1, 256, smem, st>>>(counts, world, rank, E, epr, pad, n_tile, src_base, poff, seg_counts,
                                         ntile_prefix);
  return cudaGetLastError();
}

cudaError_t launch_ep_quantize_dispatch(const void* x, int x_dtype, int n, int d, int k, const float* gamma,
                                        int gamma_is_one, const int32_t* inv_c, int terms, uint64_t term_stride,
                                        int kp, int sf_rows_n, int stacked, const int32_t* src_base,
                                        const int32_t* offsets, const int32_t* topk_idx, const float* topk_w,
                                        const float* rscale, int epr, int rank, uint32_t dst_rows,
                                        uint32_t sf_row_bytes, uint8_t* const* xq, uint8_t* const* sf_rows,
                                        void* const* meta, int* err, cudaStream_t st) {
  const uint64_t items = static_cast<uint64_t>(n) * ((d / 32 + kQBlocksPerWarp - 1) / kQBlocksPerWarp);
  if (items == 0 || k == 0) return cudaSuccess;
  const uint64_t blocks = (items + 7) / 8;
  const int grid = static_cast<int>(blocks < 148 * 64 ? blocks : 148 * 64);
  const EpDispatch ep{src_base, offsets, topk_idx, topk_w, rscale, epr, rank, dst_rows, sf_row_bytes, xq, sf_rows,
                      reinterpret_cast<uint4* const*>(meta), err};
  quantize_pairs_kernel<true><<<grid, 256, 0, st>>>(x, x_dtype, n, d, k, gamma, gamma_is_one, inv_c, terms, nullptr,
                                                    term_stride, kp, nullptr, 0, 0, sf_rows_n, stacked, ep);
  return cudaGetLastError();
}

cudaError_t launch_ep_return(const void* y_bf16, int d, int rows, const int32_t* poff, const int32_t* seg_counts,
                             int epr, const uint32_t* slot, int world, void* const* peer_ret, uint32_t ret_rows,
                             int* err, cudaStream_t st, int threads) {
  if (rows == 0 || epr == 0) return cudaSuccess;
  const int wpb = threads / 32;
  const size_t smem = (2ull * epr + 1) * sizeof(int32_t);
  {
    const cudaError_t ce = ensure_dynamic_smem(reinterpret_cast<const void*>(ep_return_kernel), smem);
    if (ce != cudaSuccess) return ce;
  }
  ep_return_kernel<<<(rows + wpb - 1) / wpb, threads, smem, st>>>(static_cast<const __nv_bfloat16*>(y_bf16),
                                                       static_cast<uint32_t>(d) * 2u, rows, poff, seg_counts, epr,
                                                       slot, world, peer_ret, ret_rows, err);
  return cudaGetLastError();
}

cudaError_t launch_ep_unpack(const void* meta, const uint8_t* sf_rows, uint32_t sf_row_bytes, int terms, int nb,
                             int rows, const int32_t* poff, const int32_t* seg_counts, int epr, float* rs, float* wt,
                             uint32_t* slot, uint8_t* xsf, uint64_t sf_term_stride, int kchunks, int pt, int stacked,
                             cudaStream_t st) {
  if (rows == 0) return cudaSuccess;
  const size_t smem = (2ull * epr + 1) * sizeof(int32_t);
  {
    const cudaError_t ce = ensure_dynamic_smem(reinterpret_cast<const void*>(ep_unpack_kernel), smem);
    if (ce != cudaSuccess) return ce;
  }
  ep_unpack_kernel<<<(rows + 7) / 8, 256, smem, st>>>(static_cast<const uint4*>(meta), sf_rows, sf_row_bytes, terms, nb,
                                                       rows, poff, seg_counts, epr, rs, wt, slot, xsf, sf_term_stride,
                                                       kchunks, pt, stacked);
  return cudaGetLastError();
}

cudaError_t launch_iota(int32_t* a, int n, cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  iota_kernel<<<(n + 255) / 256, 256, 0, st>>>(a, n);
  return cudaGetLastError();
}

cudaError_t launch_split_meta(const uint32_t* meta, int R, float* rscale, int32_t* expert, float* weight,
                              uint32_t* slot, cudaStream_t st) {
  if (R == 0) return cudaSuccess;
  split_meta_kernel<<<(R + 255) / 256, 256, 0, st>>>(reinterpret_cast<const uint4*>(meta), R, rscale, expert, weight,
                                                      slot);
  return cudaGetLastError();
}


cudaError_t launch_simt_w1(const void* x, int x_dtype, int d, int k, const float* gamma, const float* rscale,
                           const uint8_t* w1q, const uint8_t* w1sf, const float* b1, int fp, int kp1, int E,
                           const int32_t* poff, const int32_t* counts, const int32_t* perm_p, float alpha, float limit,
                           float* act, cudaStream_t st) {
  dim3 grid((fp + 7) / 8, E);
  simt_w1_kernel<<<grid, 256, 0, st>>>(x, x_dtype, d, k, gamma, rscale, w1q, w1sf, b1, fp, kp1, poff, counts, perm_p,
                                       alpha, limit, act);
  return cudaGetLastError();
}

cudaError_t launch_simt_w2(const float* act, int fp, int d, int k, const uint8_t* w2q, const uint8_t* w2sf,
                           const float* b2, float bias_mult, int kp2, int E, const int32_t* poff,
                           const int32_t* counts, const int32_t* perm_p, const float* topk_w, float* y_pair,
                           cudaStream_t st) {
  dim3 grid((d + 7) / 8, E);
  simt_w2_kernel<<<grid, 256, 0, st>>>(act, fp, d, k, w2q, w2sf, b2, bias_mult, kp2, poff, counts, perm_p, topk_w,
                                       y_pair);
  return cudaGetLastError();
}

}  // namespace mxmoe
