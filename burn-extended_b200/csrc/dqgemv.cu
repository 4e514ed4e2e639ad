// dqgemv.cu -- fused MXFP4 dequant-GEMV expert FFN for decode batches (at
// most a few routed pairs), on CUDA cores: W1 + SwiGLU-clamp, W2 + bias +
// route weight and (in the fused forward) the expert-order combine with the
// residual, in one launch.
//
// Replaces, for few-token batches, the per-element byte-wise dequant loops of
// w1_swiglu_dense_kernel / w2_scatter_dense_kernel (src/quant/gpu.rs:89-192)
// and the per-expert accumulation of src/moe/mod.rs:279-411: there every
// token-row thread re-reads each weight byte and recomputes exp(s * ln 2) per
// element; here each weight byte crosses HBM once per forward, is decoded two
// codes per instruction, and serves every routed pair of its expert.
//
// Work split (no host sync, one block per SM, cooperative launch):
//   W1: the GLU units of the touched experts, laid end to end in increasing
//       expert order, are cut into gridDim.x equal contiguous ranges; block b
//       computes range b for all of its expert's pairs.
//   W2: the d output columns are cut into gridDim.x equal ranges; block b
//       computes its columns for every touched expert, so it holds all k
//       contributions of its columns and (fused forward) adds them in
//       increasing expert order plus the residual and writes y itself.
//   Between the two phases the blocks meet once on a grid-wide arrival
//   counter (bounded wait; on timeout a status code and the arrival count
//   are recorded and the kernel runs to its end).
//
// Data movement: a copy warp streams the block's weight ranges (contiguous
// rows: a W1 chunk is up to 8 GLU rows plus their 8 linear partner rows, a
// W2 chunk up to a slot's worth of output rows, each with its E8M0 scale
// rows) into a ring of shared-memory slots with cp.async.bulk (L2
// evict-first), one mbarrier pair per slot, keeping about 48 KB in flight per
// SM (its share of HBM bandwidth times latency; more only lengthens the
// memory queues the compute warps' own reads wait in).  It runs ahead into W2
// while W1 is computed, so the W2 weights are on chip when the grid barrier
// opens.  The block's small reads (token rows, biases) are issued before the
// weight stream.  Items (a W1 GLU unit = two rows, or a W2 column pair) go to
// the 16 compute warps round robin over the block's whole sequence.
//
// Math: lane l covers the 32-column blocks kb = l + 32 i of both rows (one
// 16-byte code load each, conflict-free), decodes them with
// cvt.rn.f16x2.e2m1x2 and multiplies pairs of columns with packed f16 FMAs
// against the activation rows staged in shared memory as f16: each E2M1 value
// times the f16 activation rounds once, the 16 products of a block half sum
// in f16 (the activation scales keep |sum| <= 16 * 6 * 512), the two halves
// and every block after that in f32.  Per block the sum is scaled once by
// 2^(s - 127); the warp then reduces all (row, pair) sums at once by halving
// exchanges.  The K loop is unrolled at compile time (KI blocks per lane) and
// the pair count is dispatched to unrolled variants.
//
// Activations: W1 stages one router-normalized token row per token (x *
// (1/rms) * gamma as f16, written by the router), W2 the f16 SwiGLU row of
// each pair; both carry a power of two that bounds them by 512 (|x_hat| <=
// sqrt(d) * max|gamma| after RmsNorm; |act| <= max(limit, 0.28 / alpha) *
// (limit + 1) after the clamp), which keeps the f16 block sums finite.  The
// swizzle puts lane l's four 16-byte pieces of a 32-column block 512 bytes
// apart, so a quarter warp reads 128 contiguous bytes.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>

#include "kernels.h"
#include "launch_util.h"
#include "layout.cuh"
#include "ptx.cuh"

namespace mxmoe {

namespace {

constexpr int kDqWarps = 16;                     // compute warps per block
constexpr int kDqConsumers = 32 * kDqWarps;
constexpr int kDqThreads = kDqConsumers + 32;    // + the copy warp
constexpr int kDqMaxPairs = 8;                   // routed pairs per launch
constexpr int kDqMaxSlots = 8;
constexpr int kDqMaxCols = 64;                   // W2 output columns per block
constexpr int kDqMaxUnits = 256;                 // W1 GLU units per block
constexpr int kDqRows = 2;                       // weight rows per item
// per-block float scratch after the staged rows: W2 partial sums, W1 / W2 biases
constexpr int kDqScratchFloats = kDqMaxPairs * kDqMaxCols + 2 * kDqMaxUnits + kDqMaxPairs * kDqMaxCols;
// status codes of this kernel (the layer's status word)
constexpr int kDqErrGrid = 8;  // the blocks did not all finish W1 in time
constexpr int kDqErrCopy = 9;  // a weight chunk did not land, or a slot was not released, in time

// Build-time timeline probe (-DMXMOE_DQ_TRACE, never in the shipped build):
// lane 0 of every warp stamps %globaltimer at fixed event slots.
#ifdef MXMOE_DQ_TRACE
constexpr int kDqTraceSlots = 64;
__device__ unsigned long long g_dq_trace[160 * 17 * kDqTraceSlots];
#define DQ_T(k)                                                                                  \
  do {                                                                                           \
    if ((threadIdx.x & 31) == 0 && blockIdx.x < 160 && (k) < kDqTraceSlots)                      \
      g_dq_trace[(blockIdx.x * 17 + (threadIdx.x >> 5)) * kDqTraceSlots + (k)] = global_timer_ns(); \
  } while (0)
#else
#define DQ_T(k) \
  do {          \
  } while (0)
#endif

__device__ __forceinline__ __half2 u32_h2(uint32_t u) {
  __half2 h;
  memcpy(&h, &u, 4);
  return h;
}

// E2M1 code word (8 codes, low nibble first) -> four f16x2 (low half = even column).
__device__ __forceinline__ void e2m1x8_to_f16x2(uint32_t w, uint32_t (&h)[4]) {
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "mov.b32 {b0, b1, b2, b3}, %4;\n\t"
      "cvt.rn.f16x2.e2m1x2 %0, b0;\n\t"
      "cvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %2, b2;\n\t"
      "cvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
      : "=r"(h[0]), "=r"(h[1]), "=r"(h[2]), "=r"(h[3])
      : "r"(w));
}

// 2^(s - 127) for an E8M0 byte (0 -> 2^-127, 255 -> inf, as the format's
// exponent range gives).
__device__ __forceinline__ float e8m0_to_f32(uint32_t s) {
  return s == 0 ? __int_as_float(0x00400000) : __int_as_float(static_cast<int>(s) << 23);
}

// Index (in 16-byte pieces) of piece q (columns 8q .. 8q + 7) of 32-column
// block kb of staged row p, rows ki * 128 pieces apart.
__device__ __forceinline__ int dq_piece(int p, int ki, int kb, int q) {
  return p * ki * 128 + ((kb >> 5) * 4 + q) * 32 + (kb & 31);
}


// 8 consecutive source values -> f32 (f16 sources were written earlier in
// this forward by other blocks: read through L2).
__device__ __forceinline__ void dq_src8(const void* p, int dtype, float (&v)[8]) {
  if (dtype == kDqSrcF32) {
    const float4 a = __ldg(static_cast<const float4*>(p)), b = __ldg(static_cast<const float4*>(p) + 1);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  } else if (dtype == kDqSrcBf16) {
    const uint4 u = __ldg(static_cast<const uint4*>(p));
    const uint32_t wd[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      v[2 * h] = __uint_as_float(wd[h] << 16);
      v[2 * h + 1] = __uint_as_float(wd[h] & 0xFFFF0000u);
    }
  } else {
    const uint4 u = __ldcg(static_cast<const uint4*>(p));
    const uint32_t wd[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&wd[h]));
      v[2 * h] = f.x;
      v[2 * h + 1] = f.y;
    }
  }
}

// Sum over the warp of V values per lane (V a power of two <= 32) in
// V - 1 + (5 - log2 V) shuffles: halving exchanges leave lane L with value
// L % V of its group, then butterflies finish it.  Returns lane L's total of
// value L % V.
template <int V>
__device__ __forceinline__ float dq_warp_reduce(float (&v)[V], int lane) {
#pragma unroll
  for (int h = V / 2; h >= 1; h /= 2) {
    const bool upper = (lane & h) != 0;
#pragma unroll
    for (int i = 0; i < h; ++i) {
      const float send = upper ? v[i] : v[i + h];
      const float keep = upper ? v[i + h] : v[i];
      v[i] = keep + __shfl_xor_sync(0xFFFFFFFFu, send, h);
    }
  }
  float r = v[0];
#pragma unroll
  for (int o = V; o < 32; o *= 2) r += __shfl_xor_sync(0xFFFFFFFFu, r, o);
  return r;
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async4(uint32_t dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }
// The compute warps' own barrier (the copy warp never joins it).
__device__ __forceinline__ void dq_bar() { asm volatile("bar.sync 1, %0;" ::"n"(kDqConsumers) : "memory"); }

// The routed pairs of this launch, sorted by (expert, pair): rank r is pair
// pair[r] of token tok[r] on local expert exp[r] with route weight w[r].
// Touched expert i (increasing) is te_exp[i], owning ranks te_lo[i] ..
// te_lo[i + 1] - 1.  W1 stages one row per token (row t = token t), W2 one
// per rank (ident).
struct DqTable {
  int pair[kDqMaxPairs], tok[kDqMaxPairs], exp[kDqMaxPairs];
  float w[kDqMaxPairs];
  int te_exp[kDqMaxPairs], te_lo[kDqMaxPairs + 1];
  int ident[kDqMaxPairs];
  int n, nt;
};

// One piece of a block's weight stream.
struct DqChunk {
  int w2;   // 0: W1 GLU units r0 .. r0 + len - 1; 1: W2 rows (output columns) r0 ..
  int ei;   // touched-expert number
  int r0, len;
};

// A block's chunk sequence: its W1 units [u, u1) of the touched experts' GLU
// units laid end to end (expert-major), in pieces of at most cu units that
// stay inside one 64-unit GLU block; then, for each touched expert in
// increasing order, its output rows [c0, c1) of W2 in pieces of at most cr.
// The copy warp and the compute warps walk the same sequence.
struct DqWalk {
  int u, u1, fp, cu;
  int ei, nt, c, c0, c1, cr;
  __device__ bool next(DqChunk& ch) {
    if (u < u1) {
      const int e = u / fp, m = u - e * fp;
      const int len = min(min(u1 - u, cu), kGluBlock - m % kGluBlock);
      ch = DqChunk{0, e, m, len};
      u += len;
      return true;
    }
    while (ei < nt) {
      if (c < c1) {
        const int len = min(c1 - c, cr);
        ch = DqChunk{1, ei, c, len};
        c += len;
        return true;
      }
      ++ei;
      c = c0;
    }
    return false;
  }
};

// Synchronous W1 staging from the token rows x (when no f16 rows were
// prepared): rows t < ntok of x * (1/rms) * gamma * x_scale as f16, in
// dq_piece order.  Consecutive threads read consecutive 16-byte pieces.
__device__ void dq_stage_x(uint4* xs, const DqParams& a, int ntok, int ki) {
  const int kbr = a.d / 32;
  for (int t = 0; t < ntok; ++t) {
    const float rs = __ldcg(a.rscale + t) * a.x_scale;
    for (int p = threadIdx.x; p < 4 * kbr; p += kDqConsumers) {
      const int kb = p >> 2, q = p & 3, c = kb * 32 + q * 8;
      float v[8];
      dq_src8(static_cast<const char*>(a.x) + (static_cast<uint64_t>(t) * a.d + c) * (a.x_dtype == kDqSrcF32 ? 4 : 2),
              a.x_dtype, v);
      const float4 g0 = __ldg(reinterpret_cast<const float4*>(a.gamma + c));
      const float4 g1 = __ldg(reinterpret_cast<const float4*>(a.gamma + c) + 1);
      v[0] *= g0.x; v[1] *= g0.y; v[2] *= g0.z; v[3] *= g0.w; v[4] *= g1.x; v[5] *= g1.y; v[6] *= g1.z; v[7] *= g1.w;
      uint4 o;
      uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const __half2 hv = __floats2half2_rn(v[2 * h] * rs, v[2 * h + 1] * rs);
        ow[h] = *reinterpret_cast<const uint32_t*>(&hv);
      }
      xs[dq_piece(t, ki, kb, q)] = o;
    }
  }
}

// Asynchronous staging of n f16 rows of K columns into xs (dq_piece order),
// staged row j from base + key[j] * stride: one 16-byte copy per piece,
// issued by the compute threads; the caller commits and waits.
__device__ __forceinline__ void dq_stage_async(uint4* xs, const __half* base, const int* key, uint64_t stride, int n,
                                               int K, int ki) {
  const int kbr = K / 32;
  for (int j = 0; j < n; ++j) {
    const __half* src = base + static_cast<uint64_t>(key[j]) * stride;
    for (int p = threadIdx.x; p < 4 * kbr; p += kDqConsumers) {
      const int kb = p >> 2, q = p & 3;
      cp_async16(smem_u32(xs + dq_piece(j, ki, kb, q)), src + kb * 32 + q * 8);
    }
  }
}

__host__ __device__ constexpr int dq_pow2(int n) { return n <= 1 ? 1 : n <= 2 ? 2 : n <= 4 ? 4 : 8; }

// Dot products of two weight rows (codes c0 / c1, scale rows s0 / s1) with
// the staged rows of ranks j0 .. j0 + NP - 1 (staged row rix[rank]), reduced
// over the warp: lane L returns the sum of (row (L % V) / NPP, rank j0 +
// L % NPP), V = 2 * NPP.  Fully unrolled over the KI 32-column blocks of a
// lane; lanes past the last block read zero codes.
template <int KI, int NP>
__device__ __forceinline__ float dq_dot(const uint8_t* c0, const uint8_t* c1, const uint8_t* s0, const uint8_t* s1,
                                        const uint4* xs, const int* rix, int kbr, int lane, int j0) {
  constexpr int NPP = dq_pow2(NP);
  float acc[kDqRows * NPP];
#pragma unroll
  for (int i = 0; i < kDqRows * NPP; ++i) acc[i] = 0.0f;
  int row[NP];
#pragma unroll
  for (int j = 0; j < NP; ++j) row[j] = rix[j0 + j];
#pragma unroll
  for (int i = 0; i < KI; ++i) {
    const int kb = lane + 32 * i;
    const bool ok = kb < kbr;
    uint32_t h[kDqRows][4][4];
    float sc[kDqRows];
#pragma unroll
    for (int r = 0; r < kDqRows; ++r) {
      uint4 cw = make_uint4(0u, 0u, 0u, 0u);
      if (ok) cw = *reinterpret_cast<const uint4*>((r ? c1 : c0) + kb * 16);
      e2m1x8_to_f16x2(cw.x, h[r][0]);
      e2m1x8_to_f16x2(cw.y, h[r][1]);
      e2m1x8_to_f16x2(cw.z, h[r][2]);
      e2m1x8_to_f16x2(cw.w, h[r][3]);
      sc[r] = ok ? e8m0_to_f32((r ? s1 : s0)[kb]) : 0.0f;
    }
#pragma unroll
    for (int j = 0; j < NP; ++j) {
      uint4 xv[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) xv[q] = xs[dq_piece(row[j], KI, kb, q)];
#pragma unroll
      for (int r = 0; r < kDqRows; ++r) {
        // packed f16 products summed in f16 over the block's 32 columns (two
        // chains of 8), then one f32 scale step
        __half2 p0 = __float2half2_rn(0.0f), p1 = p0;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          p0 = __hfma2(u32_h2(h[r][q][0]), u32_h2(xv[q].x), p0);
          p1 = __hfma2(u32_h2(h[r][q][1]), u32_h2(xv[q].y), p1);
          p0 = __hfma2(u32_h2(h[r][q][2]), u32_h2(xv[q].z), p0);
          p1 = __hfma2(u32_h2(h[r][q][3]), u32_h2(xv[q].w), p1);
        }
        const float2 f = __half22float2(__hadd2(p0, p1));
        acc[r * NPP + j] = fmaf(f.x + f.y, sc[r], acc[r * NPP + j]);
      }
    }
  }
  return dq_warp_reduce<kDqRows * NPP>(acc, lane);
}

// W1 item: GLU unit m of one expert (its GLU row c0/s0 and linear row c1/s1)
// against ranks j0 .. j0 + NP - 1 -> the SwiGLU values of those pairs.
template <int KI, int NP>
__device__ __forceinline__ void dq_w1_item(const DqParams& a, const DqTable& tb, const uint8_t* c0, const uint8_t* c1,
                                           const uint8_t* s0, const uint8_t* s1, const uint4* xs, int lane, int j0,
                                           int m, float bias) {
  constexpr int NPP = dq_pow2(NP);
  const float v = dq_dot<KI, NP>(c0, c1, s0, s1, xs, tb.tok, a.d / 32, lane, j0);
  // lane j (< NPP) holds the GLU row's sum of rank j0 + j, lane NPP + j the linear row's
  const float vl = __shfl_sync(0xFFFFFFFFu, v, (lane + NPP) & 31);
  const float bg = __shfl_sync(0xFFFFFFFFu, bias, 0), bl = __shfl_sync(0xFFFFFFFFu, bias, 1);
  if (lane < NP) {
    const float xg = fminf(v * a.inv_x_scale + bg, a.limit);
    const float xl = fmaxf(-a.limit, fminf(vl * a.inv_x_scale + bl, a.limit));
    const float act = (xg / (1.0f + expf(-a.alpha * xg))) * (xl + 1.0f);
    a.act[static_cast<uint64_t>(tb.pair[j0 + lane]) * a.fp + m] = __float2half_rn(act * a.act_scale);
  }
}

// W2 item: output columns col, col + 1 (nrow of them valid) of one expert
// against ranks j0 .. j0 + NP - 1: (sum / act_scale + b2) * route weight,
// into the block's partial sums (fused) or the pair rows of y_pair.
template <int KI, int NP>
__device__ __forceinline__ void dq_w2_item(const DqParams& a, const DqTable& tb, const uint8_t* c0, const uint8_t* c1,
                                           const uint8_t* s0, const uint8_t* s1, const uint4* xs, int lane, int j0,
                                           int col, int nrow, int col0, float bias, float* partial) {
  constexpr int NPP = dq_pow2(NP);
  const float v = dq_dot<KI, NP>(c0, c1, s0, s1, xs, tb.ident, a.fp / 32, lane, j0);
  const int vi = lane % (kDqRows * NPP), r = vi / NPP, j = vi % NPP;
  const float br = __shfl_sync(0xFFFFFFFFu, bias, r);
  if (lane < kDqRows * NPP && j < NP && r < nrow) {
    const int rank = j0 + j;
    const float val = (v * a.inv_act_scale + br) * tb.w[rank];
    if (a.fused)
      partial[rank * kDqMaxCols + col + r - col0] = val;
    else
      a.y_pair[static_cast<uint64_t>(__ldg(a.inv + tb.pair[rank])) * a.d + col + r] = val;
  }
}

template <int KI, bool W2>
__device__ __forceinline__ void dq_item(const DqParams& a, const DqTable& tb, const uint8_t* c0, const uint8_t* c1,
                                        const uint8_t* s0, const uint8_t* s1, const uint4* xs, int lane, int j0,
                                        int np, int r0, int nrow, int col0, float bias, float* partial) {
  // groups of up to four ranks, each with its own unrolled kernel
  for (int g = 0; g < np; g += 4) {
    switch (min(4, np - g)) {
#define DQ_CASE(N)                                                                                \
  case N:                                                                                         \
    if (W2)                                                                                       \
      dq_w2_item<KI, N>(a, tb, c0, c1, s0, s1, xs, lane, j0 + g, r0, nrow, col0, bias, partial); \
    else                                                                                          \
      dq_w1_item<KI, N>(a, tb, c0, c1, s0, s1, xs, lane, j0 + g, r0, bias);                      \
    break;
      DQ_CASE(1)
      DQ_CASE(2)
      DQ_CASE(3)
      DQ_CASE(4)
#undef DQ_CASE
    }
  }
}

template <int KI>
__global__ void __launch_bounds__(kDqThreads, 1) mxmoe_dqgemv_ffn_kernel(const DqParams a) {
  extern __shared__ __align__(128) uint8_t dq_smem[];
  __shared__ DqTable tb;
  __shared__ __align__(8) uint64_t full_bar[kDqMaxSlots], empty_bar[kDqMaxSlots];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = a.slots;
  const uint32_t SB = a.slot_bytes;
  uint8_t* slots = dq_smem;
  uint4* xs = reinterpret_cast<uint4*>(dq_smem + static_cast<size_t>(S) * SB);
  float* partial = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(xs) + static_cast<size_t>(a.xs_rows) * KI * 2048);
  float* bias1 = partial + kDqMaxPairs * kDqMaxCols;  // [unit][GLU, linear] of the block's W1 units
  float* bias2 = bias1 + 2 * kDqMaxUnits;             // [touched expert][column] of the block's W2 columns
  const uint32_t rb1 = static_cast<uint32_t>(a.kp1) / 2, rb2 = static_cast<uint32_t>(a.kp2) / 2;
  // set-up that reads nothing from earlier kernels runs before the wait:
  // staged columns past K stay finite (zero) for the lanes that read them
  if (threadIdx.x == kDqConsumers) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], kDqWarps);
    }
    fence_barrier_init();
  }
  for (int i = threadIdx.x; i < a.xs_rows * KI * 128; i += kDqThreads) xs[i] = make_uint4(0u, 0u, 0u, 0u);
  // what the kernel reads next comes from the kernels just before
  griddep_wait();
  griddep_launch_dependents();
  DQ_T(0);
  if (warp == 0) {
    // the pairs, sorted by (expert, pair) with a rank count over the lanes
    int id = -1;
    float w = 0.0f;
    if (lane < a.P) {
      id = __ldcg(a.topk_idx + lane);
      w = __ldcg(a.topk_w + lane);
    }
    const bool ok = lane < a.P && id >= 0 && id < a.E;
    const uint32_t key = ok ? (static_cast<uint32_t>(id) << 3) | static_cast<uint32_t>(lane) : 0xFFFFFFFFu;
    int rank = 0;
#pragma unroll
    for (int j = 0; j < kDqMaxPairs; ++j) rank += __shfl_sync(0xFFFFFFFFu, key, j) < key ? 1 : 0;
    const int nv = __popc(__ballot_sync(0xFFFFFFFFu, ok));
    if (ok) {
      tb.pair[rank] = lane;
      tb.tok[rank] = lane / a.pair_k;
      tb.exp[rank] = id;
      tb.w[rank] = w;
    }
    if (lane < kDqMaxPairs) tb.ident[lane] = lane;
    __syncwarp();
    const int er = lane < nv ? tb.exp[lane] : -1;
    const int eprev = __shfl_up_sync(0xFFFFFFFFu, er, 1);
    const bool first = lane < nv && (lane == 0 || eprev != er);
    const uint32_t fm = __ballot_sync(0xFFFFFFFFu, first);
    if (first) {
      const int i = __popc(fm & ((1u << lane) - 1u));
      tb.te_exp[i] = er;
      tb.te_lo[i] = lane;
    }
    if (lane == 0) {
      tb.n = nv;
      tb.nt = __popc(fm);
      tb.te_lo[__popc(fm)] = nv;
    }
    // fused forward: block 0 writes the canonical routing maps
    if (a.fused && blockIdx.x == 0 && lane < a.P) {
      a.inv_c[lane] = ok ? rank : -1;
      if (ok) a.perm_c[rank] = lane;
    }
  }
  __syncthreads();
  DQ_T(1);
  if (a.fused && blockIdx.x == 0) {
    for (int e = threadIdx.x; e <= a.E; e += kDqThreads) {
      int c = 0;
      for (int r = 0; r < tb.n; ++r) c += tb.exp[r] < e ? 1 : 0;
      a.offsets[e] = c;
    }
  }
  const int B = gridDim.x, b = blockIdx.x, nt = tb.nt;
  const int U = nt * a.fp;
  DqWalk walk;
  // (32-bit products: U <= 8 * 4096 and d <= 4096 times at most a few hundred blocks)
  walk.u = U * b / B;
  walk.u1 = U * (b + 1) / B;
  walk.fp = a.fp;
  walk.cu = a.cu;
  walk.c0 = a.d * b / B;
  walk.c1 = a.d * (b + 1) / B;
  walk.c = walk.c0;
  walk.ei = 0;
  walk.nt = nt;
  walk.cr = a.cr;
  const int ubase = walk.u, nu = walk.u1 - walk.u;
  const int ntok = (a.P + a.pair_k - 1) / a.pair_k;  // tokens of the launch
  const int col0 = walk.c0, ncol = walk.c1 - walk.c0;
  const unsigned long long limit = a.wait_ns ? a.wait_ns : kWaitTimeoutNs;

  // The block's small reads (the W1 input rows and the biases of its rows)
  // are issued first; the weight stream is queued behind them.
  if (warp < kDqWarps) {
    if (a.xh != nullptr) dq_stage_async(xs, a.xh, tb.ident, a.d, ntok, a.d, KI);
    for (int i = threadIdx.x; i < 2 * nu; i += kDqConsumers) {
      const int u = ubase + i / 2, e = tb.te_exp[u / a.fp], m = u % a.fp;
      cp_async4(smem_u32(bias1 + i), a.b1 + static_cast<uint64_t>(e) * (2u * a.fp) + w1_packed_row(m, i & 1));
    }
    for (int i = threadIdx.x; i < nt * ncol; i += kDqConsumers) {
      const int ei = i / ncol, cc = i - ei * ncol;
      cp_async4(smem_u32(bias2 + ei * kDqMaxCols + cc), a.b2 + static_cast<uint64_t>(tb.te_exp[ei]) * a.d + col0 + cc);
    }
    cp_async_commit();
  }
  __syncthreads();

  if (warp == kDqWarps) {
    // ---------------------------------------------------------------- copy warp
    // Chunk c goes to slot c % S once the slot's previous chunk is consumed,
    // and only after chunk c - ahead has landed.
    if (lane == 0) {
      const uint64_t pol = l2_evict_first_policy();
      DqChunk ch;
      for (int c = 0; walk.next(ch); ++c) {
        const int sl = c % S, use = c / S;
        uint8_t* dst = slots + static_cast<size_t>(sl) * SB;
        if (use > 0 && !mbar_wait(&empty_bar[sl], (use - 1) & 1, a.err, kDqErrCopy, limit)) break;
        if (c >= a.ahead) {
          const int p = c - a.ahead;
          if (!mbar_wait(&full_bar[p % S], (p / S) & 1, a.err, kDqErrCopy, limit)) break;
        }
        const int e = tb.te_exp[ch.ei];
        if (!ch.w2) {
          const uint64_t base = static_cast<uint64_t>(e) * 2u * a.fp;
          const uint64_t g = base + w1_packed_row(ch.r0, 0), l = base + w1_packed_row(ch.r0, 1);
          const uint32_t cb = ch.len * rb1, sb = ch.len * a.sr1;
          mbar_arrive_expect_tx(&full_bar[sl], 2u * (cb + sb));
          bulk_load_hint(dst, a.w1q + g * rb1, cb, &full_bar[sl], pol);
          bulk_load_hint(dst + a.cu * rb1, a.w1q + l * rb1, cb, &full_bar[sl], pol);
          bulk_load_hint(dst + 2u * a.cu * rb1, a.w1sr + g * a.sr1, sb, &full_bar[sl], pol);
          bulk_load_hint(dst + 2u * a.cu * rb1 + a.cu * a.sr1, a.w1sr + l * a.sr1, sb, &full_bar[sl], pol);
        } else {
          const uint64_t row = static_cast<uint64_t>(e) * a.d + ch.r0;
          const uint32_t cb = ch.len * rb2, sb = ch.len * a.sr2;
          mbar_arrive_expect_tx(&full_bar[sl], cb + sb);
          bulk_load_hint(dst, a.w2q + row * rb2, cb, &full_bar[sl], pol);
          bulk_load_hint(dst + a.cr * rb2, a.w2sr + row * a.sr2, sb, &full_bar[sl], pol);
        }
      }
    }
    return;
  }

  // ------------------------------------------------------------------ compute warps
  // W1 input: the router's f16 token rows (copies above), or x normalized here
  if (a.xh == nullptr) dq_stage_x(xs, a, ntok, KI);
  cp_async_wait_all();
  dq_bar();
  DQ_T(2);
  // The grid barrier: every block's SwiGLU rows are written before any block
  // reads them; then the block stages its pairs' SwiGLU rows.
  auto grid_barrier = [&]() {
    dq_bar();  // this block's act writes are done
    if (threadIdx.x == 0) {
      __threadfence();
      // (test hook: block 0 stays silent, so every block's wait runs out)
      if (!(a.skip_arrival && blockIdx.x == 0)) atomicAdd(a.sync, 1);
      const unsigned long long t0 = global_timer_ns();
      while (true) {
        int v;
        asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(a.sync) : "memory");
        if (v >= static_cast<int>(gridDim.x)) break;
        if (global_timer_ns() - t0 > limit) {
          // the first timeout also records the arrivals seen and expected
          if (atomicCAS(a.err, 0, kDqErrGrid) == 0) {
            a.err[2] = -1;
            a.err[3] = v;
            a.err[4] = static_cast<int>(gridDim.x);
          }
          break;
        }
      }
    }
    dq_bar();
    DQ_T(4);
    dq_stage_async(xs, a.act, tb.pair, a.fp, tb.n, a.fp, KI);
    cp_async_commit();
    cp_async_wait_all();
    dq_bar();
    DQ_T(5);
  };
  // Items go to the compute warps round robin over the block's whole W1 unit
  // sequence (then its W2 column pairs), so chunks smaller than 16 items
  // still keep every warp busy; every warp releases every chunk.
  DqChunk ch;
  bool in_w2 = false;
  int item0 = 0;  // block-relative index of the chunk's first item
  for (int c = 0; walk.next(ch); ++c) {
    if (ch.w2 && !in_w2) {
      DQ_T(3);
      grid_barrier();
      in_w2 = true;
      item0 = 0;
    }
    const int sl = c % S;
    const uint8_t* sb = slots + static_cast<size_t>(sl) * SB;
    const int j0 = tb.te_lo[ch.ei], np = tb.te_lo[ch.ei + 1] - j0;
    const int nitem = ch.w2 ? (ch.len + 1) / 2 : ch.len;
    const int first = (warp - item0 % kDqWarps + kDqWarps) % kDqWarps;
    if (first < nitem) mbar_wait(&full_bar[sl], (c / S) & 1, a.err, kDqErrCopy, limit);
    if (!ch.w2) {
      const uint8_t* sc = sb + 2u * a.cu * rb1;
      for (int i = first; i < nitem; i += kDqWarps) {
        const int m = ch.r0 + i, j = item0 + i;
        const float bias = lane < kDqRows ? bias1[2 * j + lane] : 0.0f;
        dq_item<KI, false>(a, tb, sb + i * rb1, sb + (a.cu + i) * rb1, sc + i * a.sr1, sc + (a.cu + i) * a.sr1, xs,
                           lane, j0, np, m, 2, col0, bias, partial);
      }
    } else {
      const uint8_t* sc = sb + a.cr * rb2;
      for (int i = first; i < nitem; i += kDqWarps) {
        const int r = 2 * i, nrow = min(2, ch.len - r), r1 = r + nrow - 1, col = ch.r0 + r;
        const float bias = lane < nrow ? bias2[ch.ei * kDqMaxCols + col - col0 + lane] * a.bias_mult : 0.0f;
        dq_item<KI, true>(a, tb, sb + r * rb2, sb + r1 * rb2, sc + r * a.sr2, sc + r1 * a.sr2, xs, lane, j0, np, col,
                          nrow, col0, bias, partial);
      }
    }
    item0 += nitem;
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty_bar[sl]);
  }
  if (!in_w2) grid_barrier();  // a block without W2 rows still meets the others
  if (!a.fused) return;
  // fused forward: y = x + the pairs' rows of each token in increasing expert order
  dq_bar();
  for (int idx = threadIdx.x; idx < a.n_tok * ncol; idx += kDqConsumers) {
    const int t = idx / ncol, cc = idx - t * ncol, col = col0 + cc;
    float acc = 0.0f;
    for (int r = 0; r < tb.n; ++r)
      if (tb.tok[r] == t) acc = __fadd_rn(acc, partial[r * kDqMaxCols + cc]);
    const uint64_t o = static_cast<uint64_t>(t) * a.d + col;
    if (a.residual) {
      const float xv = a.x_dtype == kDqSrcF32 ? __ldg(static_cast<const float*>(a.x) + o)
                                              : __bfloat162float(__ldg(static_cast<const __nv_bfloat16*>(a.x) + o));
      acc = __fadd_rn(xv, acc);
    }
    if (a.y_dtype == kDqSrcF32)
      static_cast<float*>(a.y)[o] = acc;
    else
      static_cast<__nv_bfloat16*>(a.y)[o] = __float2bfloat16_rn(acc);
  }
  DQ_T(6);
}

// Cooperative launch: the blocks meet between W1 and W2, so all of them must
// be resident at once.
template <int KI>
cudaError_t dq_launch(const DqParams& a, size_t smem, int grid, cudaStream_t st) {
  const auto fn = mxmoe_dqgemv_ffn_kernel<KI>;
  const cudaError_t e = ensure_dynamic_smem(reinterpret_cast<const void*>(fn), smem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kDqThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2]{};
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  // a runtime that refuses the two attributes together gets the cooperative
  // launch alone (the kernel then starts after the router completes)
  static bool pdl_refused = false;
  cfg.numAttrs = pdl_enabled() && !pdl_refused ? 2 : 1;
  cudaError_t r = cudaLaunchKernelEx(&cfg, fn, a);
  if (r != cudaSuccess && cfg.numAttrs == 2 && r != cudaErrorStreamCaptureInvalidated &&
      r != cudaErrorStreamCaptureUnsupported) {
    cudaGetLastError();
    pdl_refused = true;
    cfg.numAttrs = 1;
    r = cudaLaunchKernelEx(&cfg, fn, a);
  }
  return r;
}

}  // namespace

#ifdef MXMOE_DQ_TRACE
extern "C" __attribute__((visibility("default"))) int mxmoe_dq_trace_dump(unsigned long long* host, size_t n) {
  return cudaMemcpyFromSymbol(host, g_dq_trace, n * sizeof(unsigned long long)) == cudaSuccess ? 0 : 1;
}
extern "C" __attribute__((visibility("default"))) int mxmoe_dq_trace_clear() {
  static unsigned long long zero[160 * 17 * kDqTraceSlots];
  return cudaMemcpyToSymbol(g_dq_trace, zero, sizeof(zero)) == cudaSuccess ? 0 : 1;
}
#endif

cudaError_t launch_dqgemv_ffn(DqParams a, int num_sms, size_t smem_limit, cudaStream_t st) {
  const int grid = num_sms;
  if (a.d % 32 != 0 || a.fp % 64 != 0 || a.d > kDqMaxK || a.fp > kDqMaxK || a.P < 0 || a.P > kDqMaxPairs ||
      grid <= 0 || a.d > kDqMaxCols * grid || (kDqMaxPairs * a.fp + grid - 1) / grid > kDqMaxUnits)
    return cudaErrorInvalidValue;
  const uint32_t rb1 = static_cast<uint32_t>(a.kp1) / 2, rb2 = static_cast<uint32_t>(a.kp2) / 2;
  const uint32_t unit = 2u * (rb1 + a.sr1), row2 = rb2 + a.sr2;
  const int ki = (std::max(a.d, a.fp) / 32 + 31) / 32;
  a.xs_rows = dq_pow2(std::max(a.P, 1));
  const size_t fixed = static_cast<size_t>(a.xs_rows) * ki * 2048 + kDqScratchFloats * sizeof(float);
  const size_t budget = smem_limit > fixed + 2048 ? smem_limit - fixed - 2048 : 0;
  // Chunks of 8 GLU units (two chunks feed the 16 compute warps); about 48 KB
  // in flight per SM, the rest of the ring holding landed chunks.
  a.slots = 0;
  for (int cu : {8, 4, 2, 1}) {
    const uint32_t sb = (std::max(cu * unit, 2u * row2) + 127u) / 128u * 128u;
    const int s = static_cast<int>(std::min<size_t>(kDqMaxSlots, budget / sb));
    if (s >= 3 || (cu == 1 && s >= 2)) {
      a.cu = cu;
      a.slot_bytes = sb;
      a.slots = s;
      break;
    }
  }
  if (a.slots == 0) return cudaErrorInvalidValue;
  a.cr = static_cast<int>(a.slot_bytes / row2) & ~1;
  a.ahead = std::max(1, std::min(a.slots - 1, static_cast<int>((48u * 1024u + a.slot_bytes - 1) / a.slot_bytes)));
  const size_t smem = static_cast<size_t>(a.slots) * a.slot_bytes + fixed;
  switch (ki) {
    case 1: return dq_launch<1>(a, smem, grid, st);
    case 2: return dq_launch<2>(a, smem, grid, st);
    case 3: return dq_launch<3>(a, smem, grid, st);
    default: return dq_launch<4>(a, smem, grid, st);
  }
}

}  // namespace mxmoe
