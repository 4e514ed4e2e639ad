// dqgemv.cu -- fused MXFP4 dequant-GEMV expert FFN for decode batches (at
// most a few routed pairs), on CUDA cores: W1 + SwiGLU-clamp and W2 + bias +
// route weight in one launch.
//
// Replaces, for few-token batches, the per-element byte-wise dequant loops of
// w1_swiglu_dense_kernel / w2_scatter_dense_kernel (src/quant/gpu.rs:89-192):
// there every token-row thread re-reads each weight byte and recomputes
// exp(s * ln 2) per element; here each weight byte crosses HBM once per
// forward, is decoded two codes per instruction, and serves every routed pair
// of its expert.
//
// Work split (no host sync): one block per SM.  Each block finds the experts
// with routed pairs, serves expert b % nt of the nt touched ones, and walks
// that expert's W1 and then W2 row items with the other blocks of the same
// expert (block-strided).  Untouched experts cost nothing.
//
// Block = 16 warps, each streaming its own items through a private ring of
// shared-memory stages with 16-byte cp.async copies (L2 evict-first): D - 1
// items in flight while one is computed.  An item is two weight rows (W1: a
// GLU unit's GLU and linear row; W2: output columns 2m, 2m + 1) with their
// E8M0 scale rows (a row-major copy of the scales kept for this kernel).
// Items are taken in order from a per-block counter; W2's weights are
// already arriving while the last W1 items are computed.
//
// Math: lane l covers the 32-column blocks kb = l + 32 i of both rows (one
// 16-byte code load each, conflict-free), decodes them with
// cvt.rn.f16x2.e2m1x2 and multiplies with `fma.rn.f32.f16` against the
// activation rows staged in shared memory as f16: the E2M1 value times the
// f16 activation is exact, the sum is f32.  Per block the sum is scaled once
// by 2^(s - 127); the warp then reduces all (row, pair) sums at once by
// halving exchanges.  The K loop is unrolled at compile time (KI blocks per
// lane) and the pair count is dispatched to unrolled variants, so the
// instruction stream has no runtime predicates or divergent branches.
//
// Activations: W1 stages the router's normalized token rows (x * (1/rms) *
// gamma as f16, written by the router), W2 the f16 SwiGLU rows W1 wrote;
// both carry a power of two that keeps them in f16's normal range (|x_hat| <=
// sqrt(d) * max|gamma| after RmsNorm; |act| <= max(limit, 0.28 / alpha) *
// (limit + 1) after the clamp).  The swizzle puts lane l's four 16-byte pieces
// of a 32-column block 512 bytes apart, so a quarter warp reads 128
// contiguous bytes.  The staged rows are copied before the weight stream
// starts: behind it they would wait for every SM's weight requests.
//
// W1 -> W2: W2 needs every SwiGLU column of its expert, written by all blocks
// of that expert.  The blocks meet on a per-expert arrival counter in global
// memory, zeroed before every forward.  The launch is cooperative (all blocks
// resident at once), and the wait is bounded: on timeout it records a status
// code and the kernel carries on to its end.
//
// Fused mode (mxmoe_forward): no permutation kernel runs before this one; the
// blocks take their pairs from the canonical top-k ids, and the last block to
// finish adds each token's pair rows in increasing expert order plus the
// residual and writes the canonical routing maps.  The forward is then the
// router and this kernel.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>

#include "kernels.h"
#include "launch_util.h"
#include "layout.cuh"
#include "ptx.cuh"

namespace mxmoe {

namespace {

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

constexpr int kDqWarps = 16;  // warps per block
constexpr int kDqThreads = 32 * kDqWarps;
constexpr int kDqRows = 2;  // weight rows per item
// status codes of this kernel (the layer's status word)
constexpr int kDqErrExpert = 8;  // the blocks of an expert did not all finish W1 in time

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

// a0 += the even-column products, a1 += the odd ones, over 8 columns: w (four
// f16x2 weights) times x (four f16x2 activations), exact products, f32 sums.
__device__ __forceinline__ void fma8_f16_f32(float& a0, float& a1, const uint32_t (&w)[4], uint4 x) {
  asm("{\n\t.reg .f16 wl0, wh0, wl1, wh1, wl2, wh2, wl3, wh3, xl0, xh0, xl1, xh1, xl2, xh2, xl3, xh3;\n\t"
      "mov.b32 {wl0, wh0}, %2;\n\t"
      "mov.b32 {wl1, wh1}, %3;\n\t"
      "mov.b32 {wl2, wh2}, %4;\n\t"
      "mov.b32 {wl3, wh3}, %5;\n\t"
      "mov.b32 {xl0, xh0}, %6;\n\t"
      "mov.b32 {xl1, xh1}, %7;\n\t"
      "mov.b32 {xl2, xh2}, %8;\n\t"
      "mov.b32 {xl3, xh3}, %9;\n\t"
      "fma.rn.f32.f16 %0, wl0, xl0, %0;\n\t"
      "fma.rn.f32.f16 %1, wh0, xh0, %1;\n\t"
      "fma.rn.f32.f16 %0, wl1, xl1, %0;\n\t"
      "fma.rn.f32.f16 %1, wh1, xh1, %1;\n\t"
      "fma.rn.f32.f16 %0, wl2, xl2, %0;\n\t"
      "fma.rn.f32.f16 %1, wh2, xh2, %1;\n\t"
      "fma.rn.f32.f16 %0, wl3, xl3, %0;\n\t"
      "fma.rn.f32.f16 %1, wh3, xh3, %1;\n\t}"
      : "+f"(a0), "+f"(a1)
      : "r"(w[0]), "r"(w[1]), "r"(w[2]), "r"(w[3]), "r"(x.x), "r"(x.y), "r"(x.z), "r"(x.w));
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


struct DqSlot {
  int e;     // local expert
  int g, G;  // this block's index among the G blocks of its expert
};

// The touched experts (count > 0) in increasing index are numbered 0..nt-1;
// block b serves number b % nt as block b / nt of its group.  Every warp
// computes the same answer.  Counts are read through L2.
__device__ __forceinline__ bool dq_find_slot(const int32_t* counts, int E, const int (&cnt_r)[4], DqSlot& s) {
  const int lane = threadIdx.x & 31;
  // experts below 128 come from the preloaded counts, the rest are loaded
  uint32_t mask[4];
  int nt = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    mask[i] = __ballot_sync(0xFFFFFFFFu, cnt_r[i] > 0);
    nt += __popc(mask[i]);
  }
  for (int base = 128; base < E; base += 32) {
    const int e = base + lane;
    nt += __popc(__ballot_sync(0xFFFFFFFFu, e < E && __ldcg(counts + e) > 0));
  }
  if (nt == 0) return false;
  const int B = gridDim.x, b = blockIdx.x;
  const int slot = b % nt;
  s.g = b / nt;
  s.G = (B - slot + nt - 1) / nt;
  int seen = 0;
  for (int base = 0; base < E; base += 32) {
    const int e = base + lane;
    uint32_t m = 0;
    if (base < 128) {
#pragma unroll
      for (int i = 0; i < 4; ++i)
        if (base == 32 * i) m = mask[i];
    } else {
      m = __ballot_sync(0xFFFFFFFFu, e < E && __ldcg(counts + e) > 0);
    }
    const int n = __popc(m);
    if (slot < seen + n) {
      for (int r = slot - seen; r > 0; --r) m &= m - 1;
      s.e = base + __ffs(m) - 1;
      return true;
    }
    seen += n;
  }
  return false;
}

// Position of the r-th set bit (r < popc(m)).
__device__ __forceinline__ int dq_nth_bit(uint32_t m, int r) {
  for (; r > 0; --r) m &= m - 1;
  return __ffs(m) - 1;
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

// Synchronous W1 staging from the token rows x (when no f16 rows were
// prepared): np rows of x * (1/rms) * gamma * x_scale as f16, in dq_piece
// order.  Piece p of a row is (kb = p / 4, q = p % 4): consecutive threads
// read consecutive 16-byte pieces of the source row.
__device__ void dq_stage_x(uint4* xs, const DqParams& a, int ki, int p0, int base, int np) {
  const int kbr = a.d / 32;
  for (int j = 0; j < np; ++j) {
    const int t = __ldcg(a.perm + p0 + base + j) / a.pair_k;
    const float rs = __ldcg(a.rscale + t) * a.x_scale;
    for (int p = threadIdx.x; p < 4 * kbr; p += kDqThreads) {
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
      xs[dq_piece(j, ki, kb, q)] = o;
    }
  }
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
// Asynchronous staging of np f16 rows of K columns into xs (dq_piece order),
// row j at rows[j] (shared memory, filled by the caller): one 16-byte copy per
// piece, issued by all threads; the caller commits and waits.
__device__ __forceinline__ void dq_stage_async(uint4* xs, const __half* const* rows, int K, int ki, int np) {
  const int kbr = K / 32;
  for (int j = 0; j < np; ++j) {
    const __half* src = rows[j];
    for (int p = threadIdx.x; p < 4 * kbr; p += kDqThreads) {
      const int kb = p >> 2, q = p & 3;
      cp_async16(smem_u32(xs + dq_piece(j, ki, kb, q)), src + kb * 32 + q * 8);
    }
  }
}

// Item t of a block's sequence: W1 items (passes x c1), then W2 items (passes x c2).
struct DqItem {
  bool w2;
  int pass, m;
};
__device__ __forceinline__ DqItem dq_item(int t, int n1, int c1, int c2, int g, int G, int passes) {
  DqItem it;
  it.w2 = t >= n1;
  const int u = it.w2 ? t - n1 : t;
  const int c = it.w2 ? c2 : c1;
  it.pass = passes == 1 ? 0 : u / c;  // one pass is the common case: no division
  it.m = g + (u - it.pass * c) * G;
  return it;
}

// Weight rows of an item: W1 item m = GLU unit m (its GLU row, then its
// linear row, in the packed order); W2 item m = output columns 2m, 2m + 1.
__device__ __forceinline__ uint32_t dq_row(const DqItem& it, int r) {
  return it.w2 ? 2u * it.m + r : w1_packed_row(static_cast<uint32_t>(it.m), static_cast<uint32_t>(r));
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint64_t pol) {
  asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "l"(pol)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// The warp's copies of item t into its stage buffer: the codes of the two
// rows, then their scale rows, 16 bytes per lane and instruction.
__device__ __forceinline__ void dq_issue(const DqParams& a, int e, const DqItem& it, uint8_t* buf, int lane,
                                         uint64_t pol) {
  const uint32_t rb = static_cast<uint32_t>(it.w2 ? a.kp2 : a.kp1) / 2, sr = it.w2 ? a.sr2 : a.sr1;
  const uint32_t rows = it.w2 ? static_cast<uint32_t>(a.d) : 2u * a.fp;
  const uint8_t* q = (it.w2 ? a.w2q : a.w1q) + static_cast<uint64_t>(e) * rows * rb;
  const uint8_t* sc = (it.w2 ? a.w2sr : a.w1sr) + static_cast<uint64_t>(e) * rows * sr;
  const uint32_t dst = smem_u32(buf);
#pragma unroll
  for (int r = 0; r < kDqRows; ++r) {
    const uint64_t row = dq_row(it, r);
    for (uint32_t k = lane * 16u; k < rb; k += 512u) cp_async16(dst + r * rb + k, q + row * rb + k, pol);
    for (uint32_t k = lane * 16u; k < sr; k += 512u) cp_async16(dst + kDqRows * rb + r * sr + k, sc + row * sr + k, pol);
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

__host__ __device__ constexpr int dq_pow2(int n) { return n <= 1 ? 1 : n <= 2 ? 2 : n <= 4 ? 4 : 8; }

// Dot products of the item's two weight rows (stage buffer sb) with staged
// rows j0 .. j0 + NP - 1, reduced over the warp: lane L returns the sum of
// (row (L % V) / NPP, pair L % NPP), V = 2 * NPP.  Fully unrolled over the
// KI 32-column blocks of a lane; lanes past the last block read zero codes.
template <int KI, int NP>
__device__ __forceinline__ float dq_dot(const uint8_t* sb, uint32_t rb, uint32_t sr, const uint4* xs, int kbr,
                                        int lane, int j0) {
  constexpr int NPP = dq_pow2(NP);
  float acc[kDqRows * NPP];
#pragma unroll
  for (int i = 0; i < kDqRows * NPP; ++i) acc[i] = 0.0f;
#pragma unroll
  for (int i = 0; i < KI; ++i) {
    const int kb = lane + 32 * i;
    const bool ok = kb < kbr;
    uint32_t h[kDqRows][4][4];
    float sc[kDqRows];
#pragma unroll
    for (int r = 0; r < kDqRows; ++r) {
      uint4 cw = make_uint4(0u, 0u, 0u, 0u);
      if (ok) cw = *reinterpret_cast<const uint4*>(sb + r * rb + kb * 16);
      e2m1x8_to_f16x2(cw.x, h[r][0]);
      e2m1x8_to_f16x2(cw.y, h[r][1]);
      e2m1x8_to_f16x2(cw.z, h[r][2]);
      e2m1x8_to_f16x2(cw.w, h[r][3]);
      sc[r] = ok ? e8m0_to_f32(sb[kDqRows * rb + r * sr + kb]) : 0.0f;
    }
#pragma unroll
    for (int j = 0; j < NP; ++j) {
      uint4 xv[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) xv[q] = xs[dq_piece(j0 + j, KI, kb, q)];
#pragma unroll
      for (int r = 0; r < kDqRows; ++r) {
        float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;  // four short chains
        fma8_f16_f32(a0, a1, h[r][0], xv[0]);
        fma8_f16_f32(a2, a3, h[r][1], xv[1]);
        fma8_f16_f32(a0, a1, h[r][2], xv[2]);
        fma8_f16_f32(a2, a3, h[r][3], xv[3]);
        acc[r * NPP + j] = fmaf((a0 + a1) + (a2 + a3), sc[r], acc[r * NPP + j]);
      }
    }
  }
  return dq_warp_reduce<kDqRows * NPP>(acc, lane);
}

// One item's outputs for staged rows j0 .. j0 + NP - 1 of its pass.
template <int KI, int NP>
__device__ __forceinline__ void dq_finish(const DqParams& a, const DqItem& it, const uint8_t* sb, const uint4* xs,
                                          const float* rw, const int* pos_s, int lane, int j0, float bias) {
  constexpr int NPP = dq_pow2(NP);
  const uint32_t rb = static_cast<uint32_t>(it.w2 ? a.kp2 : a.kp1) / 2, sr = it.w2 ? a.sr2 : a.sr1;
  const int kbr = (it.w2 ? a.fp : a.d) / 32;
  const float v = dq_dot<KI, NP>(sb, rb, sr, xs, kbr, lane, j0);
  const int vi = lane % (kDqRows * NPP), r = vi / NPP, j = vi % NPP;
  const float br = __shfl_sync(0xFFFFFFFFu, bias, r);
  if (!it.w2) {
    // lane j (< NPP) holds the GLU row's sum of pair j, lane NPP + j the linear row's
    const float vl = __shfl_sync(0xFFFFFFFFu, v, (lane + NPP) & 31);
    const float bl = __shfl_sync(0xFFFFFFFFu, bias, 1);
    if (lane < NP) {
      const float xg = fminf(v * a.inv_x_scale + br, a.limit);
      const float xl = fmaxf(-a.limit, fminf(vl * a.inv_x_scale + bl, a.limit));
      const float act = (xg / (1.0f + expf(-a.alpha * xg))) * (xl + 1.0f);
      a.act[static_cast<uint64_t>(pos_s[j0 + lane]) * a.fp + it.m] = __float2half_rn(act * a.act_scale);
    }
  } else if (lane < kDqRows * NPP && j < NP) {
    a.y_pair[static_cast<uint64_t>(pos_s[j0 + j]) * a.d + 2 * it.m + r] = (v * a.inv_act_scale + br) * rw[j0 + j];
  }
}

// D: stage buffers per warp (D - 1 items in flight while one is computed).
// Fused mode (a.fused, at most 64 routed pairs): no permutation kernel runs
// before this one.  Each block derives the touched experts and its expert's
// pairs from the canonical top-k ids; act and y_pair rows are indexed by the
// canonical pair t * k + s; the last block to finish adds the k pair rows of
// every token in increasing expert order (plus the residual), as the combine
// kernel does, and writes the canonical routing maps (offsets, perm, inv).
__device__ void dq_combine_and_maps(const DqParams& a, const int32_t* tk_s) {
  const int P = a.P, k = a.pair_k, n = a.n_tok, d = a.d;
  // canonical maps: stable sort of the pairs by expert id
  for (int e = threadIdx.x; e <= a.E; e += kDqThreads) {
    int c = 0;
    for (int p = 0; p < P; ++p) c += tk_s[p] < e;
    a.offsets[e] = c;
  }
  for (int p = threadIdx.x; p < P; p += kDqThreads) {
    const int id = tk_s[p];
    int pos = 0;
    for (int q = 0; q < P; ++q) pos += tk_s[q] < id || (tk_s[q] == id && q < p);
    a.perm_c[pos] = p;
    a.inv_c[p] = pos;
  }
  // y[t] = x[t] + sum over the token's pairs in increasing expert order
  const int c4 = d / 4;
  for (int i = threadIdx.x; i < n * c4; i += kDqThreads) {
    const int t = i / c4, c = (i - t * c4) * 4;
    int ord[kMaxTopK], ex[kMaxTopK];
    for (int q = 0; q < k; ++q) {
      ord[q] = t * k + q;
      ex[q] = tk_s[t * k + q];
    }
    for (int q = 1; q < k; ++q)
      for (int b = q; b > 0 && ex[b - 1] > ex[b]; --b) {
        int tmp = ex[b]; ex[b] = ex[b - 1]; ex[b - 1] = tmp;
        tmp = ord[b]; ord[b] = ord[b - 1]; ord[b - 1] = tmp;
      }
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int q = 0; q < k; ++q) {
      const float4 v = __ldcg(reinterpret_cast<const float4*>(a.y_pair + static_cast<uint64_t>(ord[q]) * d + c));
      acc.x = __fadd_rn(acc.x, v.x); acc.y = __fadd_rn(acc.y, v.y);
      acc.z = __fadd_rn(acc.z, v.z); acc.w = __fadd_rn(acc.w, v.w);
    }
    if (a.residual) {
      float xv[4];
      if (a.x_dtype == kDqSrcF32) {
        const float4 f = __ldg(reinterpret_cast<const float4*>(static_cast<const float*>(a.x) + static_cast<uint64_t>(t) * d + c));
        xv[0] = f.x; xv[1] = f.y; xv[2] = f.z; xv[3] = f.w;
      } else {
        const uint2 u = __ldg(reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(a.x) + static_cast<uint64_t>(t) * d + c));
        xv[0] = __uint_as_float(u.x << 16); xv[1] = __uint_as_float(u.x & 0xFFFF0000u);
        xv[2] = __uint_as_float(u.y << 16); xv[3] = __uint_as_float(u.y & 0xFFFF0000u);
      }
      acc.x = __fadd_rn(xv[0], acc.x); acc.y = __fadd_rn(xv[1], acc.y);
      acc.z = __fadd_rn(xv[2], acc.z); acc.w = __fadd_rn(xv[3], acc.w);
    }
    if (a.y_dtype == kDqSrcF32) {
      *reinterpret_cast<float4*>(static_cast<float*>(a.y) + static_cast<uint64_t>(t) * d + c) = acc;
    } else {
      const __nv_bfloat162 lo = __floats2bfloat162_rn(acc.x, acc.y), hi = __floats2bfloat162_rn(acc.z, acc.w);
      *reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(a.y) + static_cast<uint64_t>(t) * d + c) =
          make_uint2(*reinterpret_cast<const uint32_t*>(&lo), *reinterpret_cast<const uint32_t*>(&hi));
    }
  }
}

// D: stage buffers per warp (D - 1 items in flight while one is computed).
template <int D, int KI>
__global__ void __launch_bounds__(kDqThreads, 1) mxmoe_dqgemv_ffn_kernel(const DqParams a) {
  extern __shared__ __align__(128) uint8_t dq_smem[];
  __shared__ uint32_t present[32];  // fused mode: touched experts (E <= 1024) as a bit set
  __shared__ int32_t tk_s[64];      // fused mode: the canonical top-k ids
  __shared__ int last_block;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int ki = KI;  // 32-column blocks per lane (staged row stride: KI * 1024 columns)
  uint4* xs = reinterpret_cast<uint4*>(dq_smem + static_cast<size_t>(kDqWarps) * D * a.stage_bytes);
  float* rw = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(xs) + static_cast<size_t>(a.ps) * ki * 2048);
  int* pos_s = reinterpret_cast<int*>(rw + 16);
  const __half** rows_s = reinterpret_cast<const __half**>(pos_s + 16);
  int* next = reinterpret_cast<int*>(rows_s + 16);
  // set-up that reads nothing from earlier kernels runs before the wait:
  // staged columns past K stay finite (zero) for the lanes that read them
  if (threadIdx.x == 0) *next = 0;
  if (threadIdx.x < 32) present[threadIdx.x] = 0u;
  for (int i = threadIdx.x; i < a.ps * KI * 128; i += kDqThreads) xs[i] = make_uint4(0u, 0u, 0u, 0u);
  // what the kernel reads next comes from the kernels just before
  griddep_wait();
  griddep_launch_dependents();
  DQ_T(0);
  DqSlot s;
  int e, cnt, p0;
  uint32_t pm[2] = {0u, 0u};  // the expert's pairs among the (at most 64) routed pairs
  if (a.fused) {
    if (threadIdx.x < a.P) {
      const int id = __ldcg(a.topk_idx + threadIdx.x);
      tk_s[threadIdx.x] = id;
      atomicOr(&present[id >> 5], 1u << (id & 31));
    }
    __syncthreads();
    // touched experts in increasing index: number b % nt serves this block
    const uint32_t w = present[lane];
    int pre = __popc(w);
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xFFFFFFFFu, pre, o);
      if (lane >= o) pre += v;
    }
    const int nt = __shfl_sync(0xFFFFFFFFu, pre, 31);
    const int slot = blockIdx.x % nt;
    s.g = blockIdx.x / nt;
    s.G = (gridDim.x - slot + nt - 1) / nt;
    const uint32_t hit = __ballot_sync(0xFFFFFFFFu, pre > slot);
    const int wl = __ffs(hit) - 1;  // word holding the slot-th touched expert
    const int before = __shfl_sync(0xFFFFFFFFu, pre - __popc(w), wl);
    e = 32 * wl + dq_nth_bit(__shfl_sync(0xFFFFFFFFu, w, wl), slot - before);
#pragma unroll
    for (int i = 0; i < 2; ++i) pm[i] = __ballot_sync(0xFFFFFFFFu, 32 * i + lane < a.P && tk_s[32 * i + lane] == e);
    cnt = __popc(pm[0]) + __popc(pm[1]);
    p0 = 0;
  } else {
    // one round of independent loads: the pair counts and offsets of up to
    // 128 experts
    constexpr int kCR = 4;
    int cnt_r[kCR], off_r[kCR];
#pragma unroll
    for (int i = 0; i < kCR; ++i) {
      const int ex = 32 * i + lane;
      cnt_r[i] = ex < a.E ? __ldcg(a.counts + ex) : 0;
      off_r[i] = ex < a.E ? __ldcg(a.poff + ex) : 0;
    }
    if (!dq_find_slot(a.counts, a.E, cnt_r, s)) return;
    e = s.e;
    if (e < 32 * kCR) {
      int c = 0, o = 0;
#pragma unroll
      for (int i = 0; i < kCR; ++i)
        if (e / 32 == i) {
          c = cnt_r[i];
          o = off_r[i];
        }
      cnt = __shfl_sync(0xFFFFFFFFu, c, e & 31);
      p0 = __shfl_sync(0xFFFFFFFFu, o, e & 31);
    } else {
      cnt = __ldcg(a.counts + e);
      p0 = __ldcg(a.poff + e);
    }
  }
  DQ_T(1);
  const int passes = (cnt + a.ps - 1) / a.ps;
  const int items1 = a.fp, items2 = a.d / 2;
  const int c1 = s.g < items1 ? (items1 - s.g + s.G - 1) / s.G : 0;
  const int c2 = s.g < items2 ? (items2 - s.g + s.G - 1) / s.G : 0;
  const int n1 = passes * c1, total = n1 + passes * c2;
  uint8_t* ring = dq_smem + static_cast<size_t>(warp) * D * a.stage_bytes;
  DQ_T(60);
  // Stages one pass's activation rows: W1 the router's f16 token rows (or,
  // without them, x normalized here), W2 the SwiGLU rows; the rows' pair
  // positions go to pos_s and their route weights to rw.  Copies are
  // committed as one group.
  auto stage = [&](bool w2, int pass) {
    const int base = pass * a.ps, np = min(a.ps, cnt - base);
    __syncthreads();  // the previous pass's rows (and the zero fill) are done with
    if (threadIdx.x < np) {
      const int r = base + threadIdx.x;
      int pair, pos;
      if (a.fused) {
        const int c0 = __popc(pm[0]);
        pair = r < c0 ? dq_nth_bit(pm[0], r) : 32 + dq_nth_bit(pm[1], r - c0);
        pos = pair;
      } else {
        pos = p0 + r;
        pair = __ldcg(a.perm + pos);
      }
      pos_s[threadIdx.x] = pos;
      rows_s[threadIdx.x] = w2 ? a.act + static_cast<uint64_t>(pos) * a.fp
                               : (a.xh ? a.xh + static_cast<uint64_t>(pair / a.pair_k) * a.d : nullptr);
      if (w2) rw[threadIdx.x] = __ldg(a.topk_w + pair);
    }
    __syncthreads();
    if (!w2 && a.xh == nullptr)
      dq_stage_x(xs, a, ki, p0, base, np);
    else
      dq_stage_async(xs, rows_s, w2 ? a.fp : a.d, ki, np);
    cp_async_commit();
  };
  stage(false, 0);
  const uint64_t pol = l2_evict_first_policy();
  auto claim = [&]() {
    int t = 0;
    if (lane == 0) t = atomicAdd(next, 1);
    return __shfl_sync(0xFFFFFFFFu, t, 0);
  };
  // The staged rows land first: issued after the weight stream they would
  // queue behind every SM's weight requests (microseconds), issued alone they
  // take one round trip.  Then the warp's pipeline is primed with D - 1 items.
  cp_async_wait<0>();
  DQ_T(62);
  int queue[D];
#pragma unroll
  for (int q = 0; q < D - 1; ++q) {
    queue[q] = claim();
    if (queue[q] < total)
      dq_issue(a, e, dq_item(queue[q], n1, c1, c2, s.g, s.G, passes), ring + q * a.stage_bytes, lane, pol);
    cp_async_commit();
  }
  const int nphases = 2 * passes;
  DQ_T(2);
  __syncthreads();
  DQ_T(3);
  int nitem = 0;
  int phase = 0;
  int* arrive = a.sync + e;  // zeroed before every forward
  for (int seq = 0;; ++seq) {
    // keep D - 1 items in flight: claim and issue one more, then wait for the oldest
    queue[D - 1] = claim();
    if (queue[D - 1] < total)
      dq_issue(a, e, dq_item(queue[D - 1], n1, c1, c2, s.g, s.G, passes), ring + ((seq + D - 1) % D) * a.stage_bytes,
               lane, pol);
    cp_async_commit();
    const int t = queue[0];
#pragma unroll
    for (int q = 0; q < D - 1; ++q) queue[q] = queue[q + 1];
    const DqItem it = t < total ? dq_item(t, n1, c1, c2, s.g, s.G, passes) : DqItem{true, passes, 0};
    // the epilogue's bias values, fetched while the item's weights arrive
    float bias = 0.0f;
    if (t < total && lane < kDqRows)
      bias = it.w2 ? __ldg(a.b2 + static_cast<uint64_t>(e) * a.d + dq_row(it, lane)) * a.bias_mult
                   : __ldg(a.b1 + static_cast<uint64_t>(e) * (2u * a.fp) + dq_row(it, lane));
    const int ph = t < total ? (it.w2 ? passes + it.pass : it.pass) : nphases;
    // cross every phase boundary before this item (all warps do, in order)
    while (phase < ph && phase + 1 < nphases) {
      ++phase;
      DQ_T(56);
      __syncthreads();  // the previous phase's items are done
      DQ_T(57);
      const bool to_w2 = phase >= passes;
      if (phase == passes) {
        if (threadIdx.x == 0) {
          // this block's SwiGLU columns are written: meet the expert's other blocks
          __threadfence();
          // (test hook: block 0 stays silent, so its expert's wait runs out)
          if (!(a.skip_arrival && blockIdx.x == 0)) atomicAdd(arrive, 1);
          const unsigned long long t0 = global_timer_ns();
          const unsigned long long limit = a.wait_ns ? a.wait_ns : kWaitTimeoutNs;
          while (true) {
            int v;
            asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(arrive) : "memory");
            if (v >= s.G) break;
            if (global_timer_ns() - t0 > limit) {
              atomicCAS(a.err, 0, kDqErrExpert);
              break;
            }
          }
        }
      }
      DQ_T(58);
      stage(to_w2, to_w2 ? phase - passes : phase);
      cp_async_wait<0>();
      __syncthreads();
      DQ_T(59);
    }
    if (t >= total) break;
    if (nitem < 12) DQ_T(4 + 4 * nitem);
    cp_async_wait<D - 1>();  // this item's group has landed
    __syncwarp();
    if (nitem < 12) DQ_T(5 + 4 * nitem);
    const uint8_t* sb = ring + (seq % D) * a.stage_bytes;
    const int np = min(a.ps, cnt - it.pass * a.ps);
    // groups of up to four staged rows, each with its own unrolled kernel
    for (int j0 = 0; j0 < np; j0 += 4) {
      switch (min(4, np - j0)) {
        case 1: dq_finish<KI, 1>(a, it, sb, xs, rw, pos_s, lane, j0, bias); break;
        case 2: dq_finish<KI, 2>(a, it, sb, xs, rw, pos_s, lane, j0, bias); break;
        case 3: dq_finish<KI, 3>(a, it, sb, xs, rw, pos_s, lane, j0, bias); break;
        default: dq_finish<KI, 4>(a, it, sb, xs, rw, pos_s, lane, j0, bias); break;
      }
    }
    __syncwarp();  // the buffer is refilled by a later dq_issue of this warp
    if (nitem < 12) DQ_T(6 + 4 * nitem);
    ++nitem;
  }
  cp_async_wait<0>();
  if (a.fused) {
    // the last block to finish combines (every block's y_pair rows are written)
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence();
      last_block = atomicAdd(a.done, 1) == static_cast<int>(gridDim.x) - 1;
    }
    __syncthreads();
    if (last_block) {
      __threadfence();
      dq_combine_and_maps(a, tk_s);
    }
  }
  DQ_T(63);
}

// Cooperative launch: the blocks of an expert wait for each other between W1
// and W2, so all blocks must be resident at once.
template <int D, int KI>
cudaError_t dq_launch(const DqParams& a, size_t smem, int grid, cudaStream_t st) {
  const auto fn = mxmoe_dqgemv_ffn_kernel<D, KI>;
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
  // launch alone (the kernel then starts after the permutation completes)
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

size_t dq_smem_bytes(const DqParams& a, int D) {
  const int ki = (std::max(a.d, a.fp) / 32 + 31) / 32;
  return static_cast<size_t>(kDqWarps) * D * a.stage_bytes + static_cast<size_t>(a.ps) * ki * 2048 +
         16 * sizeof(float) + 16 * sizeof(int) + 16 * sizeof(void*) + 16;
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

cudaError_t launch_dqgemv_ffn(DqParams a, int max_pairs_per_expert, int max_experts, int num_sms, size_t smem_limit,
                              cudaStream_t st) {
  if (a.d % 32 != 0 || a.fp % 64 != 0 || a.d > kDqMaxK || a.fp > kDqMaxK || a.ps <= 0 || a.ps > 16)
    return cudaErrorInvalidValue;
  const uint32_t rb1 = static_cast<uint32_t>(a.kp1) / 2, rb2 = static_cast<uint32_t>(a.kp2) / 2;
  a.stage_bytes = (kDqRows * std::max(rb1 + a.sr1, rb2 + a.sr2) + 127u) / 128u * 128u;
  // three stage buffers per warp when they fit beside the staged rows, else two
  const int D = dq_smem_bytes(a, 3) + 2048 <= smem_limit ? 3 : 2;
  const size_t smem = dq_smem_bytes(a, D);
  if (smem + 2048 > smem_limit) return cudaErrorInvalidValue;
  (void)max_pairs_per_expert;
  const int grid = std::max(num_sms, max_experts);  // every touched expert gets a block
  const int ki = (std::max(a.d, a.fp) / 32 + 31) / 32;
  if (D == 3) {
    switch (ki) {
      case 1: return dq_launch<3, 1>(a, smem, grid, st);
      case 2: return dq_launch<3, 2>(a, smem, grid, st);
      case 3: return dq_launch<3, 3>(a, smem, grid, st);
      default: return dq_launch<3, 4>(a, smem, grid, st);
    }
  }
  switch (ki) {
    case 1: return dq_launch<2, 1>(a, smem, grid, st);
    case 2: return dq_launch<2, 2>(a, smem, grid, st);
    case 3: return dq_launch<2, 3>(a, smem, grid, st);
    default: return dq_launch<2, 4>(a, smem, grid, st);
  }
}

}  // namespace mxmoe
