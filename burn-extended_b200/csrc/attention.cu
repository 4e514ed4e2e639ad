// attention.cu -- the streaming multi-query attention step of GPT-OSS decoder
// blocks (src/attention/streaming_mqa.rs:239-435) on the GPU:
//   Q/K/V projections -> RoPE with an absolute offset -> rolling KV cache
//   (sink tokens kept, oldest evicted) -> windowed attention with optional
//   sinks logits, quiet softmax and additive bias -> output projection.
//
// Cache: the reference keeps [batch, cache_len, kv_heads, d_k] in logical
// order and rolls the non-sink part left on eviction (src/attention/
// cache_ops.rs:74-117), an O(cache) copy per step once full.  Here the
// non-sink part is a ring: logical index l >= sink lives at physical
// sink + (l - sink + head) mod (cap - sink), and an eviction of n tokens is
// head += n.  Every logical index the reference reads holds the same value.
//
// Kernels:
//   proj_gemv_kernel    y[r][j] = sum_c x[r][c] W[j][c] + b[j], weights stored
//                       output-major (bf16 or f32), a warp per output, its
//                       weight row in registers before the grid-dependency
//                       wait, one or two token rows, f32 sums; the output
//                       projection writes y in the caller's dtype.  Wider
//                       steps are GEMMs and go to cuBLAS.
//   rope_cache_kernel   rotates q and k of every (row, head) by the position
//                       (interleaved pairs, as burn's RotaryEncoding), writes
//                       k and v into the cache at their ring slots.
//   attn_split_kernel   one block per (query row, KV head, key split), a warp
//                       per query head of the group (shared K / V reads); a
//                       lane scores one key per step, the warp keeps a
//                       running max / sum and a V accumulator;
//   attn_merge_kernel   merges the splits (flash-decoding); the sinks column
//                       and the quiet-softmax 1 join the normalizer.
#include <cublas_v2.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <new>
#include <vector>

#include "../../include/mxmoe.h"
#include "launch_util.h"

namespace mxmoe {
// shared with api.cu
int set_last_error(int code, const char* msg);
}  // namespace mxmoe

namespace {

using mxmoe::griddep_wait;

int afail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  return mxmoe::set_last_error(code, buf);
}

#define A_CUDA(expr)                                                                            \
  do {                                                                                          \
    const cudaError_t e_ = (expr);                                                              \
    if (e_ != cudaSuccess) return afail(MXMOE_ERR_CUDA, "%s: %s", #expr, cudaGetErrorString(e_)); \
  } while (0)
#define A_TRY(expr)            \
  do {                         \
    const int r_ = (expr);     \
    if (r_ != MXMOE_OK) return r_; \
  } while (0)

struct ADevice {
  int prev = -1;
  explicit ADevice(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~ADevice() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

template <typename T>
int aalloc(T** p, size_t n) {
  *p = nullptr;
  if (n == 0) return MXMOE_OK;
  const cudaError_t e = cudaMalloc(reinterpret_cast<void**>(p), n * sizeof(T));
  if (e != cudaSuccess) return afail(MXMOE_ERR_OOM, "cudaMalloc(%zu bytes): %s", n * sizeof(T), cudaGetErrorString(e));
  return MXMOE_OK;
}
template <typename T>
void afree(T*& p) {
  if (p) cudaFree(p);
  p = nullptr;
}

constexpr int kGemvWarps = 8;    // outputs per block
constexpr int kAttnWarps = 8;
constexpr int kMaxHeadDim = 256;
constexpr int kMaxSplits = 32;
constexpr int kTileKeys = 32;  // keys per staged attention tile

// 8 consecutive weights from a 16-byte (bf16) or two 16-byte (f32) loads.
__device__ __forceinline__ void ld_w8(const void* w, int wdtype, size_t i, float (&o)[8]) {
  if (wdtype == MXMOE_BF16) {
    const uint4 u = __ldg(reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(w) + i));
    const uint32_t v[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      o[2 * h] = __uint_as_float(v[h] << 16);
      o[2 * h + 1] = __uint_as_float(v[h] & 0xFFFF0000u);
    }
  } else {
    const float4 a = __ldg(reinterpret_cast<const float4*>(static_cast<const float*>(w) + i));
    const float4 b = __ldg(reinterpret_cast<const float4*>(static_cast<const float*>(w) + i) + 1);
    o[0] = a.x; o[1] = a.y; o[2] = a.z; o[3] = a.w; o[4] = b.x; o[5] = b.y; o[6] = b.z; o[7] = b.w;
  }
}

// y[r][j] = sum_c x[r][c] * W[j][c] + b[j] for rows r < R, outputs j < J.
// x: [R][K] (f32 or bf16), W: [J][K] output-major, K % 8 == 0, y f32 or
// bf16 (ld = J).  One warp per output j; lane l owns the 8-element pieces
// l, l + 32, ...  The first kProjPf pieces of the warp's weight row (K <=
// 3072 in one go) are loaded into registers BEFORE the grid-dependency wait:
// the weights do not depend on the kernel before, so their HBM round trip
// overlaps that kernel's tail.  One- and two-row steps hold 8 pieces and run
// three blocks per SM, wider steps 12 pieces and two blocks.  Token rows are staged in shared memory as f32, NR (1, 2, 4 or 8) per pass.
constexpr int kProjPf = 12;
template <bool WBF16, int NR>
__global__ void __launch_bounds__(32 * kGemvWarps, NR <= 2 ? 3 : 2)
    proj_gemv_kernel(const void* __restrict__ x, int x_dtype, int R, int K, const void* __restrict__ W,
                     const float* __restrict__ bias, int J, void* __restrict__ y, int y_dtype) {
  extern __shared__ __align__(16) float xs_dense[];  // [NR][K]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int j = blockIdx.x * kGemvWarps + warp;
  const int npiece = K / 8;
  constexpr int PF = NR <= 2 ? 8 : kProjPf;  // fewer pieces where more blocks share an SM
  uint4 wr[PF];
  if (WBF16 && j < J) {
    const uint4* wrow = reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(W) + static_cast<size_t>(j) * K);
#pragma unroll
    for (int i = 0; i < PF; ++i)
      if (lane + 32 * i < npiece) wr[i] = __ldg(wrow + lane + 32 * i);
  }
  const float bj = (j < J && bias) ? __ldg(bias + j) : 0.0f;
  griddep_wait();
  for (int r0 = 0; r0 < R; r0 += NR) {
    const int nr = min(NR, R - r0);
    __syncthreads();
    if (x_dtype == MXMOE_BF16) {
      const uint4* xv = reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(x) + static_cast<size_t>(r0) * K);
      for (int i = threadIdx.x; i < nr * K / 8; i += blockDim.x) {
        const uint4 u = __ldg(xv + i);
        const uint32_t v[4] = {u.x, u.y, u.z, u.w};
        float4 lo, hi;
        lo.x = __uint_as_float(v[0] << 16); lo.y = __uint_as_float(v[0] & 0xFFFF0000u);
        lo.z = __uint_as_float(v[1] << 16); lo.w = __uint_as_float(v[1] & 0xFFFF0000u);
        hi.x = __uint_as_float(v[2] << 16); hi.y = __uint_as_float(v[2] & 0xFFFF0000u);
        hi.z = __uint_as_float(v[3] << 16); hi.w = __uint_as_float(v[3] & 0xFFFF0000u);
        reinterpret_cast<float4*>(xs_dense)[2 * i] = lo;
        reinterpret_cast<float4*>(xs_dense)[2 * i + 1] = hi;
      }
    } else {
      const float4* xv = reinterpret_cast<const float4*>(static_cast<const float*>(x) + static_cast<size_t>(r0) * K);
      for (int i = threadIdx.x; i < nr * K / 4; i += blockDim.x) reinterpret_cast<float4*>(xs_dense)[i] = __ldg(xv + i);
    }
    __syncthreads();
    if (j >= J) continue;
    float acc[NR];
#pragma unroll
    for (int r = 0; r < NR; ++r) acc[r] = 0.0f;
    auto piece = [&](int p, const float (&w)[8]) {
#pragma unroll
      for (int r = 0; r < NR; ++r) {
        if (r < nr) {
          const float4 a = *reinterpret_cast<const float4*>(xs_dense + r * K + 8 * p);
          const float4 b = *reinterpret_cast<const float4*>(xs_dense + r * K + 8 * p + 4);
          acc[r] = fmaf(a.x, w[0], acc[r]); acc[r] = fmaf(a.y, w[1], acc[r]);
          acc[r] = fmaf(a.z, w[2], acc[r]); acc[r] = fmaf(a.w, w[3], acc[r]);
          acc[r] = fmaf(b.x, w[4], acc[r]); acc[r] = fmaf(b.y, w[5], acc[r]);
          acc[r] = fmaf(b.z, w[6], acc[r]); acc[r] = fmaf(b.w, w[7], acc[r]);
        }
      }
    };
    if (WBF16) {
#pragma unroll
      for (int i = 0; i < PF; ++i) {
        const int p = lane + 32 * i;
        if (p < npiece) {
          const uint32_t v[4] = {wr[i].x, wr[i].y, wr[i].z, wr[i].w};
          float w[8];
#pragma unroll
          for (int h = 0; h < 4; ++h) {
            w[2 * h] = __uint_as_float(v[h] << 16);
            w[2 * h + 1] = __uint_as_float(v[h] & 0xFFFF0000u);
          }
          piece(p, w);
        }
      }
    }
    for (int p = lane + (WBF16 ? 32 * PF : 0); p < npiece; p += 32) {
      float w[8];
      ld_w8(W, WBF16 ? MXMOE_BF16 : MXMOE_F32, static_cast<size_t>(j) * K + 8 * p, w);
      piece(p, w);
    }
#pragma unroll
    for (int r = 0; r < NR; ++r) {
      float v = acc[r];
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
      if (lane == 0 && r < nr) {
        const size_t o = static_cast<size_t>(r0 + r) * J + j;
        if (y_dtype == MXMOE_F32)
          static_cast<float*>(y)[o] = v + bj;
        else
          static_cast<__nv_bfloat16*>(y)[o] = __float2bfloat16_rn(v + bj);
      }
    }
  }
}

// Physical cache slot of logical index l.
__device__ __forceinline__ int ring_slot(int l, int sink, int cap, int head) {
  return l < sink ? l : sink + (l - sink + head) % (cap - sink);
}

struct RopeArgs {
  const float* theta;  // [rope_dim / 2] inverse frequencies (scaled), null: no RoPE
  float concentration; // multiplies cos and sin (YaRN)
  int rope_dim;        // even part of d_k that rotates
  int by_head;         // reference compat: the rotation index runs over heads, not tokens
};

// qkv: [B * T][(nH + 2 kvH) * dk] f32 (rows b * T + t).  Rotates q (in
// place) and k, then writes k and v to the cache [B][cap][kvH][dk] at the
// ring slot of logical local_start + t.
__global__ void rope_cache_kernel(float* __restrict__ qkv, int B, int T, int nH, int kvH, int dk, int start_pos,
                                  RopeArgs rope, float* __restrict__ kc, float* __restrict__ vc, int cap, int sink,
                                  int head, int local_start) {
  griddep_wait();
  const int row = blockIdx.x;  // b * T + t
  const int b = row / T, t = row - b * T;
  const int width = (nH + 2 * kvH) * dk;
  float* r = qkv + static_cast<size_t>(row) * width;
  const int slot = ring_slot(local_start + t, sink, cap, head);
  // q heads then k heads rotate; v is copied
  for (int i = threadIdx.x; i < (nH + kvH) * (dk / 2); i += blockDim.x) {
    const int hh = i / (dk / 2), pr = i - hh * (dk / 2);  // head (q then k) and pair index
    const int c = 2 * pr;
    float* base = r + hh * dk;
    if (rope.theta != nullptr && c + 1 < rope.rope_dim) {
      const int hidx = hh < nH ? hh : hh - nH;
      const float pos = static_cast<float>(start_pos + (rope.by_head ? hidx : t));
      const float ang = pos * rope.theta[pr];
      float sn, cs;
      sincosf(ang, &sn, &cs);
      cs *= rope.concentration;
      sn *= rope.concentration;
      const float a = base[c], bb = base[c + 1];
      base[c] = a * cs - bb * sn;
      base[c + 1] = bb * cs + a * sn;
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < kvH * dk; i += blockDim.x) {
    const size_t dst = (static_cast<size_t>(b) * cap + slot) * kvH * dk + i;
    kc[dst] = r[nH * dk + i];
    vc[dst] = r[(nH + kvH) * dk + i];
  }
}

struct AttnArgs {
  const float* qkv;       // [B*T][(nH + 2 kvH) dk], q rotated
  const float* kc;        // cache [B][cap][kvH][dk]
  const float* vc;
  int B, T, nH, kvH, dk, cap, sink, head;
  int win_start, win_len; // logical window [win_start, win_start + win_len)
  int splits, split_len;  // the window in `splits` key ranges of split_len keys
  float scale;            // 1 / sqrt(d_k) (1 when pre-scaled)
  const float* sinks;     // [nH] or null
  const float* bias;      // [B][nH][T][win_len] or null
  int quiet;
  float* ctx;             // [B*T][nH * dk] (splits == 1)
  float* part_ml;         // [B*T][nH][splits][2] running max / sum per split (splits > 1)
  float* part_acc;        // [B*T][nH][splits][dk]
};

// The finished row of one head: the sinks column and the quiet-softmax 1
// join the normalizer (src/attention/core.rs:37-55).
__device__ __forceinline__ float attn_norm(float m, float l, const AttnArgs& a, int h, float& M) {
  const float sink = a.sinks ? a.sinks[h] : -INFINITY;
  M = fmaxf(m, sink);
  float L = (m == -INFINITY) ? 0.0f : l * expf(m - M);
  if (a.sinks) L += expf(sink - M);
  if (a.quiet) L += expf(-M);
  return L;
}

__device__ __forceinline__ void cp_async16_a(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
               "l"(src)
               : "memory");
}

// One block per (row = b * T + t, KV head x group of up to 8 query heads,
// key split); warp w takes query head kvh * G + 8 hg + w.  The block stages
// its keys in tiles of 32 (K and V rows, padded to d_k + 4 floats so a
// lane's row reads are conflict-free) through a double-buffered cp.async
// ring, so every K / V byte is read once per block and the next tile's loads
// overlap the current tile's math.  A lane scores one key per tile (q in
// shared memory); the warp keeps a running max / sum and a V accumulator
// (lane owns columns lane + 32 i).  One split writes the context row itself;
// several write their partial max / sum / accumulator for attn_merge_kernel.
__global__ void __launch_bounds__(32 * kAttnWarps) attn_split_kernel(const AttnArgs a) {
  extern __shared__ __align__(16) float kv_s[];  // [2 buffers][K, V][kTileKeys][dk + 4]
  __shared__ __align__(16) float q_s[kAttnWarps][kMaxHeadDim];
  const int dk = a.dk, G = a.nH / a.kvH, hgroups = (G + kAttnWarps - 1) / kAttnWarps;
  const int row = blockIdx.x, kvh = blockIdx.y / hgroups, hg = blockIdx.y - kvh * hgroups, split = blockIdx.z;
  const int b = row / a.T, t = row - b * a.T;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = hg * kAttnWarps + warp, h = kvh * G + g;
  const bool active = g < G;
  const int width = (a.nH + 2 * a.kvH) * dk, ld = dk + 4, dq = dk / 4;
  const int j_lo = split * a.split_len, j_hi = min(a.win_len, j_lo + a.split_len);
  const int ntiles = (j_hi - j_lo + kTileKeys - 1) / kTileKeys;
  constexpr int kPer = kMaxHeadDim / 32;
  const int per = (dk + 31) / 32;
  griddep_wait();
  auto load_tile = [&](int buf, int tile) {
    float* base = kv_s + static_cast<size_t>(buf) * 2 * kTileKeys * ld;
    for (int idx = threadIdx.x; idx < 2 * kTileKeys * dq; idx += blockDim.x) {
      const int which = idx / (kTileKeys * dq), rem = idx - which * kTileKeys * dq;
      const int key = rem / dq, c4 = rem - key * dq;
      const int j = j_lo + tile * kTileKeys + key;
      if (j < j_hi) {
        const int slot = ring_slot(a.win_start + j, a.sink, a.cap, a.head);
        const float* src = (which ? a.vc : a.kc) + ((static_cast<size_t>(b) * a.cap + slot) * a.kvH + kvh) * dk + 4 * c4;
        cp_async16_a(base + (which * kTileKeys + key) * ld + 4 * c4, src);
      }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  if (ntiles > 0) load_tile(0, 0);
  if (active)
    for (int i = lane; i < dk; i += 32) q_s[warp][i] = a.qkv[static_cast<size_t>(row) * width + h * dk + i];
  float m = -INFINITY, l = 0.0f;
  float acc[kPer];
#pragma unroll
  for (int i = 0; i < kPer; ++i) acc[i] = 0.0f;
  const float* bias_row =
      (a.bias && active) ? a.bias + ((static_cast<size_t>(b) * a.nH + h) * a.T + t) * a.win_len : nullptr;
  for (int tile = 0; tile < ntiles; ++tile) {
    if (tile + 1 < ntiles) {
      load_tile((tile + 1) & 1, tile + 1);
      asm volatile("cp.async.wait_group 1;" ::: "memory");
    } else {
      asm volatile("cp.async.wait_group 0;" ::: "memory");
    }
    __syncthreads();
    const float* ks = kv_s + static_cast<size_t>(tile & 1) * 2 * kTileKeys * ld;
    const float* vs = ks + kTileKeys * ld;
    const int j0 = j_lo + tile * kTileKeys, nk = min(kTileKeys, j_hi - j0);
    if (active) {
      float s = -INFINITY;
      if (lane < nk) {
        const float4* kr = reinterpret_cast<const float4*>(ks + lane * ld);
        const float4* qv = reinterpret_cast<const float4*>(q_s[warp]);
        float d0 = 0.0f, d1 = 0.0f;
        for (int c = 0; c < dq; c += 2) {
          const float4 k0 = kr[c], q0 = qv[c];
          d0 = fmaf(q0.x, k0.x, d0); d0 = fmaf(q0.y, k0.y, d0); d0 = fmaf(q0.z, k0.z, d0); d0 = fmaf(q0.w, k0.w, d0);
          if (c + 1 < dq) {
            const float4 k1 = kr[c + 1], q1 = qv[c + 1];
            d1 = fmaf(q1.x, k1.x, d1); d1 = fmaf(q1.y, k1.y, d1); d1 = fmaf(q1.z, k1.z, d1); d1 = fmaf(q1.w, k1.w, d1);
          }
        }
        s = (d0 + d1) * a.scale;
        if (bias_row) s += bias_row[j0 + lane];
      }
      float mb = s;
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) mb = fmaxf(mb, __shfl_xor_sync(0xFFFFFFFFu, mb, o));
      const float mn = fmaxf(m, mb);
      const float p = (lane < nk && s != -INFINITY) ? expf(s - mn) : 0.0f;
      const float corr = (m == -INFINITY) ? 0.0f : expf(m - mn);
      float ps = p;
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) ps += __shfl_xor_sync(0xFFFFFFFFu, ps, o);
      l = l * corr + ps;
#pragma unroll
      for (int i = 0; i < kPer; ++i) acc[i] *= corr;
      m = mn;
      for (int u = 0; u < nk; ++u) {
        const float pu = __shfl_sync(0xFFFFFFFFu, p, u);
        const float* vr = vs + u * ld;
#pragma unroll
        for (int i = 0; i < kPer; ++i)
          if (i < per && lane + 32 * i < dk) acc[i] = fmaf(pu, vr[lane + 32 * i], acc[i]);
      }
    }
    __syncthreads();  // the buffer is refilled by the next tile's loads
  }
  if (!active) return;
  if (a.splits == 1) {
    float M;
    const float L = attn_norm(m, l, a, h, M);
    const float f = (L > 0.0f && m != -INFINITY) ? expf(m - M) / L : 0.0f;
#pragma unroll
    for (int i = 0; i < kPer; ++i)
      if (i < per && lane + 32 * i < dk) a.ctx[static_cast<size_t>(row) * a.nH * dk + h * dk + lane + 32 * i] = acc[i] * f;
  } else {
    const size_t pi = (static_cast<size_t>(row) * a.nH + h) * a.splits + split;
    if (lane == 0) {
      a.part_ml[2 * pi] = m;
      a.part_ml[2 * pi + 1] = l;
    }
#pragma unroll
    for (int i = 0; i < kPer; ++i)
      if (i < per && lane + 32 * i < dk) a.part_acc[pi * dk + lane + 32 * i] = acc[i];
  }
}

// One warp per (row, head): merges the splits' running max / sum /
// accumulator, then normalizes with the sinks column and the quiet 1.
__global__ void attn_merge_kernel(const AttnArgs a) {
  griddep_wait();
  const int wid = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  const int rows = a.B * a.T;
  if (wid >= rows * a.nH) return;
  const int row = wid / a.nH, h = wid - row * a.nH, dk = a.dk;
  const size_t p0 = static_cast<size_t>(wid) * a.splits;
  float m = -INFINITY;
  for (int s = 0; s < a.splits; ++s) m = fmaxf(m, a.part_ml[2 * (p0 + s)]);
  float M;
  float l = 0.0f;
  for (int s = 0; s < a.splits; ++s) {
    const float ms = a.part_ml[2 * (p0 + s)];
    if (ms != -INFINITY) l += a.part_ml[2 * (p0 + s) + 1] * expf(ms - m);
  }
  const float L = attn_norm(m, l, a, h, M);
  for (int c = lane; c < dk; c += 32) {
    float v = 0.0f;
    for (int s = 0; s < a.splits; ++s) {
      const float ms = a.part_ml[2 * (p0 + s)];
      if (ms != -INFINITY) v += a.part_acc[(p0 + s) * dk + c] * expf(ms - M);
    }
    a.ctx[static_cast<size_t>(row) * a.nH * dk + h * dk + c] = L > 0.0f ? v / L : 0.0f;
  }
}

template <bool WBF16, int NR>
cudaError_t launch_proj(const void* x, int x_dtype, int R, int K, const void* W, const float* bias, int J, void* y,
                        int y_dtype, cudaStream_t st) {
  const auto fn = proj_gemv_kernel<WBF16, NR>;
  const size_t smem = static_cast<size_t>(NR) * K * sizeof(float);
  const cudaError_t e = mxmoe::ensure_dynamic_smem(reinterpret_cast<const void*>(fn), smem);
  if (e != cudaSuccess) return e;
  return mxmoe::launch_kernel(fn, dim3((J + kGemvWarps - 1) / kGemvWarps), dim3(32 * kGemvWarps), smem, st, x, x_dtype,
                              R, K, W, bias, J, y, y_dtype);
}

// One or two token rows per launch (wider steps are GEMMs, see wide_proj).
cudaError_t launch_gemv(const void* x, int x_dtype, int R, int K, const void* W, int wdtype, const float* bias, int J,
                        void* y, int y_dtype, cudaStream_t st) {
  if (R <= 1)
    return wdtype == MXMOE_BF16 ? launch_proj<true, 1>(x, x_dtype, R, K, W, bias, J, y, y_dtype, st)
                                : launch_proj<false, 1>(x, x_dtype, R, K, W, bias, J, y, y_dtype, st);
  return wdtype == MXMOE_BF16 ? launch_proj<true, 2>(x, x_dtype, R, K, W, bias, J, y, y_dtype, st)
                              : launch_proj<false, 2>(x, x_dtype, R, K, W, bias, J, y, y_dtype, st);
}

// Steps of more than kGemvMaxRows token rows are GEMMs (M = rows; measured
// at batch 8: 160 us per step on the GEMV kernel): they go to cuBLAS (a
// plain library GEMM, f32 accumulation).  f32 activations against bf16
// weights are split into two bf16 terms (hi = bf16(x), lo = bf16(x - hi)),
// whose two products sum to x W within about 2^-16 of |x|.
constexpr int kGemvMaxRows = 2;

__global__ void split_bf16_kernel(const float* __restrict__ x, size_t n, __nv_bfloat16* __restrict__ hi,
                                  __nv_bfloat16* __restrict__ lo) {
  griddep_wait();
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const float v = x[i];
    const __nv_bfloat16 h = __float2bfloat16_rn(v);
    hi[i] = h;
    lo[i] = __float2bfloat16_rn(v - __bfloat162float(h));
  }
}

__global__ void widen_bf16_kernel(const __nv_bfloat16* __restrict__ x, size_t n, float* __restrict__ y) {
  griddep_wait();
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x)
    y[i] = __bfloat162float(x[i]);
}

// y[r][j] = acc[r][j] + b[j], in y's dtype (acc may alias y when it is f32).
__global__ void bias_out_kernel(const float* acc, size_t rows, int J, const float* __restrict__ bias, void* y,
                                int y_dtype) {
  griddep_wait();
  const size_t n = rows * static_cast<size_t>(J);
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const float v = acc[i] + (bias ? bias[i % J] : 0.0f);
    if (y_dtype == MXMOE_F32)
      static_cast<float*>(y)[i] = v;
    else
      static_cast<__nv_bfloat16*>(y)[i] = __float2bfloat16_rn(v);
  }
}

dim3 grid_for(size_t n) { return dim3(static_cast<unsigned>(std::min<size_t>((n + 255) / 256, 2368))); }

}  // namespace

struct mxmqa_layer {
  mxmqa_config cfg{};
  int groups = 1;
  int wdtype = MXMOE_F32;
  void* wqkv = nullptr;   // [(nH + 2 kvH) dk][d] output-major
  float* bqkv = nullptr;  // [(nH + 2 kvH) dk]
  void* wo = nullptr;     // [d][nH dk]
  float* bo = nullptr;    // [d]
  float* sinks = nullptr; // [nH] module sinks (learned_sinks), or null
  float* theta = nullptr; // [rope_dim / 2]
  float concentration = 1.0f;
  int rope_dim = 0;
  bool ready = false;
  // per-forward scratch
  float* qkv = nullptr;
  float* ctx = nullptr;
  float* part = nullptr;  // split partials: [rows][nH][splits][2] then [rows][nH][splits][dk]
  size_t cap_rows = 0, cap_part = 0;
  int num_sms = 148;
  // wide steps (cuBLAS): handle and scratch for split / widened rows and the f32 product
  cublasHandle_t blas = nullptr;
  void* wide = nullptr;
  size_t cap_wide = 0;
};

struct mxmqa_cache {
  int device = 0;
  uint32_t batch = 0, cap = 0, sink = 0, kv_heads = 0, head_dim = 0;
  uint64_t global_end = 0, local_end = 0;
  uint32_t head = 0;  // ring offset of the non-sink part
  float* k = nullptr;
  float* v = nullptr;
};

namespace {

// Burn Linear weight [d_in][d_out] (host, f32 or bf16) -> output-major
// [d_out][d_in] at dst + row0 * d_in.
void transpose_into(const void* w, int dtype, size_t d_in, size_t d_out, std::vector<uint16_t>& dst16,
                    std::vector<float>& dst32, size_t row0) {
  for (size_t i = 0; i < d_in; ++i)
    for (size_t o = 0; o < d_out; ++o) {
      const size_t s = i * d_out + o, d = (row0 + o) * d_in + i;
      if (dtype == MXMOE_BF16)
        dst16[d] = static_cast<const uint16_t*>(w)[s];
      else
        dst32[d] = static_cast<const float*>(w)[s];
    }
}

void bias_into(const void* b, int dtype, size_t n, float* dst) {
  for (size_t i = 0; i < n; ++i) {
    if (!b) {
      dst[i] = 0.0f;
    } else if (dtype == MXMOE_BF16) {
      const uint32_t u = static_cast<uint32_t>(static_cast<const uint16_t*>(b)[i]) << 16;
      std::memcpy(&dst[i], &u, 4);
    } else {
      dst[i] = static_cast<const float*>(b)[i];
    }
  }
}

cudaStream_t as_stream_a(void* s) { return static_cast<cudaStream_t>(s); }

}  // namespace

namespace {

const char* blas_status(cublasStatus_t s) {
  switch (s) {
    case CUBLAS_STATUS_NOT_INITIALIZED: return "not initialized";
    case CUBLAS_STATUS_ALLOC_FAILED: return "allocation failed";
    case CUBLAS_STATUS_INVALID_VALUE: return "invalid value";
    case CUBLAS_STATUS_ARCH_MISMATCH: return "architecture mismatch";
    case CUBLAS_STATUS_EXECUTION_FAILED: return "execution failed";
    case CUBLAS_STATUS_NOT_SUPPORTED: return "not supported";
    default: return "error";
  }
}
#define A_BLAS(expr)                                                                          \
  do {                                                                                        \
    const cublasStatus_t s_ = (expr);                                                         \
    if (s_ != CUBLAS_STATUS_SUCCESS) return afail(MXMOE_ERR_CUDA, "%s: %s", #expr, blas_status(s_)); \
  } while (0)

// y[R][J] = x[R][K] W[J][K]^T + b for R > kGemvMaxRows.  Column-major view:
// C (J x R, ld J) = op(W) (J x K) * x (K x R).  The product lands in f32
// (out32, or scratch), then bias_out_kernel adds the bias in y's dtype.
int wide_proj(mxmqa_layer* L, const void* x, int x_dtype, int R, int K, const void* W, const float* bias, int J,
              void* y, int y_dtype, float* out32, cudaStream_t st) {
  if (!L->blas) A_BLAS(cublasCreate(&L->blas));
  A_BLAS(cublasSetStream(L->blas, st));
  const size_t nx = static_cast<size_t>(R) * K, ny = static_cast<size_t>(R) * J;
  const size_t need = 2 * nx * 2 + nx * 4 + (out32 ? 0 : ny * 4);
  if (L->cap_wide < need) {
    afree(L->wide);
    L->cap_wide = 0;
    A_TRY(aalloc(reinterpret_cast<uint8_t**>(&L->wide), need));
    L->cap_wide = need;
  }
  __nv_bfloat16* hi = static_cast<__nv_bfloat16*>(L->wide);
  __nv_bfloat16* lo = hi + nx;
  float* xf = reinterpret_cast<float*>(lo + nx);
  float* c = out32 ? out32 : xf + nx;
  const float one = 1.0f, zero = 0.0f;
  if (L->wdtype == MXMOE_F32) {
    const float* xa = static_cast<const float*>(x);
    if (x_dtype == MXMOE_BF16) {
      A_CUDA(mxmoe::launch_kernel(widen_bf16_kernel, grid_for(nx), dim3(256), 0, st,
                                  static_cast<const __nv_bfloat16*>(x), nx, xf));
      xa = xf;
    }
    A_BLAS(cublasSgemm(L->blas, CUBLAS_OP_T, CUBLAS_OP_N, J, R, K, &one, static_cast<const float*>(W), K, xa, K, &zero,
                       c, J));
  } else if (x_dtype == MXMOE_BF16) {
    A_BLAS(cublasGemmEx(L->blas, CUBLAS_OP_T, CUBLAS_OP_N, J, R, K, &one, W, CUDA_R_16BF, K, x, CUDA_R_16BF, K, &zero,
                        c, CUDA_R_32F, J, CUBLAS_COMPUTE_32F, CUBLAS_GEMM_DEFAULT));
  } else {
    A_CUDA(mxmoe::launch_kernel(split_bf16_kernel, grid_for(nx), dim3(256), 0, st, static_cast<const float*>(x), nx, hi,
                                lo));
    A_BLAS(cublasGemmEx(L->blas, CUBLAS_OP_T, CUBLAS_OP_N, J, R, K, &one, W, CUDA_R_16BF, K, hi, CUDA_R_16BF, K, &zero,
                        c, CUDA_R_32F, J, CUBLAS_COMPUTE_32F, CUBLAS_GEMM_DEFAULT));
    A_BLAS(cublasGemmEx(L->blas, CUBLAS_OP_T, CUBLAS_OP_N, J, R, K, &one, W, CUDA_R_16BF, K, lo, CUDA_R_16BF, K, &one,
                        c, CUDA_R_32F, J, CUBLAS_COMPUTE_32F, CUBLAS_GEMM_DEFAULT));
  }
  A_CUDA(mxmoe::launch_kernel(bias_out_kernel, grid_for(ny), dim3(256), 0, st, static_cast<const float*>(c),
                              static_cast<size_t>(R), J, bias, y, y_dtype));
  return MXMOE_OK;
}

// The projection of one step: the GEMV kernel up to kGemvMaxRows rows, cuBLAS above.
int project(mxmqa_layer* L, const void* x, int x_dtype, int R, int K, const void* W, const float* bias, int J, void* y,
            int y_dtype, cudaStream_t st) {
  if (R <= kGemvMaxRows) {
    A_CUDA(launch_gemv(x, x_dtype, R, K, W, L->wdtype, bias, J, y, y_dtype, st));
    return MXMOE_OK;
  }
  return wide_proj(L, x, x_dtype, R, K, W, bias, J, y, y_dtype, y_dtype == MXMOE_F32 ? static_cast<float*>(y) : nullptr,
                   st);
}

}  // namespace

extern "C" {

int mxmqa_create(const mxmqa_config* cfg, mxmqa_layer** out) {
  if (!cfg || !out) return afail(MXMOE_ERR_INVALID_ARG, "null argument");
  *out = nullptr;
  if (cfg->d_model == 0 || cfg->n_heads == 0 || cfg->kv_heads == 0 || cfg->head_dim == 0)
    return afail(MXMOE_ERR_INVALID_ARG, "zero dimension");
  if (cfg->n_heads % cfg->kv_heads != 0)
    return afail(MXMOE_ERR_INVALID_ARG, "n_heads must be divisible by kv_heads");
  if (cfg->head_dim % 4 != 0 || cfg->head_dim > static_cast<uint32_t>(kMaxHeadDim) || cfg->d_model % 8 != 0 ||
      (cfg->n_heads * cfg->head_dim) % 8 != 0)
    return afail(MXMOE_ERR_UNSUPPORTED, "head_dim must be a multiple of 4 and at most %d, d_model a multiple of 8",
                 kMaxHeadDim);
  mxmqa_layer* L = new (std::nothrow) mxmqa_layer();
  if (!L) return afail(MXMOE_ERR_OOM, "host allocation failed");
  L->cfg = *cfg;
  L->groups = static_cast<int>(cfg->n_heads / cfg->kv_heads);
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, cfg->device) == cudaSuccess && sms > 0)
    L->num_sms = sms;
  *out = L;
  return MXMOE_OK;
}

int mxmqa_destroy(mxmqa_layer* L) {
  if (!L) return MXMOE_OK;
  ADevice g(L->cfg.device);
  afree(L->wqkv); afree(L->bqkv); afree(L->wo); afree(L->bo); afree(L->sinks); afree(L->theta);
  afree(L->qkv); afree(L->ctx); afree(L->part); afree(L->wide);
  if (L->blas) cublasDestroy(L->blas);
  delete L;
  return MXMOE_OK;
}

int mxmqa_set_weights(mxmqa_layer* L, const void* wq, const void* bq, const void* wk, const void* bk, const void* wv,
                      const void* bv, const void* wo, const void* bo, mxmoe_dtype dtype, void* stream) {
  if (!L || !wq || !wk || !wv || !wo) return afail(MXMOE_ERR_INVALID_ARG, "null weight");
  if (dtype != MXMOE_F32 && dtype != MXMOE_BF16) return afail(MXMOE_ERR_INVALID_ARG, "bad dtype");
  ADevice g(L->cfg.device);
  const size_t d = L->cfg.d_model, dk = L->cfg.head_dim, nH = L->cfg.n_heads, kvH = L->cfg.kv_heads;
  const size_t jq = nH * dk, jk = kvH * dk, J = jq + 2 * jk;
  std::vector<uint16_t> w16(dtype == MXMOE_BF16 ? J * d : 0), o16(dtype == MXMOE_BF16 ? d * jq : 0);
  std::vector<float> w32(dtype == MXMOE_F32 ? J * d : 0), o32(dtype == MXMOE_F32 ? d * jq : 0);
  transpose_into(wq, dtype, d, jq, w16, w32, 0);
  transpose_into(wk, dtype, d, jk, w16, w32, jq);
  transpose_into(wv, dtype, d, jk, w16, w32, jq + jk);
  transpose_into(wo, dtype, jq, d, o16, o32, 0);
  std::vector<float> b(J), bo32(d);
  bias_into(bq, dtype, jq, b.data());
  bias_into(bk, dtype, jk, b.data() + jq);
  bias_into(bv, dtype, jk, b.data() + jq + jk);
  bias_into(bo, dtype, d, bo32.data());
  afree(L->wqkv); afree(L->bqkv); afree(L->wo); afree(L->bo);
  const size_t es = dtype == MXMOE_BF16 ? 2 : 4;
  A_TRY(aalloc(reinterpret_cast<uint8_t**>(&L->wqkv), J * d * es));
  A_TRY(aalloc(reinterpret_cast<uint8_t**>(&L->wo), d * jq * es));
  A_TRY(aalloc(&L->bqkv, J));
  A_TRY(aalloc(&L->bo, d));
  cudaStream_t st = as_stream_a(stream);
  A_CUDA(cudaMemcpyAsync(L->wqkv, dtype == MXMOE_BF16 ? static_cast<const void*>(w16.data()) : w32.data(), J * d * es,
                         cudaMemcpyHostToDevice, st));
  A_CUDA(cudaMemcpyAsync(L->wo, dtype == MXMOE_BF16 ? static_cast<const void*>(o16.data()) : o32.data(), d * jq * es,
                         cudaMemcpyHostToDevice, st));
  A_CUDA(cudaMemcpyAsync(L->bqkv, b.data(), J * 4, cudaMemcpyHostToDevice, st));
  A_CUDA(cudaMemcpyAsync(L->bo, bo32.data(), d * 4, cudaMemcpyHostToDevice, st));
  A_CUDA(cudaStreamSynchronize(st));
  L->wdtype = dtype;
  L->ready = true;
  return MXMOE_OK;
}

int mxmqa_set_sinks(mxmqa_layer* L, const float* sinks) {
  if (!L) return afail(MXMOE_ERR_INVALID_ARG, "null layer");
  ADevice g(L->cfg.device);
  afree(L->sinks);
  if (!sinks) return MXMOE_OK;
  A_TRY(aalloc(&L->sinks, L->cfg.n_heads));
  A_CUDA(cudaMemcpy(L->sinks, sinks, L->cfg.n_heads * sizeof(float), cudaMemcpyHostToDevice));
  return MXMOE_OK;
}

int mxmqa_set_rope(mxmqa_layer* L, const mxmqa_rope* rope) {
  if (!L) return afail(MXMOE_ERR_INVALID_ARG, "null layer");
  ADevice g(L->cfg.device);
  afree(L->theta);
  L->rope_dim = 0;
  if (!rope) return MXMOE_OK;
  const int dk = static_cast<int>(L->cfg.head_dim);
  const int rd = dk & ~1;  // the even part of d_k rotates (src/attention/streaming_mqa.rs:287)
  if (rd == 0) return MXMOE_OK;
  // burn RotaryEncodingConfig::init: theta_i = 1 / base^(2i / rd), i < rd / 2,
  // then the NTK / YaRN interpolation of src/rope/mod.rs:11-50 when
  // scaling_factor > 1, which also scales cos and sin by 0.1 ln(s) + 1.
  std::vector<float> th(rd / 2);
  const float base = rope->theta > 0.0f ? rope->theta : 10000.0f;
  for (int i = 0; i < rd / 2; ++i) th[i] = 1.0f / std::pow(base, static_cast<float>(2 * i) / static_cast<float>(rd));
  float conc = 1.0f;
  if (rope->scaling_factor > 1.0f) {
    const float d_model = static_cast<float>(rd) * 2.0f, d_half = d_model / 2.0f, log_base = std::log(base);
    const float two_pi = 6.28318530717958647692f;
    const float low = d_half * std::log(rope->initial_context / (rope->ntk_beta * two_pi)) / log_base;
    const float high = d_half * std::log(rope->initial_context / (rope->ntk_alpha * two_pi)) / log_base;
    if (!(low > 0.0f && high > 0.0f && low < high && high < d_half - 1.0f))
      return afail(MXMOE_ERR_INVALID_ARG, "NTK/YaRN thresholds out of range (low %g, high %g)", low, high);
    for (int i = 0; i < rd / 2; ++i) {
      const float idx = std::log(th[i]) * (-d_model / 2.0f / log_base);
      const float ramp = std::min(1.0f, std::max(0.0f, (idx - low) / (high - low)));
      th[i] = (th[i] / rope->scaling_factor) * (1.0f - ramp) + th[i] * ramp;
    }
    conc = 0.1f * std::log(rope->scaling_factor) + 1.0f;
  }
  A_TRY(aalloc(&L->theta, th.size()));
  A_CUDA(cudaMemcpy(L->theta, th.data(), th.size() * sizeof(float), cudaMemcpyHostToDevice));
  L->rope_dim = rd;
  L->concentration = conc;
  return MXMOE_OK;
}

int mxmqa_cache_create(const mxmqa_layer* L, uint32_t batch, uint32_t cache_len, uint32_t sink_tokens,
                       mxmqa_cache** out) {
  if (!L || !out) return afail(MXMOE_ERR_INVALID_ARG, "null argument");
  *out = nullptr;
  if (batch == 0 || cache_len == 0 || sink_tokens > cache_len)
    return afail(MXMOE_ERR_INVALID_ARG, "batch and cache_len must be positive, sink_tokens <= cache_len");
  ADevice g(L->cfg.device);
  mxmqa_cache* C = new (std::nothrow) mxmqa_cache();
  if (!C) return afail(MXMOE_ERR_OOM, "host allocation failed");
  C->device = L->cfg.device;
  C->batch = batch;
  C->cap = cache_len;
  C->sink = sink_tokens;
  C->kv_heads = L->cfg.kv_heads;
  C->head_dim = L->cfg.head_dim;
  const size_t n = static_cast<size_t>(batch) * cache_len * C->kv_heads * C->head_dim;
  int rc = aalloc(&C->k, n);
  if (rc == MXMOE_OK) rc = aalloc(&C->v, n);
  if (rc == MXMOE_OK && (cudaMemset(C->k, 0, n * 4) != cudaSuccess || cudaMemset(C->v, 0, n * 4) != cudaSuccess))
    rc = afail(MXMOE_ERR_CUDA, "cudaMemset of the cache failed");
  if (rc != MXMOE_OK) {
    afree(C->k);
    afree(C->v);
    delete C;
    return rc;
  }
  *out = C;
  return MXMOE_OK;
}

int mxmqa_cache_reset(mxmqa_cache* C) {
  if (!C) return afail(MXMOE_ERR_INVALID_ARG, "null cache");
  C->global_end = C->local_end = 0;
  C->head = 0;
  return MXMOE_OK;
}

int mxmqa_cache_state(const mxmqa_cache* C, uint64_t* global_end, uint64_t* local_end) {
  if (!C) return afail(MXMOE_ERR_INVALID_ARG, "null cache");
  if (global_end) *global_end = C->global_end;
  if (local_end) *local_end = C->local_end;
  return MXMOE_OK;
}

int mxmqa_cache_destroy(mxmqa_cache* C) {
  if (!C) return MXMOE_OK;
  ADevice g(C->device);
  afree(C->k);
  afree(C->v);
  delete C;
  return MXMOE_OK;
}

int mxmqa_forward_streaming(mxmqa_layer* L, mxmqa_cache* C, const void* x, mxmoe_dtype x_dtype, uint32_t batch,
                            uint32_t seq_len, uint64_t start_pos, uint32_t window, const float* sinks,
                            const float* attn_bias, void* y, mxmoe_dtype y_dtype, void* stream) {
  if (!L || !C) return afail(MXMOE_ERR_INVALID_ARG, "null layer or cache");
  if (!L->ready) return afail(MXMOE_ERR_NOT_READY, "weights not set");
  if ((x_dtype != MXMOE_F32 && x_dtype != MXMOE_BF16) || (y_dtype != MXMOE_F32 && y_dtype != MXMOE_BF16))
    return afail(MXMOE_ERR_INVALID_ARG, "bad dtype");
  if (batch != C->batch) return afail(MXMOE_ERR_INVALID_ARG, "batch %u != cache batch %u", batch, C->batch);
  if (C->device != L->cfg.device || C->kv_heads != L->cfg.kv_heads || C->head_dim != L->cfg.head_dim)
    return afail(MXMOE_ERR_INVALID_ARG, "cache does not belong to this layer's shape or device");
  if (seq_len == 0) return MXMOE_OK;
  if (!x || !y) return afail(MXMOE_ERR_INVALID_ARG, "null x or y");
  if (reinterpret_cast<uintptr_t>(x) % 16 != 0) return afail(MXMOE_ERR_INVALID_ARG, "x must be 16-byte aligned");
  ADevice g(L->cfg.device);
  cudaStream_t st = as_stream_a(stream);
  mxmoe::PdlScope pdl(true);
  const int nH = static_cast<int>(L->cfg.n_heads), kvH = static_cast<int>(L->cfg.kv_heads);
  const int dk = static_cast<int>(L->cfg.head_dim), d = static_cast<int>(L->cfg.d_model);
  const int R = static_cast<int>(batch * seq_len);
  const int J = (nH + 2 * kvH) * dk;
  // Cache bookkeeping exactly as src/attention/streaming_mqa.rs:313-370 and
  // evict_and_roll_mqa (src/attention/cache_ops.rs:74-117), with the roll as
  // a ring offset.
  const uint64_t num_new = seq_len, current_end = start_pos + num_new;
  if (current_end < C->global_end) return afail(MXMOE_ERR_INVALID_ARG, "start_pos must be non-decreasing");
  const uint64_t sink = C->sink, cap = C->cap;
  const uint64_t delta = current_end - C->global_end;
  const uint64_t need = C->local_end + delta;
  // Work on copies; the cache state changes only once every check passed.
  uint64_t head = C->head, local_end = C->local_end;
  if (need > cap) {
    const uint64_t num_evicted = need - cap;
    const uint64_t avail = local_end > sink ? local_end - sink : 0;
    if (!(avail == 0 || num_evicted >= avail)) head = (head + num_evicted) % (cap - sink);
    local_end = local_end > num_evicted ? local_end - num_evicted : 0;
  }
  local_end += delta;
  if (local_end < num_new || local_end > cap)
    return afail(MXMOE_ERR_INVALID_ARG, "chunk of %llu tokens does not fit the cache state",
                 (unsigned long long)num_new);
  const uint64_t local_start = local_end - num_new;
  uint64_t active_len = local_end;
  if (window != 0) {
    // The reference's window keeps sink + min(w, local_end - sink) tokens; with
    // fewer than sink tokens cached that is longer than the cache content and
    // its reshape panics (streaming_mqa.rs:333-373): refuse the same case.
    if (local_end < sink)
      return afail(MXMOE_ERR_INVALID_ARG, "windowed attention needs at least sink_tokens (%llu) cached tokens",
                   (unsigned long long)sink);
    active_len = sink + std::min<uint64_t>(window, local_end - sink);
  }
  C->head = static_cast<uint32_t>(head);
  C->local_end = local_end;
  C->global_end = current_end;
  const uint64_t win_start = local_end > active_len ? local_end - active_len : 0;
  // Key splits (flash-decoding): enough (row, KV head, split) blocks for two
  // per SM, each split at least 128 keys (a shorter window is one block's
  // work, and a split costs a merge launch).
  const int base_blocks = R * kvH * ((L->groups + kAttnWarps - 1) / kAttnWarps);
  int splits = std::max(1, std::min({kMaxSplits, static_cast<int>((active_len + 127) / 128),
                                     (2 * L->num_sms + base_blocks - 1) / base_blocks}));
  const int split_len = static_cast<int>((active_len + splits - 1) / splits);
  splits = std::max(1, static_cast<int>((active_len + split_len - 1) / std::max(split_len, 1)));
  // scratch
  const size_t rows = static_cast<size_t>(R);
  if (L->cap_rows < rows) {
    afree(L->qkv); afree(L->ctx);
    L->cap_rows = 0;
    A_TRY(aalloc(&L->qkv, rows * J));
    A_TRY(aalloc(&L->ctx, rows * nH * dk));
    L->cap_rows = rows;
  }
  const size_t part_floats = splits > 1 ? rows * nH * splits * (dk + 2) : 0;
  if (L->cap_part < part_floats) {
    afree(L->part);
    L->cap_part = 0;
    A_TRY(aalloc(&L->part, part_floats));
    L->cap_part = part_floats;
  }
  A_TRY(project(L, x, x_dtype, R, d, L->wqkv, L->bqkv, J, L->qkv, MXMOE_F32, st));
  RopeArgs ra{};
  ra.theta = L->rope_dim ? L->theta : nullptr;
  ra.concentration = L->concentration;
  ra.rope_dim = L->rope_dim;
  ra.by_head = (L->cfg.flags & MXMQA_FLAG_ROPE_BY_HEAD) ? 1 : 0;
  A_CUDA(mxmoe::launch_kernel(rope_cache_kernel, dim3(R), dim3(128), 0, st, L->qkv, static_cast<int>(batch),
                              static_cast<int>(seq_len), nH, kvH, dk, static_cast<int>(start_pos), ra, C->k, C->v,
                              static_cast<int>(cap), static_cast<int>(sink), static_cast<int>(C->head),
                              static_cast<int>(local_start)));
  AttnArgs aa{};
  aa.qkv = L->qkv;
  aa.kc = C->k;
  aa.vc = C->v;
  aa.B = static_cast<int>(batch);
  aa.T = static_cast<int>(seq_len);
  aa.nH = nH;
  aa.kvH = kvH;
  aa.dk = dk;
  aa.cap = static_cast<int>(cap);
  aa.sink = static_cast<int>(sink);
  aa.head = static_cast<int>(C->head);
  aa.win_start = static_cast<int>(win_start);
  aa.win_len = static_cast<int>(active_len);
  aa.scale = (L->cfg.flags & MXMQA_FLAG_PRE_SCALED_QK) ? 1.0f : 1.0f / std::sqrt(static_cast<float>(dk));
  aa.sinks = sinks ? sinks : L->sinks;
  aa.bias = attn_bias;
  aa.quiet = (L->cfg.flags & MXMQA_FLAG_QUIET_SOFTMAX) ? 1 : 0;
  aa.ctx = L->ctx;
  aa.splits = splits;
  aa.split_len = split_len;
  aa.part_ml = L->part;
  aa.part_acc = L->part ? L->part + rows * nH * splits * 2 : nullptr;
  {
    const int hgroups = (L->groups + kAttnWarps - 1) / kAttnWarps;
    const size_t smem = static_cast<size_t>(2) * 2 * kTileKeys * (dk + 4) * sizeof(float);
    A_CUDA(mxmoe::ensure_dynamic_smem(reinterpret_cast<const void*>(attn_split_kernel), smem));
    A_CUDA(mxmoe::launch_kernel(attn_split_kernel, dim3(R, kvH * hgroups, splits), dim3(32 * kAttnWarps), smem, st,
                                aa));
  }
  if (splits > 1)
    A_CUDA(mxmoe::launch_kernel(attn_merge_kernel, dim3((R * nH + 7) / 8), dim3(256), 0, st, aa));
  A_TRY(project(L, L->ctx, MXMOE_F32, R, nH * dk, L->wo, L->bo, d, y, y_dtype, st));
  return MXMOE_OK;
}

}  // extern "C"
