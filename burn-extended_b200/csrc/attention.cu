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
//   dense_gemv_kernel   y[r][j] = sum_c x[r][c] W[j][c] + b[j], weights stored
//                       output-major (bf16 or f32), a warp per output and a
//                       pass of up to 8 rows, 16-byte weight loads, f32 sums.
//   rope_cache_kernel   rotates q and k of every (row, head) by the position
//                       (interleaved pairs, as burn's RotaryEncoding), writes
//                       k and v into the cache at their ring slots.
//   attn_kernel         one block per (batch, query row, head): warps split
//                       the active window; a lane scores one key per step
//                       (q in registers), the warp keeps a running max / sum
//                       and a V accumulator (lane owns d_k / 32 columns);
//                       warps merge in shared memory; the sinks column and
//                       the quiet-softmax 1 join the normalizer.
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

constexpr int kGemvRows = 8;     // rows (tokens) per pass of the projection GEMV
constexpr int kGemvWarps = 8;    // outputs per block
constexpr int kAttnWarps = 8;
constexpr int kMaxHeadDim = 256;

__device__ __forceinline__ float ld_act(const void* p, int dtype, size_t i) {
  return dtype == MXMOE_F32 ? static_cast<const float*>(p)[i]
                            : __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
}

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
// x: [R][K] (f32 or bf16), W: [J][K] output-major, K % 8 == 0.  Each warp
// owns one output j; a pass stages up to kGemvRows rows of x in shared memory
// as f32; lanes stride K in 8-element pieces.  Outputs as f32 (ld = J).
__global__ void __launch_bounds__(32 * kGemvWarps)
    dense_gemv_kernel(const void* __restrict__ x, int x_dtype, int R, int K, const void* __restrict__ W, int wdtype,
                      const float* __restrict__ bias, int J, float* __restrict__ y) {
  extern __shared__ __align__(16) float xs_dense[];  // [kGemvRows][K]
  griddep_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int j = blockIdx.x * kGemvWarps + warp;
  for (int r0 = 0; r0 < R; r0 += kGemvRows) {
    const int nr = min(kGemvRows, R - r0);
    __syncthreads();
    for (int i = threadIdx.x; i < nr * K; i += blockDim.x)
      xs_dense[i] = ld_act(x, x_dtype, static_cast<size_t>(r0) * K + i);
    __syncthreads();
    if (j >= J) continue;
    float acc[kGemvRows];
#pragma unroll
    for (int r = 0; r < kGemvRows; ++r) acc[r] = 0.0f;
    for (int c = lane * 8; c < K; c += 256) {
      float w[8];
      ld_w8(W, wdtype, static_cast<size_t>(j) * K + c, w);
#pragma unroll
      for (int r = 0; r < kGemvRows; ++r) {
        if (r < nr) {
          const float4 a = *reinterpret_cast<const float4*>(xs_dense + r * K + c);
          const float4 b = *reinterpret_cast<const float4*>(xs_dense + r * K + c + 4);
          acc[r] = fmaf(a.x, w[0], acc[r]); acc[r] = fmaf(a.y, w[1], acc[r]);
          acc[r] = fmaf(a.z, w[2], acc[r]); acc[r] = fmaf(a.w, w[3], acc[r]);
          acc[r] = fmaf(b.x, w[4], acc[r]); acc[r] = fmaf(b.y, w[5], acc[r]);
          acc[r] = fmaf(b.z, w[6], acc[r]); acc[r] = fmaf(b.w, w[7], acc[r]);
        }
      }
    }
#pragma unroll
    for (int r = 0; r < kGemvRows; ++r) {
      float v = acc[r];
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
      if (lane == 0 && r < nr) y[static_cast<size_t>(r0 + r) * J + j] = v + (bias ? bias[j] : 0.0f);
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
  float scale;            // 1 / sqrt(d_k) (1 when pre-scaled)
  const float* sinks;     // [nH] or null
  const float* bias;      // [B][nH][T][win_len] or null
  int quiet;
  float* ctx;             // [B*T][nH * dk]
};

// One block per (row = b * T + t, head h).
__global__ void __launch_bounds__(32 * kAttnWarps) attn_kernel(const AttnArgs a) {
  griddep_wait();
  const int row = blockIdx.x, h = blockIdx.y;
  const int b = row / a.T, t = row - b * a.T;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int dk = a.dk, kvh = h / (a.nH / a.kvH);
  const int width = (a.nH + 2 * a.kvH) * dk;
  __shared__ float q_s[kMaxHeadDim];
  __shared__ float m_s[kAttnWarps], l_s[kAttnWarps];
  __shared__ float acc_s[kAttnWarps][kMaxHeadDim];
  for (int i = threadIdx.x; i < dk; i += blockDim.x) q_s[i] = a.qkv[static_cast<size_t>(row) * width + h * dk + i];
  __syncthreads();
  constexpr int kPer = kMaxHeadDim / 32;  // columns per lane (upper bound)
  const int per = (dk + 31) / 32;
  float m = -INFINITY, l = 0.0f;
  float acc[kPer];
#pragma unroll
  for (int i = 0; i < kPer; ++i) acc[i] = 0.0f;
  const float* bias_row =
      a.bias ? a.bias + ((static_cast<size_t>(b) * a.nH + h) * a.T + t) * a.win_len : nullptr;
  // warp w takes keys w * 32 + lane, w * 32 + lane + 32 * kAttnWarps, ...
  for (int j0 = warp * 32; j0 < a.win_len; j0 += 32 * kAttnWarps) {
    const int j = j0 + lane;
    float s = -INFINITY;
    if (j < a.win_len) {
      const int slot = ring_slot(a.win_start + j, a.sink, a.cap, a.head);
      const float* kr = a.kc + ((static_cast<size_t>(b) * a.cap + slot) * a.kvH + kvh) * dk;
      float dot = 0.0f;
      for (int c = 0; c < dk; c += 4) {
        const float4 kv4 = *reinterpret_cast<const float4*>(kr + c);
        dot = fmaf(q_s[c], kv4.x, dot);
        dot = fmaf(q_s[c + 1], kv4.y, dot);
        dot = fmaf(q_s[c + 2], kv4.z, dot);
        dot = fmaf(q_s[c + 3], kv4.w, dot);
      }
      s = dot * a.scale;
      if (bias_row) s += bias_row[j];
    }
    // running softmax over the warp's keys
    float mb = s;
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) mb = fmaxf(mb, __shfl_xor_sync(0xFFFFFFFFu, mb, o));
    const float mn = fmaxf(m, mb);
    const float p = (j < a.win_len && s != -INFINITY) ? expf(s - mn) : 0.0f;
    const float corr = (m == -INFINITY) ? 0.0f : expf(m - mn);
    float ps = p;
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) ps += __shfl_xor_sync(0xFFFFFFFFu, ps, o);
    l = l * corr + ps;
#pragma unroll
    for (int i = 0; i < kPer; ++i) acc[i] *= corr;
    m = mn;
    // V accumulation: lane owns columns lane + 32 i
    const int nk = min(32, a.win_len - j0);
    for (int u = 0; u < nk; ++u) {
      const float pu = __shfl_sync(0xFFFFFFFFu, p, u);
      const int slot = ring_slot(a.win_start + j0 + u, a.sink, a.cap, a.head);
      const float* vr = a.vc + ((static_cast<size_t>(b) * a.cap + slot) * a.kvH + kvh) * dk;
#pragma unroll
      for (int i = 0; i < kPer; ++i)
        if (i < per && lane + 32 * i < dk) acc[i] = fmaf(pu, vr[lane + 32 * i], acc[i]);
    }
  }
  if (lane == 0) {
    m_s[warp] = m;
    l_s[warp] = l;
  }
#pragma unroll
  for (int i = 0; i < kPer; ++i)
    if (i < per && lane + 32 * i < dk) acc_s[warp][lane + 32 * i] = acc[i];
  __syncthreads();
  // merge the warps, then the sinks column and the quiet-softmax term
  float M = -INFINITY;
  for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, m_s[w]);
  const float sink = a.sinks ? a.sinks[h] : -INFINITY;
  const float Mt = fmaxf(M, sink);
  float L = 0.0f;
  for (int w = 0; w < kAttnWarps; ++w)
    if (m_s[w] != -INFINITY) L += l_s[w] * expf(m_s[w] - Mt);
  if (a.sinks) L += expf(sink - Mt);
  if (a.quiet) L += expf(-Mt);
  for (int c = threadIdx.x; c < dk; c += blockDim.x) {
    float v = 0.0f;
    for (int w = 0; w < kAttnWarps; ++w)
      if (m_s[w] != -INFINITY) v += acc_s[w][c] * expf(m_s[w] - Mt);
    a.ctx[static_cast<size_t>(row) * a.nH * dk + h * dk + c] = L > 0.0f ? v / L : 0.0f;
  }
}

__global__ void cast_rows_kernel(const float* __restrict__ src, size_t n, void* dst, int dtype) {
  griddep_wait();
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    if (dtype == MXMOE_F32)
      static_cast<float*>(dst)[i] = src[i];
    else
      static_cast<__nv_bfloat16*>(dst)[i] = __float2bfloat16_rn(src[i]);
  }
}

cudaError_t launch_gemv(const void* x, int x_dtype, int R, int K, const void* W, int wdtype, const float* bias, int J,
                        float* y, cudaStream_t st) {
  const size_t smem = static_cast<size_t>(kGemvRows) * K * sizeof(float);
  const cudaError_t e = mxmoe::ensure_dynamic_smem(reinterpret_cast<const void*>(dense_gemv_kernel), smem);
  if (e != cudaSuccess) return e;
  return mxmoe::launch_kernel(dense_gemv_kernel, dim3((J + kGemvWarps - 1) / kGemvWarps), dim3(32 * kGemvWarps), smem,
                              st, x, x_dtype, R, K, W, wdtype, bias, J, y);
}

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
  float* y32 = nullptr;
  size_t cap_rows = 0;
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
  *out = L;
  return MXMOE_OK;
}

int mxmqa_destroy(mxmqa_layer* L) {
  if (!L) return MXMOE_OK;
  ADevice g(L->cfg.device);
  afree(L->wqkv); afree(L->bqkv); afree(L->wo); afree(L->bo); afree(L->sinks); afree(L->theta);
  afree(L->qkv); afree(L->ctx); afree(L->y32);
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
  // scratch
  const size_t rows = static_cast<size_t>(R);
  if (L->cap_rows < rows) {
    afree(L->qkv); afree(L->ctx); afree(L->y32);
    L->cap_rows = 0;
    A_TRY(aalloc(&L->qkv, rows * J));
    A_TRY(aalloc(&L->ctx, rows * nH * dk));
    A_TRY(aalloc(&L->y32, rows * d));
    L->cap_rows = rows;
  }
  A_CUDA(launch_gemv(x, x_dtype, R, d, L->wqkv, L->wdtype, L->bqkv, J, L->qkv, st));
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
  A_CUDA(mxmoe::launch_kernel(attn_kernel, dim3(R, nH), dim3(32 * kAttnWarps), 0, st, aa));
  A_CUDA(launch_gemv(L->ctx, MXMOE_F32, R, nH * dk, L->wo, L->wdtype, L->bo, d, L->y32, st));
  A_CUDA(mxmoe::launch_kernel(cast_rows_kernel, dim3(std::min<size_t>((rows * d + 255) / 256, 1184)), dim3(256), 0,
                              st, static_cast<const float*>(L->y32), rows * d, y, static_cast<int>(y_dtype)));
  return MXMOE_OK;
}

}  // extern "C"
