// gemm_tc.cu -- grouped expert GEMM on the 5th-generation tensor cores.
//
// One persistent kernel serves both expert projections of the MoE block
// (reference: w1_swiglu_dense_kernel / w2_scatter_dense_kernel,
// src/quant/gpu.rs:89-146 and :148-192, launched per expert and f-tile at
// src/moe/mod.rs:316-404):
//   mode 1 (W1):  act = SwiGLUclamp(r_t * (W1_glu x_t) + b_glu, r_t * (W1_lin x_t) + b_lin)
//                 written back as two block-scaled E4M3 terms for mode 2;
//   mode 2 (W2):  y_pair = (W2 act + b2) * w_route.
// Each tile is 128 weight rows (M) x N routed pairs (N = 32..256) of one
// expert.  Operand A = MXFP4 weights exactly as stored (E2M1 codes + E8M0
// scales, loaded by TMA with the 4-bit -> byte-container expansion); operand B
// = activations as hi + lo E4M3 terms, so one k-step issues two
// kind::mxf8f6f4.block_scale MMAs into the same fp32 TMEM accumulator.
//
// Warp roles (192 threads): warp 0 = TMA producer, warp 1 = TMEM owner + MMA
// issuer, warps 2..5 = epilogue (TMEM -> registers -> global).
#include <cuda.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include "layout.cuh"
#include "ptx.cuh"
#include "quant.cuh"
#include "tc_gemm.h"

namespace mxmoe {

namespace {

constexpr int kThreads = 192;
constexpr int kEpiThreads = 128;
constexpr int kMaxStages = 8;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kSfTmemBase = 256;  // scale factors live in columns 256.. (32 per stage)
constexpr int kXchgPitch = 17;         // floats per row of the GLU/linear exchange buffer

struct SmemPlan {
  uint32_t a_bytes, b_bytes, stage_bytes;
};

__host__ __device__ inline SmemPlan smem_plan(int N, int terms) {
  SmemPlan s;
  s.a_bytes = 128 * kTileK;                     // E2M1 codes expanded to byte containers
  s.b_bytes = static_cast<uint32_t>(N) * kTileK;  // E4M3, one term
  uint32_t raw = s.a_bytes + terms * s.b_bytes + kSfAtomBytes + terms * 2 * kSfAtomBytes;
  s.stage_bytes = round_up(raw, 1024);
  return s;
}

__device__ __forceinline__ void named_bar_epi() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// Largest expert e in [0, E) whose first tile index is <= t.
__device__ __forceinline__ void decode_tile(const TcParams& p, int t, int& e, int& mt, int& nt, int& nte) {
  int lo = 0, hi = p.E;
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (p.m_tiles * __ldg(p.ntile_prefix + mid) <= t) lo = mid; else hi = mid;
  }
  e = lo;
  const int base = p.m_tiles * __ldg(p.ntile_prefix + e);
  nte = __ldg(p.ntile_prefix + e + 1) - __ldg(p.ntile_prefix + e);
  const int local = t - base;
  mt = nte > 0 ? local / nte : 0;
  nt = nte > 0 ? local % nte : 0;
}

__global__ void __launch_bounds__(kThreads, 1)
    tc_moe_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                       const TcParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const SmemPlan plan = smem_plan(p.N, p.b_terms);
  const int terms = p.b_terms;
  const int S = p.stages;
  float* xchg = reinterpret_cast<float*>(smem + S * plan.stage_bytes);
  uint64_t* bars = reinterpret_cast<uint64_t*>(xchg + 64 * kXchgPitch);
  uint64_t* full_bar = bars;
  uint64_t* empty_bar = bars + kMaxStages;
  uint64_t* tmem_full = bars + 2 * kMaxStages;
  uint64_t* tmem_empty = tmem_full + 1;
  uint64_t* drain_bar = tmem_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  int* err = p.err;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    mbar_init(tmem_full, 1);
    mbar_init(tmem_empty, kEpiThreads);
    mbar_init(drain_bar, 1);
    fence_barrier_init();
    prefetch_tmap(&tmap_a);
    prefetch_tmap(&tmap_b);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int total_tiles = p.m_tiles * __ldg(p.ntile_prefix + p.E);
  const int N = p.N;

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------------ producer
    int stage = 0;
    uint32_t phase = 0;
    uint32_t issued_parity[kMaxStages];
    bool issued[kMaxStages];
    for (int s = 0; s < kMaxStages; ++s) { issued[s] = false; issued_parity[s] = 0; }
    bool ok = true;
    for (int t = blockIdx.x; t < total_tiles && ok; t += gridDim.x) {
      int e, mt, nt, nte;
      decode_tile(p, t, e, mt, nt, nte);
      const int row0 = __ldg(p.poff + e) + nt * N;  // first activation row of the tile
      const int natoms = (N + p.sf_rows - 1) / p.sf_rows;  // scale atoms per tile and term
      const uint32_t tx = plan.a_bytes / 2 + terms * plan.b_bytes + kSfAtomBytes * (1 + terms * natoms);
      for (int kt = 0; kt < p.k_tiles; ++kt) {
        if (!mbar_wait(&empty_bar[stage], phase ^ 1u, err, kDevTimeoutEmpty)) { ok = false; break; }
        uint8_t* sb = smem + stage * plan.stage_bytes;
        mbar_arrive_expect_tx(&full_bar[stage], tx);
        tma_load_3d(sb, &tmap_a, &full_bar[stage], kt * kTileK, mt * 128, e);
        for (int term = 0; term < terms; ++term)
          tma_load_3d(sb + plan.a_bytes + term * plan.b_bytes, &tmap_b, &full_bar[stage], kt * kTileK, row0, term);
        uint8_t* sf = sb + plan.a_bytes + terms * plan.b_bytes;
        bulk_load(sf, p.a_sf + ((static_cast<uint64_t>(e) * p.m_tiles + mt) * p.k_tiles + kt) * kSfAtomBytes,
                  kSfAtomBytes, &full_bar[stage]);
        const uint64_t rb = static_cast<uint64_t>(row0) / p.sf_rows;
        for (int term = 0; term < terms; ++term)
          for (int a = 0; a < natoms; ++a)
            bulk_load(sf + kSfAtomBytes * (1 + term * 2 + a),
                      p.b_sf + term * p.b_sf_term_stride + ((rb + a) * p.k_tiles + kt) * kSfAtomBytes,
                      kSfAtomBytes, &full_bar[stage]);
        issued[stage] = true;
        issued_parity[stage] = phase;
        if (++stage == S) { stage = 0; phase ^= 1u; }
      }
    }
    // Drain: make sure no TMA write into this CTA's smem is still in flight.
    for (int s = 0; s < S; ++s)
      if (issued[s]) {
        mbar_wait(&full_bar[s], issued_parity[s], nullptr, kDevTimeoutDrain);
      }
  } else if (warp == 1 && lane == 0) {
    // ------------------------------------------------------------ MMA issuer
    int stage = 0;
    uint32_t phase = 0, acc_phase = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < total_tiles && ok; t += gridDim.x) {
      int e, mt, nt, nte;
      decode_tile(p, t, e, mt, nt, nte);
      const int natoms = (N + p.sf_rows - 1) / p.sf_rows;
      if (!mbar_wait(tmem_empty, acc_phase ^ 1u, err, kDevTimeoutTmemEmpty)) break;
      acc_phase ^= 1u;
      tc_fence_after();
      for (int kt = 0; kt < p.k_tiles; ++kt) {
        if (!mbar_wait(&full_bar[stage], phase, err, kDevTimeoutFull)) { ok = false; break; }
        tc_fence_after();
        uint8_t* sb = smem + stage * plan.stage_bytes;
        const uint32_t a_addr = smem_u32(sb);
        const uint32_t b_addr0 = smem_u32(sb + plan.a_bytes);
        const uint32_t sf_addr = smem_u32(sb + plan.a_bytes + terms * plan.b_bytes);
        const uint32_t sfa_col = kSfTmemBase + stage * 32;
        // scale factors: smem atoms -> TMEM (32 lanes x 16 B, replicated to 4 sub-partitions)
        tc_cp_32x128b_warpx4(tmem_base + sfa_col, make_smem_desc(sf_addr, 0, 128, 0));
        for (int term = 0; term < terms; ++term)
          for (int a = 0; a < natoms; ++a)
            tc_cp_32x128b_warpx4(tmem_base + sfa_col + 4 + term * 8 + a * 4,
                                 make_smem_desc(sf_addr + kSfAtomBytes * (1 + term * 2 + a), 0, 128, 0));
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const uint64_t a_desc = make_smem_desc(a_addr + kk * 32, 16, 1024, 2);
          for (int term = 0; term < terms; ++term) {
            const uint64_t b_desc = make_smem_desc(b_addr0 + term * plan.b_bytes + kk * 32, 16, 1024, 2);
            const uint32_t idesc = make_idesc_mxf8f6f4(5u, 0u, 128u, static_cast<uint32_t>(N), kk, kk);
            const uint32_t sfa = (tmem_base + sfa_col) | (static_cast<uint32_t>(kk) << 30);
            const uint32_t sfb = (tmem_base + sfa_col + 4 + term * 8) | (static_cast<uint32_t>(kk) << 30);
            tc_mma_mxf8f6f4(tmem_base, a_desc, b_desc, idesc, sfa, sfb, (kt | kk | term) != 0 ? 1u : 0u);
          }
        }
        tc_commit(&empty_bar[stage]);
        if (++stage == S) { stage = 0; phase ^= 1u; }
      }
      if (!ok) break;
      tc_commit(tmem_full);
    }
    // Drain: every MMA issued by this thread has finished before TMEM is freed.
    tc_commit(drain_bar);
    mbar_wait(drain_bar, 0, nullptr, kDevTimeoutDrain);
  } else if (warp >= 2) {
    // ------------------------------------------------------------ epilogue
    const int sp = warp & 3;              // TMEM sub-partition this warp may access
    const int m = sp * 32 + lane;         // accumulator row (weight row within the tile)
    const uint32_t trow = tmem_base + (static_cast<uint32_t>(sp * 32) << 16);
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < total_tiles; t += gridDim.x) {
      int e, mt, nt, nte;
      decode_tile(p, t, e, mt, nt, nte);
      if (!mbar_wait(tmem_full, acc_phase, err, kDevTimeoutTmemFull)) break;
      acc_phase ^= 1u;
      tc_fence_after();
      const int cnt = __ldg(p.counts + e);
      const int n_valid = min(N, cnt - nt * N);
      const int pos0 = __ldg(p.poff + e) + nt * N;
      if (p.mode == 2) {
        const int c = mt * 128 + m;
        const bool row_ok = c < p.rows_valid;
        const float bias = row_ok ? __ldg(p.bias + static_cast<uint64_t>(e) * p.bias_stride + c) * p.bias_mult : 0.f;
        for (int c0 = 0; c0 < n_valid; c0 += 16) {
          float v[16];
          tmem_ld_32x32b_x16(trow + c0, v);
          if (row_ok) {
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const int n = c0 + i;
              if (n < n_valid) {
                const int pos = pos0 + n;
                const float w = __ldg(p.topk_w + __ldg(p.perm + pos));
                p.y_pair[static_cast<uint64_t>(pos) * p.d + c] = (v[i] + bias) * w;
              }
            }
          }
        }
      } else {
        // W1: lanes 0..63 hold GLU rows, 64..127 the matching linear rows.
        const bool glu = m < 64;
        const int jl = glu ? m : m - 64;
        const int j = mt * 64 + jl;  // GLU unit index
        const uint64_t brow = static_cast<uint64_t>(e) * p.bias_stride;
        const float b_g = __ldg(p.bias + brow + mt * 128 + jl);
        const float b_l = __ldg(p.bias + brow + mt * 128 + 64 + jl);
        for (int c0 = 0; c0 < n_valid; c0 += 16) {
          float v[16];
          tmem_ld_32x32b_x16(trow + c0, v);
          if (!glu) {
#pragma unroll
            for (int i = 0; i < 16; ++i) xchg[jl * kXchgPitch + i] = v[i];
          }
          named_bar_epi();
          if (glu) {
#pragma unroll 1
            for (int i = 0; i < 16; ++i) {
              const int n = c0 + i;
              if (n >= n_valid) break;  // uniform across the warp
              const int pos = pos0 + n;
              const int tok = __ldg(p.perm + pos) / p.k;
              const float r = __ldg(p.rscale + tok);
              const float g = fmaf(v[i], r, b_g);
              const float l = fmaf(xchg[jl * kXchgPitch + i], r, b_l);
              const float xg = fminf(g, p.limit);
              const float xl = fmaxf(-p.limit, fminf(l, p.limit));
              const float a = (xg / (1.0f + expf(-p.alpha * xg))) * (xl + 1.0f);
              uint8_t code[kMaxTerms], sbyte[kMaxTerms];
              split_e4m3_terms(a, 2, code, sbyte);
              const uint64_t off = static_cast<uint64_t>(pos) * p.act_kp + j;
              p.act_codes[off] = code[0];
              p.act_codes[p.act_term_stride + off] = code[1];
              if (lane == 0) {
                const uint64_t so = sf_offset(static_cast<uint32_t>(pos), static_cast<uint32_t>(j / 32),
                                              static_cast<uint32_t>(p.act_kchunks), static_cast<uint32_t>(p.sf_rows));
                p.act_sf[so] = sbyte[0];
                p.act_sf[p.act_sf_term_stride + so] = sbyte[1];
              }
            }
          }
          named_bar_epi();
        }
      }
      tc_fence_before();
      mbar_arrive(tmem_empty);
    }
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

}  // namespace

size_t tc_gemm_smem_bytes(int N, int terms, int stages) {
  const SmemPlan plan = smem_plan(N, terms);
  return 1024 + static_cast<size_t>(stages) * plan.stage_bytes + 64 * kXchgPitch * sizeof(float) +
         (2 * kMaxStages + 4) * sizeof(uint64_t);
}

int tc_gemm_max_stages(int N, int terms, size_t smem_limit) {
  int s = kMaxStages;
  while (s > 1 && tc_gemm_smem_bytes(N, terms, s) > smem_limit) --s;
  return s;
}

cudaError_t tc_gemm_launch(const CUtensorMap& tmap_a, const CUtensorMap& tmap_b, const TcParams& p, int grid,
                           cudaStream_t stream) {
  const size_t smem = tc_gemm_smem_bytes(p.N, p.b_terms, p.stages);
  cudaError_t st = cudaFuncSetAttribute(tc_moe_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        static_cast<int>(smem));
  if (st != cudaSuccess) return st;
  tc_moe_gemm_kernel<<<grid, kThreads, smem, stream>>>(tmap_a, tmap_b, p);
  return cudaGetLastError();
}

}  // namespace mxmoe
