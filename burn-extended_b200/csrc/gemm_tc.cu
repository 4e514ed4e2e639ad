// gemm_tc.cu -- grouped expert GEMM on the 5th-generation tensor cores.
//
// Persistent kernels serving both expert projections of the MoE block
// (reference: w1_swiglu_dense_kernel / w2_scatter_dense_kernel,
// src/quant/gpu.rs:89-146 and :148-192, launched per expert and f-tile at
// src/moe/mod.rs:316-404):
//   mode 1 (W1):  act = SwiGLUclamp(r_t * (W1_glu x_t) + b_glu, r_t * (W1_lin x_t) + b_lin)
//                 written back as two block-scaled E4M3 terms for mode 2;
//   mode 2 (W2):  y_pair = (W2 act + b2) * w_route.
// Weights are the MXFP4 codes and E8M0 scales exactly as stored (TMA expands
// the 4-bit codes into byte containers in shared memory); activations are a
// sum of block-scaled E4M3 terms, so one k-step issues one
// kind::mxf8f6f4.block_scale MMA per term into the same fp32 TMEM accumulator.
//
// Three tile shapes:
//   weights-as-A (decode, few pairs per expert): 128 weight rows x N pairs,
//     N = 32..128, double-buffered accumulator;
//   tokens-as-A (prefill): 128 pairs x 256 weight rows, so that each epilogue
//     thread owns one pair's row and quantizes 32-wide blocks on its own;
//   FP4 tokens-as-A (decode, few pairs per expert): kind::mxf4 with packed
//     E2M1 weights and a four-term E2M1 activation, the four terms of 32
//     pairs stacked in one 128-row operand; W1 writes its activation in f32
//     for a separate quantization pass.  One instruction covers K = 64
//     at the cycle cost of a K = 32 mxf8f6f4 one, which halves the tensor
//     time per weight byte where decode would otherwise be MMA-bound.
// Warp roles: warp 0 = TMA producer, warp 1 = TMEM owner + MMA issuer, then the
// epilogue warps (TMEM -> registers -> global: 2..5 for weights-as-A, 2..9 for
// tokens-as-A) and one warp that moves each stage's scale factors from shared
// memory into TMEM so that the MMA thread only issues MMAs.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include "layout.cuh"
#include "ptx.cuh"
#include "quant.cuh"
#include "tc_gemm.h"
#include "launch_util.h"

namespace mxmoe {

namespace {

// weights-as-A: 7 warps (4 epilogue); tokens-as-A: 11 warps (8 epilogue, two
// per TMEM sub-partition, one per 128-column half of the accumulator).  The
// last warp copies each stage's scale factors into TMEM, off the MMA thread.
__host__ __device__ constexpr int num_threads(bool tok) { return tok ? 352 : 224; }
__host__ __device__ constexpr int sf_warp(bool tok) { return tok ? 10 : 6; }
__host__ __device__ constexpr int num_epi_threads(bool tok) { return tok ? 256 : 128; }
constexpr int kMaxStages = 8;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kSfTmemBase = 256;  // scale factors live in columns 256.. (32 per stage)
constexpr int kChunk = 32;             // weights-as-A epilogue column chunk
constexpr int kXPitch = kChunk + 1;    // linear-half exchange [64][33]
constexpr int kAPitch = 64 + 1;        // activation staging [32][65]

struct SmemPlan {
  uint32_t a_bytes, b_bytes, stage_bytes, a_terms, b_terms;
};

// Weights-as-A: A = 128 weight rows (FP4 in byte containers), B = N rows per term.
// Tokens-as-A:  A = 128 token rows per term (E4M3), B = 256 weight rows.
// Tokens-as-A loads only the PT (= pair tile) rows of each activation term;
// the MMA still reads 128 rows, the rows past PT falling into the next buffer
// of the same stage and only feeding accumulator rows that are discarded.
// Stacked tokens-as-A tiles hold both terms of PT pairs in 2 * PT rows.
__host__ __device__ inline SmemPlan smem_plan(bool tok, int N, int terms, int PT, bool stacked, bool fp4 = false) {
  SmemPlan s;
  if (fp4) {
    // packed E2M1 rows of K = 256 (128 bytes): 4 * PT activation rows, 256 weight rows
    s.a_terms = 1;
    s.b_terms = 1;
    s.a_bytes = static_cast<uint32_t>(kF4Terms) * static_cast<uint32_t>(PT) * 128u;
    s.b_bytes = 256u * 128u;
  } else if (!tok) {
    s.a_terms = 1;
    s.b_terms = terms;
    s.a_bytes = 128 * kTileK;
    s.b_bytes = static_cast<uint32_t>(N) * kTileK;
  } else if (stacked) {
    s.a_terms = 1;
    s.b_terms = 1;
    s.a_bytes = 2u * static_cast<uint32_t>(PT) * kTileK;
    s.b_bytes = 256 * kTileK;
  } else {
    s.a_terms = terms;
    s.b_terms = 1;
    s.a_bytes = static_cast<uint32_t>(PT) * kTileK;
    s.b_bytes = 256 * kTileK;
  }
  const uint32_t raw = s.a_terms * s.a_bytes + s.b_terms * s.b_bytes + 6 * kSfAtomBytes;
  s.stage_bytes = round_up(raw, 1024);
  return s;
}

__host__ __device__ inline uint32_t epi_smem_bytes(bool tok) {
  return tok ? 0u : static_cast<uint32_t>((64 * kXPitch + kChunk * kAPitch + 2 * kChunk) * sizeof(float));
}

__device__ __forceinline__ void named_bar_epi() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// Tile t -> (expert e, weight tile wt, pair tile pt).  Tiles of expert e are
// [m_tiles * prefix[e], m_tiles * prefix[e+1]), ordered weight tile major so
// that the pair tiles sharing one weight tile run on neighbouring CTAs and
// meet it in L2.
__device__ __forceinline__ void decode_tile(const TcParams& p, int t, int& e, int& wt, int& pt) {
  int lo = 0, hi = p.E;
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (p.m_tiles * __ldg(p.ntile_prefix + mid) <= t) lo = mid; else hi = mid;
  }
  e = lo;
  const int base = p.m_tiles * __ldg(p.ntile_prefix + e);
  const int nte = __ldg(p.ntile_prefix + e + 1) - __ldg(p.ntile_prefix + e);
  const int local = t - base;
  wt = nte > 0 ? local / nte : 0;
  pt = nte > 0 ? local % nte : 0;
}

__device__ __forceinline__ float swiglu_clamp(float g, float l, float alpha, float limit) {
  const float xg = fminf(g, limit);
  const float xl = fmaxf(-limit, fminf(l, limit));
  // x * sigmoid(alpha x) with the fast exponential and divide (relative error
  // ~1e-7, far inside the layer tolerance); a huge exponent gives 0.
  return __fdividef(xg, 1.0f + __expf(-alpha * xg)) * (xl + 1.0f);
}

// Scale byte of (row pos, term t, k block kb) in the activation atom arrays:
// plain (one atom per sf_rows rows and term, term arrays act_sf_term_stride
// apart) or stacked (layout.cuh, stacked_sf_offset).
__device__ __forceinline__ uint64_t act_sf_offset(const TcParams& p, int pos, int t, int kb) {
  if (p.stacked)
    return stacked_sf_offset(static_cast<uint32_t>(pos), static_cast<uint32_t>(t), static_cast<uint32_t>(kb),
                             static_cast<uint32_t>(p.act_kchunks), static_cast<uint32_t>(p.sf_rows));
  return t * p.act_sf_term_stride + sf_offset(static_cast<uint32_t>(pos), static_cast<uint32_t>(kb),
                                              static_cast<uint32_t>(p.act_kchunks),
                                              static_cast<uint32_t>(p.sf_rows));
}

__device__ __forceinline__ void store_block_terms(const TcParams& p, int pos, int j0,
                                                  const uint32_t (&words)[kMaxTerms][8],
                                                  const uint8_t (&sbyte)[kMaxTerms]) {
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    const uint64_t off =
        p.stacked ? static_cast<uint64_t>(stacked_code_row(static_cast<uint32_t>(pos), static_cast<uint32_t>(t),
                                                                       static_cast<uint32_t>(p.sf_rows))) *
                            p.act_kp + j0
                  : t * p.act_term_stride + static_cast<uint64_t>(pos) * p.act_kp + j0;
    uint4* dst = reinterpret_cast<uint4*>(p.act_codes + off);
    dst[0] = make_uint4(words[t][0], words[t][1], words[t][2], words[t][3]);
    dst[1] = make_uint4(words[t][4], words[t][5], words[t][6], words[t][7]);
    p.act_sf[act_sf_offset(p, pos, t, j0 / 32)] = sbyte[t];
  }
}

// W2 output row of a pair: this GPU's y_pair (row pos) or, for the
// expert-parallel return, the source GPU's buffer at the pair's return slot.
__device__ __forceinline__ __nv_bfloat16* w2_out_row(const TcParams& p, int pos, int pair) {
  if (p.ret_ptrs != nullptr) {
    const uint32_t slot = __ldg(p.ret_slot + pair);
    return static_cast<__nv_bfloat16*>(p.ret_ptrs[slot >> 24]) + static_cast<uint64_t>(slot & 0xFFFFFFu) * p.d;
  }
  return p.y_pair_bf16 + static_cast<uint64_t>(p.y_by_pair ? pair : pos) * p.d;
}

// 8 outputs (bias, route weight) -> 8 bf16 in one 16-byte store.
__device__ __forceinline__ void store_w2_8(__nv_bfloat16* dst, const float* v, float4 b0, float4 b1, float bm,
                                           float w) {
  const __nv_bfloat162 a = __floats2bfloat162_rn(fmaf(b0.x, bm, v[0]) * w, fmaf(b0.y, bm, v[1]) * w);
  const __nv_bfloat162 b = __floats2bfloat162_rn(fmaf(b0.z, bm, v[2]) * w, fmaf(b0.w, bm, v[3]) * w);
  const __nv_bfloat162 c = __floats2bfloat162_rn(fmaf(b1.x, bm, v[4]) * w, fmaf(b1.y, bm, v[5]) * w);
  const __nv_bfloat162 e = __floats2bfloat162_rn(fmaf(b1.z, bm, v[6]) * w, fmaf(b1.w, bm, v[7]) * w);
  *reinterpret_cast<uint4*>(dst) =
      make_uint4(*reinterpret_cast<const uint32_t*>(&a), *reinterpret_cast<const uint32_t*>(&b),
                 *reinterpret_cast<const uint32_t*>(&c), *reinterpret_cast<const uint32_t*>(&e));
}

// kKind: 0 = weights-as-A, 1 = tokens-as-A, 2 = FP4 tokens-as-A (stacked).
template <int kKind>
__global__ void __launch_bounds__(num_threads(kKind != 0), 1)
    tc_moe_gemm_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
                       const TcParams p) {
  constexpr bool kTok = kKind != 0;
  constexpr bool kF4 = kKind == 2;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const SmemPlan plan = smem_plan(kTok, p.N, p.b_terms, p.sf_rows, kTok && p.stacked, kF4);
  const int S = p.stages;
  float* epi = reinterpret_cast<float*>(smem + S * plan.stage_bytes);
  uint64_t* bars = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(epi) + epi_smem_bytes(kTok));
  uint64_t* full_bar = bars;
  uint64_t* empty_bar = bars + kMaxStages;
  uint64_t* tmem_full = bars + 2 * kMaxStages;  // [2]
  uint64_t* tmem_empty = tmem_full + 2;         // [2]
  uint64_t* drain_bar = tmem_full + 4;
  uint64_t* sf_drain = tmem_full + 5;
  uint64_t* sf_full = tmem_full + 6;  // [kMaxStages] scale factors of the stage are in TMEM
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sf_full + kMaxStages);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  int* err = p.err;
  const unsigned long long wait_ns = p.wait_ns ? p.wait_ns : kWaitTimeoutNs;
  const int N = p.N;                             // weights-as-A: pairs per tile; tokens-as-A: 256
  const int PT = kTok ? p.sf_rows : N;           // pairs per tile
  const int nacc = (!kTok && N <= 128) ? 2 : 1;  // accumulator buffers
  const int terms = p.b_terms;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tmem_full[b], 1);
      mbar_init(&tmem_empty[b], num_epi_threads(kTok));
    }
    mbar_init(drain_bar, 1);
    mbar_init(sf_drain, 1);
    for (int s = 0; s < S; ++s) mbar_init(&sf_full[s], 1);
    fence_barrier_init();
    prefetch_tmap(&tmap_w);
    prefetch_tmap(&tmap_x);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int t_lo = p.m_tiles * __ldg(p.ntile_prefix + p.e_lo);
  const int total_tiles = p.m_tiles * __ldg(p.ntile_prefix + (p.e_hi > 0 ? p.e_hi : p.E));
  // With a programmatic launch the setup above overlapped the previous
  // kernel.  So can the first weight boxes: the tile list comes from the
  // permutation, which completed before the previous kernel started its
  // work, and the weights never change -- prefetch them into L2, then wait
  // for the previous kernel's output (the activation operand).
  if (kTok && warp == 0 && lane == 0 && t_lo + static_cast<int>(blockIdx.x) < total_tiles) {
    int e, wt, pt;
    decode_tile(p, t_lo + static_cast<int>(blockIdx.x), e, wt, pt);
    const int nk = min(p.stages, p.k_tiles);
    for (int kt = 0; kt < nk; ++kt) tma_prefetch_3d(&tmap_w, kt * (kF4 ? 128 : kTileK), wt * 256, e);
  }
  griddep_wait();
  const int natoms_x = kTok ? 1 : (N + p.sf_rows - 1) / p.sf_rows;  // activation atoms per term
  const int natoms_w = kTok ? 2 : 1;                                 // weight atoms

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------------ producer
    int stage = 0;
    uint32_t phase = 0;
    uint32_t issued_parity[kMaxStages];
    bool issued[kMaxStages];
    for (int s = 0; s < kMaxStages; ++s) {
      issued[s] = false;
      issued_parity[s] = 0;
    }
    const uint32_t w_tx = (kTok ? 256 : 128) * kTileK / 2;  // packed FP4 bytes
    const uint32_t x_tx = PT * kTileK;                      // E4M3 bytes per term
    const int nsf_x = (kTok && p.stacked) ? 1 : terms * natoms_x;  // activation scale atoms per stage
    const uint32_t tx = w_tx + terms * x_tx + kSfAtomBytes * (natoms_w + nsf_x);
    const uint64_t w_policy = kF4 ? l2_evict_first_policy() : 0;
    bool ok = true;
    for (int t = t_lo + static_cast<int>(blockIdx.x); t < total_tiles && ok; t += gridDim.x) {
      int e, wt, pt;
      decode_tile(p, t, e, wt, pt);
      const int row0 = __ldg(p.poff + e) + pt * PT;  // first activation row of the tile
      const uint64_t rbx = static_cast<uint64_t>(row0) / p.sf_rows;
      for (int kt = 0; kt < p.k_tiles; ++kt) {
        if (!mbar_wait(&empty_bar[stage], phase ^ 1u, err, kDevTimeoutEmpty, wait_ns)) {
          ok = false;
          break;
        }
        if (p.skip_stage && blockIdx.x == 0 && t == t_lo && kt == 0) {
          // test hook: this stage is never armed; the MMA issuer's wait for it runs out
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
          }
          continue;
        }
        uint8_t* sb = smem + stage * plan.stage_bytes;
        uint8_t* w_s = kTok ? sb + plan.a_terms * plan.a_bytes : sb;
        uint8_t* x_s = kTok ? sb : sb + plan.a_bytes;
        const uint32_t x_stride = kTok ? plan.a_bytes : plan.b_bytes;
        uint8_t* sf = sb + plan.a_terms * plan.a_bytes + plan.b_terms * plan.b_bytes;
        if constexpr (kF4) {
          // one stage = K 256: the weight tile's packed rows, the tile's 4 * PT
          // stacked activation rows, and the scale atoms of the stage's one or
          // two 128-K chunks (weights: the 256-row atom pair per chunk,
          // adjacent chunks contiguous; activation: one atom per chunk)
          const int nch = min(2, p.k_chunks - 2 * kt);
          const uint64_t tile = static_cast<uint64_t>(row0 / PT);
          mbar_arrive_expect_tx(&full_bar[stage], plan.a_bytes + plan.b_bytes +
                                                      static_cast<uint32_t>(nch) * (kWSfPairBytes + kSfAtomBytes));
          // weights and their scales are read once per step: evict them first
          tma_load_3d_hint(w_s, &tmap_w, &full_bar[stage], kt * 128, wt * 256, e, w_policy);
          tma_load_3d(x_s, &tmap_x, &full_bar[stage], kt * 128, static_cast<int>(tile) * kF4Terms * PT, 0);
          bulk_load_hint(sf,
                         p.a_sf + ((static_cast<uint64_t>(e) * p.w_row_pairs + wt) * p.k_chunks + 2 * kt) *
                                      kWSfPairBytes,
                         static_cast<uint32_t>(nch) * kWSfPairBytes, &full_bar[stage], w_policy);
          bulk_load(sf + 2 * kWSfPairBytes, p.b_sf + (tile * p.k_chunks + 2 * kt) * kSfAtomBytes,
                    static_cast<uint32_t>(nch) * kSfAtomBytes, &full_bar[stage]);
          issued[stage] = true;
          issued_parity[stage] = phase;
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
          }
          continue;
        }
        mbar_arrive_expect_tx(&full_bar[stage], tx);
        tma_load_3d(w_s, &tmap_w, &full_bar[stage], kt * kTileK, wt * (kTok ? 256 : 128), e);
        if (kTok && p.stacked) {
          // the tile's stacked code rows (stacked_code_row) are consecutive:
          // one box of 2 * PT rows of the flat code map
          tma_load_3d(x_s, &tmap_x, &full_bar[stage], kt * kTileK, (row0 / PT) * 2 * PT, 0);
        } else {
          for (int term = 0; term < terms; ++term)
            tma_load_3d(x_s + term * x_stride, &tmap_x, &full_bar[stage], kt * kTileK, row0, term);
        }
        // scale atoms in smem: [weights x natoms_w][term 0 x natoms_x][term 1 ...]
        // weight atoms: the tile's pair of 128-row atoms is adjacent (w_sf_offset);
        // a 128-row weights-as-A tile takes its half
        {
          const int wp = kTok ? wt : wt / 2;
          const uint64_t src = ((static_cast<uint64_t>(e) * p.w_row_pairs + wp) * p.k_tiles + kt) * kWSfPairBytes +
                               (kTok ? 0 : (wt & 1) * kSfAtomBytes);
          bulk_load(sf, p.a_sf + src, kSfAtomBytes * natoms_w, &full_bar[stage]);
        }
        if (kTok && p.stacked) {
          bulk_load(sf + kSfAtomBytes * natoms_w, p.b_sf + (rbx * p.k_tiles + kt) * kSfAtomBytes, kSfAtomBytes,
                    &full_bar[stage]);
        } else {
          for (int term = 0; term < terms; ++term)
            for (int a = 0; a < natoms_x; ++a)
              bulk_load(sf + kSfAtomBytes * (natoms_w + term * natoms_x + a),
                        p.b_sf + term * p.b_sf_term_stride + ((rbx + a) * p.k_tiles + kt) * kSfAtomBytes,
                        kSfAtomBytes, &full_bar[stage]);
        }
        issued[stage] = true;
        issued_parity[stage] = phase;
        if (++stage == S) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
    // Drain: no TMA write into this CTA's shared memory may still be in flight.
    for (int s = 0; s < S; ++s)
      if (issued[s]) mbar_wait(&full_bar[s], issued_parity[s], nullptr, kDevTimeoutDrain);
  } else if (warp == 1 && lane == 0) {
    // ------------------------------------------------------------ MMA issuer
    int stage = 0;
    uint32_t phase = 0;
    uint32_t acc_phase[2] = {0, 0};
    int acc = 0;
    // tokens-as-A: A = x (E4M3, fmt 0), B = w (E2M1, fmt 5), M = 128 pairs, N = 256 rows
    // weights-as-A: A = w (E2M1),       B = x (E4M3),        M = 128 rows,  N = pairs
    const uint32_t a_fmt = kTok ? 0u : 5u, b_fmt = kTok ? 5u : 0u;
    const uint32_t mma_n = kTok ? 256u : static_cast<uint32_t>(N);
    bool ok = true;
    for (int t = t_lo + static_cast<int>(blockIdx.x); t < total_tiles && ok; t += gridDim.x) {
      if (!mbar_wait(&tmem_empty[acc], acc_phase[acc] ^ 1u, err, kDevTimeoutTmemEmpty, wait_ns)) break;
      acc_phase[acc] ^= 1u;
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * 128);
      for (int kt = 0; kt < p.k_tiles; ++kt) {
        // the scale-factor warp waits for the stage's TMA data, copies the
        // scales into TMEM and commits sf_full: data and scales are then ready.
        // FP4 tiles copy their scales from this thread instead (below): a copy
        // issued by another thread queues behind this thread's MMAs, and
        // waiting for its commit would drain the tensor pipe every stage.
        if (!mbar_wait(kF4 ? &full_bar[stage] : &sf_full[stage], phase, err, kDevTimeoutFull, wait_ns)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint8_t* sb = smem + stage * plan.stage_bytes;
        const uint32_t w_addr = smem_u32(kTok ? sb + plan.a_terms * plan.a_bytes : sb);
        const uint32_t x_addr = smem_u32(kTok ? sb : sb + plan.a_bytes);
        const uint32_t x_stride = kTok ? plan.a_bytes : plan.b_bytes;
        const uint32_t col0 = kSfTmemBase + stage * 32;
        const int mma_terms = (kTok && p.stacked) ? 1 : terms;
        if constexpr (kF4) {
          // A = stacked activation terms, B = weights; scale columns: weights
          // col0 + 8 * chunk (+4 for rows 128..255), activation col0 + 16 + 4 * chunk
          const int nk = kt == p.k_tiles - 1 ? p.last_mmas : 4;
          {
            // scale atoms of the stage's one or two 128-K chunks -> TMEM; the
            // tcgen05 ops of one thread run in issue order, so the MMAs below
            // read them, and a later stage's copies into these columns wait
            // for these MMAs
            const uint32_t sf_addr = smem_u32(sb + plan.a_bytes + plan.b_bytes);
            const int nch = min(2, p.k_chunks - 2 * kt);
            for (int c = 0; c < nch; ++c) {
              for (int ra = 0; ra < 2; ++ra)
                tc_cp_32x128b_warpx4(tmem_base + col0 + c * 8 + ra * 4,
                                     make_smem_desc(sf_addr + c * kWSfPairBytes + ra * kSfAtomBytes, 0, 128, 0));
              tc_cp_32x128b_warpx4(tmem_base + col0 + 16 + c * 4,
                                   make_smem_desc(sf_addr + 2 * kWSfPairBytes + c * kSfAtomBytes, 0, 128, 0));
            }
          }
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            if (kk < nk) {
              const uint32_t sid = static_cast<uint32_t>(kk & 1) * 2u;
              const uint64_t w_desc = make_smem_desc(w_addr + kk * 32, 16, 1024, 2);
              const uint64_t x_desc = make_smem_desc(x_addr + kk * 32, 16, 1024, 2);
              const uint32_t sf_w = (tmem_base + col0 + static_cast<uint32_t>(kk >> 1) * 8u) | (sid << 30);
              const uint32_t sf_x = (tmem_base + col0 + 16u + static_cast<uint32_t>(kk >> 1) * 4u) | (sid << 30);
              tc_mma_mxf4(d_tmem, x_desc, w_desc, make_idesc_mxf4(128u, 256u, sid, sid), sf_x, sf_w,
                          (kt | kk) != 0 ? 1u : 0u);
            }
          }
        } else {
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint64_t w_desc = make_smem_desc(w_addr + kk * 32, 16, 1024, 2);
            for (int term = 0; term < mma_terms; ++term) {
              const uint64_t x_desc = make_smem_desc(x_addr + term * x_stride + kk * 32, 16, 1024, 2);
              const uint32_t idesc = make_idesc_mxf8f6f4(a_fmt, b_fmt, 128u, mma_n, kk, kk);
              const uint32_t sf_w = (tmem_base + col0) | (static_cast<uint32_t>(kk) << 30);
              const uint32_t sf_x = (tmem_base + col0 + 8 + term * 8) | (static_cast<uint32_t>(kk) << 30);
              const uint32_t accum = (kt | kk | term) != 0 ? 1u : 0u;
              if (kTok)
                tc_mma_mxf8f6f4(d_tmem, x_desc, w_desc, idesc, sf_x, sf_w, accum);
              else
                tc_mma_mxf8f6f4(d_tmem, w_desc, x_desc, idesc, sf_w, sf_x, accum);
            }
          }
        }
        tc_commit(&empty_bar[stage]);
        if (++stage == S) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (!ok) break;
      tc_commit(&tmem_full[acc]);
      if (++acc == nacc) acc = 0;
    }
    // Drain: every MMA issued by this thread has finished before TMEM is freed.
    tc_commit(drain_bar);
    mbar_wait(drain_bar, 0, nullptr, kDevTimeoutDrain);
  } else if (!kF4 && warp == sf_warp(kTok) && lane == 0) {
    // ------------------------------------------------------------ scale factors -> TMEM
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    const int mma_terms = (kTok && p.stacked) ? 1 : terms;
    for (int t = t_lo + static_cast<int>(blockIdx.x); t < total_tiles && ok; t += gridDim.x) {
      for (int kt = 0; kt < p.k_tiles; ++kt) {
        if (!mbar_wait(&full_bar[stage], phase, err, kDevTimeoutFull, wait_ns)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint8_t* sb = smem + stage * plan.stage_bytes;
        const uint32_t sf_addr = smem_u32(sb + plan.a_terms * plan.a_bytes + plan.b_terms * plan.b_bytes);
        const uint32_t col0 = kSfTmemBase + stage * 32;
        // TMEM scale columns of this stage: weights at col0 (4 per 128 rows),
        // activation term q at col0 + 8 + 8q (4 per 128 rows).
        for (int a = 0; a < natoms_w; ++a)
          tc_cp_32x128b_warpx4(tmem_base + col0 + a * 4, make_smem_desc(sf_addr + kSfAtomBytes * a, 0, 128, 0));
        for (int term = 0; term < mma_terms; ++term)
          for (int a = 0; a < natoms_x; ++a)
            tc_cp_32x128b_warpx4(tmem_base + col0 + 8 + term * 8 + a * 4,
                                 make_smem_desc(sf_addr + kSfAtomBytes * (natoms_w + term * natoms_x + a), 0, 128, 0));
        tc_commit(&sf_full[stage]);
        if (++stage == S) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
    tc_commit(sf_drain);
    mbar_wait(sf_drain, 0, nullptr, kDevTimeoutDrain);
  } else if (warp >= 2 && warp < 2 + num_epi_threads(kTok) / 32) {
    // ------------------------------------------------------------ epilogue
    const int sp = warp & 3;          // TMEM sub-partition this warp may access
    const int m = sp * 32 + lane;     // accumulator row
    const int et = threadIdx.x - 64;  // epilogue thread id
    uint32_t acc_phase[2] = {0, 0};
    int acc = 0;
    float* xl = epi;                   // [64][kXPitch] linear half (weights-as-A)
    float* as = epi + 64 * kXPitch;    // [kChunk][kAPitch] activations (weights-as-A)
    float* rs = as + kChunk * kAPitch; // [kChunk] 1/rms per column
    // Tokens-as-A: the first pass (t < 0) is dry -- zeros instead of an
    // accumulator, no stores -- and runs while the first tile's MMAs do, so
    // the epilogue's long straight-line code is in the instruction cache
    // before the first real accumulator arrives.
    for (int t = t_lo + static_cast<int>(blockIdx.x) - (kTok ? static_cast<int>(gridDim.x) : 0); t < total_tiles;
         t += gridDim.x) {
      const bool dry = kTok && t < t_lo;
      int e = 0, wt = 0, pt = 0;
      if (!dry) {
        decode_tile(p, t, e, wt, pt);
        if (!mbar_wait(&tmem_full[acc], acc_phase[acc], err, kDevTimeoutTmemFull, wait_ns)) break;
        acc_phase[acc] ^= 1u;
        tc_fence_after();
      }
      const uint32_t trow = tmem_base + static_cast<uint32_t>(acc * 128) + (static_cast<uint32_t>(sp * 32) << 16);
      const int cnt = dry ? PT : __ldg(p.counts + e);
      const int n_valid = min(PT, cnt - pt * PT);
      const int pos0 = dry ? 0 : __ldg(p.poff + e) + pt * PT;
      const uint64_t bias_e = static_cast<uint64_t>(e) * p.bias_stride;
      if (kTok) {
        // Thread = pair row m; this warp owns columns [half*128, half*128 + 128)
        // of the 256 weight rows of tile wt.  The accumulator is copied to
        // registers and released before any math, so the next tile's MMAs
        // overlap this epilogue.
        const int half = (warp - 2) >> 2;
        float v[128];
        if (dry) {
#pragma unroll
          for (int i = 0; i < 128; ++i) v[i] = 0.0f;
        } else {
#pragma unroll
          for (int q = 0; q < 4; ++q) tmem_ld_32x32b_x32(trow + half * 128 + q * 32, v + q * 32);
          tmem_wait_ld();
          tc_fence_before();
          mbar_arrive(&tmem_empty[acc]);
          if (++acc == nacc) acc = 0;
        }
        if constexpr (kF4) {
          // Lane L holds term L / 8 of pair sp * 8 + L % 8.  Two butterfly
          // steps (lane ^ 16, lane ^ 8) sum the four terms and leave each lane
          // a quarter of the warp's 128 columns: W2 columns 32 * (L / 8) ..
          // + 31; W1 the GLU units 16 * (L / 8) .. + 15 with their linear
          // partners 64 columns later.
          const int tq = lane >> 3;
          const bool up1 = (tq >> 1) != 0, up2 = (tq & 1) != 0;
          const int jr = sp * 8 + (lane & 7);
          if (p.mode == 2) {
            float g1[64];
#pragma unroll
            for (int j = 0; j < 64; ++j) {
              const float recv = __shfl_xor_sync(0xFFFFFFFFu, up1 ? v[j] : v[64 + j], 16);
              g1[j] = (up1 ? v[64 + j] : v[j]) + recv;
            }
            float g2[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const float recv = __shfl_xor_sync(0xFFFFFFFFu, up2 ? g1[j] : g1[32 + j], 8);
              g2[j] = (up2 ? g1[32 + j] : g1[j]) + recv;
            }
            if (jr >= n_valid) continue;
            const int pos = pos0 + jr;
            const int pair = __ldg(p.perm + pos);
            const float w = __ldg(p.topk_w + pair);
            const int cf0 = wt * 256 + half * 128 + 32 * tq;
            const float4* bb = reinterpret_cast<const float4*>(p.bias + bias_e + cf0);
            __nv_bfloat16* dst = w2_out_row(p, pos, pair) + cf0;
#pragma unroll
            for (int q = 0; q < 4; ++q)
              if (!dry && cf0 + 8 * q < p.rows_valid)
                store_w2_8(dst + 8 * q, g2 + 8 * q, __ldg(bb + 2 * q), __ldg(bb + 2 * q + 1), p.bias_mult, w);
          } else {
            float g1[64];
#pragma unroll
            for (int j = 0; j < 64; ++j) {
              const int cl = j < 32 ? j : j + 32;
              const float recv = __shfl_xor_sync(0xFFFFFFFFu, up1 ? v[cl] : v[cl + 32], 16);
              g1[j] = (up1 ? v[cl + 32] : v[cl]) + recv;
            }
            float g2[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const int cl = j < 16 ? j : j + 16;
              const float recv = __shfl_xor_sync(0xFFFFFFFFu, up2 ? g1[cl] : g1[cl + 16], 8);
              g2[j] = (up2 ? g1[cl + 16] : g1[cl]) + recv;
            }
            // SwiGLU in f32 to the activation rows [pos][units]; a separate
            // pass splits them into the four-term E2M1 operand of W2 (doing
            // that here would make this epilogue slower than the tile's MMAs)
            const int unit0 = wt * 128 + half * 64 + 16 * tq;  // GLU unit of g2[0]
            if (jr < n_valid && unit0 < p.units && !dry) {
              const int pos = pos0 + jr;
              const int pair = __ldg(p.perm + pos);
              const float r = __ldg(p.rscale + pair / p.k);
              const float4* bb = reinterpret_cast<const float4*>(p.bias + bias_e + wt * 256 + half * 128 + 16 * tq);
              float4* dst = reinterpret_cast<float4*>(p.act_f32 + static_cast<uint64_t>(pos) * p.units + unit0);
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                const float4 bg = __ldg(bb + q);       // GLU biases
                const float4 bl = __ldg(bb + 16 + q);  // linear biases (64 columns later)
                float4 o;
                o.x = swiglu_clamp(fmaf(g2[4 * q + 0], r, bg.x), fmaf(g2[16 + 4 * q + 0], r, bl.x), p.alpha, p.limit);
                o.y = swiglu_clamp(fmaf(g2[4 * q + 1], r, bg.y), fmaf(g2[16 + 4 * q + 1], r, bl.y), p.alpha, p.limit);
                o.z = swiglu_clamp(fmaf(g2[4 * q + 2], r, bg.z), fmaf(g2[16 + 4 * q + 2], r, bl.z), p.alpha, p.limit);
                o.w = swiglu_clamp(fmaf(g2[4 * q + 3], r, bg.w), fmaf(g2[16 + 4 * q + 3], r, bl.w), p.alpha, p.limit);
                dst[q] = o;
              }
            }
          }
          continue;
        }
        if (p.stacked) {
          // Lane L < 16 holds the hi-term row of pair sp*16 + L, lane L + 16 its
          // lo-term row.  The two lanes swap partial sums so that each ends
          // with hi + lo for half of the columns and finishes that half:
          // W1 lower lane GLU units [0, 32) of this half (columns 0..31 and
          // 64..95), upper lane units [32, 64); W2 lower lane columns 0..63,
          // upper lane 64..127.
          const bool upper = lane >= 16;
          float g[64];
          if (p.mode == 2) {
#pragma unroll
            for (int j = 0; j < 64; ++j) {
              const float recv = __shfl_xor_sync(0xFFFFFFFFu, upper ? v[j] : v[64 + j], 16);
              g[j] = (upper ? v[64 + j] : v[j]) + recv;
            }
          } else {
#pragma unroll
            for (int j = 0; j < 64; ++j) {
              const int cl = j < 32 ? j : j + 32, cu = cl + 32;
              const float recv = __shfl_xor_sync(0xFFFFFFFFu, upper ? v[cl] : v[cu], 16);
              g[j] = (upper ? v[cu] : v[cl]) + recv;
            }
          }
          const int jr = sp * 16 + (lane & 15);
          if (jr >= n_valid) continue;
          const int pos = pos0 + jr;
          const int pair = __ldg(p.perm + pos);
          if (p.mode == 2) {
            const float w = __ldg(p.topk_w + pair);
            const int cf0 = wt * 256 + half * 128 + (upper ? 64 : 0);
            const float4* bb = reinterpret_cast<const float4*>(p.bias + bias_e + cf0);
            __nv_bfloat16* dst = w2_out_row(p, pos, pair) + cf0;
#pragma unroll
            for (int q = 0; q < 8; ++q)
              if (!dry && cf0 + 8 * q < p.rows_valid)
                store_w2_8(dst + 8 * q, g + 8 * q, __ldg(bb + 2 * q), __ldg(bb + 2 * q + 1), p.bias_mult, w);
          } else {
            const int unit0 = wt * 128 + half * 64 + (upper ? 32 : 0);  // GLU unit of g[0]
            if (unit0 >= p.units) continue;
            const float r = __ldg(p.rscale + pair / p.k);
            const float4* bb =
                reinterpret_cast<const float4*>(p.bias + bias_e + wt * 256 + half * 128 + (upper ? 32 : 0));
            float a[32];
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              const float4 bg = __ldg(bb + q);       // GLU biases
              const float4 bl = __ldg(bb + 16 + q);  // linear biases (64 columns later)
              a[4 * q + 0] = swiglu_clamp(fmaf(g[4 * q + 0], r, bg.x), fmaf(g[32 + 4 * q + 0], r, bl.x), p.alpha, p.limit);
              a[4 * q + 1] = swiglu_clamp(fmaf(g[4 * q + 1], r, bg.y), fmaf(g[32 + 4 * q + 1], r, bl.y), p.alpha, p.limit);
              a[4 * q + 2] = swiglu_clamp(fmaf(g[4 * q + 2], r, bg.z), fmaf(g[32 + 4 * q + 2], r, bl.z), p.alpha, p.limit);
              a[4 * q + 3] = swiglu_clamp(fmaf(g[4 * q + 3], r, bg.w), fmaf(g[32 + 4 * q + 3], r, bl.w), p.alpha, p.limit);
            }
            uint32_t words[kMaxTerms][8];
            uint8_t sbyte[kMaxTerms];
            quantize_block32(a, 2, words, sbyte);
            if (!dry) store_block_terms(p, pos, unit0, words, sbyte);
          }
          continue;
        }
        const int jrow = m;  // pair index within the tile
        const bool valid = jrow < n_valid;
        const int pos = pos0 + jrow;
        if (!valid) continue;
        const int pair = __ldg(p.perm + pos);
        if (p.mode == 2) {
          const float w = __ldg(p.topk_w + pair);
          const int cf0 = wt * 256 + half * 128;  // output feature of v[0]
          const float4* bb = reinterpret_cast<const float4*>(p.bias + bias_e + cf0);
          __nv_bfloat16* dst = w2_out_row(p, pos, pair) + cf0;
#pragma unroll
          for (int q = 0; q < 16; ++q)
            if (!dry && cf0 + 8 * q < p.rows_valid)
              store_w2_8(dst + 8 * q, v + 8 * q, __ldg(bb + 2 * q), __ldg(bb + 2 * q + 1), p.bias_mult, w);
        } else {
          const int unit0 = wt * 128 + half * 64;  // GLU unit of v[0]
          if (unit0 >= p.units) continue;
          const float r = __ldg(p.rscale + pair / p.k);
          const float4* bb = reinterpret_cast<const float4*>(p.bias + bias_e + wt * 256 + half * 128);
#pragma unroll
          for (int sb = 0; sb < 2; ++sb) {
            float a[32];
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              const float4 bg = __ldg(bb + sb * 8 + q);       // GLU biases
              const float4 bl = __ldg(bb + 16 + sb * 8 + q);  // linear biases (64 columns later)
              const float* gv = v + sb * 32 + 4 * q;
              const float* lv = v + 64 + sb * 32 + 4 * q;
              a[4 * q + 0] = swiglu_clamp(fmaf(gv[0], r, bg.x), fmaf(lv[0], r, bl.x), p.alpha, p.limit);
              a[4 * q + 1] = swiglu_clamp(fmaf(gv[1], r, bg.y), fmaf(lv[1], r, bl.y), p.alpha, p.limit);
              a[4 * q + 2] = swiglu_clamp(fmaf(gv[2], r, bg.z), fmaf(lv[2], r, bl.z), p.alpha, p.limit);
              a[4 * q + 3] = swiglu_clamp(fmaf(gv[3], r, bg.w), fmaf(lv[3], r, bl.w), p.alpha, p.limit);
            }
            uint32_t words[kMaxTerms][8];
            uint8_t sbyte[kMaxTerms];
            quantize_block32(a, 2, words, sbyte);
            if (!dry) store_block_terms(p, pos, unit0 + sb * 32, words, sbyte);
          }
        }
        continue;
      } else {
        // weights-as-A: thread = weight row m of tile wt; columns = pairs
        if (p.mode == 2) {
          const int c = wt * 128 + m;
          const bool row_ok = c < p.rows_valid;
          const float bias = row_ok ? __ldg(p.bias + bias_e + c) * p.bias_mult : 0.f;
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
          // lanes 0..63: GLU rows, 64..127: linear rows of units j0..j0+63
          const bool glu = m < 64;
          const int jl = glu ? m : m - 64;
          const int j0 = wt * 64;
          const float b_g = __ldg(p.bias + bias_e + wt * 128 + jl);
          const float b_l = __ldg(p.bias + bias_e + wt * 128 + 64 + jl);
          for (int c0 = 0; c0 < n_valid; c0 += kChunk) {
            float v[kChunk];
            tmem_ld_32x32b_x16(trow + c0, *reinterpret_cast<float(*)[16]>(&v[0]));
            tmem_ld_32x32b_x16(trow + c0 + 16, *reinterpret_cast<float(*)[16]>(&v[16]));
            if (!glu) {
#pragma unroll
              for (int i = 0; i < kChunk; ++i) xl[jl * kXPitch + i] = v[i];
            }
            if (et < kChunk) {
              const int n = c0 + et;
              rs[et] = n < n_valid ? __ldg(p.rscale + __ldg(p.perm + pos0 + n) / p.k) : 0.f;
            }
            named_bar_epi();
            if (glu) {
#pragma unroll 4
              for (int i = 0; i < kChunk; ++i) {
                const float r = rs[i];
                as[i * kAPitch + jl] =
                    swiglu_clamp(fmaf(v[i], r, b_g), fmaf(xl[jl * kXPitch + i], r, b_l), p.alpha, p.limit);
              }
            }
            named_bar_epi();
            // two 32-unit blocks per column: thread et -> (column et / 2, block et % 2)
            if (et < 2 * kChunk) {
              const int col = et >> 1, blk = et & 1;
              const int n = c0 + col;
              if (n < n_valid && j0 + blk * 32 < p.units) {
                float a[32];
#pragma unroll
                for (int i = 0; i < 32; ++i) a[i] = as[col * kAPitch + blk * 32 + i];
                uint32_t words[kMaxTerms][8];
                uint8_t sbyte[kMaxTerms];
                quantize_block32(a, 2, words, sbyte);
                store_block_terms(p, pos0 + n, j0 + blk * 32, words, sbyte);
              }
            }
            named_bar_epi();
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&tmem_empty[acc]);
      if (++acc == nacc) acc = 0;
    }
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

}  // namespace

size_t tc_gemm_smem_bytes(bool tokens_as_a, int N, int terms, int stages, int pair_tile, bool stacked, bool fp4) {
  const SmemPlan plan = smem_plan(tokens_as_a, N, terms, pair_tile, tokens_as_a && stacked, fp4);
  return 1024 + static_cast<size_t>(stages) * plan.stage_bytes + epi_smem_bytes(tokens_as_a) +
         (3 * kMaxStages + 10) * sizeof(uint64_t);
}

int tc_gemm_max_stages(bool tokens_as_a, int N, int terms, size_t smem_limit, int pair_tile, bool stacked,
                       bool fp4) {
  int s = kMaxStages - 1;  // 7 stages x 32 scale columns fit above column 256
  while (s > 1 && tc_gemm_smem_bytes(tokens_as_a, N, terms, s, pair_tile, stacked, fp4) > smem_limit) --s;
  return s;
}

cudaError_t tc_gemm_launch(bool tokens_as_a, const CUtensorMap& tmap_w, const CUtensorMap& tmap_x,
                           const TcParams& p, int grid, cudaStream_t stream) {
  const size_t smem =
      tc_gemm_smem_bytes(tokens_as_a, p.N, p.b_terms, p.stages, p.sf_rows, p.stacked != 0, p.fp4 != 0);
  const auto fn = tokens_as_a ? (p.fp4 ? tc_moe_gemm_kernel<2> : tc_moe_gemm_kernel<1>) : tc_moe_gemm_kernel<0>;
  cudaError_t st = ensure_dynamic_smem(reinterpret_cast<const void*>(fn), smem);
  if (st != cudaSuccess) return st;
  return launch_kernel(fn, dim3(grid), dim3(num_threads(tokens_as_a)), smem, stream, tmap_w, tmap_x, p);
}

}  // namespace mxmoe
