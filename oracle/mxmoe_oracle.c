/*
 * mxmoe_oracle.c -- CPU restatement of burn-extended's MXFP4 MoE hot path.
 * TEST INFRASTRUCTURE ONLY (the checker, never the product); see the header.
 *
 * Build: oracle/Makefile (gcc -O2 -fopenmp -ffp-contract=off).  Contraction is
 * off so that every a*b+c below rounds twice unless fmaf() is written out,
 * which is what the CUDA router does with __fmul_rn/__fmaf_rn.
 */
#include "mxmoe_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* E2M1 code -> value; src/loader/mxfp4.rs:11-13 (and src/quant/gpu.rs:116-119).
 * Codes 8..15 are the negatives of 0..7, including -0.0 for code 8. */
static const float kFp4[16] = {0.0f,  0.5f,  1.0f,  1.5f,  2.0f,  3.0f,
                               4.0f,  6.0f,  -0.0f, -0.5f, -1.0f, -1.5f,
                               -2.0f, -3.0f, -4.0f, -6.0f};

/* Exact 2^e in f32 for any integer e (src/loader/mxfp4.rs:67 uses powi). */
static float exp2i(int e) { return ldexpf(1.0f, e); }

int orc_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

/* src/loader/mxfp4.rs:57-79 */
void orc_dequant_mxfp4_bytes(const uint8_t* blocks, size_t rows_total, size_t b,
                             const uint8_t* scales, float* out) {
  for (size_t r = 0; r < rows_total; ++r) {
    const float scale = exp2i((int)scales[r] - 127);
    for (size_t i = 0; i < b; ++i) {
      const uint8_t byte = blocks[r * b + i];
      out[r * 2 * b + 2 * i] = kFp4[byte & 0x0F] * scale;
      out[r * 2 * b + 2 * i + 1] = kFp4[byte >> 4] * scale;
    }
  }
}

/* src/quant/gpu.rs:124-134 (W1) and :183-187 (W2), with the exact power of
 * two of src/loader/mxfp4.rs:67-68 in place of exp((s - ue8 - 127) * ln 2). */
void orc_dequant_rows(const uint8_t* blocks, const uint8_t* scales, size_t rows,
                      size_t cols, size_t bpr, size_t gpr, int ue8_offset,
                      float* out) {
  for (size_t r = 0; r < rows; ++r) {
    for (size_t c = 0; c < cols; ++c) {
      const uint8_t byte = blocks[r * bpr + (c >> 1)];
      const uint8_t nib = (c & 1) ? (byte >> 4) : (byte & 0x0F);
      const int e = (int)scales[r * gpr + (c >> 5)] - 127 - ue8_offset;
      out[r * cols + c] = kFp4[nib] * exp2i(e);
    }
  }
}

/* Sum of 32 lane partials in the order of a shuffle-xor butterfly with
 * offsets 16, 8, 4, 2, 1 (the order the CUDA router reduces in). */
static float butterfly32(float p[32]) {
  for (int off = 16; off >= 1; off >>= 1)
    for (int i = 0; i < off; ++i) p[i] = p[i] + p[i + off];
  return p[0];
}

/* Router: src/moe/mod.rs:109 (RmsNorm), :110 (Linear gate), :272-276 (top-k,
 * softmax over the k selected logits).
 * Pinned definitions (Burn's own are outside the reference, unpinned):
 *   ss     = sum_c x[c]^2, as 32 lane chains c = l, l+32, ... (fmaf), then
 *            butterfly32;
 *   r      = 1 / sqrtf(ss / d + eps);
 *   normed = (x * r) * gamma, each product rounded;
 *   logit  = butterfly32(lane chains of fmaf(normed[c], W[e][c], acc)) + b[e];
 *   top-k  = largest logits, ties to the lower expert index;
 *   w      = expf(v - v_max) / sum (sum in slot order).                      */
void orc_topk_softmax(size_t n, uint32_t E, uint32_t k, const float* logits,
                      int32_t* topk_idx, float* topk_w) {
  for (size_t t = 0; t < n; ++t) {
    const float* lg = logits + t * E;
    int32_t idx[256];
    float val[256];
    for (uint32_t s = 0; s < k; ++s) {
      int best = -1;
      for (uint32_t e = 0; e < E; ++e) {
        int taken = 0;
        for (uint32_t q = 0; q < s; ++q) taken |= (idx[q] == (int32_t)e);
        if (taken) continue;
        if (best < 0 || lg[e] > lg[best]) best = (int)e;
      }
      idx[s] = best;
      val[s] = lg[best];
    }
    float ex[256];
    float sum = 0.0f;
    for (uint32_t s = 0; s < k; ++s) {
      ex[s] = expf(val[s] - val[0]);
      sum = sum + ex[s];
    }
    for (uint32_t s = 0; s < k; ++s) {
      if (topk_idx) topk_idx[t * k + s] = idx[s];
      if (topk_w) topk_w[t * k + s] = ex[s] / sum;
    }
  }
}

void orc_route(const orc_cfg* cfg, size_t n, const float* x, const float* gamma,
               const float* gate_w, const float* gate_b, float* normed_out,
               float* rscale_out, float* logits_out, int32_t* topk_idx,
               float* topk_w) {
  const size_t d = cfg->d_model;
  const uint32_t E = cfg->num_experts;
  float* logits = logits_out ? logits_out : (float*)malloc(n * E * sizeof(float));
#pragma omp parallel
  {
    float* nrm = (float*)malloc(d * sizeof(float));
#pragma omp for schedule(static)
    for (long long tt = 0; tt < (long long)n; ++tt) {
      const size_t t = (size_t)tt;
      const float* xr = x + t * d;
      float p[32];
      for (int l = 0; l < 32; ++l) {
        float acc = 0.0f;
        for (size_t c = (size_t)l; c < d; c += 32) acc = fmaf(xr[c], xr[c], acc);
        p[l] = acc;
      }
      const float ss = butterfly32(p);
      const float r = 1.0f / sqrtf(ss / (float)d + cfg->rms_eps);
      for (size_t c = 0; c < d; ++c) nrm[c] = (xr[c] * r) * gamma[c];
      if (normed_out) memcpy(normed_out + t * d, nrm, d * sizeof(float));
      if (rscale_out) rscale_out[t] = r;
      for (uint32_t e = 0; e < E; ++e) {
        const float* w = gate_w + (size_t)e * d;
        for (int l = 0; l < 32; ++l) {
          float acc = 0.0f;
          for (size_t c = (size_t)l; c < d; c += 32) acc = fmaf(nrm[c], w[c], acc);
          p[l] = acc;
        }
        logits[t * E + e] = butterfly32(p) + gate_b[e];
      }
    }
    free(nrm);
  }
  orc_topk_softmax(n, E, cfg->experts_per_token, logits, topk_idx, topk_w);
  if (!logits_out) free(logits);
}

/* Canonical permutation (replaces the dense per-expert mask of
 * src/moe/mod.rs:279-288): pairs p = t*k + s are stably sorted by expert id.
 * offsets[E+1] are exclusive prefix counts, perm[pos] = p, inv[p] = pos. */
void orc_permute(size_t n, uint32_t k, uint32_t E, const int32_t* topk_idx,
                 int32_t* offsets, int32_t* perm, int32_t* inv) {
  const size_t P = n * k;
  int32_t* cnt = (int32_t*)calloc(E + 1, sizeof(int32_t));
  for (size_t p = 0; p < P; ++p) cnt[topk_idx[p]]++;
  int32_t run = 0;
  for (uint32_t e = 0; e < E; ++e) {
    offsets[e] = run;
    run += cnt[e];
    cnt[e] = offsets[e];
  }
  offsets[E] = run;
  for (size_t p = 0; p < P; ++p) {
    const int32_t pos = cnt[topk_idx[p]]++;
    perm[pos] = (int32_t)p;
    inv[p] = pos;
  }
  free(cnt);
}

/* src/quant/gpu.rs:140-145 and src/activation/mod.rs:32-40: the GLU half is
 * clamped from above only, the linear half on both sides. */
float orc_swiglu(float g, float l, float alpha, float limit) {
  const float xg = fminf(g, limit);
  const float xl = fmaxf(-limit, fminf(l, limit));
  const float sig = 1.0f / (1.0f + expf(-alpha * xg));
  return (xg * sig) * (xl + 1.0f);
}

/* Expert FFN over externally supplied routing.
 * W1 row j (src/quant/gpu.rs:112-137): split-half pairs GLU row j with linear
 * row f + j (src/moe/mod.rs:320-321, :336-337); ORC_FLAG_INTERLEAVED_GLU pairs
 * rows 2j and 2j+1 (src/activation/mod.rs:28-30).  Dots run sequentially over
 * c = 0..K-1 in f32 as in the reference kernel loops (:120-137, :179-189).
 * W2 bias: once (mathematical intent) or once per 256-wide f tile
 * (ORC_FLAG_BIAS_PER_FTILE, the reference's behaviour at src/quant/gpu.rs:191
 * with the f-tiling of src/moe/mod.rs:316-317).
 * Combine (src/moe/mod.rs:279, :405, :411): per token the expert terms
 * (dot + b2) * w are summed in increasing expert index, then x is added. */
void orc_moe_experts(const orc_cfg* cfg, size_t n, const float* x,
                     const float* normed, const int32_t* topk_idx,
                     const float* topk_w, const uint8_t* w1_blocks,
                     const uint8_t* w1_scales, const float* b1,
                     const uint8_t* w2_blocks, const uint8_t* w2_scales,
                     const float* b2, float* y, int nthreads) {
  const size_t d = cfg->d_model, f = cfg->ffn_hidden;
  const uint32_t E = cfg->num_experts, k = cfg->experts_per_token;
  const size_t P = n * k;
  const size_t bpr1 = (d + 1) / 2, gpr1 = (d + 31) / 32;
  const size_t bpr2 = (f + 1) / 2, gpr2 = (f + 31) / 32;
  const int interleaved = (cfg->flags & ORC_FLAG_INTERLEAVED_GLU) != 0;
  const float bias_rep =
      (cfg->flags & ORC_FLAG_BIAS_PER_FTILE) ? (float)((f + 255) / 256) : 1.0f;
  const int ue8 = cfg->ue8_offset;
  if (nthreads <= 0) nthreads = orc_num_threads();

  int32_t* offsets = (int32_t*)malloc((E + 1) * sizeof(int32_t));
  int32_t* perm = (int32_t*)malloc(P * sizeof(int32_t));
  int32_t* inv = (int32_t*)malloc(P * sizeof(int32_t));
  orc_permute(n, k, E, topk_idx, offsets, perm, inv);

  float* act = (float*)malloc(P * f * sizeof(float));     /* [pos][f] */
  float* contrib = (float*)malloc(P * d * sizeof(float)); /* [pos][d] */

  for (uint32_t e = 0; e < E; ++e) {
    const int32_t p0 = offsets[e], p1 = offsets[e + 1];
    if (p1 == p0) continue;
    const uint8_t* wb1 = w1_blocks + (size_t)e * 2 * f * bpr1;
    const uint8_t* ws1 = w1_scales + (size_t)e * 2 * f * gpr1;
    const uint8_t* wb2 = w2_blocks + (size_t)e * d * bpr2;
    const uint8_t* ws2 = w2_scales + (size_t)e * d * gpr2;
#pragma omp parallel num_threads(nthreads)
    {
      const size_t wmax = d > f ? d : f;
      float* rg = (float*)malloc(wmax * sizeof(float));
      float* rl = (float*)malloc(wmax * sizeof(float));
#pragma omp for schedule(static)
      for (long long jj = 0; jj < (long long)f; ++jj) {
        const size_t j = (size_t)jj;
        const size_t row_g = interleaved ? 2 * j : j;
        const size_t row_l = interleaved ? 2 * j + 1 : f + j;
        orc_dequant_rows(wb1 + row_g * bpr1, ws1 + row_g * gpr1, 1, d, bpr1, gpr1, ue8, rg);
        orc_dequant_rows(wb1 + row_l * bpr1, ws1 + row_l * gpr1, 1, d, bpr1, gpr1, ue8, rl);
        const float bg = b1[(size_t)e * 2 * f + row_g];
        const float bl = b1[(size_t)e * 2 * f + row_l];
        for (int32_t pos = p0; pos < p1; ++pos) {
          const float* in = normed + (size_t)(perm[pos] / (int32_t)k) * d;
          float sg = 0.0f, sl = 0.0f;
          for (size_t c = 0; c < d; ++c) {
            sg = sg + in[c] * rg[c];
            sl = sl + in[c] * rl[c];
          }
          act[(size_t)pos * f + j] =
              orc_swiglu(sg + bg, sl + bl, cfg->swiglu_alpha, cfg->swiglu_limit);
        }
      }
#pragma omp for schedule(static)
      for (long long cc = 0; cc < (long long)d; ++cc) {
        const size_t c = (size_t)cc;
        orc_dequant_rows(wb2 + c * bpr2, ws2 + c * gpr2, 1, f, bpr2, gpr2, ue8, rg);
        const float bb = b2[(size_t)e * d + c] * bias_rep;
        for (int32_t pos = p0; pos < p1; ++pos) {
          const float* a = act + (size_t)pos * f;
          float s = 0.0f;
          for (size_t j = 0; j < f; ++j) s = s + a[j] * rg[j];
          contrib[(size_t)pos * d + c] = (s + bb) * topk_w[perm[pos]];
        }
      }
      free(rg);
      free(rl);
    }
  }

  const int residual = (cfg->flags & ORC_FLAG_NO_RESIDUAL) == 0;
#pragma omp parallel for num_threads(nthreads) schedule(static)
  for (long long tt = 0; tt < (long long)n; ++tt) {
    const size_t t = (size_t)tt;
    /* slots of this token in increasing expert order */
    int32_t order[256];
    for (uint32_t s = 0; s < k; ++s) order[s] = (int32_t)s;
    for (uint32_t a = 1; a < k; ++a)
      for (uint32_t b = a; b > 0 && topk_idx[t * k + order[b - 1]] > topk_idx[t * k + order[b]]; --b) {
        const int32_t tmp = order[b];
        order[b] = order[b - 1];
        order[b - 1] = tmp;
      }
    for (size_t c = 0; c < d; ++c) {
      float acc = 0.0f;
      for (uint32_t s = 0; s < k; ++s)
        acc = acc + contrib[(size_t)inv[t * k + order[s]] * d + c];
      y[t * d + c] = residual ? x[t * d + c] + acc : acc;
    }
  }
  free(offsets);
  free(perm);
  free(inv);
  free(act);
  free(contrib);
}

void orc_moe_forward(const orc_cfg* cfg, size_t n, const float* x,
                     const float* gamma, const float* gate_w, const float* gate_b,
                     const uint8_t* w1_blocks, const uint8_t* w1_scales,
                     const float* b1, const uint8_t* w2_blocks,
                     const uint8_t* w2_scales, const float* b2, float* y,
                     int32_t* topk_idx_out, float* topk_w_out, int nthreads) {
  const size_t d = cfg->d_model;
  const uint32_t k = cfg->experts_per_token;
  float* normed = (float*)malloc(n * d * sizeof(float));
  int32_t* ti = topk_idx_out ? topk_idx_out : (int32_t*)malloc(n * k * sizeof(int32_t));
  float* tw = topk_w_out ? topk_w_out : (float*)malloc(n * k * sizeof(float));
  orc_route(cfg, n, x, gamma, gate_w, gate_b, normed, NULL, NULL, ti, tw);
  orc_moe_experts(cfg, n, x, normed, ti, tw, w1_blocks, w1_scales, b1, w2_blocks,
                  w2_scales, b2, y, nthreads);
  free(normed);
  if (!topk_idx_out) free(ti);
  if (!topk_w_out) free(tw);
}
