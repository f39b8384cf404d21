/*
 * riallm_oracle.c -- CPU restatement of riallm's block quantization and MoE
 * block forward. TEST INFRASTRUCTURE ONLY (the parity reference and the
 * timed CPU port); the product never links it. PARITY UNPINNED: see riallm_oracle.h.
 *
 * Build: oracle/Makefile (gcc -O2 -fopenmp -ffp-contract=off). Contraction
 * must stay off: every rounding step below is meant literally.
 */
#include "riallm_oracle.h"

#include <float.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------ bf16 */

uint16_t ro_f32_to_bf16(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
  uint32_t rounding_bias = 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)((u + rounding_bias) >> 16);
}

float ro_bf16_to_f32(uint16_t b) {
  uint32_t u = ((uint32_t)b) << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

static inline float round_bf16(float f) { return ro_bf16_to_f32(ro_f32_to_bf16(f)); }

/* ------------------------------------------------------- quantization.rs */

/* NF4 code table, src/quantization.rs:127-130. */
static const float kNf4Table[16] = {
    -1.0f,   -0.6962f, -0.5250f, -0.3900f, -0.2750f, -0.1750f,
    -0.0850f, -0.0150f, 0.0f,    0.0150f,  0.0850f,  0.1750f,
    0.2750f, 0.3900f,  0.5250f,  0.6962f};

uint64_t ro_num_blocks(int32_t qtype, uint64_t n) {
  uint64_t b = qtype == RO_FOUR_BIT ? 64 : 128;
  return (n + b - 1) / b;
}

uint64_t ro_data_bytes(int32_t qtype, uint64_t n) {
  if (qtype == RO_EIGHT_BIT) return n;
  /* 64-element blocks, ceil(len/2) bytes each; only the last block can be
   * odd, so the total is ceil(n/2). */
  return (n + 1) / 2;
}

/* Rust f32::clamp(min, max): NaN stays NaN. */
static inline float rust_clamp(float x, float lo, float hi) {
  if (x < lo) x = lo;
  if (x > hi) x = hi;
  return x;
}

/* src/quantization.rs:179-196: nearest table entry to clamp(v,-1,1); the
 * first minimum wins (strict <); NaN distances never win, giving 0. */
static inline uint8_t nf4_code(float value) {
  float normalized = rust_clamp(value, -1.0f, 1.0f);
  float min_dist = FLT_MAX;
  uint8_t q = 0;
  for (int i = 0; i < 16; ++i) {
    float dist = fabsf(normalized - kNf4Table[i]);
    if (dist < min_dist) {
      min_dist = dist;
      q = (uint8_t)i;
    }
  }
  return q;
}

void ro_quantize_nf4(const float* v, uint64_t n, uint8_t* data, float* scales,
                     float* zeros) {
  const uint64_t bs = 64;
  int64_t nb = (int64_t)((n + bs - 1) / bs);
  /* Blocks are independent; block b's bytes start at 32 b (only the last
   * block can be shorter than 64 elements). */
#pragma omp parallel for schedule(static)
  for (int64_t b = 0; b < nb; ++b) {
    uint64_t o = (uint64_t)b * 32;
    uint64_t start = b * bs;
    uint64_t end = start + bs < n ? start + bs : n;
    uint64_t len = end - start;
    const float* blk = v + start;
    /* fold(0.0, |a,&b| a.max(b.abs())) -- fmaxf ignores NaN like f32::max */
    float abs_max = 0.0f;
    for (uint64_t i = 0; i < len; ++i) abs_max = fmaxf(abs_max, fabsf(blk[i]));
    /* Iterator::sum for f32: sequential, starting at -0.0 (Rust >= 1.82). */
    float sum = -0.0f;
    for (uint64_t i = 0; i < len; ++i) sum += blk[i];
    float mean = sum / (float)len;
    scales[b] = abs_max / 1.0f;
    zeros[b] = mean;
    for (uint64_t i = 0; i < len; i += 2) {
      float v1 = blk[i];
      float v2 = i + 1 < len ? blk[i + 1] : 0.0f;
      uint8_t q1 = nf4_code(v1);
      uint8_t q2 = nf4_code(v2);
      data[o++] = (uint8_t)((q2 << 4) | q1);
    }
  }
}

/* Rust `f32 as u8`: saturating, NaN -> 0. */
static inline uint8_t rust_as_u8(float t) {
  if (t != t) return 0;
  if (t <= 0.0f) return 0;
  if (t >= 255.0f) return 255;
  return (uint8_t)t;
}

void ro_quantize_int8(const float* v, uint64_t n, uint8_t* data, float* scales,
                      float* zeros) {
  const uint64_t bs = 128;
  int64_t nb = (int64_t)((n + bs - 1) / bs);
#pragma omp parallel for schedule(static)
  for (int64_t b = 0; b < nb; ++b) {
    uint64_t start = (uint64_t)b * bs;
    uint64_t end = start + bs < n ? start + bs : n;
    uint64_t len = end - start;
    const float* blk = v + start;
    float mn = INFINITY, mx = -INFINITY;
    for (uint64_t i = 0; i < len; ++i) mn = fminf(mn, blk[i]);
    for (uint64_t i = 0; i < len; ++i) mx = fmaxf(mx, blk[i]);
    float scale = (mx - mn) / 255.0f;
    float zero_point = mn;
    scales[b] = scale;
    zeros[b] = zero_point;
    for (uint64_t i = 0; i < len; ++i) {
      float t = (blk[i] - zero_point) / scale;
      t = roundf(t); /* f32::round: half away from zero */
      t = rust_clamp(t, 0.0f, 255.0f);
      data[start + i] = rust_as_u8(t);
    }
  }
}

uint64_t ro_dequantize_nf4(const uint8_t* data, uint64_t n_bytes,
                           const float* scales, uint64_t n_scales,
                           const float* zeros, uint64_t n_zeros,
                           uint64_t numel, uint64_t block_size, float* out) {
  uint64_t w = 0;
  uint64_t scale_idx = 0;
  for (uint64_t i = 0; i < n_bytes; ++i) {
    uint8_t byte = data[i];
    float low = (float)(byte & 0x0F);
    float high = (float)((byte >> 4) & 0x0F);
    float scale = scale_idx < n_scales ? scales[scale_idx] : 1.0f;
    float zero = scale_idx < n_zeros ? zeros[scale_idx] : 0.0f;
    out[w++] = (low - zero) * scale;
    uint64_t element_idx = i * 2;
    if ((element_idx + 2) % block_size == 0) scale_idx += 1;
    if (element_idx + 1 < numel) {
      scale = scale_idx < n_scales ? scales[scale_idx] : 1.0f;
      zero = scale_idx < n_zeros ? zeros[scale_idx] : 0.0f;
      out[w++] = (high - zero) * scale;
    }
  }
  return w;
}

uint64_t ro_dequantize_int8(const uint8_t* data, uint64_t n_bytes,
                            const float* scales, uint64_t n_scales,
                            const float* zeros, uint64_t n_zeros,
                            uint64_t block_size, float* out) {
  for (uint64_t i = 0; i < n_bytes; ++i) {
    float value = (float)data[i];
    uint64_t b = i / block_size;
    float scale = b < n_scales ? scales[b] : 1.0f;
    float zero = b < n_zeros ? zeros[b] : 0.0f;
    out[i] = (value - zero) * scale;
  }
  return n_bytes;
}

void ro_tensor_span_f32(const ro_qtensor* t, uint64_t start, uint64_t len,
                        int32_t bf16_round, float* out) {
  if (t->qtype == RO_NONE) {
    const float* d = (const float*)t->data;
    for (uint64_t i = 0; i < len; ++i) out[i] = d[start + i];
  } else if (t->qtype == RO_FOUR_BIT) {
    const uint8_t* d = (const uint8_t*)t->data;
    uint64_t bs = (uint64_t)t->block_size;
    for (uint64_t i = 0; i < len; ++i) {
      uint64_t e = start + i;
      uint8_t byte = d[e >> 1];
      float q = (float)((e & 1) ? (byte >> 4) & 0x0F : byte & 0x0F);
      uint64_t b = (e + 1) / bs; /* closed form of the running index */
      float scale = b < t->n_scales ? t->scales[b] : 1.0f;
      float zero = b < t->n_zero_points ? t->zero_points[b] : 0.0f;
      out[i] = (q - zero) * scale;
    }
  } else {
    const uint8_t* d = (const uint8_t*)t->data;
    uint64_t bs = (uint64_t)t->block_size;
    for (uint64_t i = 0; i < len; ++i) {
      uint64_t e = start + i;
      uint64_t b = e / bs;
      float scale = b < t->n_scales ? t->scales[b] : 1.0f;
      float zero = b < t->n_zero_points ? t->zero_points[b] : 0.0f;
      out[i] = ((float)d[e] - zero) * scale;
    }
  }
  if (bf16_round)
    for (uint64_t i = 0; i < len; ++i) out[i] = round_bf16(out[i]);
}

/* ---------------------------------------------------------------- router */

/* e^x by Cody & Waite's argument reduction x = n*ln2 + r (ln2 split into a
 * 16-bit head and a tail so n*ln2_hi is exact), then the degree-7 Taylor
 * polynomial of e^r on |r| <= ln2/2 in Horner form with fused multiply-adds
 * (truncation error < 6e-9 relative), scaled by 2^n. Inputs below -87 give 0
 * (the softmax only feeds x - max <= 0). Every step is an IEEE operation
 * with one rounding, so the CUDA router reproduces it bit for bit. */
float ro_expf(float x) {
  if (x != x) return x;
  if (x < -87.0f) return 0.0f;
  if (x > 88.0f) return INFINITY;
  const float log2e = 0x1.715476p+0f;  /* float(log2 e) */
  const float ln2_hi = 0x1.62e4p-1f;    /* 0.693145751953125, 16 bits */
  const float ln2_lo = 0x1.7f7d1cp-20f; /* float(ln2 - ln2_hi) */
  float t = x * log2e;
  float n = rintf(t);
  float r = fmaf(-n, ln2_hi, x);
  r = fmaf(-n, ln2_lo, r);
  float p = 0x1.a01a02p-13f;      /* 1/7! */
  p = fmaf(p, r, 0x1.6c16c2p-10f); /* 1/6! */
  p = fmaf(p, r, 0x1.111112p-7f);  /* 1/5! */
  p = fmaf(p, r, 0x1.555556p-5f);  /* 1/4! */
  p = fmaf(p, r, 0x1.555556p-3f);  /* 1/3! */
  p = fmaf(p, r, 0.5f);
  p = fmaf(p, r, 1.0f);
  p = fmaf(p, r, 1.0f);
  int ni = (int)n;
  /* 2^n for n in [-126, 127] as an exact float */
  uint32_t bits = (uint32_t)(ni + 127) << 23;
  float scale;
  memcpy(&scale, &bits, 4);
  return p * scale;
}

static float router_dot(const float* xf, const float* w, int32_t H) {
  float lane[32];
  int32_t nchunk = H / 8;
  for (int l = 0; l < 32; ++l) {
    float acc = 0.0f;
    for (int32_t c = l; c < nchunk; c += 32)
      for (int j = 0; j < 8; ++j) acc = fmaf(xf[8 * c + j], w[8 * c + j], acc);
    lane[l] = acc;
  }
  for (int off = 16; off >= 1; off >>= 1) {
    float nl[32];
    for (int l = 0; l < 32; ++l) nl[l] = lane[l] + lane[l ^ off];
    memcpy(lane, nl, sizeof(lane));
  }
  return lane[0];
}

static void x_row_f32(const void* x, int32_t x_bf16, int32_t H, int32_t t,
                      float* xf) {
  if (x_bf16) {
    const uint16_t* xb = (const uint16_t*)x + (uint64_t)t * H;
    for (int32_t h = 0; h < H; ++h) xf[h] = ro_bf16_to_f32(xb[h]);
  } else {
    memcpy(xf, (const float*)x + (uint64_t)t * H, sizeof(float) * H);
  }
}

void ro_router(const void* x, int32_t x_bf16, int32_t T, int32_t H,
               const float* wg, int32_t E, int32_t k, float* logits,
               float* probs, int32_t* topk_idx, float* topk_w) {
#pragma omp parallel
  {
    float* xf = (float*)malloc(sizeof(float) * H);
    float* lg = (float*)malloc(sizeof(float) * E);
    float* ex = (float*)malloc(sizeof(float) * E);
    float* p = (float*)malloc(sizeof(float) * E);
    char* taken = (char*)malloc(E);
#pragma omp for schedule(static)
    for (int32_t t = 0; t < T; ++t) {
      x_row_f32(x, x_bf16, H, t, xf);
      for (int32_t e = 0; e < E; ++e) lg[e] = router_dot(xf, wg + (uint64_t)e * H, H);
      float m = -INFINITY;
      for (int32_t e = 0; e < E; ++e) m = fmaxf(m, lg[e]);
      for (int32_t e = 0; e < E; ++e) ex[e] = ro_expf(lg[e] - m);
      float s = 0.0f;
      for (int32_t e = 0; e < E; ++e) s += ex[e];
      for (int32_t e = 0; e < E; ++e) p[e] = ex[e] / s;
      if (logits) memcpy(logits + (uint64_t)t * E, lg, sizeof(float) * E);
      if (probs) memcpy(probs + (uint64_t)t * E, p, sizeof(float) * E);
      memset(taken, 0, E);
      int32_t sel[256];
      for (int32_t j = 0; j < k; ++j) {
        int32_t best = -1;
        for (int32_t e = 0; e < E; ++e) {
          if (taken[e]) continue;
          if (best < 0 || p[e] > p[best]) best = e;
        }
        taken[best] = 1;
        sel[j] = best;
      }
      float ssum = 0.0f;
      for (int32_t j = 0; j < k; ++j) ssum += p[sel[j]];
      for (int32_t j = 0; j < k; ++j) {
        if (topk_idx) topk_idx[(uint64_t)t * k + j] = sel[j];
        if (topk_w) topk_w[(uint64_t)t * k + j] = p[sel[j]] / ssum;
      }
    }
    free(xf);
    free(lg);
    free(ex);
    free(p);
    free(taken);
  }
}

void ro_bucket(const int32_t* topk_idx, int32_t T, int32_t k, int32_t E,
               int32_t* counts, int32_t* offsets, int32_t* perm_pair) {
  int64_t P = (int64_t)T * k;
  for (int32_t e = 0; e < E; ++e) counts[e] = 0;
  for (int64_t p = 0; p < P; ++p) counts[topk_idx[p]] += 1;
  offsets[0] = 0;
  for (int32_t e = 0; e < E; ++e) offsets[e + 1] = offsets[e] + counts[e];
  int32_t* fill = (int32_t*)calloc((size_t)E, sizeof(int32_t));
  for (int64_t p = 0; p < P; ++p) {
    int32_t e = topk_idx[p];
    perm_pair[offsets[e] + fill[e]++] = (int32_t)p;
  }
  free(fill);
}

/* ------------------------------------------------------------- MoE block */

static inline float silu(float g) { return g / (1.0f + expf(-g)); }

/* out_rows[j][r] = x_rows[j] . W[row0 + r], r in [0,R), one weight row of
 * length K at a time (dequantized once, used by every token). */
static void rows_matvec(const ro_qtensor* W, uint64_t row0, int32_t R, int32_t K,
                        int32_t bf16, const float* xr, int32_t n, float* outr,
                        int32_t ld_out) {
#pragma omp parallel
  {
    float* row = (float*)malloc(sizeof(float) * K);
#pragma omp for schedule(static)
    for (int32_t r = 0; r < R; ++r) {
      ro_tensor_span_f32(W, (row0 + (uint64_t)r) * (uint64_t)K, (uint64_t)K, bf16, row);
      for (int32_t j = 0; j < n; ++j) {
        const float* xv = xr + (uint64_t)j * K;
        double acc = 0.0;
        for (int32_t c = 0; c < K; ++c) acc += (double)xv[c] * (double)row[c];
        outr[(uint64_t)j * ld_out + r] = (float)acc;
      }
    }
    free(row);
  }
}

void ro_moe_forward(const ro_moe_weights* w, const void* x, int32_t act_bf16,
                    int32_t T, int32_t H, int32_t I, int32_t E, int32_t k,
                    float* out, int32_t* topk_idx, float* topk_w,
                    int32_t* counts, int32_t n_threads) {
#ifdef _OPENMP
  int prev_threads = omp_get_max_threads();
  if (n_threads > 0) omp_set_num_threads(n_threads);
#else
  (void)n_threads;
#endif
  uint64_t P = (uint64_t)T * k;
  float* xf = (float*)malloc(sizeof(float) * (uint64_t)T * H);
  for (int32_t t = 0; t < T; ++t) x_row_f32(x, act_bf16, H, t, xf + (uint64_t)t * H);
  float* wg = (float*)malloc(sizeof(float) * (uint64_t)E * H);
  ro_tensor_span_f32(&w->gate, 0, (uint64_t)E * H, 0, wg);
  int32_t* idx = (int32_t*)malloc(sizeof(int32_t) * P);
  float* tw = (float*)malloc(sizeof(float) * P);
  ro_router(x, act_bf16, T, H, wg, E, k, NULL, NULL, idx, tw);
  int32_t* cnt = (int32_t*)malloc(sizeof(int32_t) * E);
  int32_t* off = (int32_t*)malloc(sizeof(int32_t) * (E + 1));
  int32_t* perm = (int32_t*)malloc(sizeof(int32_t) * P);
  ro_bucket(idx, T, k, E, cnt, off, perm);
  memset(out, 0, sizeof(float) * (uint64_t)T * H);

  int32_t max_n = 0;
  for (int32_t e = 0; e < E; ++e) max_n = cnt[e] > max_n ? cnt[e] : max_n;
  int32_t nrows = max_n > T ? max_n : T;
  float* xs = (float*)malloc(sizeof(float) * (uint64_t)nrows * H);
  float* proj = (float*)malloc(sizeof(float) * (uint64_t)nrows * 2 * I);
  float* hb = (float*)malloc(sizeof(float) * (uint64_t)nrows * I);
  float* y = (float*)malloc(sizeof(float) * (uint64_t)nrows * H);

  for (int32_t e = 0; e < E; ++e) {
    int32_t n = cnt[e];
    if (n == 0) continue;
    for (int32_t j = 0; j < n; ++j) {
      int32_t tok = perm[off[e] + j] / k;
      memcpy(xs + (uint64_t)j * H, xf + (uint64_t)tok * H, sizeof(float) * H);
    }
    rows_matvec(&w->gate_up_proj, (uint64_t)e * 2 * I, 2 * I, H, act_bf16, xs, n,
                proj, 2 * I);
    for (int32_t j = 0; j < n; ++j)
      for (int32_t i = 0; i < I; ++i) {
        float g = proj[(uint64_t)j * 2 * I + i];
        float u = proj[(uint64_t)j * 2 * I + I + i];
        float hv = silu(g) * u;
        hb[(uint64_t)j * I + i] = act_bf16 ? round_bf16(hv) : hv;
      }
    rows_matvec(&w->down_proj, (uint64_t)e * H, H, I, act_bf16, hb, n, y, H);
    for (int32_t j = 0; j < n; ++j) {
      int32_t pr = perm[off[e] + j];
      int32_t tok = pr / k;
      /* src/model.rs:800-802: the routing weight is cast to the activation
       * dtype before it scales the expert output (bf16 rounding in bf16
       * mode); the product and the sum stay float32. */
      float wt = act_bf16 ? round_bf16(tw[pr]) : tw[pr];
      float* o = out + (uint64_t)tok * H;
      const float* yv = y + (uint64_t)j * H;
      for (int32_t h = 0; h < H; ++h) o[h] = o[h] + yv[h] * wt;
    }
  }

  if (w->shared_gate_proj.data != NULL) {
    int32_t Is = w->shared_intermediate;
    float* sg = (float*)malloc(sizeof(float) * (uint64_t)T * Is);
    float* su = (float*)malloc(sizeof(float) * (uint64_t)T * Is);
    float* sh = (float*)malloc(sizeof(float) * (uint64_t)T * Is);
    float* sy = (float*)malloc(sizeof(float) * (uint64_t)T * H);
    float* sgate = (float*)malloc(sizeof(float) * (uint64_t)T);
    rows_matvec(&w->shared_gate_proj, 0, Is, H, act_bf16, xf, T, sg, Is);
    rows_matvec(&w->shared_up_proj, 0, Is, H, act_bf16, xf, T, su, Is);
    for (uint64_t i = 0; i < (uint64_t)T * Is; ++i) {
      float hv = silu(sg[i]) * su[i];
      sh[i] = act_bf16 ? round_bf16(hv) : hv;
    }
    rows_matvec(&w->shared_down_proj, 0, H, Is, act_bf16, sh, T, sy, H);
    rows_matvec(&w->shared_expert_gate, 0, 1, H, 0, xf, T, sgate, 1);
    for (int32_t t = 0; t < T; ++t) {
      float gsig = 1.0f / (1.0f + expf(-sgate[t]));
      float* o = out + (uint64_t)t * H;
      for (int32_t h = 0; h < H; ++h) o[h] = o[h] + sy[(uint64_t)t * H + h] * gsig;
    }
    free(sg);
    free(su);
    free(sh);
    free(sy);
    free(sgate);
  }

  if (topk_idx) memcpy(topk_idx, idx, sizeof(int32_t) * P);
  if (topk_w) memcpy(topk_w, tw, sizeof(float) * P);
  if (counts) memcpy(counts, cnt, sizeof(int32_t) * E);
  free(xf);
  free(wg);
  free(idx);
  free(tw);
  free(cnt);
  free(off);
  free(perm);
  free(xs);
  free(proj);
  free(hb);
  free(y);
#ifdef _OPENMP
  if (n_threads > 0) omp_set_num_threads(prev_threads);
#endif
}
