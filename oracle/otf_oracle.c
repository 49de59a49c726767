/*
 * otf_oracle.c -- CPU restatement of OTF-LLM's quantized-decode path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity oracle and the timed CPU
 * baseline; nothing in the shipped library links it.  Only tests/, the smoke
 * check and bench.py's CPU-baseline leg load it, and only as the checker.
 *
 * Every function restates one piece of the reference package otf_llm
 * (GT-Labs-AI/otf-llm-engine, v4.1.0); the file:line each one follows is in
 * its comment.  Half-precision values are carried as uint16_t bit patterns and
 * converted with _Float16 (IEEE-754 binary16, round-to-nearest-even), which is
 * the rounding torch applies on CPU.
 */
#include <stdint.h>
#include <string.h>
#include <stdlib.h>
#include <math.h>
#ifdef _OPENMP
#include <omp.h>
#endif

typedef uint16_t h16;

static inline float h2f(h16 v) { _Float16 h; memcpy(&h, &v, 2); return (float)h; }
static inline h16 f2h(float f) { _Float16 h = (_Float16)f; h16 v; memcpy(&v, &h, 2); return v; }

int orc_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

void orc_set_num_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}

/* Code k of row n sits at bits 2*(k%4) of byte k/4 (pack_2bit_uint8,
 * otf_llm/symmetric_2bit_engine.py:100-107; unpack in
 * otf_llm/otf_2bit_quantizer.py:58-63).  codes: uint8 [N, K]. */
void orc_unpack_codes(const uint8_t* packed, int64_t ld_packed, int64_t N, int64_t K, uint8_t* codes) {
  #pragma omp parallel for schedule(static)
  for (int64_t n = 0; n < N; ++n)
    for (int64_t k = 0; k < K; ++k)
      codes[n * K + k] = (packed[n * ld_packed + k / 4] >> (2 * (k % 4))) & 3u;
}

/* Inverse of orc_unpack_codes: pack_2bit_uint8 (otf_llm/symmetric_2bit_engine.py:100-107). */
void orc_pack_codes(const uint8_t* codes, int64_t N, int64_t K, uint8_t* packed) {
  #pragma omp parallel for schedule(static)
  for (int64_t n = 0; n < N; ++n)
    for (int64_t b = 0; b < K / 4; ++b) {
      const uint8_t* c = codes + n * K + 4 * b;
      packed[n * (K / 4) + b] = (uint8_t)((c[0] & 3) | ((c[1] & 3) << 2) | ((c[2] & 3) << 4) | ((c[3] & 3) << 6));
    }
}

/*
 * fp32 restatement of one quantized linear layer (the numeric oracle).
 *
 *   xm[m,k]  = fp16(x[m,k] * mask[k])                 mask multiply in fp16,
 *                                                     otf_llm/otf_triton_2bit_kernel.py:178-179
 *   w[n,k]   = cb[q[n,k]] * s[n,k/G] (+ z[n,k/G])     byte-LUT dequant, :189-192 (symmetric);
 *                                                     unpack_2bit_uint8 with zeros,
 *                                                     otf_llm/otf_2bit_quantizer.py:65-71
 *   y[m,n]   = sum_k xm*w + bias[n] + sum_j x[m,idx_j]*ov[n,j]
 *                                                     otf_llm/symmetric_2bit_engine.py:218-232
 *   y        = clamp(y, -65504, 65504)                :234 (skipped when clamp == 0, as
 *                                                     OTF2BitLinear.forward does not clamp)
 * Everything after the fp16 inputs is fp32 with a double accumulator; y is fp32 [M, N].
 * Optional pointers may be NULL.
 */
void orc_linear_f32(const h16* x, int64_t ldx, const uint8_t* packed, int64_t ld_packed,
                    const h16* scales, int64_t ld_scales, const h16* zeros, int64_t ld_zeros,
                    const float* cb4, const h16* mask, const int64_t* oidx, int64_t n_out,
                    const h16* ovals, int64_t ld_ovals, const h16* bias, float* y, int64_t ldy,
                    int64_t M, int64_t N, int64_t K, int64_t G, int clamp) {
  float* xm = (float*)malloc(sizeof(float) * (size_t)(M * K));
  for (int64_t m = 0; m < M; ++m)
    for (int64_t k = 0; k < K; ++k) {
      float v = h2f(x[m * ldx + k]);
      xm[m * K + k] = mask ? h2f(f2h(v * h2f(mask[k]))) : v;
    }
  #pragma omp parallel for schedule(static)
  for (int64_t n = 0; n < N; ++n) {
    for (int64_t m = 0; m < M; ++m) {
      double acc = 0.0;
      for (int64_t g = 0; g < K / G; ++g) {
        float s = h2f(scales[n * ld_scales + g]);
        float z = zeros ? h2f(zeros[n * ld_zeros + g]) : 0.0f;
        for (int64_t k = g * G; k < (g + 1) * G; ++k) {
          unsigned q = (packed[n * ld_packed + k / 4] >> (2 * (k % 4))) & 3u;
          float w = cb4[q] * s + z;
          acc += (double)xm[m * K + k] * (double)w;
        }
      }
      if (bias) acc += (double)h2f(bias[n]);
      for (int64_t j = 0; j < n_out; ++j)
        acc += (double)h2f(x[m * ldx + oidx[j]]) * (double)h2f(ovals[n * ld_ovals + j]);
      float r = (float)acc;
      if (clamp) r = fminf(fmaxf(r, -65504.0f), 65504.0f);
      y[m * ldy + n] = r;
    }
  }
  free(xm);
}

/*
 * The reference's own CPU algorithm for SymmetricOTF2BitLinear.forward, ported
 * step for step so that its cost can be timed (it is the reference arm of the
 * benchmark).  Per call it materialises the fp16 weight matrix through the
 * 256x4 byte LUT and the fp16 scale product (otf_llm/otf_triton_2bit_kernel.py:
 * 149-161 and :189-192, both in fp16), multiplies the masked fp16 activations
 * with it (:193, fp32 accumulate), clamps (:194), then adds bias and the fp16
 * outlier product and clamps again (otf_llm/symmetric_2bit_engine.py:227-234).
 * wbuf must hold N*K halves (scratch for the materialised matrix).  y is fp16.
 */
void orc_lut_linear(const h16* x, int64_t ldx, const uint8_t* packed, int64_t ld_packed,
                    const h16* scales, int64_t ld_scales, const h16* cb4_h, const h16* mask,
                    const int64_t* oidx, int64_t n_out, const h16* ovals, int64_t ld_ovals,
                    const h16* bias, h16* y, int64_t ldy, int64_t M, int64_t N, int64_t K, int64_t G,
                    h16* wbuf) {
  h16 lut[256][4];
  for (int b = 0; b < 256; ++b)
    for (int i = 0; i < 4; ++i) lut[b][i] = cb4_h[(b >> (2 * i)) & 3];
  float* xm = (float*)malloc(sizeof(float) * (size_t)(M * K));
  for (int64_t m = 0; m < M; ++m)
    for (int64_t k = 0; k < K; ++k) {
      float v = h2f(x[m * ldx + k]);
      xm[m * K + k] = mask ? h2f(f2h(v * h2f(mask[k]))) : v;
    }
  #pragma omp parallel for schedule(static)
  for (int64_t n = 0; n < N; ++n) {
    h16* wr = wbuf + n * K;
    for (int64_t k4 = 0; k4 < K / 4; ++k4) {
      const h16* c = lut[packed[n * ld_packed + k4]];
      float s = h2f(scales[n * ld_scales + (4 * k4) / G]);
      for (int i = 0; i < 4; ++i) wr[4 * k4 + i] = f2h(h2f(c[i]) * s);
    }
  }
  #pragma omp parallel for schedule(static)
  for (int64_t n = 0; n < N; ++n) {
    const h16* wr = wbuf + n * K;
    for (int64_t m = 0; m < M; ++m) {
      float acc = 0.0f;
      for (int64_t k = 0; k < K; ++k) acc += xm[m * K + k] * h2f(wr[k]);
      acc = fminf(fmaxf(acc, -65504.0f), 65504.0f);
      h16 yh = f2h(acc);
      if (bias) yh = f2h(h2f(yh) + h2f(bias[n]));
      if (n_out > 0) {
        float o = 0.0f;
        for (int64_t j = 0; j < n_out; ++j) o += h2f(x[m * ldx + oidx[j]]) * h2f(ovals[n * ld_ovals + j]);
        yh = f2h(h2f(yh) + h2f(f2h(o)));
      }
      float r = fminf(fmaxf(h2f(yh), -65504.0f), 65504.0f);
      y[m * ldy + n] = f2h(r);
    }
  }
  free(xm);
}

/*
 * INT8 shared-vocabulary LM head, fp32 restatement of QuantizedLinearHead.forward
 * (otf_llm/symmetric_2bit_engine.py:75-91): logits[m,v] = sum_d x[m,d]*w[v,d] * s[v],
 * then nan_to_num(nan=0, +-inf=+-65504) (:90).  The reference computes the product in
 * fp16 chunks (:84-88); this oracle keeps fp32, and clamps to the range the fp16 path
 * can produce.  logits: fp32 [M, V].
 */
void orc_i8_head(const h16* x, int64_t ldx, const int8_t* w, int64_t ldw, const h16* scales,
                 float* logits, int64_t ldl, int64_t M, int64_t V, int64_t D) {
  #pragma omp parallel for schedule(static)
  for (int64_t v = 0; v < V; ++v) {
    float s = h2f(scales[v]);
    for (int64_t m = 0; m < M; ++m) {
      double acc = 0.0;
      for (int64_t d = 0; d < D; ++d) acc += (double)h2f(x[m * ldx + d]) * (double)w[v * ldw + d];
      float r = (float)(acc * (double)s);
      if (isnan(r)) r = 0.0f;
      r = fminf(fmaxf(r, -65504.0f), 65504.0f);
      logits[m * ldl + v] = r;
    }
  }
}

/* Greedy pick over fp32 logits: first index of the maximum (torch.argmax order). */
void orc_argmax_rows(const float* logits, int64_t ldl, int64_t M, int64_t V, int64_t* out) {
  for (int64_t m = 0; m < M; ++m) {
    int64_t best = 0;
    float bv = logits[m * ldl];
    for (int64_t v = 1; v < V; ++v)
      if (logits[m * ldl + v] > bv) { bv = logits[m * ldl + v]; best = v; }
    out[m] = best;
  }
}

/*
 * INT8 embedding gather, QuantizedEmbedding.forward (otf_llm/symmetric_2bit_engine.py:41-47):
 * out[t,:] = fp16( fp16(w[id_t,:]) * s[id_t] ).  The product of two halves is exact in
 * fp32, so rounding it once to fp16 reproduces the fp16 multiply bit for bit.
 * Returns the number of ids outside [0, V) (those rows are left untouched).
 */
int64_t orc_i8_embed(const int64_t* ids, int64_t n_ids, const int8_t* w, int64_t ldw, const h16* scales,
                     h16* out, int64_t ldo, int64_t V, int64_t D) {
  int64_t bad = 0;
  for (int64_t t = 0; t < n_ids; ++t) {
    int64_t id = ids[t];
    if (id < 0 || id >= V) { ++bad; continue; }
    float s = h2f(scales[id]);
    for (int64_t d = 0; d < D; ++d) out[t * ldo + d] = f2h((float)w[id * ldw + d] * s);
  }
  return bad;
}

/* Row-wise absmax INT8 quantisation, quantize_from_fp16
 * (otf_llm/symmetric_2bit_engine.py:26-39): s = max(absmax/127, 1e-8) in fp32,
 * q = clamp(round_half_even(w/s), -127, 127); the stored scale is fp16(s). */
void orc_i8_quantize(const h16* wf, int64_t ldw, int64_t V, int64_t D, int8_t* q, h16* scales) {
  #pragma omp parallel for schedule(static)
  for (int64_t v = 0; v < V; ++v) {
    float mx = 0.0f;
    for (int64_t d = 0; d < D; ++d) mx = fmaxf(mx, fabsf(h2f(wf[v * ldw + d])));
    float s = fmaxf(mx / 127.0f, 1e-8f);
    for (int64_t d = 0; d < D; ++d) {
      float r = nearbyintf(h2f(wf[v * ldw + d]) / s);
      r = fminf(fmaxf(r, -127.0f), 127.0f);
      q[v * D + d] = (int8_t)r;
    }
    scales[v] = f2h(s);
  }
}

/* Symmetric 2-bit quantizer, Symmetric2BitQuantizer.quantize_tensor
 * (otf_llm/symmetric_2bit_engine.py:109-169, packing :100-107), in fp32 with every product
 * and sum rounded on its own (no fused multiply-add) and the sums in this fixed order:
 *   column sums of squares over row chunks of QUANT_IMPACT_ROWS rows (row order inside a
 *   chunk, then chunk order), sqrt, times act[c];
 *   group sums: TL = min(32, G/4) partial sums, partial l taking elements 4l..4l+3 of each
 *   slab of 4*TL elements in slab order, then combined pairwise (l + TL/2, ..., l + 1).
 * Anchors: the k columns of largest impact, descending, ties to the lower index, NaN above
 * everything.  The torch reference sums in an order that depends on the device and vector
 * width; the two agree except for scales next to an fp16 rounding boundary (one ulp apart). */
#define QUANT_IMPACT_ROWS 256

static inline uint32_t order_key(float f) {
  uint32_t b;
  memcpy(&b, &f, 4);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

static const float* g_sort_keys;
static int cmp_impact(const void* a, const void* b) {
  const int64_t i = *(const int64_t*)a, j = *(const int64_t*)b;
  const uint32_t ki = order_key(g_sort_keys[i]), kj = order_key(g_sort_keys[j]);
  if (ki != kj) return ki > kj ? -1 : 1;
  return i < j ? -1 : (i > j);
}

__attribute__((optimize("fp-contract=off")))
static float team_sum(const float* v, int G, float* lanes) {
  const int TL = G / 4 < 32 ? G / 4 : 32, S = G / (4 * TL);
  for (int l = 0; l < TL; ++l) {
    float acc = 0.0f;
    int first = 1;
    for (int s = 0; s < S; ++s)
      for (int e = 0; e < 4; ++e) {
        const float p = v[s * 4 * TL + 4 * l + e];
        acc = first ? p : acc + p;
        first = 0;
      }
    lanes[l] = acc;
  }
  for (int o = TL / 2; o > 0; o >>= 1)
    for (int l = 0; l < o; ++l) lanes[l] = lanes[l] + lanes[l + o];
  return lanes[0];
}

__attribute__((optimize("fp-contract=off")))
void orc_quantize_2b(const float* W, int64_t ldw, int64_t N, int64_t K, int64_t G, const float* act, int64_t k,
                     const float* cb, uint8_t* packed, h16* scales, h16* outliers, int64_t* idx) {
  uint8_t* keep = (uint8_t*)malloc((size_t)K);
  memset(keep, 1, (size_t)K);
  if (k > 0) {
    const int64_t nch = (N + QUANT_IMPACT_ROWS - 1) / QUANT_IMPACT_ROWS;
    float* imp = (float*)malloc((size_t)K * sizeof(float));
    #pragma omp parallel for schedule(static)
    for (int64_t c = 0; c < K; ++c) {
      float tot = 0.0f;
      for (int64_t ch = 0; ch < nch; ++ch) {
        float acc = 0.0f;
        const int64_t r1 = (ch + 1) * QUANT_IMPACT_ROWS < N ? (ch + 1) * QUANT_IMPACT_ROWS : N;
        for (int64_t r = ch * QUANT_IMPACT_ROWS; r < r1; ++r) {
          const float v = W[r * ldw + c];
          const float p = v * v;
          acc = acc + p;
        }
        tot = ch == 0 ? acc : tot + acc;
      }
      float v = sqrtf(tot);
      if (act) v = v * act[c];
      imp[c] = v;
    }
    int64_t* order = (int64_t*)malloc((size_t)K * sizeof(int64_t));
    for (int64_t c = 0; c < K; ++c) order[c] = c;
    g_sort_keys = imp;
    qsort(order, (size_t)K, sizeof(int64_t), cmp_impact);
    for (int64_t j = 0; j < k; ++j) {
      idx[j] = order[j];
      keep[order[j]] = 0;
    }
    for (int64_t n = 0; n < N; ++n)
      for (int64_t j = 0; j < k; ++j) outliers[n * k + j] = f2h(W[n * ldw + idx[j]]);
    free(order);
    free(imp);
  }
  const int64_t ng = K / G;
  #pragma omp parallel for schedule(static)
  for (int64_t n = 0; n < N; ++n) {
    float w[256], kp[256], t[256], lanes[32];
    uint8_t q[256];
    for (int64_t g = 0; g < ng; ++g) {
      int cnt = 0;
      for (int64_t i = 0; i < G; ++i) {
        const int64_t c = g * G + i;
        kp[i] = keep[c] ? 1.0f : 0.0f;
        w[i] = keep[c] ? W[n * ldw + c] : 0.0f;
        cnt += keep[c];
      }
      for (int64_t i = 0; i < G; ++i) t[i] = w[i] * w[i];
      const float ss = team_sum(t, (int)G, lanes);
      const float nact = cnt > 1 ? (float)cnt : 1.0f;
      float s = sqrtf(ss / nact + 1e-8f) / 0.95f;
      s = s > 1e-8f ? s : 1e-8f;
      for (int it = 0; it < 5; ++it) {
        const float d = s > 1e-8f ? s : 1e-8f;
        float cq[256];
        for (int64_t i = 0; i < G; ++i) {
          const float z = w[i] / d;
          float best = fabsf(z - cb[0]);
          int b = 0;
          for (int j = 1; j < 4; ++j) {
            const float dj = fabsf(z - cb[j]);
            if (dj < best) { best = dj; b = j; }
          }
          q[i] = (uint8_t)b;
          cq[i] = cb[b] * kp[i];
        }
        for (int64_t i = 0; i < G; ++i) t[i] = w[i] * cq[i];
        const float num = team_sum(t, (int)G, lanes);
        for (int64_t i = 0; i < G; ++i) t[i] = cq[i] * cq[i];
        const float den = team_sum(t, (int)G, lanes);
        s = num / (den > 1e-8f ? den : 1e-8f);
        s = s > 1e-8f ? s : 1e-8f;
      }
      for (int64_t i = 0; i < G; i += 4)
        packed[n * (K / 4) + (g * G + i) / 4] =
            (uint8_t)(q[i] | (q[i + 1] << 2) | (q[i + 2] << 4) | (q[i + 3] << 6));
      scales[n * ng + g] = f2h(s);
    }
  }
  free(keep);
}

/* fp16 <-> fp32 helpers exported for the Python side of the oracle. */
void orc_h2f(const h16* in, float* out, int64_t n) { for (int64_t i = 0; i < n; ++i) out[i] = h2f(in[i]); }
void orc_f2h(const float* in, h16* out, int64_t n) { for (int64_t i = 0; i < n; ++i) out[i] = f2h(in[i]); }
