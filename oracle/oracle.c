/*
 * CPU ORACLE — test infrastructure only, never part of the product path.
 *
 * A plain-C restatement of the reference's llama-webgpu decode step
 * (bilalba/ChonkLM src/lib/llama-wgsl-runtime.ts, "runToken" :1025-1150) and
 * of every WGSL compute shader that step dispatches for GGUF models.  Each
 * function cites the shader it restates.  All arithmetic is IEEE fp32 in the
 * shaders' operation order; this file must be compiled with
 * -ffp-contract=off and without -ffast-math so products and sums are rounded
 * one at a time, as the WGSL expressions are written.
 *
 * Pinning: the dequantizers are pinned bit-for-bit against gguf-py 0.19.0
 * (llama.cpp's own Python reader of these block formats, whose numpy decode
 * uses the same fp32 operation order) by tests/test_oracle_golden.py.  Every
 * kernel of runToken (matvecs, embeddings, norms, RoPE stores, attention,
 * activations, residual adds, argmax stages) is pinned against the
 * reference's own WGSL text, run on the CPU by the oracle/wgsl.py
 * interpreter (tests/golden/wgsl_golden.npz, tests/test_wgsl_golden.py):
 * bit for bit where the shader's arithmetic is specified, within a few ulps
 * through pow / cos / sin / exp / tanh / inverseSqrt.  The graph order of
 * runToken (:1039-1124) is restated from the TypeScript, which cannot run
 * here (no JavaScript runtime).
 *
 * Two accumulation modes for matvec / attention dot products:
 *   OR_MODE_WGSL  : 128 per-thread strided partial sums + tree reduction,
 *                   exactly as GGUF_*_MATVEC_WGSL (:2202-2613) reduce;
 *   OR_MODE_F64   : fp64 accumulation ("truth") for tolerance checks.
 */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#define GT_F32 0
#define GT_F16 1
#define GT_Q5_0 6
#define GT_Q5_1 7
#define GT_Q8_0 8
#define GT_Q4_K 12
#define GT_Q5_K 13
#define GT_Q6_K 14

#define OR_MODE_WGSL 0
#define OR_MODE_F64 1

/* f16ToF32, llama-wgsl-runtime.ts:1837-1844 (exact, subnormals kept).  WGSL
 * unpack2x16float is also exact for every finite half. */
static float f16_to_f32(uint16_t h) {
  float sign = (h & 0x8000) ? -1.0f : 1.0f;
  int e = (h >> 10) & 0x1f;
  int frac = h & 0x3ff;
  if (e == 0) return sign * ldexpf((float)frac, -24);
  if (e == 0x1f) return frac ? NAN : sign * INFINITY;
  return sign * ldexpf((float)(1024 + frac), e - 25);
}

static inline uint32_t byte_at(const uint8_t* b, size_t i) { return b[i]; }
static inline float f16_at(const uint8_t* b, size_t i) {
  return f16_to_f32((uint16_t)(b[i] | (b[i + 1] << 8)));
}
static inline int32_t i8_at(const uint8_t* b, size_t i) { return (int8_t)b[i]; }
static inline uint32_t u32_at(const uint8_t* b, size_t i) {
  return (uint32_t)b[i] | ((uint32_t)b[i + 1] << 8) | ((uint32_t)b[i + 2] << 16) | ((uint32_t)b[i + 3] << 24);
}

int or_block_weights(int t) {
  switch (t) {
    case GT_F32: case GT_F16: return 1;
    case GT_Q5_0: case GT_Q5_1: case GT_Q8_0: return 32;
    case GT_Q4_K: case GT_Q5_K: case GT_Q6_K: return 256;
  }
  return 0;
}
int or_block_bytes(int t) {
  switch (t) {
    case GT_F32: return 4;
    case GT_F16: return 2;
    case GT_Q5_0: return 22;
    case GT_Q5_1: return 24;
    case GT_Q8_0: return 34;
    case GT_Q4_K: return 144;
    case GT_Q5_K: return 176;
    case GT_Q6_K: return 210;
  }
  return 0;
}

/* scale_min_k4, llama-wgsl-runtime.ts:2387-2394 */
static void scale_min_k4(const uint8_t* q, uint32_t j, uint32_t* d, uint32_t* m) {
  if (j < 4) {
    *d = q[j] & 63u;
    *m = q[j + 4] & 63u;
  } else {
    *d = (q[j + 4] & 15u) | ((q[j - 4] >> 6) << 4);
    *m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
  }
}

/* Weight (row-relative byte pointer `row`, column `col`) for each GGUF type.
 * Formulas and operation order follow the WGSL dequantizers:
 *   Q5_0 :2234-2245   Q5_1 :2280-2289   Q8_0 :2321-2327
 *   Q4_K :2396-2410   Q5_K :2479-2494   Q6_K :2560-2580                    */
static float weight_at(int t, const uint8_t* row, uint32_t col) {
  switch (t) {
    case GT_F32: { float f; memcpy(&f, row + 4 * (size_t)col, 4); return f; }
    case GT_F16: return f16_at(row, 2 * (size_t)col);
    case GT_Q5_0: case GT_Q5_1: {
      uint32_t block = col >> 5, within = col & 31u;
      size_t base = (size_t)block * (t == GT_Q5_0 ? 22 : 24);
      uint32_t qh = u32_at(row, base + (t == GT_Q5_0 ? 2 : 4));
      uint32_t q_byte = byte_at(row, base + (t == GT_Q5_0 ? 6 : 8) + (within & 15u));
      uint32_t low4 = within >= 16u ? (q_byte >> 4) : (q_byte & 15u);
      uint32_t high = (qh >> within) & 1u;
      uint32_t qv = low4 | (high << 4);
      if (t == GT_Q5_0) return f16_at(row, base) * (float)((int32_t)qv - 16);
      return f16_at(row, base) * (float)qv + f16_at(row, base + 2);
    }
    case GT_Q8_0: {
      uint32_t block = col >> 5, within = col & 31u;
      size_t base = (size_t)block * 34;
      return (float)i8_at(row, base + 2 + within) * f16_at(row, base);
    }
    case GT_Q4_K: case GT_Q5_K: {
      uint32_t sb = col >> 8, within = col & 255u;
      uint32_t group64 = within >> 6, lane = within & 31u;
      int high = (within & 32u) != 0;
      size_t base = (size_t)sb * (t == GT_Q4_K ? 144 : 176);
      float d = f16_at(row, base), dmin = f16_at(row, base + 2);
      uint32_t sc, mn;
      scale_min_k4(row + base + 4, group64 * 2 + (high ? 1 : 0), &sc, &mn);
      if (t == GT_Q4_K) {
        uint32_t q_byte = byte_at(row, base + 16 + group64 * 32 + lane);
        uint32_t qv = high ? (q_byte >> 4) : (q_byte & 15u);
        return d * (float)sc * (float)qv - dmin * (float)mn;
      } else {
        uint32_t q_byte = byte_at(row, base + 48 + group64 * 32 + lane);
        uint32_t low4 = high ? (q_byte >> 4) : (q_byte & 15u);
        uint32_t qh_mask = (high ? 2u : 1u) << (group64 * 2);
        uint32_t high_bit = (byte_at(row, base + 16 + lane) & qh_mask) != 0 ? 16u : 0u;
        return d * (float)sc * (float)(low4 + high_bit) - dmin * (float)mn;
      }
    }
    case GT_Q6_K: {
      uint32_t sb = col >> 8, within = col & 255u;
      uint32_t half = within >> 7, local = within & 127u;
      uint32_t lane = local & 31u, quarter = local >> 5;
      size_t base = (size_t)sb * 210;
      size_t ql_base = base + half * 64, qh_base = base + 128 + half * 32, sc_base = base + 192 + half * 8;
      uint32_t ql = byte_at(row, ql_base + lane + ((quarter & 1u) ? 32 : 0));
      uint32_t lo = quarter < 2 ? (ql & 15u) : (ql >> 4);
      uint32_t qh = (byte_at(row, qh_base + lane) >> (quarter * 2)) & 3u;
      int32_t q = (int32_t)(lo | (qh << 4)) - 32;
      int32_t scale = i8_at(row, sc_base + (lane >> 4) + quarter * 2);
      return f16_at(row, base + 208) * (float)scale * (float)q;
    }
  }
  return NAN;
}

size_t or_row_bytes(int t, int k) { return (size_t)(k / or_block_weights(t)) * or_block_bytes(t); }

/* Dequantize `n` rows of `k` weights. */
void or_dequant(int t, const uint8_t* w, int k, int n, float* out) {
  size_t rb = or_row_bytes(t, k);
#pragma omp parallel for schedule(static)
  for (int r = 0; r < n; r++)
    for (int c = 0; c < k; c++) out[(size_t)r * k + c] = weight_at(t, w + rb * r, (uint32_t)c);
}

/* Embedding row `token` times EMBEDDING_SCALE, GGUF_*_EMBEDDING_WGSL
 * (:2615-2866).  The shaders multiply the finished weight expression by the
 * scale, i.e. (w) * ES with w rounded first. */
void or_embedding(int t, const uint8_t* table, int k, uint32_t token, float scale, float* out) {
  const uint8_t* row = table + or_row_bytes(t, k) * token;
  for (int c = 0; c < k; c++) out[c] = weight_at(t, row, (uint32_t)c) * scale;
}

/* One row of weights into out[0..k), each value computed by the same
 * expression, in the same operation order, as weight_at (the per-block
 * factors d*sc and dmin*m are the leading products of that expression, so
 * hoisting them per sub-block leaves every rounding unchanged). */
static void dequant_row(int t, const uint8_t* row, int k, float* out) {
  switch (t) {
    case GT_Q4_K: case GT_Q5_K: {
      const size_t bb = t == GT_Q4_K ? 144 : 176;
      for (int sb = 0; sb < k / 256; sb++) {
        const size_t base = (size_t)sb * bb;
        const float d = f16_at(row, base), dmin = f16_at(row, base + 2);
        for (uint32_t j = 0; j < 8; j++) {
          uint32_t sc, mn;
          scale_min_k4(row + base + 4, j, &sc, &mn);
          const float a = d * (float)sc, b = dmin * (float)mn;
          const uint32_t group64 = j >> 1, high = j & 1u;
          float* o = out + 256 * sb + 64 * group64 + 32 * high;
          for (uint32_t lane = 0; lane < 32; lane++) {
            uint32_t qv;
            if (t == GT_Q4_K) {
              const uint32_t q_byte = row[base + 16 + group64 * 32 + lane];
              qv = high ? (q_byte >> 4) : (q_byte & 15u);
            } else {
              const uint32_t q_byte = row[base + 48 + group64 * 32 + lane];
              const uint32_t low4 = high ? (q_byte >> 4) : (q_byte & 15u);
              const uint32_t qh_mask = (high ? 2u : 1u) << (group64 * 2);
              qv = low4 + ((row[base + 16 + lane] & qh_mask) != 0 ? 16u : 0u);
            }
            o[lane] = a * (float)qv - b;
          }
        }
      }
      return;
    }
    case GT_Q6_K: {
      for (int sb = 0; sb < k / 256; sb++) {
        const size_t base = (size_t)sb * 210;
        const float d = f16_at(row, base + 208);
        for (uint32_t half = 0; half < 2; half++)
          for (uint32_t quarter = 0; quarter < 4; quarter++)
            for (uint32_t lane = 0; lane < 32; lane++) {
              const uint32_t ql = row[base + half * 64 + lane + ((quarter & 1u) ? 32 : 0)];
              const uint32_t lo = quarter < 2 ? (ql & 15u) : (ql >> 4);
              const uint32_t qh = (row[base + 128 + half * 32 + lane] >> (quarter * 2)) & 3u;
              const int32_t q = (int32_t)(lo | (qh << 4)) - 32;
              const int32_t scale = (int8_t)row[base + 192 + half * 8 + (lane >> 4) + quarter * 2];
              out[256 * sb + 128 * half + 32 * quarter + lane] = d * (float)scale * (float)q;
            }
      }
      return;
    }
    case GT_Q8_0: {
      for (int b = 0; b < k / 32; b++) {
        const size_t base = (size_t)b * 34;
        const float d = f16_at(row, base);
        for (int i = 0; i < 32; i++) out[32 * b + i] = (float)(int8_t)row[base + 2 + i] * d;
      }
      return;
    }
    case GT_Q5_0: case GT_Q5_1: {
      const size_t bb = t == GT_Q5_0 ? 22 : 24;
      for (int b = 0; b < k / 32; b++) {
        const size_t base = (size_t)b * bb;
        const uint32_t qh = u32_at(row, base + (t == GT_Q5_0 ? 2 : 4));
        const float d = f16_at(row, base);
        const float m = t == GT_Q5_1 ? f16_at(row, base + 2) : 0.0f;
        for (uint32_t w = 0; w < 32; w++) {
          const uint32_t q_byte = row[base + (t == GT_Q5_0 ? 6 : 8) + (w & 15u)];
          const uint32_t qv = (w >= 16u ? (q_byte >> 4) : (q_byte & 15u)) | (((qh >> w) & 1u) << 4);
          out[32 * b + w] = t == GT_Q5_0 ? d * (float)((int32_t)qv - 16) : d * (float)qv + m;
        }
      }
      return;
    }
    default:
      for (int c = 0; c < k; c++) out[c] = weight_at(t, row, (uint32_t)c);
  }
}

/* GGUF_*_MATVEC_WGSL main (:2247-2277 and siblings): 128 threads stride k,
 * `sum = sum + input[k] * w`, then a stride-64..1 tree. */
void or_matvec(int t, const uint8_t* w, int k, int n, const float* x, float* y, int mode) {
  size_t rb = or_row_bytes(t, k);
  /* rows are independent: spreading them over host threads changes no result */
#pragma omp parallel
  {
    float* wr = (float*)malloc((size_t)k * sizeof(float));
#pragma omp for schedule(static)
    for (int r = 0; r < n; r++) {
      dequant_row(t, w + rb * r, k, wr);
      if (mode == OR_MODE_F64) {
        double s = 0.0;
        for (int c = 0; c < k; c++) s += (double)x[c] * (double)wr[c];
        y[r] = (float)s;
        continue;
      }
      float partial[128];
      for (int tid = 0; tid < 128; tid++) {
        float sum = 0.0f;
        for (int c = tid; c < k; c += 128) {
          float p = x[c] * wr[c];
          sum = sum + p;
        }
        partial[tid] = sum;
      }
      for (int stride = 64; stride >= 1; stride >>= 1)
        for (int tid = 0; tid < stride; tid++) partial[tid] = partial[tid] + partial[tid + stride];
      y[r] = partial[0];
    }
    free(wr);
  }
}

/* RMS_NORM_WGSL :1910-1949 (256 threads, stride-128..1 tree). */
static float rms_inv(const float* v, int n, float eps) {
  float partial[256];
  for (int tid = 0; tid < 256; tid++) {
    float sum = 0.0f;
    for (int i = tid; i < n; i += 256) { float sq = v[i] * v[i]; sum = sum + sq; }
    partial[tid] = sum;
  }
  for (int stride = 128; stride >= 1; stride >>= 1)
    for (int tid = 0; tid < stride; tid++) partial[tid] = partial[tid] + partial[tid + stride];
  return 1.0f / sqrtf(partial[0] / (float)n + eps);
}

void or_rms_norm(const float* in, const float* w, float* out, int n, float eps) {
  float inv = rms_inv(in, n, eps);
  for (int i = 0; i < n; i++) { float a = in[i] * inv; out[i] = a * w[i]; }
}

/* ADD_RMS_NORM_WGSL :1951-1992: io = a + io, out = rmsnorm(io) * w. */
void or_add_rms_norm(const float* a, float* io, const float* w, float* out, int n, float eps) {
  for (int i = 0; i < n; i++) io[i] = a[i] + io[i];
  or_rms_norm(io, w, out, n, eps);
}

/* rope_angle (:2885-2888): pow(f32(theta), -2*d/HEAD_DIM) * pos, theta is the
 * u32 Math.round(layer theta) the host passes (:1477). */
static float rope_angle(uint32_t theta, uint32_t d, uint32_t hd, uint32_t pos) {
  float e = (-2.0f * (float)d) / (float)hd;
  float inv = powf((float)theta, e);
  return (float)pos * inv;
}

static void rope_pair(float a, float b, float ang, float* o0, float* o1) {
  float co = cosf(ang), si = sinf(ang);
  float t0 = a * co, t1 = b * si, t2 = a * si, t3 = b * co;
  *o0 = t0 - t1;
  *o1 = t2 + t3;
}

/* ROPE_STORE_WGSL (:2868-2927, split halves) and ROPE_STORE_INTERLEAVED_WGSL
 * (:3122-3184, adjacent pairs).  q is rotated in place; k is rotated into
 * key_cache at pos; v is copied into value_cache.  Cache layout
 * [kv_head][max_context][head_dim] (:2915). */
void or_rope_store(float* q, const float* k, const float* v, float* kc, float* vc, int heads, int kv_heads,
                   int hd, int max_ctx, int pos, uint32_t theta, int interleaved) {
  int half = hd / 2;
  for (int h = 0; h < heads; h++)
    for (int d = 0; d < half; d++) {
      int i0 = interleaved ? h * hd + 2 * d : h * hd + d;
      int i1 = interleaved ? i0 + 1 : i0 + half;
      float ang = rope_angle(theta, (uint32_t)d, (uint32_t)hd, (uint32_t)pos);
      rope_pair(q[i0], q[i1], ang, &q[i0], &q[i1]);
    }
  for (int h = 0; h < kv_heads; h++) {
    size_t cb = ((size_t)h * max_ctx + pos) * hd;
    for (int d = 0; d < half; d++) {
      int s0 = interleaved ? 2 * d : d, s1 = interleaved ? 2 * d + 1 : d + half;
      float ang = rope_angle(theta, (uint32_t)d, (uint32_t)hd, (uint32_t)pos);
      rope_pair(k[h * hd + s0], k[h * hd + s1], ang, &kc[cb + s0], &kc[cb + s1]);
    }
    for (int d = 0; d < hd; d++) vc[cb + d] = v[h * hd + d];
  }
}

/* Per-head RMS with the 256-wide tree of QK_NORM_ROPE_STORE_WGSL (:2962-2986). */
static float head_rms_inv(const float* v, int hd, float eps) {
  float partial[256];
  for (int d = 0; d < 256; d++) partial[d] = d < hd ? v[d] * v[d] : 0.0f;
  for (int stride = 128; stride >= 1; stride >>= 1)
    for (int d = 0; d < stride; d++) partial[d] = partial[d] + partial[d + stride];
  return 1.0f / sqrtf(partial[0] / (float)hd + eps);
}

/* QK_NORM_ROPE_STORE_WGSL (:2929-3023) and _INTERLEAVED (:3186-3283):
 * per-head RMSNorm of q (into q_out) and k, RoPE, KV store. */
void or_qk_norm_rope_store(const float* q, const float* k, const float* v, const float* qw, const float* kw,
                           float* q_out, float* kc, float* vc, int heads, int kv_heads, int hd, int max_ctx,
                           int pos, uint32_t theta, float eps, int interleaved) {
  int half = hd / 2;
  int group = heads / kv_heads;
  for (int h = 0; h < heads; h++) {
    const float* qh = q + (size_t)h * hd;
    float inv = head_rms_inv(qh, hd, eps);
    for (int d = 0; d < half; d++) {
      int s0 = interleaved ? 2 * d : d, s1 = interleaved ? 2 * d + 1 : d + half;
      float a0 = qh[s0] * inv, b0 = qh[s1] * inv;
      float a = a0 * qw[s0], b = b0 * qw[s1];
      float ang = rope_angle(theta, (uint32_t)d, (uint32_t)hd, (uint32_t)pos);
      rope_pair(a, b, ang, &q_out[h * hd + s0], &q_out[h * hd + s1]);
    }
    if (h % group != 0) continue;
    int kvh = h / group;
    const float* kh = k + (size_t)kvh * hd;
    float kinv = head_rms_inv(kh, hd, eps);
    size_t cb = ((size_t)kvh * max_ctx + pos) * hd;
    for (int d = 0; d < half; d++) {
      int s0 = interleaved ? 2 * d : d, s1 = interleaved ? 2 * d + 1 : d + half;
      float a0 = kh[s0] * kinv, b0 = kh[s1] * kinv;
      float a = a0 * kw[s0], b = b0 * kw[s1];
      float ang = rope_angle(theta, (uint32_t)d, (uint32_t)hd, (uint32_t)pos);
      rope_pair(a, b, ang, &kc[cb + s0], &kc[cb + s1]);
    }
    for (int d = 0; d < hd; d++) vc[cb + d] = v[kvh * hd + d];
  }
}

/* ATTENTION_SCORE_WGSL (:3385-3437) + ATTENTION_VALUE_WGSL (:3439-3490).
 * window start: pos+1-window when window != 0 and pos+1 > window (:3405). */
void or_attention(const float* q, const float* kc, const float* vc, float* out, float* scores, int heads,
                  int kv_heads, int hd, int max_ctx, int pos, int window, float attn_scale, int mode) {
  int group = heads / kv_heads;
  uint32_t start = (window != 0 && (uint32_t)pos + 1u > (uint32_t)window) ? (uint32_t)pos + 1u - (uint32_t)window : 0u;
  /* heads are independent (each owns its row of `scores`) */
#pragma omp parallel for schedule(static)
  for (int h = 0; h < heads; h++) {
    int kvh = h / group;
    for (uint32_t t = start; t <= (uint32_t)pos; t++) {
      const float* kr = kc + ((size_t)kvh * max_ctx + t) * hd;
      float s;
      if (mode == OR_MODE_F64) {
        double acc = 0.0;
        for (int d = 0; d < hd; d++) acc += (double)q[h * hd + d] * (double)kr[d];
        s = (float)acc;
      } else {
        float partial[256];
        for (int d = 0; d < 256; d++) partial[d] = d < hd ? q[h * hd + d] * kr[d] : 0.0f;
        for (int stride = 128; stride >= 1; stride >>= 1)
          for (int d = 0; d < stride; d++) partial[d] = partial[d] + partial[d + stride];
        s = partial[0];
      }
      scores[(size_t)h * max_ctx + t] = s * attn_scale;
    }
    float* sc = scores + (size_t)h * max_ctx;
    float m = -3.402823e38f;
    for (uint32_t t = start; t <= (uint32_t)pos; t++) m = fmaxf(m, sc[t]);
    float den = 0.0f;
    /* sc[t] becomes exp(score - max): the same value for every d below */
    for (uint32_t t = start; t <= (uint32_t)pos; t++) { sc[t] = expf(sc[t] - m); den = den + sc[t]; }
    /* per d the terms are added in position order, as the WGSL loop does;
     * the loops are only nested position-outer for cache locality */
    if (mode == OR_MODE_F64) {
      double acc[256];
      for (int d = 0; d < hd; d++) acc[d] = 0.0;
      for (uint32_t t = start; t <= (uint32_t)pos; t++) {
        const double p = (double)sc[t] / (double)den;
        const float* vr = vc + ((size_t)kvh * max_ctx + t) * hd;
        for (int d = 0; d < hd; d++) acc[d] += p * (double)vr[d];
      }
      for (int d = 0; d < hd; d++) out[h * hd + d] = (float)acc[d];
    } else {
      float acc[256];
      for (int d = 0; d < hd; d++) acc[d] = 0.0f;
      for (uint32_t t = start; t <= (uint32_t)pos; t++) {
        const float p = sc[t] / den;
        const float* vr = vc + ((size_t)kvh * max_ctx + t) * hd;
        for (int d = 0; d < hd; d++) {
          float pv = p * vr[d];
          acc[d] = acc[d] + pv;
        }
      }
      for (int d = 0; d < hd; d++) out[h * hd + d] = acc[d];
    }
  }
}

/* SILU_MUL_WGSL :3529-3547 */
void or_silu_mul(const float* g, const float* u, float* out, int n) {
  for (int i = 0; i < n; i++) { float s = g[i] / (1.0f + expf(-g[i])); out[i] = s * u[i]; }
}

/* gelu_tanh :3578-3590 (NaN -> 0, |x| > 10 shortcuts) */
static float gelu_tanh(float x) {
  if (x != x) return 0.0f;
  if (x > 10.0f) return x;
  if (x < -10.0f) return 0.0f;
  const float c = 0.7978845608028654f;
  float x3 = 0.044715f * x;
  x3 = x3 * x;
  x3 = x3 * x;
  float inner = c * (x + x3);
  float hx = 0.5f * x;
  return hx * (1.0f + tanhf(inner));
}

void or_gelu_tanh_mul(const float* g, const float* u, float* out, int n) {
  for (int i = 0; i < n; i++) out[i] = gelu_tanh(g[i]) * u[i];
}

/* ADD_WGSL :3492-3508 / ADD_CLAMP_WGSL :3510-3527 */
void or_add(const float* a, float* io, int n, int clamp) {
  for (int i = 0; i < n; i++) {
    float v = a[i] + io[i];
    io[i] = clamp ? fminf(fmaxf(v, -65000.0f), 65000.0f) : v;
  }
}

/* `better` of ARGMAX_STAGE1/2 (:3665-3673): NaN never wins, ties -> lower index. */
static int better(float v, uint32_t i, float bv, uint32_t bi) {
  if (v != v) return 0;
  if (bv != bv) return 1;
  return (v > bv) || (v == bv && i < bi);
}

/* ARGMAX_STAGE1_WGSL (:3645-3726): per-256 chunk (value, index) after the
 * repetition penalty; the penalty is passed as Math.round(p*1000) (:1661). */
void or_argmax_stage1(const float* logits, int vocab, const uint32_t* penalty_ids, int penalty_count,
                      uint32_t penalty_milli, float* cand_val, uint32_t* cand_idx) {
  int groups = (vocab + 255) / 256;
  float penalty = (float)penalty_milli / 1000.0f;
  for (int g = 0; g < groups; g++) {
    float vals[256];
    uint32_t idx[256];
    for (int l = 0; l < 256; l++) {
      uint32_t i = (uint32_t)g * 256u + (uint32_t)l;
      if (i < (uint32_t)vocab) {
        float v = logits[i];
        if (penalty_count > 0) {
          int hit = 0;
          for (int j = 0; j < penalty_count; j++) if (penalty_ids[j] == i) { hit = 1; break; }
          if (hit) v = v > 0.0f ? v / penalty : v * penalty;
        }
        vals[l] = v;
        idx[l] = i;
      } else {
        vals[l] = -3.402823e38f;
        idx[l] = 0xffffffffu;
      }
    }
    for (int stride = 128; stride >= 1; stride >>= 1)
      for (int l = 0; l < stride; l++)
        if (better(vals[l + stride], idx[l + stride], vals[l], idx[l])) { vals[l] = vals[l + stride]; idx[l] = idx[l + stride]; }
    cand_val[g] = vals[0];
    cand_idx[g] = idx[0];
  }
}

/* ARGMAX_STAGE2_WGSL (:3728-3791) */
uint32_t or_argmax_stage2(const float* cand_val, const uint32_t* cand_idx, int groups) {
  float vals[256];
  uint32_t idx[256];
  for (int l = 0; l < 256; l++) {
    float bv = -3.402823e38f;
    uint32_t bi = 0xffffffffu;
    for (int i = l; i < groups; i += 256)
      if (better(cand_val[i], cand_idx[i], bv, bi)) { bv = cand_val[i]; bi = cand_idx[i]; }
    vals[l] = bv;
    idx[l] = bi;
  }
  for (int stride = 128; stride >= 1; stride >>= 1)
    for (int l = 0; l < stride; l++)
      if (better(vals[l + stride], idx[l + stride], vals[l], idx[l])) { vals[l] = vals[l + stride]; idx[l] = idx[l + stride]; }
  return idx[0];
}

/* ------------------------------------------------------------------------ */
/* Whole-step restatement of LlamaWgslEngine.runToken (:1025-1150).          */

typedef struct {
  int type; int k; int n; const uint8_t* data;
} or_weight;

typedef struct {
  const float *input_norm, *post_norm, *pre_ffn_norm, *post_ffn_norm, *q_norm, *k_norm;
  or_weight q, k, v, o, gate, up, down;
  int rope_theta;        /* Math.round(layer theta) (:1477) */
  int window;            /* 0 = full attention (:1548-1559) */
} or_layer;

typedef struct {
  int hidden, intermediate, vocab, layers, heads, kv_heads, head_dim;
  int context_length;
  float norm_eps, qk_norm_eps, embedding_scale, attn_scale;
  int is_gemma3;         /* architecture == "gemma3" (:1044) */
  int interleaved_rope;  /* ropeLayout == "interleaved" (:402) */
  int qk_norm;           /* q/k norm tensors present (:399) */
  int mode;              /* OR_MODE_WGSL / OR_MODE_F64 */
} or_cfg;

typedef struct {
  or_cfg c;
  or_weight embed, lm_head;
  const float* final_norm;
  or_layer* layers;
  float **kcache, **vcache;
  float *hA, *hB, *hC, *norm, *q, *qn, *k, *v, *attn, *gate, *up, *ff, *logits, *scores;
  float* cand_val;
  uint32_t* cand_idx;
  int pos;
} or_engine;

or_engine* or_create(const or_cfg* c) {
  or_engine* e = (or_engine*)calloc(1, sizeof(or_engine));
  e->c = *c;
  e->layers = (or_layer*)calloc((size_t)c->layers, sizeof(or_layer));
  e->kcache = (float**)calloc((size_t)c->layers, sizeof(float*));
  e->vcache = (float**)calloc((size_t)c->layers, sizeof(float*));
  size_t kv = (size_t)c->kv_heads * c->head_dim * c->context_length;
  for (int i = 0; i < c->layers; i++) {
    e->kcache[i] = (float*)calloc(kv, sizeof(float));
    e->vcache[i] = (float*)calloc(kv, sizeof(float));
  }
  int qd = c->heads * c->head_dim, kvd = c->kv_heads * c->head_dim;
  e->hA = calloc((size_t)c->hidden, 4); e->hB = calloc((size_t)c->hidden, 4); e->hC = calloc((size_t)c->hidden, 4);
  e->norm = calloc((size_t)c->hidden, 4);
  e->q = calloc((size_t)qd, 4); e->qn = calloc((size_t)qd, 4); e->attn = calloc((size_t)qd, 4);
  e->k = calloc((size_t)kvd, 4); e->v = calloc((size_t)kvd, 4);
  e->gate = calloc((size_t)c->intermediate, 4); e->up = calloc((size_t)c->intermediate, 4);
  e->ff = calloc((size_t)c->intermediate, 4);
  e->logits = calloc((size_t)c->vocab, 4);
  e->scores = calloc((size_t)c->heads * c->context_length, 4);
  int groups = (c->vocab + 255) / 256;
  e->cand_val = calloc((size_t)groups, 4);
  e->cand_idx = calloc((size_t)groups, 4);
  return e;
}

void or_set_embedding(or_engine* e, int type, const uint8_t* data) {
  e->embed.type = type; e->embed.k = e->c.hidden; e->embed.n = e->c.vocab; e->embed.data = data;
}
void or_set_lm_head(or_engine* e, int type, const uint8_t* data) {
  e->lm_head.type = type; e->lm_head.k = e->c.hidden; e->lm_head.n = e->c.vocab; e->lm_head.data = data;
}
void or_set_final_norm(or_engine* e, const float* w) { e->final_norm = w; }

/* slot: 0 q 1 k 2 v 3 o 4 gate 5 up 6 down */
void or_set_layer_weight(or_engine* e, int layer, int slot, int type, int k, int n, const uint8_t* data) {
  or_layer* L = &e->layers[layer];
  or_weight* w = slot == 0 ? &L->q : slot == 1 ? &L->k : slot == 2 ? &L->v : slot == 3 ? &L->o
               : slot == 4 ? &L->gate : slot == 5 ? &L->up : &L->down;
  w->type = type; w->k = k; w->n = n; w->data = data;
}
/* slot: 0 input 1 post_attn 2 pre_ffn 3 post_ffn 4 q_norm 5 k_norm */
void or_set_layer_norm(or_engine* e, int layer, int slot, const float* w) {
  or_layer* L = &e->layers[layer];
  switch (slot) {
    case 0: L->input_norm = w; break;
    case 1: L->post_norm = w; break;
    case 2: L->pre_ffn_norm = w; break;
    case 3: L->post_ffn_norm = w; break;
    case 4: L->q_norm = w; break;
    case 5: L->k_norm = w; break;
  }
}
void or_set_layer_rope(or_engine* e, int layer, int theta, int window) {
  e->layers[layer].rope_theta = theta;
  e->layers[layer].window = window;
}

void or_reset(or_engine* e) {
  e->pos = 0;
  size_t kv = (size_t)e->c.kv_heads * e->c.head_dim * e->c.context_length;
  for (int i = 0; i < e->c.layers; i++) {
    memset(e->kcache[i], 0, kv * 4);
    memset(e->vcache[i], 0, kv * 4);
  }
}
int or_position(or_engine* e) { return e->pos; }
void or_set_position(or_engine* e, int pos) { e->pos = pos; }
const float* or_logits(or_engine* e) { return e->logits; }
const float* or_hidden(or_engine* e) { return e->hA; }

static void mv(or_engine* e, const float* x, const or_weight* w, float* y) {
  or_matvec(w->type, w->data, w->k, w->n, x, y, e->c.mode);
}

/* One token.  Returns the greedy argmax id (stage 2) when need_logits, else 0;
 * stage-1 candidates are left in cand_val/cand_idx.  Returns -1 when the
 * context is exhausted (:1030-1033). */
int64_t or_run_token(or_engine* e, uint32_t token, int need_logits, const uint32_t* penalty_ids, int penalty_count,
                     uint32_t penalty_milli) {
  const or_cfg* c = &e->c;
  if (e->pos >= c->context_length) return -1;
  int H = c->hidden;
  or_embedding(e->embed.type, e->embed.data, H, token, c->embedding_scale, e->hA);
  float* residual = e->hA;
  float* other = e->hB;
  for (int li = 0; li < c->layers; li++) {
    or_layer* L = &e->layers[li];
    float* kc = e->kcache[li];
    float* vc = e->vcache[li];
    if (c->is_gemma3) {                                        /* :1044-1067 */
      or_rms_norm(residual, L->input_norm, e->norm, H, c->norm_eps);
      mv(e, e->norm, &L->q, e->q);
      mv(e, e->norm, &L->k, e->k);
      mv(e, e->norm, &L->v, e->v);
      or_qk_norm_rope_store(e->q, e->k, e->v, L->q_norm, L->k_norm, e->qn, kc, vc, c->heads, c->kv_heads,
                            c->head_dim, c->context_length, e->pos, (uint32_t)L->rope_theta, c->qk_norm_eps,
                            c->interleaved_rope);
      or_attention(e->qn, kc, vc, e->attn, e->scores, c->heads, c->kv_heads, c->head_dim, c->context_length,
                   e->pos, L->window, c->attn_scale, c->mode);
      mv(e, e->attn, &L->o, e->hB);
      or_rms_norm(e->hB, L->post_norm, e->hC, H, c->norm_eps);
      or_add(residual, e->hC, H, 1);
      residual = e->hC;
      or_rms_norm(residual, L->pre_ffn_norm, e->norm, H, c->norm_eps);
      mv(e, e->norm, &L->gate, e->gate);
      mv(e, e->norm, &L->up, e->up);
      or_gelu_tanh_mul(e->gate, e->up, e->ff, L->gate.n);
      mv(e, e->ff, &L->down, e->hB);
      or_rms_norm(e->hB, L->post_ffn_norm, e->hA, H, c->norm_eps);
      or_add(residual, e->hA, H, 1);
      residual = e->hA;
      other = e->hB;
    } else {                                                   /* :1068-1103 */
      or_rms_norm(residual, L->input_norm, e->norm, H, c->norm_eps);
      mv(e, e->norm, &L->q, e->q);
      mv(e, e->norm, &L->k, e->k);
      mv(e, e->norm, &L->v, e->v);
      const float* qa;
      if (L->q_norm && L->k_norm) {
        or_qk_norm_rope_store(e->q, e->k, e->v, L->q_norm, L->k_norm, e->qn, kc, vc, c->heads, c->kv_heads,
                              c->head_dim, c->context_length, e->pos, (uint32_t)L->rope_theta, c->qk_norm_eps,
                              c->interleaved_rope);
        qa = e->qn;
      } else {
        or_rope_store(e->q, e->k, e->v, kc, vc, c->heads, c->kv_heads, c->head_dim, c->context_length, e->pos,
                      (uint32_t)L->rope_theta, c->interleaved_rope);
        qa = e->q;
      }
      or_attention(qa, kc, vc, e->attn, e->scores, c->heads, c->kv_heads, c->head_dim, c->context_length,
                   e->pos, L->window, c->attn_scale, c->mode);
      mv(e, e->attn, &L->o, other);
      or_add_rms_norm(residual, other, L->post_norm, e->norm, H, c->norm_eps);
      { float* t = residual; residual = other; other = t; }
      mv(e, e->norm, &L->gate, e->gate);
      mv(e, e->norm, &L->up, e->up);
      or_silu_mul(e->gate, e->up, e->ff, L->gate.n);
      mv(e, e->ff, &L->down, other);
      or_add(residual, other, H, 0);
      { float* t = residual; residual = other; other = t; }
    }
  }
  int64_t best = 0;
  if (need_logits) {                                           /* :1106-1124 */
    or_rms_norm(residual, e->final_norm, e->norm, H, c->norm_eps);
    mv(e, e->norm, &e->lm_head, e->logits);
    or_argmax_stage1(e->logits, c->vocab, penalty_ids, penalty_count, penalty_milli, e->cand_val, e->cand_idx);
    best = or_argmax_stage2(e->cand_val, e->cand_idx, (c->vocab + 255) / 256);
  }
  if (residual != e->hA) memcpy(e->hA, residual, (size_t)H * 4);
  e->pos += 1;
  return best;
}

const float* or_cand_val(or_engine* e) { return e->cand_val; }
const uint32_t* or_cand_idx(or_engine* e) { return e->cand_idx; }
const float* or_kcache(or_engine* e, int layer) { return e->kcache[layer]; }
const float* or_vcache(or_engine* e, int layer) { return e->vcache[layer]; }

void or_destroy(or_engine* e) {
  if (!e) return;
  for (int i = 0; i < e->c.layers; i++) { free(e->kcache[i]); free(e->vcache[i]); }
  free(e->kcache); free(e->vcache); free(e->layers);
  free(e->hA); free(e->hB); free(e->hC); free(e->norm); free(e->q); free(e->qn); free(e->attn);
  free(e->k); free(e->v); free(e->gate); free(e->up); free(e->ff); free(e->logits); free(e->scores);
  free(e->cand_val); free(e->cand_idx);
  free(e);
}
