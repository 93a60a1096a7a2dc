// Decode-step phases for the B200 engine.
//
// One token of LlamaWgslEngine.runToken (llama-wgsl-runtime.ts:1025-1150) is a
// list of phases.  Each phase is a device function over (cta, ncta) so the
// same code runs either as one kernel launch per phase (CUDA-graph mode) or
// inside one persistent cooperative kernel with a grid barrier between phases
// (megakernel mode).  The reference's ~14 dispatches per layer become 5
// phases: the elementwise shaders (RMSNorm, SiLU/GeLU-mul, residual add and
// clamp, QK-norm + RoPE + KV store, embedding) are folded into the
// prologue/epilogue of the matvec or attention phase that consumes them.
#pragma once
#include <cuda_fp16.h>
#include <math.h>
#include <stdint.h>

#include "ck_layout.cuh"

#define CK_THREADS 256
#define CK_WARPS 8
#define CK_KMAX 3072          // longest matvec input (x) handled (3 units per lane)
#define CK_GMAX 8             // q heads per kv head handled by one attention unit
#define CK_HDMAX 256          // head_dim handled
#define CK_SAMPLE_MAX 1024    // ARGMAX_STAGE1 candidates handled by the sampler
#define CK_MIN_SPLIT 32       // positions per attention split (lower bound)

// device error bits (CkState::err)
#define CK_DERR_TOKEN 1
#define CK_DERR_BARRIER 2
#define CK_DERR_SAMPLE 4

struct CkState {
  int pos;                  // position the next token is written to
  int err;                  // sticky CK_DERR_* bits
  uint32_t next_token;      // argmax / sampled id of the last logits step
  uint32_t draw;            // Philox draw index of the next sampled token
  int abort_flag;           // megakernel: a barrier gave up
  uint32_t bar;             // megakernel barrier arrivals (reset per launch)
  // sampling options (sampling.ts) -- written by the host per call; doubles
  // because the reference's options are JS numbers
  double temperature;
  double top_p;
  double pen_d;             // repetition penalty as given (CPU re-penalty, sampling.ts:35-43)
  int top_k;
  uint32_t pen_milli;       // Math.round(penalty*1000) (llama-wgsl-runtime.ts:1661)
  int pen_src;              // 0: history tokens[0..pos], 1: explicit list
  int pen_count;            // explicit list length
  int sampling;             // needsSamplingReadback (sampling.ts:9-16)
  int chain;                // write next_token into tokens[pos+1]
  int pad0;
  unsigned long long seed;  // Philox key
};

struct CkDev {
  CkState* st;
  uint32_t* tokens;         // [ctx] token at each position
  uint32_t* pen_list;       // [ctx] explicit penalty ids
  uint32_t* pen_mask;       // [ceil(vocab/32)] bit set of penalized ids
  float* logits;            // [vocab]
  float* cand_val;          // [ceil(vocab/256)]
  uint32_t* cand_idx;
  int vocab;
  int ctx;
};

enum { PRO_COPY = 0, PRO_NORM = 1, PRO_SILU = 2, PRO_GELU = 3, PRO_GEMMA = 4 };
enum { PH_EMBED = 0, PH_MATVEC = 1, PH_ATTN = 2, PH_ARGMAX1 = 3, PH_ARGMAX2 = 4, PH_SAMPLE = 5, PH_FINISH = 6 };

struct Pro {
  int kind;
  const float* a;           // NORM/COPY: source; SILU/GELU: gate; GEMMA: sub-layer output
  const float* b;           // SILU/GELU: up
  const float* w0;          // NORM: weight; GEMMA: weight of the following pre-norm
  const float* w1;          // GEMMA: post-norm weight of the sub-layer output
  const float* rin;         // GEMMA: residual in
  float* rout;              // GEMMA: residual out (written by CTA 0)
  float eps;
};

struct MvSeg {
  const uint8_t* w;
  float* out;
  const float* add;         // y = add + W x when non-null (residual epilogue)
  Lay L;
  int n;
};

struct MvPhase {
  Pro pro;
  int k;
  int nseg;
  MvSeg seg[3];
};

struct AttnPhase {
  const float *q, *k, *v;   // raw projections
  const float *qw, *kw;     // QK-norm weights (null when the model has none)
  void *kc, *vc;            // this layer's cache [kv_head][ctx][head_dim]
  float* out;               // [heads * head_dim]
  float* part;              // split partials [kvh][smax][G][hd + 2]
  unsigned* counter;        // [kvh] finished splits (last CTA merges, resets)
  int heads, kvh, hd, ctx, window, interleaved, kv_f32, smax;
  uint32_t theta;
  float eps, scale;
};

struct EmbedPhase {
  const uint8_t* w;
  Lay L;
  float* out;
  float scale;
  int need_logits;
};

struct Phase {
  int kind;
  int grid;                 // CTAs for a standalone launch
  union {
    MvPhase mv;
    AttnPhase at;
    EmbedPhase em;
    int need_logits;        // PH_FINISH
  };
};

// ---------------------------------------------------------------------------
struct SmemMv {
  float xf[CK_KMAX];
  int8_t xh[CK_KMAX];
  int8_t xl[CK_KMAX];
  float sx[CK_KMAX / 32];
  int s16[CK_KMAX / 16];
  float red[CK_WARPS * 2];
};
struct SmemAt {
  float qs[CK_GMAX * CK_HDMAX];
  float wacc[CK_WARPS * 1024];
  float wm[CK_WARPS * CK_GMAX];
  float wl[CK_WARPS * CK_GMAX];
  float inv[CK_GMAX + 1];
  int last;
};
struct SmemSm {
  double val[CK_SAMPLE_MAX];
  uint32_t idx[CK_SAMPLE_MAX];
  double prob[CK_SAMPLE_MAX];
  int n;
};
union Smem {
  SmemMv mv;
  SmemAt at;
  SmemSm sm;
};

// ---------------------------------------------------------------------------
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Sum over the CTA; `red` needs CK_WARPS floats.  All threads get the result.
__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int i = 0; i < CK_WARPS; i++) t += red[i];
  return t;
}

__device__ __forceinline__ float rms_inv(float ss, int n, float eps) {
  return 1.0f / sqrtf(ss / (float)n + eps);
}

// gelu_tanh of GELU_TANH_MUL_WGSL (llama-wgsl-runtime.ts:3578-3590)
__device__ __forceinline__ float gelu_tanh(float x) {
  if (x != x) return 0.f;
  if (x > 10.f) return x;
  if (x < -10.f) return 0.f;
  const float c = 0.7978845608028654f;
  return 0.5f * x * (1.0f + tanhf(c * (x + 0.044715f * x * x * x)));
}

// Build the matvec input x (fp32) in shared memory.  Mirrors, per kind:
//   NORM  RMS_NORM_WGSL (:1910-1949)        out = (in * inv) * w
//   COPY  the attention output feeding o_proj
//   SILU  SILU_MUL_WGSL (:3529-3547)        (g / (1 + exp(-g))) * u
//   GELU  GELU_TANH_MUL_WGSL (:3568-3599)
//   GEMMA rmsNorm(post) -> ADD_CLAMP (:3510-3527) -> rmsNorm(pre), the gemma3
//         sandwich of runToken (:1050-1064); CTA 0 stores the new residual.
__device__ void build_x(const Pro& p, int k, SmemMv& s, int cta) {
  const int tid = threadIdx.x;
  float* xf = s.xf;
  if (p.kind == PRO_COPY) {
    for (int i = tid; i < k; i += CK_THREADS) xf[i] = p.a[i];
  } else if (p.kind == PRO_NORM) {
    float ss = 0.f;
    for (int i = tid; i < k; i += CK_THREADS) {
      float v = p.a[i];
      xf[i] = v;
      ss += v * v;
    }
    float inv = rms_inv(block_sum(ss, s.red), k, p.eps);
    for (int i = tid; i < k; i += CK_THREADS) xf[i] = (xf[i] * inv) * p.w0[i];
  } else if (p.kind == PRO_SILU) {
    for (int i = tid; i < k; i += CK_THREADS) {
      float g = p.a[i];
      xf[i] = (g / (1.0f + expf(-g))) * p.b[i];
    }
  } else if (p.kind == PRO_GELU) {
    for (int i = tid; i < k; i += CK_THREADS) xf[i] = gelu_tanh(p.a[i]) * p.b[i];
  } else {  // PRO_GEMMA
    float ss = 0.f;
    for (int i = tid; i < k; i += CK_THREADS) {
      float v = p.a[i];
      xf[i] = v;
      ss += v * v;
    }
    float inv = rms_inv(block_sum(ss, s.red), k, p.eps);
    float ss2 = 0.f;
    for (int i = tid; i < k; i += CK_THREADS) {
      float t = (xf[i] * inv) * p.w1[i];
      float h = fminf(fmaxf(p.rin[i] + t, -65000.0f), 65000.0f);
      xf[i] = h;
      if (cta == 0) p.rout[i] = h;
      ss2 += h * h;
    }
    float inv2 = rms_inv(block_sum(ss2, s.red), k, p.eps);
    for (int i = tid; i < k; i += CK_THREADS) xf[i] = (xf[i] * inv2) * p.w0[i];
  }
  __syncthreads();
}

// Quantize xf per 32-group into X = hi*256 + lo (see XUnit).
__device__ void quant_x(int k, SmemMv& s) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int U = k >> 5;
  for (int g = warp; g < U; g += CK_WARPS) {
    float v = s.xf[32 * g + lane];
    float amax = warp_max(fabsf(v));
    float step = amax / 32639.0f;
    int X = 0;
    if (step > 0.f && amax <= 3.0e38f) {
      X = __float2int_rn(v / step);
      X = max(-32639, min(32639, X));
    }
    int hi = (X + 128) >> 8;
    int lo = X - 256 * hi;
    s.xh[32 * g + lane] = (int8_t)hi;
    s.xl[32 * g + lane] = (int8_t)lo;
    int sum = X;
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (lane == 0) {
      s.sx[g] = (amax <= 3.0e38f) ? step : __int_as_float(0x7fc00000);
      s.s16[2 * g] = sum;
    }
    if (lane == 16) s.s16[2 * g + 1] = sum;
  }
  __syncthreads();
}

__device__ __forceinline__ void load_xunit(const SmemMv& s, int c, XUnit& x) {
  const int* h = (const int*)s.xh;
  const int* l = (const int*)s.xl;
#pragma unroll
  for (int i = 0; i < 8; i++) {
    x.h[i] = h[8 * c + i];
    x.l[i] = l[8 * c + i];
  }
  x.sx = s.sx[c];
  x.sa = s.s16[2 * c];
  x.sb = s.s16[2 * c + 1];
}

// R rows of one segment: all unit loads first (memory-level parallelism), the
// lane's x units from shared memory while they are in flight, then the
// integer dots and one warp reduction per row.
template <int T, int UPL, int R>
__device__ __forceinline__ void mv_group(const MvSeg& S, int row0, const SmemMv& sm, int lane) {
  UnitRaw ur[R][UPL];
  const int U = S.L.U;
#pragma unroll
  for (int r = 0; r < R; r++) {
    int row = row0 + r;
    if (row < S.n) {
      const uint8_t* base = S.w + (size_t)row * S.L.row_bytes;
#pragma unroll
      for (int j = 0; j < UPL; j++) {
        int c = lane + 32 * j;
        if (c < U) load_unit<T>(base, S.L, c, ur[r][j]);
      }
    }
  }
  float acc[R];
#pragma unroll
  for (int r = 0; r < R; r++) acc[r] = 0.f;
#pragma unroll
  for (int j = 0; j < UPL; j++) {
    int c = lane + 32 * j;
    if (c < U) {
      XUnit xu;
      load_xunit(sm, c, xu);
#pragma unroll
      for (int r = 0; r < R; r++)
        if (row0 + r < S.n) acc[r] += unit_dot<T>(ur[r][j], xu, c);
    }
  }
#pragma unroll
  for (int r = 0; r < R; r++) {
    int row = row0 + r;
    float v = warp_sum(acc[r]);
    if (lane == 0 && row < S.n) S.out[row] = S.add ? S.add[row] + v : v;
  }
}

template <int T, int UPL, int R>
__device__ __noinline__ void mv_seg(const MvSeg& S, int first, int ngr, int nw, const SmemMv& sm, int lane) {
  for (int gi = first; gi < ngr; gi += nw) mv_group<T, UPL, R>(S, gi * R, sm, lane);
}

template <int UPL>
__device__ __forceinline__ void mv_run(const MvPhase& P, SmemMv& s, int cta, int ncta) {
  constexpr int R = UPL == 1 ? 4 : (UPL == 2 ? 2 : 1);
  build_x(P.pro, P.k, s, cta);
  quant_x(P.k, s);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  // consecutive row groups go to different CTAs first, spreading every
  // segment over all SMs
  const int gw = warp * ncta + cta, nw = ncta * CK_WARPS;
  int base = 0;
  for (int si = 0; si < P.nseg; si++) {
    const MvSeg& S = P.seg[si];
    const int ngr = (S.n + R - 1) / R;
    int first = (gw - base) % nw;
    if (first < 0) first += nw;
    switch (S.L.type) {
      case GT_Q4_K: mv_seg<GT_Q4_K, UPL, R>(S, first, ngr, nw, s, lane); break;
      case GT_Q6_K: mv_seg<GT_Q6_K, UPL, R>(S, first, ngr, nw, s, lane); break;
      case GT_Q8_0: mv_seg<GT_Q8_0, UPL, R>(S, first, ngr, nw, s, lane); break;
      case GT_Q5_0: mv_seg<GT_Q5_0, UPL, R>(S, first, ngr, nw, s, lane); break;
      case GT_Q5_1: mv_seg<GT_Q5_1, UPL, R>(S, first, ngr, nw, s, lane); break;
    }
    base += ngr;
  }
}

__device__ __forceinline__ void phase_matvec(const MvPhase& P, Smem& sm, int cta, int ncta) {
  int upl = (P.k + 1023) >> 10;
  if (upl <= 1) mv_run<1>(P, sm.mv, cta, ncta);
  else if (upl == 2) mv_run<2>(P, sm.mv, cta, ncta);
  else mv_run<3>(P, sm.mv, cta, ncta);
}

// ---------------------------------------------------------------------------
// Embedding (GGUF_*_EMBEDDING_WGSL, :2615-2866): row tokens[pos] of the
// (tied) table dequantized in WGSL order, times EMBEDDING_SCALE.  Also marks
// the repetition-penalty id set when this step computes logits.
__device__ __forceinline__ void phase_embed(const EmbedPhase& P, const CkDev& D, int cta, int ncta) {
  const CkState* st = D.st;
  int pos = st->pos;
  uint32_t token = D.tokens[pos];
  if (token >= (uint32_t)D.vocab) {
    if (cta == 0 && threadIdx.x == 0) atomicOr(&D.st->err, CK_DERR_TOKEN);
    token = 0;
  }
  const uint8_t* row = P.w + (size_t)token * P.L.row_bytes;
  for (int i = cta * CK_THREADS + threadIdx.x; i < P.L.k; i += ncta * CK_THREADS)
    P.out[i] = __fmul_rn(dequant_at(row, P.L, i), P.scale);
  if (P.need_logits && st->pen_d != 1.0) {
    int cnt = st->pen_src == 0 ? pos + 1 : st->pen_count;
    const uint32_t* ids = st->pen_src == 0 ? D.tokens : D.pen_list;
    for (int j = cta * CK_THREADS + threadIdx.x; j < cnt; j += ncta * CK_THREADS) {
      uint32_t id = ids[j];
      if (id < (uint32_t)D.vocab) atomicOr(&D.pen_mask[id >> 5], 1u << (id & 31));
    }
  }
}

// ---------------------------------------------------------------------------
// Split-K GQA decode attention with the per-head QK-norm, RoPE and KV store
// folded in.  Restates ROPE_STORE(_INTERLEAVED)_WGSL (:2868-2927, :3122-3184),
// QK_NORM_ROPE_STORE(_INTERLEAVED)_WGSL (:2929-3023, :3186-3283),
// ATTENTION_SCORE_WGSL (:3385-3437) and ATTENTION_VALUE_WGSL (:3439-3490):
// scores over [start, pos] with start = pos+1-window for windowed layers,
// scaled by 1/sqrt(head_dim), softmax, weighted sum of V.  The softmax is
// computed online per split and merged by the last split to finish.
__device__ __forceinline__ float rope_angle(uint32_t theta, int d, int hd, int pos) {
  float e = (-2.0f * (float)d) / (float)hd;
  return (float)pos * powf((float)theta, e);
}

// Normalize (optional) + rotate one head of length hd from src into dst
// (shared memory); `inv` is the head's 1/rms (ignored without weights).
__device__ __forceinline__ void rope_head(const float* src, const float* w, float inv, float* dst, int hd, int inter,
                                          uint32_t theta, int pos, int t0, int tstride) {
  int half = hd >> 1;
  for (int d = t0; d < half; d += tstride) {
    int i0 = inter ? 2 * d : d, i1 = inter ? 2 * d + 1 : d + half;
    float a = src[i0], b = src[i1];
    if (w) {
      a = (a * inv) * w[i0];
      b = (b * inv) * w[i1];
    }
    float ang = rope_angle(theta, d, hd, pos);
    float co = cosf(ang), si = sinf(ang);
    dst[i0] = a * co - b * si;
    dst[i1] = a * si + b * co;
  }
}

template <int E>
__device__ __forceinline__ void load_kv(const void* base, int kv_f32, size_t off, float (&f)[E]) {
  if (kv_f32) {
    const float* p = (const float*)base + off;
#pragma unroll
    for (int e = 0; e < E; e += 2) {
      float2 v = *(const float2*)(p + e);
      f[e] = v.x;
      f[e + 1] = v.y;
    }
  } else {
    const __half* p = (const __half*)base + off;
    if (E == 8) {
      uint4 v = *(const uint4*)p;
      const __half2* h = (const __half2*)&v;
#pragma unroll
      for (int e = 0; e < 4; e++) { float2 t = __half22float2(h[e]); f[2 * e] = t.x; f[2 * e + 1] = t.y; }
    } else if (E == 4) {
      uint2 v = *(const uint2*)p;
      const __half2* h = (const __half2*)&v;
#pragma unroll
      for (int e = 0; e < 2; e++) { float2 t = __half22float2(h[e]); f[2 * e] = t.x; f[2 * e + 1] = t.y; }
    } else {
      float2 t = __half22float2(*(const __half2*)p);
      f[0] = t.x;
      f[1] = t.y;
    }
  }
}

template <int E, int GM>
__device__ __forceinline__ void attn_unit(const AttnPhase& P, SmemAt& s, int kvh, int split, int pos) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int hd = P.hd, G = P.heads / P.kvh;
  const int start = (P.window != 0 && pos + 1 > P.window) ? pos + 1 - P.window : 0;
  const int npos = pos - start + 1;
  int chunk = (npos + P.smax - 1) / P.smax;
  if (chunk < CK_MIN_SPLIT) chunk = CK_MIN_SPLIT;
  const int S = (npos + chunk - 1) / chunk;
  if (split >= S) return;
  const int t0 = start + split * chunk;
  const int t1 = min(t0 + chunk, pos + 1);
  const bool owner = split == S - 1;   // the split holding `pos` stores K/V there

  // --- per-head 1/rms of q (and k) for the QK-norm -----------------------
  if (P.qw) {
    for (int g = warp; g < G + (owner ? 1 : 0); g += CK_WARPS) {
      const float* src = g < G ? P.q + (size_t)(kvh * G + g) * hd : P.k + (size_t)kvh * hd;
      float ss = 0.f;
      for (int d = lane; d < hd; d += 32) ss += src[d] * src[d];
      ss = warp_sum(ss);
      if (lane == 0) s.inv[g] = rms_inv(ss, hd, P.eps);
    }
  }
  __syncthreads();
  // --- q: norm + rope into shared memory; owner: k/v into the cache --------
  for (int g = 0; g < G; g++)
    rope_head(P.q + (size_t)(kvh * G + g) * hd, P.qw, P.qw ? s.inv[g] : 1.f, s.qs + g * hd, hd, P.interleaved,
              P.theta, pos, tid, CK_THREADS);
  if (owner) {
    float* kst = s.wacc;  // scratch for the rotated k row
    rope_head(P.k + (size_t)kvh * hd, P.kw, P.kw ? s.inv[G] : 1.f, kst, hd, P.interleaved, P.theta, pos, tid,
              CK_THREADS);
    __syncthreads();
    size_t cb = ((size_t)kvh * P.ctx + pos) * hd;
    for (int d = tid; d < hd; d += CK_THREADS) {
      float kv = kst[d], vv = P.v[(size_t)kvh * hd + d];
      if (P.kv_f32) {
        ((float*)P.kc)[cb + d] = kv;
        ((float*)P.vc)[cb + d] = vv;
      } else {
        ((__half*)P.kc)[cb + d] = __float2half_rn(kv);
        ((__half*)P.vc)[cb + d] = __float2half_rn(vv);
      }
    }
  }
  __syncthreads();

  // --- online softmax over this split's positions ---------------------------
  float q[GM][E], acc[GM][E], m[GM], l[GM];
#pragma unroll
  for (int g = 0; g < GM; g++) {
    m[g] = -INFINITY;
    l[g] = 0.f;
#pragma unroll
    for (int e = 0; e < E; e++) {
      q[g][e] = g < G ? s.qs[g * hd + lane * E + e] : 0.f;
      acc[g][e] = 0.f;
    }
  }
  for (int t = t0 + warp; t < t1; t += CK_WARPS) {
    float kf[E], vf[E];
    size_t off = ((size_t)kvh * P.ctx + t) * hd + lane * E;
    load_kv<E>(P.kc, P.kv_f32, off, kf);
    load_kv<E>(P.vc, P.kv_f32, off, vf);
#pragma unroll
    for (int g = 0; g < GM; g++) {
      if (g < G) {
        float d = 0.f;
#pragma unroll
        for (int e = 0; e < E; e++) d += q[g][e] * kf[e];
        float sc = warp_sum(d) * P.scale;
        float mn = fmaxf(m[g], sc);
        float c = expf(m[g] - mn), p = expf(sc - mn);
        l[g] = l[g] * c + p;
#pragma unroll
        for (int e = 0; e < E; e++) acc[g][e] = acc[g][e] * c + p * vf[e];
        m[g] = mn;
      }
    }
  }
  // --- merge the warps --------------------------------------------------------
#pragma unroll
  for (int g = 0; g < GM; g++) {
    if (g < G) {
      if (lane == 0) {
        s.wm[warp * CK_GMAX + g] = m[g];
        s.wl[warp * CK_GMAX + g] = l[g];
      }
#pragma unroll
      for (int e = 0; e < E; e++) s.wacc[warp * 1024 + g * hd + lane * E + e] = acc[g][e];
    }
  }
  __syncthreads();
  float* part = P.part + ((size_t)kvh * P.smax + split) * G * (hd + 2);
  for (int i = tid; i < G * hd; i += CK_THREADS) {
    int g = i / hd, d = i % hd;
    float M = -INFINITY;
    for (int w = 0; w < CK_WARPS; w++) M = fmaxf(M, s.wm[w * CK_GMAX + g]);
    float L = 0.f, A = 0.f;
    for (int w = 0; w < CK_WARPS; w++) {
      float wm = s.wm[w * CK_GMAX + g];
      if (wm == -INFINITY) continue;
      float f = expf(wm - M);
      L += s.wl[w * CK_GMAX + g] * f;
      A += s.wacc[w * 1024 + g * hd + d] * f;
    }
    part[g * (hd + 2) + 2 + d] = A;
    if (d == 0) {
      part[g * (hd + 2)] = M;
      part[g * (hd + 2) + 1] = L;
    }
  }
  // --- last split to finish merges all splits --------------------------------
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    unsigned prev = atomicAdd(&P.counter[kvh], 1u);
    s.last = (prev == (unsigned)(S - 1));
  }
  __syncthreads();
  if (!s.last) return;
  __threadfence();
  const float* pk = P.part + (size_t)kvh * P.smax * G * (hd + 2);
  for (int i = tid; i < G * hd; i += CK_THREADS) {
    int g = i / hd, d = i % hd;
    float M = -INFINITY;
    for (int sp = 0; sp < S; sp++) M = fmaxf(M, __ldcg(pk + ((size_t)sp * G + g) * (hd + 2)));
    float L = 0.f, A = 0.f;
    for (int sp = 0; sp < S; sp++) {
      const float* pp = pk + ((size_t)sp * G + g) * (hd + 2);
      float f = expf(__ldcg(pp) - M);
      L += __ldcg(pp + 1) * f;
      A += __ldcg(pp + 2 + d) * f;
    }
    P.out[(size_t)(kvh * G + g) * hd + d] = A / L;
  }
  if (tid == 0) P.counter[kvh] = 0u;
}

// group sizes reachable under the host's G * head_dim <= 1024 limit
template <int E>
__device__ __forceinline__ void attn_dispatch_g(const AttnPhase& P, SmemAt& s, int kvh, int split, int pos) {
  int G = P.heads / P.kvh;
  if (G <= 2) attn_unit<E, 2>(P, s, kvh, split, pos);
  else if (G <= 4 || E == 8) attn_unit<E, 4>(P, s, kvh, split, pos);
  else attn_unit<E, (E == 8 ? 4 : 8)>(P, s, kvh, split, pos);
}

__device__ __forceinline__ void phase_attn(const AttnPhase& P, Smem& sm, const CkDev& D, int cta, int ncta) {
  int pos = D.st->pos;
  int units = P.kvh * P.smax;
  for (int u = cta; u < units; u += ncta) {
    int kvh = u / P.smax, split = u % P.smax;
    if (P.hd == 64) attn_dispatch_g<2>(P, sm.at, kvh, split, pos);
    else if (P.hd == 128) attn_dispatch_g<4>(P, sm.at, kvh, split, pos);
    else attn_dispatch_g<8>(P, sm.at, kvh, split, pos);
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// ARGMAX_STAGE1_WGSL (:3645-3726) / ARGMAX_STAGE2_WGSL (:3728-3791):
// NaN never wins, ties go to the lower index.
__device__ __forceinline__ bool better(float v, uint32_t i, float bv, uint32_t bi) {
  if (v != v) return false;
  if (bv != bv) return true;
  return (v > bv) || (v == bv && i < bi);
}

__device__ __forceinline__ void block_argmax(float& v, uint32_t& i, float* sv, uint32_t* si) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    float ov = __shfl_down_sync(0xffffffffu, v, o);
    uint32_t oi = __shfl_down_sync(0xffffffffu, i, o);
    if (lane + o < 32 && better(ov, oi, v, i)) { v = ov; i = oi; }
  }
  __syncthreads();
  if (lane == 0) { sv[warp] = v; si[warp] = i; }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < CK_WARPS; w++)
      if (better(sv[w], si[w], v, i)) { v = sv[w]; i = si[w]; }
  }
}

__device__ __forceinline__ void phase_argmax1(const CkDev& D, Smem& sm, int cta, int ncta) {
  const CkState* st = D.st;
  const int groups = (D.vocab + 255) / 256;
  const bool pen = st->pen_d > 1.0;
  const float penalty = (float)st->pen_milli / 1000.0f;
  float* sv = sm.mv.red;
  uint32_t* si = (uint32_t*)(sm.mv.red + CK_WARPS);
  for (int g = cta; g < groups; g += ncta) {
    uint32_t i = (uint32_t)g * 256u + threadIdx.x;
    float v;
    uint32_t idx;
    if (i < (uint32_t)D.vocab) {
      v = D.logits[i];
      if (pen && ((D.pen_mask[i >> 5] >> (i & 31)) & 1u)) v = v > 0.f ? v / penalty : v * penalty;
      idx = i;
    } else {
      v = -3.402823e38f;
      idx = 0xffffffffu;
    }
    block_argmax(v, idx, sv, si);
    if (threadIdx.x == 0) {
      D.cand_val[g] = v;
      D.cand_idx[g] = idx;
    }
    __syncthreads();
  }
}

__device__ __forceinline__ void phase_argmax2(const CkDev& D, Smem& sm, int cta) {
  if (cta != 0) return;
  const int groups = (D.vocab + 255) / 256;
  float v = -3.402823e38f;
  uint32_t idx = 0xffffffffu;
  for (int g = threadIdx.x; g < groups; g += CK_THREADS)
    if (better(D.cand_val[g], D.cand_idx[g], v, idx)) { v = D.cand_val[g]; idx = D.cand_idx[g]; }
  block_argmax(v, idx, sm.mv.red, (uint32_t*)(sm.mv.red + CK_WARPS));
  if (threadIdx.x == 0) D.st->next_token = idx;
}

// ---------------------------------------------------------------------------
// Philox4x32-10 (Salmon, Moraes, Dror, Shaw, SC'11) and the 53-bit uniform
// draw that replaces Math.random() (sampling.ts:70).
__device__ __forceinline__ void philox4x32_10(uint32_t c[4], uint32_t k0, uint32_t k1) {
#pragma unroll
  for (int r = 0; r < 10; r++) {
    uint32_t lo0 = 0xD2511F53u * c[0], hi0 = __umulhi(0xD2511F53u, c[0]);
    uint32_t lo1 = 0xCD9E8D57u * c[2], hi1 = __umulhi(0xCD9E8D57u, c[2]);
    uint32_t n0 = hi1 ^ c[1] ^ k0, n2 = hi0 ^ c[3] ^ k1;
    c[0] = n0; c[1] = lo1; c[2] = n2; c[3] = lo0;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
}
__device__ __forceinline__ double philox_uniform(unsigned long long seed, unsigned long long off) {
  uint32_t c[4] = {(uint32_t)off, (uint32_t)(off >> 32), 0u, 0u};
  philox4x32_10(c, (uint32_t)seed, (uint32_t)(seed >> 32));
  return ((double)(c[0] >> 5) * 67108864.0 + (double)(c[1] >> 6)) / 9007199254740992.0;
}

// sampleFromCandidateBuffer (sampling.ts:23-76) on the device: re-penalty of
// seen ids, stable descending sort, top-k, temperature softmax in fp64, top-p
// cutoff at the first cdf >= topP, draw.  Single CTA.
__device__ __forceinline__ void phase_sample(const CkDev& D, Smem& smu, int cta) {
  const CkState* st = D.st;
  if (cta != 0 || !st->sampling) return;
  SmemSm& s = smu.sm;
  const int tid = threadIdx.x;
  const int groups = (D.vocab + 255) / 256;
  const int NP = CK_SAMPLE_MAX;
  const double rp = fmax(st->pen_d, 1e-6);
  for (int i = tid; i < NP; i += CK_THREADS) {
    double v = INFINITY;   // sentinel: sorts last
    uint32_t id = 0xffffffffu;
    if (i < groups) {
      float fv = D.cand_val[i];
      uint32_t ci = D.cand_idx[i];
      if (isfinite(fv) && ci != 0xffffffffu) {
        double dv = (double)fv;
        if (rp != 1.0 && ci < (uint32_t)D.vocab && ((D.pen_mask[ci >> 5] >> (ci & 31)) & 1u))
          dv = dv > 0 ? dv / rp : dv * rp;
        v = -dv;        // ascending sort of -value == descending by value
        id = ci;
      }
    }
    s.val[i] = v;
    s.idx[i] = id;
    s.prob[i] = (double)i;   // original order, the stable tie-break
  }
  __syncthreads();
  // bitonic sort by (val, original order) ascending
  for (int kk = 2; kk <= NP; kk <<= 1) {
    for (int j = kk >> 1; j > 0; j >>= 1) {
      for (int i = tid; i < NP; i += CK_THREADS) {
        int p = i ^ j;
        if (p > i) {
          bool up = (i & kk) == 0;
          double a = s.val[i], b = s.val[p];
          double oa = s.prob[i], ob = s.prob[p];
          bool gt = (a > b) || (a == b && oa > ob);
          if (gt == up) {
            s.val[i] = b; s.val[p] = a;
            s.prob[i] = ob; s.prob[p] = oa;
            uint32_t t = s.idx[i]; s.idx[i] = s.idx[p]; s.idx[p] = t;
          }
        }
      }
      __syncthreads();
    }
  }
  if (tid == 0) {
    int n = 0;
    while (n < NP && s.val[n] != INFINITY) n++;
    int k = st->top_k > 0 ? min(st->top_k, n) : n;
    uint32_t choice = n > 0 ? s.idx[0] : 0u;
    if (st->temperature > 0.0 && k > 0) {
      double T = st->temperature;
      double maxv = -s.val[0];
      double total = 0.0;
      for (int i = 0; i < k; i++) {
        s.prob[i] = exp((-s.val[i] - maxv) / T);
        total += s.prob[i];
      }
      double tp = fmin(fmax(st->top_p, 0.0), 1.0);
      int cutoff = k;
      if (tp < 1.0 && total > 0.0) {
        double cdf = 0.0;
        for (int i = 0; i < k; i++) {
          cdf += s.prob[i] / total;
          if (cdf >= tp) { cutoff = i + 1; break; }
        }
      }
      double st_total = 0.0;
      for (int i = 0; i < cutoff; i++) st_total += s.prob[i];
      double r = philox_uniform(st->seed, st->draw) * st_total;
      choice = s.idx[max(0, cutoff - 1)];
      for (int i = 0; i < cutoff; i++) {
        r -= s.prob[i];
        if (r <= 0) { choice = s.idx[i]; break; }
      }
    }
    D.st->next_token = choice;
  }
}

// End of step: clear the penalty set, chain the produced id, advance pos.
__device__ __forceinline__ void phase_finish(int need_logits, const CkDev& D, int cta) {
  if (cta != 0) return;
  CkState* st = D.st;
  int pos = st->pos;
  if (need_logits && st->pen_d != 1.0) {
    int cnt = st->pen_src == 0 ? pos + 1 : st->pen_count;
    const uint32_t* ids = st->pen_src == 0 ? D.tokens : D.pen_list;
    for (int j = threadIdx.x; j < cnt; j += CK_THREADS) {
      uint32_t id = ids[j];
      if (id < (uint32_t)D.vocab) D.pen_mask[id >> 5] = 0u;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    if (need_logits) {
      if (st->chain && pos + 1 < D.ctx) D.tokens[pos + 1] = st->next_token;
      if (st->sampling) st->draw += 1;
    }
    st->pos = pos + 1;
  }
}

// ---------------------------------------------------------------------------
__device__ __forceinline__ void run_phase(const Phase& p, Smem& sm, const CkDev& D, int cta, int ncta) {
  switch (p.kind) {
    case PH_EMBED: phase_embed(p.em, D, cta, ncta); break;
    case PH_MATVEC: phase_matvec(p.mv, sm, cta, ncta); break;
    case PH_ATTN: phase_attn(p.at, sm, D, cta, ncta); break;
    case PH_ARGMAX1: phase_argmax1(D, sm, cta, ncta); break;
    case PH_ARGMAX2: phase_argmax2(D, sm, cta); break;
    case PH_SAMPLE: phase_sample(D, sm, cta); break;
    case PH_FINISH: phase_finish(p.need_logits, D, cta); break;
  }
}

// One launch per phase (CUDA-graph mode): one kernel per phase kind so each
// gets its own register allocation.
__global__ void __launch_bounds__(CK_THREADS, 2) k_mv(const Phase* __restrict__ ph, CkDev D) {
  __shared__ SmemMv sm;
  const MvPhase& P = ph->mv;
  int upl = (P.k + 1023) >> 10;
  if (upl <= 1) mv_run<1>(P, sm, blockIdx.x, gridDim.x);
  else if (upl == 2) mv_run<2>(P, sm, blockIdx.x, gridDim.x);
  else mv_run<3>(P, sm, blockIdx.x, gridDim.x);
}
__global__ void __launch_bounds__(CK_THREADS, 2) k_attn(const Phase* __restrict__ ph, CkDev D) {
  __shared__ Smem sm;
  phase_attn(ph->at, sm, D, blockIdx.x, gridDim.x);
}
__global__ void __launch_bounds__(CK_THREADS, 2) k_misc(const Phase* __restrict__ ph, CkDev D) {
  __shared__ Smem sm;
  run_phase(*ph, sm, D, blockIdx.x, gridDim.x);
}

__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Grid-wide barrier for the cooperative megakernel.  Bounded: after ~2^21
// polls (seconds) the CTA flags CK_DERR_BARRIER + abort and returns false;
// every other CTA sees the abort flag and returns too.
__device__ bool grid_sync(CkState* st, unsigned target) {
  __shared__ int s_ok;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    atomicAdd(&st->bar, 1u);
    int ok = 1;
    unsigned spins = 0;
    while (ld_acquire_u32(&st->bar) < target) {
      if (*(volatile int*)&st->abort_flag) { ok = 0; break; }
      if (++spins > (1u << 21)) {
        atomicOr(&st->err, CK_DERR_BARRIER);
        atomicExch(&st->abort_flag, 1);
        ok = 0;
        break;
      }
      __nanosleep(64);
    }
    __threadfence();
    s_ok = ok;
  }
  __syncthreads();
  return s_ok != 0;
}

// Whole step in one cooperative launch (megakernel mode).
__global__ void __launch_bounds__(CK_THREADS, 2) k_mega(const Phase* __restrict__ ph, int nph, CkDev D) {
  __shared__ Smem sm;
  unsigned target = 0;
  for (int i = 0; i < nph; i++) {
    run_phase(ph[i], sm, D, blockIdx.x, gridDim.x);
    if (i + 1 < nph) {
      target += gridDim.x;
      if (!grid_sync(D.st, target)) return;
    }
  }
}
