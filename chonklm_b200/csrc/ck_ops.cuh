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

#define CK_THREADS 512
#define CK_WARPS 16
#define CK_KMAX 3072          // longest matvec input (x) handled (3 units per lane)
#define CK_GMAX 8             // q heads per kv head handled by one attention unit
#define CK_HDMAX 256          // head_dim handled
#define CK_SAMPLE_MAX 1024    // ARGMAX_STAGE1 candidates handled by the sampler
#define CK_MIN_SPLIT 32       // positions per attention split (lower bound)
#define CK_TILE_BYTES (64 * 1024)   // one buffer of the weight ring

// device error bits (CkState::err)
#define CK_DERR_TOKEN 1
#define CK_DERR_BARRIER 2
#define CK_DERR_SAMPLE 4

struct CkState {
  int pos;                  // position the next token is written to
  int err;                  // sticky CK_DERR_* bits
  uint32_t next_token;      // argmax / sampled id of the last logits step
  uint32_t epoch;           // steps run since the tagged buffers were cleared (starts at 1)
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
  int pad1;
  unsigned long long seed;  // Philox key
  int exact;                // sampler over the whole vocabulary (see phase_topk_local)
  int pad2;
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
  unsigned long long* trace;  // optional globaltimer stamps (null = off)
  int l2_keep;              // 1: the weights fit L2; stream them evict-last so they stay there
  // exact sampler: per-CTA top-K candidates [cta][CK_SAMPLE_MAX] and counts
  float* xhead;             // the LM head's input, written by PH_FNORM
  float* xval;
  uint32_t* xidx;
  int* xcnt;
  int xgrid;                // CTAs the candidate buffers hold
};

__device__ __forceinline__ unsigned long long gtimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
// Trace layout: k_mega: [phase][2] (CTA 0: phase start / phase end);
// k_mv: [CK_TRACE_MV_BASE + cta * 8 + stage];
// sub-stage stamps of phase i on CTA 0: [CK_TRACE_STAGE_BASE + i * 8 + stage];
// k_mega per CTA: [CK_TRACE_CTA_BASE + cta * 16 + j], j 0..3 end of phases
// 1..4, j 4..7 exit of their barriers, j 8..15 sub-stages of phase 2.
#define CK_TRACE_MV_BASE 4096
#define CK_TRACE_STAGE_BASE (CK_TRACE_MV_BASE + 8 * 1024)
#define CK_TRACE_CTA_BASE (CK_TRACE_STAGE_BASE + 8 * 512)
#define CK_TRACE_SLOTS (CK_TRACE_CTA_BASE + 16 * 1024)
// Sub-stage stamps are SM cycles (clock64): finer than the global timer, and
// only ever differenced within one CTA.
__device__ __forceinline__ void stage_mark(unsigned long long* tp, int stage) {
  if (tp && threadIdx.x == 0) tp[stage] = (unsigned long long)clock64();
}

// ---------------------------------------------------------------------------
// Tagged exchange between phases.  In the megakernel no grid barrier separates
// most phases: every activation one phase hands to the next is stored as a
// 64-bit word, value bits low and tag high, tag = epoch << 10 | producer phase
// index, in one single-copy-atomic store.  A consumer reads exactly the words
// it needs and re-reads any whose tag is not the one it expects.  Every
// phase needs all (attention: its head's) outputs of the phase before it, so
// no producer can overwrite a word another CTA has yet to read: a CTA with no
// rows in a phase skips that phase's reads.  The epoch counts steps (the
// step-end phase advances it), so words of the previous step never match.
// A tag field of 0 in a descriptor means plain floats (standalone matvec).
__device__ __forceinline__ uint32_t want_tag(uint32_t ep, int tag1) {
  return tag1 ? ((ep << 10) | (uint32_t)(tag1 - 1)) : 0u;
}
__device__ __forceinline__ unsigned long long ld_word(const float* base, size_t i, int tag1) {
  if (!tag1) return (unsigned long long)__float_as_uint(base[i]);
  unsigned long long w;
  asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(w) : "l"((const unsigned long long*)base + i) : "memory");
  return w;
}
__device__ __forceinline__ void st_word(float* base, size_t i, float v, int tag1, uint32_t ep) {
  if (!tag1) { base[i] = v; return; }
  const unsigned long long w = ((unsigned long long)want_tag(ep, tag1) << 32) | __float_as_uint(v);
  asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"((unsigned long long*)base + i), "l"(w) : "memory");
}
// The value of word w (element i), re-read until it carries `want`.  Bounded:
// after ~2^22 reads it flags the step (the host reports a device timeout)
// and returns what it has; it also stops once another CTA has given up.
__device__ __forceinline__ float word_value(unsigned long long w, const float* base, size_t i, int tag1,
                                            uint32_t want, int* err, int* abort_flag) {
  if ((uint32_t)(w >> 32) != want) {
    unsigned spins = 0;
    do {
      w = ld_word(base, i, tag1);
      if (++spins > (1u << 22)) {
        atomicOr(err, CK_DERR_BARRIER);
        atomicExch(abort_flag, 1);
        break;
      }
      if ((spins & 255u) == 0 && *(volatile int*)abort_flag) break;
    } while ((uint32_t)(w >> 32) != want);
  }
  return __uint_as_float((uint32_t)w);
}

// Bring a batch of words up to date: every round re-reads all words whose
// tag is not yet want[j], with the reads of the round in flight together, so
// the batch costs one round trip after its last producer's store lands
// (polling the words one after another would cost one each).  reread(j)
// issues the read of word j.  Bounded like word_value.
template <int N, typename Reread>
__device__ __forceinline__ void settle(unsigned long long (&w)[N], const uint32_t (&want)[N], Reread reread,
                                       int* err, int* abort_flag) {
  unsigned spins = 0;
  for (;;) {
    bool stale = false;
#pragma unroll
    for (int j = 0; j < N; j++) stale |= (uint32_t)(w[j] >> 32) != want[j];
    if (!stale) return;
    if (++spins > (1u << 22)) {
      atomicOr(err, CK_DERR_BARRIER);
      atomicExch(abort_flag, 1);
      return;
    }
    if ((spins & 255u) == 0 && *(volatile int*)abort_flag) return;
#pragma unroll
    for (int j = 0; j < N; j++)
      if ((uint32_t)(w[j] >> 32) != want[j]) w[j] = reread(j);
  }
}
__device__ __forceinline__ float word_float(unsigned long long w) { return __uint_as_float((uint32_t)w); }

enum { PRO_COPY = 0, PRO_NORM = 1, PRO_SILU = 2, PRO_GELU = 3, PRO_GEMMA = 4 };
enum { PH_EMBED = 0, PH_MATVEC = 1, PH_ATTN = 2, PH_ARGMAX1 = 3, PH_ARGMAX2 = 4, PH_SAMPLE = 5, PH_FINISH = 6,
       PH_SELECT = 7, PH_FNORM = 8, PH_HEAD = 9 };
// PH_FNORM: the LM head's prologue (final norm) on CTA 0, as plain floats in
// CkDev::xhead.  PH_HEAD: the LM head itself, xhead -> logits, run by the
// streaming matvec kernel (k_gemv) as its own launch, never by a phase kernel.

struct Pro {
  int kind;
  const float* a;           // NORM/COPY: source; SILU/GELU: gate; GEMMA: sub-layer output
  const float* b;           // SILU/GELU: up
  const float* w0;          // NORM: weight; GEMMA: weight of the following pre-norm
  const float* w1;          // GEMMA: post-norm weight of the sub-layer output
  const float* rin;         // GEMMA: residual in
  float* rout;              // GEMMA: residual out (written by CTA 0)
  float eps;
  // tags (below) of a, b, rin as read and of rout as written; 0 = plain floats
  int ta, tb, trin, trout;
};

struct MvSeg {
  const uint8_t* w;
  float* out;
  const float* add;         // y = add + W x when non-null (residual epilogue)
  Lay L;
  int n;
  int per;                  // rows per CTA of the launch this descriptor is for
  int tile_rows;            // rows that fill an empty tile (CK_TILE_BYTES / row_bytes)
  uint32_t soff;            // byte offset of this segment's rows in a packed tile
  int tout, tadd;           // tags of out as written and add as read (0 = plain)
};

enum { EPI_NONE = 0, EPI_SILU = 1, EPI_GELU = 2 };
#define CK_GLU_MAX 256        // rows per CTA a fused gate/up epilogue stages

struct MvPhase {
  Pro pro;
  int k;
  int nseg;
  int packed;               // every CTA's rows of all segments fit one tile
  int epi;                  // EPI_SILU / EPI_GELU: segments 0, 1 are gate, up
  int tglu;                 // tag of glu_out as written
  float* glu_out;           // with epi: act(gate) * up, the down projection's input
  MvSeg seg[3];
};

struct AttnPhase {
  const float *q, *k, *v;   // raw projections
  const float *qw, *kw;     // QK-norm weights (null when the model has none)
  void *kc, *vc;            // this layer's cache [kv_head][ctx][head_dim]
  const float* inv_freq;    // [head_dim/2] theta^(-2d/head_dim) of this layer
  float* out;               // [heads * head_dim]
  float* part;              // split partials [kvh][smax][G][hd + 2], tagged words
  int heads, kvh, hd, ctx, window, interleaved, kv_f32, smax;
  int group;                // q heads per kv head (heads / kvh)
  int tqkv, tout;           // tags of q/k/v as read and of out as written
  uint32_t theta;
  float eps, scale;
};

struct EmbedPhase {
  const uint8_t* w;
  Lay L;
  float* out;
  float scale;
  int need_logits;
  int tout;                 // tag of out as written
};

struct __align__(16) Phase {
  int kind;
  int grid;                 // CTAs for a standalone launch
  int index;                // position in its schedule (trace slots)
  int barrier_after;        // megakernel: grid barrier before the next phase
  union {
    MvPhase mv;
    AttnPhase at;
    EmbedPhase em;
    int need_logits;        // PH_FINISH
  };
};
static_assert(sizeof(Phase) % 16 == 0, "phase descriptors are bulk-copied");

// Host: the row partition of every matvec segment of `p` for a launch of
// `grid` CTAs (CTA c owns rows [c*per, min(n, (c+1)*per))) and the rows that
// fill an empty tile.  Every row fits a tile (rows are <= 3072 weights).
// A phase is packed when a CTA's full share of every segment fits one tile:
// then segment s sits at a fixed offset (the shares before it); otherwise
// each segment is cut into tiles of its own.
inline void set_partition(Phase& p, int grid) {
  if (p.kind != PH_MATVEC) return;
  uint32_t off = 0;
  for (int i = 0; i < p.mv.nseg; i++) {
    MvSeg& s = p.mv.seg[i];
    s.per = (s.n + grid - 1) / grid;
    s.tile_rows = (int)(CK_TILE_BYTES / s.L.row_bytes);
    s.soff = off;
    off += (uint32_t)s.per * s.L.row_bytes;
  }
  p.mv.packed = off <= CK_TILE_BYTES ? 1 : 0;
  if (!p.mv.packed)
    for (int i = 0; i < p.mv.nseg; i++) p.mv.seg[i].soff = 0;
}

// ---------------------------------------------------------------------------
struct SmemMv {
  float xf[CK_KMAX];
  alignas(16) int8_t xh[CK_KMAX];
  int8_t xl[CK_KMAX];
  float sx[CK_KMAX / 32];
  alignas(8) int s16[CK_KMAX / 16];
  float red[CK_WARPS * 2];
  float glu[2][CK_GLU_MAX];        // this CTA's gate and up rows (fused epilogue)
};
struct SmemAt {
  float qs[CK_GMAX * CK_HDMAX];
  float raw[CK_GMAX * CK_HDMAX];   // q rows as produced by the projection
  float kvw[4][CK_HDMAX];          // k, v, q-norm weight, k-norm weight
  float wacc[CK_WARPS * CK_HDMAX];
  float kst[CK_HDMAX];             // the new k row after norm + rope
  float wm[CK_WARPS];
  float wl[CK_WARPS];
  float wf[CK_WARPS];              // each warp's weight exp(m_w - M) in its head's merge
  float hm[CK_GMAX], hl[CK_GMAX];  // per head: merged max and sum of this split
  float2 cs[CK_HDMAX / 2];
  float inv[CK_GMAX + 1];
};
struct SmemSm {
  double val[CK_SAMPLE_MAX];
  uint32_t idx[CK_SAMPLE_MAX];
  double prob[CK_SAMPLE_MAX];
  double dtotal;                   // the sampler's fp64 sum of the k weights
  int n;
  // exact sampler (radix select): histogram, warp counts, running bases,
  // per-CTA list offsets
  int hist[256];
  int cnt[CK_WARPS];
  int base, eqbase, rem, total;
  uint32_t prefix;
  int off[1024];
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
__device__ void build_x(const Pro& p, int k, SmemMv& s, int cta, uint32_t ep, int* err, int* abort_flag) {
  // Every global load of the prologue is issued in one round into registers
  // before anything is stored: interleaving them with the shared-memory
  // stores lets the compiler serialise each load behind the previous store.
  constexpr int PER = CK_KMAX / CK_THREADS;
  const int tid = threadIdx.x;
  const int kind = p.kind;
  float* xf = s.xf;
  float va[PER], vb[PER], vc[PER], vd[PER];
  const bool act = kind == PRO_SILU || kind == PRO_GELU;
  const float* pb = act ? p.b : p.w0;
  const int tb = act ? p.tb : 0, trin = kind == PRO_GEMMA ? p.trin : 0;
  const uint32_t wa = want_tag(ep, p.ta), wb = want_tag(ep, tb), wr = want_tag(ep, trin);
  unsigned long long x[3 * PER];        // a, b, rin words
  uint32_t want[3 * PER];
#pragma unroll
  for (int j = 0; j < PER; j++) {
    const int i = tid + j * CK_THREADS;
    const bool ok = i < k;
    x[j] = ok ? ld_word(p.a, i, p.ta) : ((unsigned long long)wa << 32);
    x[PER + j] = (ok && kind != PRO_COPY) ? ld_word(pb, i, tb) : ((unsigned long long)wb << 32);
    vc[j] = (ok && kind == PRO_GEMMA) ? p.w1[i] : 0.f;
    x[2 * PER + j] = (ok && kind == PRO_GEMMA) ? ld_word(p.rin, i, trin) : ((unsigned long long)wr << 32);
    want[j] = wa;
    want[PER + j] = wb;
    want[2 * PER + j] = wr;
  }
  settle(x, want, [&](int j) {
    const int i = tid + (j % PER) * CK_THREADS;
    return j < PER ? ld_word(p.a, i, p.ta) : j < 2 * PER ? ld_word(pb, i, tb) : ld_word(p.rin, i, trin);
  }, err, abort_flag);
#pragma unroll
  for (int j = 0; j < PER; j++) {
    va[j] = word_float(x[j]);
    vb[j] = word_float(x[PER + j]);
    vd[j] = word_float(x[2 * PER + j]);
  }
  if (kind == PRO_COPY) {
#pragma unroll
    for (int j = 0; j < PER; j++) {
      const int i = tid + j * CK_THREADS;
      if (i < k) xf[i] = va[j];
    }
  } else if (kind == PRO_NORM) {
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < PER; j++) ss += va[j] * va[j];
    const float inv = rms_inv(block_sum(ss, s.red), k, p.eps);
#pragma unroll
    for (int j = 0; j < PER; j++) {
      const int i = tid + j * CK_THREADS;
      if (i < k) xf[i] = (va[j] * inv) * vb[j];
    }
  } else if (kind == PRO_SILU) {
#pragma unroll
    for (int j = 0; j < PER; j++) {
      const int i = tid + j * CK_THREADS;
      const float g = va[j];
      if (i < k) xf[i] = (g / (1.0f + expf(-g))) * vb[j];
    }
  } else if (kind == PRO_GELU) {
#pragma unroll
    for (int j = 0; j < PER; j++) {
      const int i = tid + j * CK_THREADS;
      if (i < k) xf[i] = gelu_tanh(va[j]) * vb[j];
    }
  } else {  // PRO_GEMMA: t = rmsnorm(a) * w1; h = clamp(rin + t); x = rmsnorm(h) * w0
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < PER; j++) ss += va[j] * va[j];
    const float inv = rms_inv(block_sum(ss, s.red), k, p.eps);
    float ss2 = 0.f;
#pragma unroll
    for (int j = 0; j < PER; j++) {
      const int i = tid + j * CK_THREADS;
      const float t = (va[j] * inv) * vc[j];
      const float h = fminf(fmaxf(vd[j] + t, -65000.0f), 65000.0f);
      va[j] = h;
      if (i < k) {
        if (cta == 0) st_word(p.rout, i, h, p.trout, ep);
        ss2 += h * h;
      }
    }
    const float inv2 = rms_inv(block_sum(ss2, s.red), k, p.eps);
#pragma unroll
    for (int j = 0; j < PER; j++) {
      const int i = tid + j * CK_THREADS;
      if (i < k) xf[i] = (va[j] * inv2) * vb[j];
    }
  }
  __syncthreads();
}

// Quantize xf per 32-group into X = hi*256 + lo (see XUnit): half a warp per
// group, two elements per lane, so k <= 3072 takes a single pass.
__device__ void quant_x(int k, SmemMv& s) {
  const int lane = threadIdx.x & 31, half = (threadIdx.x >> 4) & 1, warp = threadIdx.x >> 5;
  const int U = k >> 5;
  const int hl = lane & 15;
  // the loop condition is warp-uniform (shuffles need the whole warp)
  for (int gp = warp; 2 * gp < U; gp += CK_WARPS) {
    const int g = 2 * gp + half;
    const bool ok = g < U;
    float2 v = ok ? *(const float2*)(s.xf + 32 * g + 2 * hl) : make_float2(0.f, 0.f);
    float amax = fmaxf(fabsf(v.x), fabsf(v.y));
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const bool fin = amax <= 3.0e38f;
    const float step = amax * (1.0f / 32639.0f);
    const float inv = (step > 0.f && fin) ? 32639.0f / amax : 0.f;
    int X0 = max(-32639, min(32639, __float2int_rn(v.x * inv)));
    int X1 = max(-32639, min(32639, __float2int_rn(v.y * inv)));
    int h0 = (X0 + 128) >> 8, h1 = (X1 + 128) >> 8;
    int l0 = X0 - 256 * h0, l1 = X1 - 256 * h1;
    int sum = X0 + X1;
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (!ok) continue;
    *(short*)(s.xh + 32 * g + 2 * hl) = (short)((h0 & 0xFF) | (h1 << 8));
    *(short*)(s.xl + 32 * g + 2 * hl) = (short)((l0 & 0xFF) | (l1 << 8));
    // lanes 0..7 hold weights 0..15 of the group, lanes 8..15 weights 16..31
    if (hl == 0) s.sx[g] = fin ? step : __int_as_float(0x7fc00000);
    if (hl == 0) s.s16[2 * g] = sum;
    if (hl == 8) s.s16[2 * g + 1] = sum;
  }
  __syncthreads();
}

// The x unit of column c: two 16-byte shared loads per plane (a scalar load
// per word would be an 8-way bank conflict at the 32-byte unit stride).
__device__ __forceinline__ void load_xunit(const SmemMv& s, int c, XUnit& x) {
  const int4* h = (const int4*)s.xh + 2 * c;
  const int4* l = (const int4*)s.xl + 2 * c;
  const int4 h0 = h[0], h1 = h[1], l0 = l[0], l1 = l[1];
  x.h[0] = h0.x; x.h[1] = h0.y; x.h[2] = h0.z; x.h[3] = h0.w;
  x.h[4] = h1.x; x.h[5] = h1.y; x.h[6] = h1.z; x.h[7] = h1.w;
  x.l[0] = l0.x; x.l[1] = l0.y; x.l[2] = l0.z; x.l[3] = l0.w;
  x.l[4] = l1.x; x.l[5] = l1.y; x.l[6] = l1.z; x.l[7] = l1.w;
  x.sx = s.sx[c];
  const int2 ss = *(const int2*)(s.s16 + 2 * c);
  x.sa = ss.x;
  x.sb = ss.y;
}

// ---------------------------------------------------------------------------
// Weight streaming: each CTA owns a contiguous row range of every matvec
// segment (rows are self-contained and 16-byte aligned in the device layout),
// packed into tiles of at most CK_TILE_BYTES.  One issuer thread copies tiles into a
// two-buffer shared-memory ring with cp.async.bulk (TMA bulk copy into this
// CTA's own shared memory) completing on an mbarrier; the ring runs ahead across phases, so
// the next matvec's weights are in flight while this CTA is in a grid barrier
// or an attention phase.  Consumers read the tile from shared memory.
#define CK_ISSUER (CK_THREADS - 32)   // lane 0 of the last warp copies tiles
// Dynamic shared memory: [tile buffer 0][tile buffer 1][3 mbarriers, 128 B][phase descriptors]
#define CK_DYN_BARS (2 * CK_TILE_BYTES)
#define CK_DYN_PHASES (2 * CK_TILE_BYTES + 128)
#define CK_PHASE_SMEM_MAX (56 * 1024)   // 160 phases of 352 bytes (31 layers)
#define CK_DYN_SMEM_MAX (CK_DYN_PHASES + CK_PHASE_SMEM_MAX)

struct Cursor {
  int phase, seg, row;
};

// Ring state.  The buffers, barriers and staged descriptors sit at fixed
// offsets of the dynamic shared memory (no registers); the issuer's cursor
// lives in shared memory (one thread uses it); every thread keeps the count
// of consumed tiles, which is CTA-uniform.
struct Ring {
  unsigned consumed;       // tiles consumed so far
  int ok;                  // 0 once a wait gave up
};
struct IssueState {
  Cursor issue;            // next row to copy
  unsigned issued;         // tiles copied so far
  int nph;                 // phases staged for this launch
  int keep;                // L2 hint of the weight copies (CkDev::l2_keep)
};
__device__ __forceinline__ uint8_t* dyn_smem() {
  extern __shared__ __align__(128) uint8_t ck_dyn[];
  return ck_dyn;
}
__device__ __forceinline__ uint8_t* ring_buf(unsigned tile) {
  return dyn_smem() + (size_t)(tile & 1) * CK_TILE_BYTES;
}
__device__ __forceinline__ IssueState& issue_state() {
  __shared__ IssueState st;
  return st;
}

// A CTA's tiles of a phase, followed identically by the issuer and the
// consumers: a packed phase is one tile holding the CTA's rows of every
// segment at the segment's fixed offset; otherwise segment by segment in
// tiles of tile_rows rows.  The row partition (CTA c owns rows
// [c*per, min(n, (c+1)*per))) and the tile shapes are precomputed on the host
// for the launch's grid, so the walk has no division and no dependent chain.
__device__ __forceinline__ void seg_range(const MvSeg& S, int cta, int& lo, int& hi) {
  lo = min(S.n, cta * S.per);
  hi = min(S.n, lo + S.per);
}

// The row ranges ("pieces") of one tile, at most one per segment, kept as
// scalars so they stay in registers.  Flat row t of the tile belongs to
// piece (t >= st1) + (t >= st2).
struct TileList {
  int n, total;            // pieces, rows
  int st1, st2;            // first flat row of pieces 1 and 2
  int seg0, seg1, seg2;    // segment of each piece
  int r00, r01, r02;       // first output row of each piece
  uint32_t off0, off1, off2;   // byte offset of each piece in the tile
};
__device__ __forceinline__ int pick3(int p, int a, int b, int c) { return p == 0 ? a : (p == 1 ? b : c); }
__device__ __forceinline__ uint32_t pick3u(int p, uint32_t a, uint32_t b, uint32_t c) {
  return p == 0 ? a : (p == 1 ? b : c);
}
__device__ __forceinline__ void tile_clear(TileList& T) {
  T.n = 0; T.total = 0; T.st1 = T.st2 = 1 << 30;
  T.seg0 = T.seg1 = T.seg2 = 0; T.r00 = T.r01 = T.r02 = 0; T.off0 = T.off1 = T.off2 = 0u;
}
__device__ __forceinline__ void tile_add(TileList& T, int seg, int r0, int rows, uint32_t off) {
  if (T.n == 0) { T.seg0 = seg; T.r00 = r0; T.off0 = off; }
  else if (T.n == 1) { T.seg1 = seg; T.r01 = r0; T.off1 = off; T.st1 = T.total; }
  else { T.seg2 = seg; T.r02 = r0; T.off2 = off; T.st2 = T.total; }
  T.n++;
  T.total += rows;
}

// Next tile of phase m for this CTA from position (seg, row) (seg = 0,
// row = -1 at the start of the phase); false when the phase has no more.
__device__ __forceinline__ bool next_tile(const MvPhase& m, int cta, int& seg, int& row, TileList& T) {
  tile_clear(T);
  if (m.packed) {
    if (seg != 0) return false;
    seg = 1;
#pragma unroll
    for (int i = 0; i < 3; i++) {
      if (i < m.nseg) {
        int lo, hi;
        seg_range(m.seg[i], cta, lo, hi);
        if (hi > lo) tile_add(T, i, lo, hi - lo, m.seg[i].soff);
      }
    }
    return T.total > 0;
  }
  while (seg < m.nseg) {
    const MvSeg& S = m.seg[seg];
    int lo, hi;
    seg_range(S, cta, lo, hi);
    if (row < lo) row = lo;
    if (row >= hi) { seg++; row = -1; continue; }
    const int take = min(S.tile_rows, hi - row);
    tile_add(T, seg, row, take, 0u);
    row += take;
    return true;
  }
  return false;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t* b, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
__device__ __forceinline__ void mbar_expect_tx(uint64_t* b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)), "r"(bytes) : "memory");
}
// expect_tx without an arrival: one per copy of a tile, then one arrive
__device__ __forceinline__ void mbar_expect_tx_only(uint64_t* b, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(b)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* b, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(done)
      : "r"(smem_u32(b)), "r"(parity)
      : "memory");
  return done != 0;
}
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}
// Same, with an L2 cache hint for weights.  By default evict-first: weights
// larger than L2 are read once per token and should not push activations,
// norms or the KV cache out.  keep = 1 (every weight of the model fits L2):
// evict-last, so the next token reads them from L2 instead of HBM.
__device__ __forceinline__ void bulk_g2s_stream(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                                int keep = 0) {
  uint64_t pol;
  if (keep) asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
  else asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(pol)
      : "memory");
}

// Issuer thread: copy the next tile (if any) into buffer issued & 1, one bulk
// copy per piece, each preceded by its expect_tx; the single arrival after
// the last copy lets the barrier's phase complete.
__device__ __forceinline__ void ring_issue(int cta) {
  IssueState& is = issue_state();
  Cursor& c = is.issue;
  const Phase* ph = (const Phase*)(dyn_smem() + CK_DYN_PHASES);
  TileList T;
  while (c.phase < is.nph) {
    const Phase& p = ph[c.phase];
    if (p.kind == PH_MATVEC && next_tile(p.mv, cta, c.seg, c.row, T)) {
      const int b = is.issued & 1;
      uint64_t* bar = (uint64_t*)(dyn_smem() + CK_DYN_BARS) + b;
      uint8_t* dst = ring_buf(b);
      for (int i = 0; i < T.n; i++) {
        const int sg = pick3(i, T.seg0, T.seg1, T.seg2);
        const int r0 = pick3(i, T.r00, T.r01, T.r02);
        const int rows = (i + 1 < T.n ? pick3(i + 1, 0, T.st1, T.st2) : T.total) - pick3(i, 0, T.st1, T.st2);
        const MvSeg& S = p.mv.seg[sg];
        const uint32_t rb = S.L.row_bytes, bytes = (uint32_t)rows * rb;
        mbar_expect_tx_only(bar, bytes);
        bulk_g2s_stream(dst + pick3u(i, T.off0, T.off1, T.off2), S.w + (size_t)r0 * rb, bytes, bar, is.keep);
      }
      mbar_arrive(bar);
      is.issued++;
      return;
    }
    c.phase++; c.seg = 0; c.row = -1;
  }
}

// Shared-memory layout of the streaming kernels (dynamic part):
//   [tile buffer 0][tile buffer 1][3 mbarriers, 128 B][phase descriptors]

// Start of a launch: init the barriers, stage the phase descriptors in shared
// memory with one bulk copy (every later descriptor read is a shared-memory
// read), then put the first two weight tiles in flight.  Returns the staged
// descriptors, or null when the wait gave up.
__device__ __forceinline__ const Phase* launch_start(Ring& R, const Phase* gph, int nph, int cta, int* err, int* abort_flag,
                                                    int keep) {
  uint8_t* dyn = dyn_smem();
  uint64_t* bars = (uint64_t*)(dyn + CK_DYN_BARS);
  Phase* sph = (Phase*)(dyn + CK_DYN_PHASES);
  if (threadIdx.x == 0) {
    mbar_init(bars, 1);
    mbar_init(bars + 1, 1);
    mbar_init(bars + 2, 1);
    mbar_fence_init();
    uint32_t bytes = (uint32_t)(nph * sizeof(Phase));
    mbar_expect_tx(bars + 2, bytes);
    bulk_g2s(sph, gph, bytes, bars + 2);
  }
  if (threadIdx.x == CK_ISSUER) {
    IssueState& is = issue_state();
    is.issue.phase = 0; is.issue.seg = 0; is.issue.row = -1;
    is.issued = 0;
    is.nph = nph;
    is.keep = keep;
  }
  __syncthreads();
  unsigned spins = 0;
  while (!mbar_try_wait(bars + 2, 0)) {
    if (++spins > (1u << 20)) {
      atomicOr(err, CK_DERR_BARRIER);
      atomicExch(abort_flag, 1);
      return nullptr;
    }
  }
  R.consumed = 0;
  R.ok = 1;
  if (threadIdx.x == CK_ISSUER) {
    ring_issue(cta);
    ring_issue(cta);
  }
  return sph;
}

// Wait for tile `consumed` (bounded: ~seconds, then flags and gives up).
__device__ __forceinline__ bool ring_wait(const Ring& R, int* err, int* abort_flag) {
  uint64_t* bar = (uint64_t*)(dyn_smem() + CK_DYN_BARS) + (R.consumed & 1);
  uint32_t par = (R.consumed >> 1) & 1u;
  unsigned spins = 0;
  while (!mbar_try_wait(bar, par)) {
    if (++spins > (1u << 20)) {
      if (err) atomicOr(err, CK_DERR_BARRIER);
      if (abort_flag) atomicExch(abort_flag, 1);
      return false;
    }
    if ((spins & 1023u) == 0 && abort_flag && *(volatile int*)abort_flag) return false;
  }
  return true;
}

// After every thread finished reading tile `consumed`: free its buffer and
// refill it with the tile two ahead.
__device__ __forceinline__ void ring_release(Ring& R, int cta) {
  __syncthreads();
  R.consumed++;
  if (threadIdx.x == CK_ISSUER && issue_state().issued < R.consumed + 2) ring_issue(cta);
}

// Rows of a tile, read from shared memory, as one flat list over the tile's
// pieces so every warp has rows even when each piece is short (a QKV tile
// holds a few rows of each projection).  A warp step covers rows t and
// t + CK_WARPS (ONE) or row t: first every unit of those rows is unpacked
// into registers (step_unpack: needs only the weights), then dotted with x
// (step_dot).  The first step of a phase is unpacked before x exists, under
// the latency of the prologue's loads.  With one unit per lane (ONE, k <= 1024)
// the lane's x unit stays in registers (every segment of a phase has the
// same k); with 2-3 units per lane the x units are read from shared memory
// per unit.  The block type is a runtime switch inside the unpack: compiling
// the row loop per type multiplies register pressure past the budget.
template <bool ONE>
struct MvStep {
  static constexpr int R = ONE ? 2 : 1;        // rows per warp step
  static constexpr int UPL = 1;                // units per lane (ONE steps only)
  U8 u[R][UPL];
  int sg[R], orow[R];
};

template <bool ONE, unsigned TM>
__device__ __forceinline__ void step_unpack(const MvPhase& P, const uint8_t* tb, const TileList& T, int t,
                                            MvStep<ONE>& w) {
  const int lane = threadIdx.x & 31;
  const int U = P.seg[0].L.U;
#pragma unroll
  for (int i = 0; i < MvStep<ONE>::R; i++) {
    const int tt = t + i * CK_WARPS;
    const int pc = (tt >= T.st1) + (tt >= T.st2);
    w.sg[i] = pick3(pc, T.seg0, T.seg1, T.seg2);
    const int local = tt - pick3(pc, 0, T.st1, T.st2);
    w.orow[i] = pick3(pc, T.r00, T.r01, T.r02) + local;
    if (tt < T.total) {
      const MvSeg& S = P.seg[w.sg[i]];
      const uint8_t* row = tb + pick3u(pc, T.off0, T.off1, T.off2) + (uint32_t)local * S.L.row_bytes;
      const int type = S.L.type;
#pragma unroll
      for (int j = 0; j < MvStep<ONE>::UPL; j++) {
        const int c = lane + 32 * j;
        if (c < U) unpack_unit<false, TM>(type, row, S.L, c, w.u[i][j]);
      }
    }
  }
}

// Store one output row: y = add + v, or, with a fused gate/up epilogue, the
// CTA's staging row in shared memory.
__device__ __forceinline__ void mv_store(const MvPhase& P, int sg, int orow, float v, SmemMv& s, int cta,
                                         uint32_t ep, int* err, int* abort_flag) {
  const MvSeg& S = P.seg[sg];
  if (P.epi) {
    s.glu[sg][orow - cta * S.per] = v;
  } else {
    if (S.add) {
      const uint32_t want = want_tag(ep, S.tadd);
      v = word_value(ld_word(S.add, orow, S.tadd), S.add, orow, S.tadd, want, err, abort_flag) + v;
    }
    st_word(S.out, orow, v, S.tout, ep);
  }
}

template <bool ONE>
__device__ __forceinline__ void step_dot(const MvPhase& P, const TileList& T, int t, const MvStep<ONE>& w,
                                         SmemMv& s, const XUnit& x0, float xscale, int cta, uint32_t ep, int* err,
                                         int* abort_flag) {
  constexpr int R = MvStep<ONE>::R;
  const int lane = threadIdx.x & 31;
  const int U = P.seg[0].L.U;
  float acc[R];
#pragma unroll
  for (int i = 0; i < R; i++) {
    acc[i] = 0.f;
    if (t + i * CK_WARPS < T.total) {
#pragma unroll
      for (int j = 0; j < MvStep<ONE>::UPL; j++) {
        const int c = lane + 32 * j;
        if (c < U) {
          if (ONE) {
            acc[i] += unit_dot8(w.u[i][j], x0);
          } else {
            XUnit xj;
            load_xunit(s, c, xj);
            acc[i] += unit_dot8(w.u[i][j], xj);
          }
        }
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
#pragma unroll
    for (int i = 0; i < R; i++) acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], o);
#pragma unroll
  for (int i = 0; i < R; i++) {
    if (lane == i && t + i * CK_WARPS < T.total)
      mv_store(P, w.sg[i], w.orow[i], xscale * acc[i], s, cta, ep, err, abort_flag);
  }
}

// Warp steps t0, t0 + R*CK_WARPS, ... of a tile.  With 2-3 units per lane
// each unit is unpacked and dotted in turn (its x unit read from shared
// memory), which keeps a single unpacked unit live.
template <bool ONE, unsigned TM>
__device__ __forceinline__ void mv_tile(const MvPhase& P, const uint8_t* tb, const TileList& T, int t0,
                                        SmemMv& s, const XUnit& x0, float xscale, int cta, uint32_t ep, int* err,
                                        int* abort_flag) {
  constexpr int R = MvStep<ONE>::R;
  if (ONE) {
    for (int t = t0; t < T.total; t += R * CK_WARPS) {
      MvStep<true> w;
      step_unpack<true, TM>(P, tb, T, t, w);
      step_dot<true>(P, T, t, w, s, x0, xscale, cta, ep, err, abort_flag);
    }
    return;
  }
  const int lane = threadIdx.x & 31;
  const int U = P.seg[0].L.U;
  const int upl = (U + 31) >> 5;
  for (int t = t0; t < T.total; t += CK_WARPS) {
    const int pc = (t >= T.st1) + (t >= T.st2);
    const int sg = pick3(pc, T.seg0, T.seg1, T.seg2);
    const int local = t - pick3(pc, 0, T.st1, T.st2);
    const MvSeg& S = P.seg[sg];
    const uint8_t* row = tb + pick3u(pc, T.off0, T.off1, T.off2) + (uint32_t)local * S.L.row_bytes;
    const int type = S.L.type;
    float acc = 0.f;
#pragma unroll 1
    for (int j = 0; j < upl; j++) {
      const int c = lane + 32 * j;
      if (c < U) {
        U8 u;
        unpack_unit<false, TM>(type, row, S.L, c, u);
        XUnit xj;
        load_xunit(s, c, xj);
        acc += unit_dot8(u, xj);
      }
    }
    acc = warp_sum(acc);
    if (lane == 0) mv_store(P, sg, pick3(pc, T.r00, T.r01, T.r02) + local, xscale * acc, s, cta, ep, err, abort_flag);
  }
}

// Prologue loads (fused path): element 32 g + lane of every group g of this
// warp, issued before anything waits on them.
template <int GPW>
__device__ __forceinline__ void prologue_load(const Pro& p, int k, float (&va)[GPW], float (&vb)[GPW], uint32_t ep,
                                              int* err, int* abort_flag) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int U = k >> 5, kind = p.kind;
  const bool act = kind == PRO_SILU || kind == PRO_GELU;   // b is an activation, else a weight
  const float* pb = act ? p.b : p.w0;
  const int tb = act ? p.tb : 0;
  const uint32_t wa = want_tag(ep, p.ta), wb = want_tag(ep, tb);
  unsigned long long x[2 * GPW];       // a words, then b words
  uint32_t want[2 * GPW];
#pragma unroll
  for (int j = 0; j < GPW; j++) {
    const int g = warp + j * CK_WARPS;
    const int i = 32 * g + lane;
    x[j] = g < U ? ld_word(p.a, i, p.ta) : ((unsigned long long)wa << 32);
    x[GPW + j] = (g < U && kind != PRO_COPY) ? ld_word(pb, i, tb) : ((unsigned long long)wb << 32);
    want[j] = wa;
    want[GPW + j] = wb;
  }
  settle(x, want, [&](int j) {
    const int i = 32 * (warp + (j % GPW) * CK_WARPS) + lane;
    return j < GPW ? ld_word(p.a, i, p.ta) : ld_word(pb, i, tb);
  }, err, abort_flag);
#pragma unroll
  for (int j = 0; j < GPW; j++) {
    va[j] = word_float(x[j]);
    vb[j] = word_float(x[GPW + j]);
  }
}

// Fused prologue for COPY / NORM / SILU / GELU: one warp per 32-group, one
// element per lane, into the quantized form of quant_x.  The RMS scale of
// NORM is a scalar over the whole vector, so x is quantized without it (the
// per-group quantization is scale-invariant) and the caller applies it to
// each output row: y = inv * (W (a * w)), the RMS_NORM_WGSL product
// (a * inv) * w with the scalar moved past the dot.  Returns that scale.
template <int GPW>
__device__ float prologue_quant(const Pro& p, int k, const float (&va)[GPW], const float (&vb)[GPW], SmemMv& s) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int U = k >> 5, kind = p.kind;
  // the kind switch sits outside the group loop so the groups interleave
  float ss = 0.f, vx[GPW];
  if (kind == PRO_COPY) {
#pragma unroll
    for (int j = 0; j < GPW; j++) vx[j] = va[j];
  } else if (kind == PRO_NORM) {
#pragma unroll
    for (int j = 0; j < GPW; j++) { vx[j] = va[j] * vb[j]; ss += va[j] * va[j]; }
  } else if (kind == PRO_SILU) {
#pragma unroll
    for (int j = 0; j < GPW; j++) vx[j] = (va[j] / (1.0f + expf(-va[j]))) * vb[j];
  } else {
#pragma unroll
    for (int j = 0; j < GPW; j++) vx[j] = gelu_tanh(va[j]) * vb[j];
  }
#pragma unroll
  for (int j = 0; j < GPW; j++) {
    const int g = warp + j * CK_WARPS;
    const bool ok = g < U;                           // warp-uniform
    const float v = vx[j];
    const float amax = warp_max(fabsf(v));
    const bool fin = amax <= 3.0e38f;
    const float step = amax * (1.0f / 32639.0f);
    const float inv = (step > 0.f && fin) ? 32639.0f / amax : 0.f;
    const int X = max(-32639, min(32639, __float2int_rn(v * inv)));
    const int h = (X + 128) >> 8;
    int sum = X;
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (ok) {
      s.xh[32 * g + lane] = (int8_t)h;
      s.xl[32 * g + lane] = (int8_t)(X - 256 * h);
      if (lane == 0) s.sx[g] = fin ? step : __int_as_float(0x7fc00000);
      if ((lane & 15) == 0) s.s16[2 * g + (lane >> 4)] = sum;
    }
  }
  if (kind == PRO_NORM) {
    ss = warp_sum(ss);
    if (lane == 0) s.red[warp] = ss;
  }
  __syncthreads();
  if (kind != PRO_NORM) return 1.0f;
  float t = 0.f;
#pragma unroll
  for (int w = 0; w < CK_WARPS; w++) t += s.red[w];
  return rms_inv(t, k, p.eps);
}

// One matvec phase on this CTA.  GPW = 32-groups of x per warp (k <= 512 *
// GPW); ONE (k <= 1024) keeps the lane's x unit in registers.
template <int GPW, unsigned TM>
__device__ __forceinline__ void mv_run_t(const MvPhase& P, SmemMv& s, Ring& R, int cta, int* err, int* abort_flag,
                                         unsigned long long* tp, uint32_t ep) {
  constexpr bool ONE = GPW <= 2;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int seg = 0, row = -1;
  TileList T;
  // a CTA without rows in this phase reads nothing (its reads could race the
  // next writer of the input, which does not wait for this CTA)
  if (!next_tile(P, cta, seg, row, T)) return;
  stage_mark(tp, 0);
  float xscale = 1.0f;
  if (P.pro.kind == PRO_GEMMA) {
    build_x(P.pro, P.k, s, cta, ep, err, abort_flag);
    quant_x(P.k, s);
  } else {
    float va[GPW], vb[GPW];
    prologue_load<GPW>(P.pro, P.k, va, vb, ep, err, abort_flag);
    xscale = prologue_quant<GPW>(P.pro, P.k, va, vb, s);
  }
  stage_mark(tp, 1);
  XUnit x0;
  if (ONE && lane < (P.k >> 5)) load_xunit(s, lane, x0);
  bool first = true;
  do {
    if (!ring_wait(R, err, abort_flag)) { R.ok = 0; return; }
    if (first) stage_mark(tp, 2);
    mv_tile<ONE, TM>(P, ring_buf(R.consumed), T, warp, s, x0, xscale, cta, ep, err, abort_flag);
    if (first) stage_mark(tp, 3);
    first = false;
    ring_release(R, cta);
  } while (next_tile(P, cta, seg, row, T));
  if (P.epi) {
    // fused SILU_MUL_WGSL (:3529-3547) / GELU_TANH_MUL_WGSL (:3568-3599) over
    // this CTA's rows (the release above synchronised the staging rows)
    int lo, hi;
    seg_range(P.seg[0], cta, lo, hi);
    for (int i = threadIdx.x; i < hi - lo; i += CK_THREADS) {
      const float g = s.glu[0][i], u = s.glu[1][i];
      st_word(P.glu_out, lo + i, P.epi == EPI_SILU ? (g / (1.0f + expf(-g))) * u : gelu_tanh(g) * u, P.tglu, ep);
    }
  }
  stage_mark(tp, 4);
}

template <unsigned TM>
__device__ __forceinline__ void mv_run(const MvPhase& P, SmemMv& s, Ring& R, int cta, int* err, int* abort_flag,
                                       unsigned long long* tp, uint32_t ep) {
  const int U = P.k >> 5;
  if (U <= 2 * CK_WARPS) mv_run_t<2, TM>(P, s, R, cta, err, abort_flag, tp, ep);
  else if (U <= 4 * CK_WARPS) mv_run_t<4, TM>(P, s, R, cta, err, abort_flag, tp, ep);
  else mv_run_t<CK_KMAX / 32 / CK_WARPS, TM>(P, s, R, cta, err, abort_flag, tp, ep);
}

template <unsigned TM = CK_TM_ALL>
__device__ __forceinline__ void phase_matvec(const MvPhase& P, Smem& sm, Ring& R, int cta, int* err,
                                             int* abort_flag, unsigned long long* tp, uint32_t ep) {
  mv_run<TM>(P, sm.mv, R, cta, err, abort_flag, tp, ep);
}

// ---------------------------------------------------------------------------
// Embedding (GGUF_*_EMBEDDING_WGSL, :2615-2866): row tokens[pos] of the
// (tied) table dequantized in WGSL order, times EMBEDDING_SCALE.  Also marks
// the repetition-penalty id set when this step computes logits.
__device__ __forceinline__ void phase_embed(const EmbedPhase& P, const CkDev& D, int cta, int ncta, int pos,
                                            uint32_t ep) {
  const CkState* st = D.st;
  uint32_t token = D.tokens[pos];
  if (token >= (uint32_t)D.vocab) {
    if (cta == 0 && threadIdx.x == 0) atomicOr(&D.st->err, CK_DERR_TOKEN);
    token = 0;
  }
  const uint8_t* row = P.w + (size_t)token * P.L.row_bytes;
  for (int i = cta * CK_THREADS + threadIdx.x; i < P.L.k; i += ncta * CK_THREADS)
    st_word(P.out, i, __fmul_rn(dequant_at(row, P.L, i), P.scale), P.tout, ep);
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
// theta^(-2d/hd) for d < hd/2, the inverse frequency of rope_angle
// (llama-wgsl-runtime.ts:2885-2888), built once per layer at load time.
__global__ void k_inv_freq(float* out, uint32_t theta, int hd) {
  int d = threadIdx.x;
  if (d < hd / 2) out[d] = powf((float)theta, (-2.0f * (float)d) / (float)hd);
}

// Normalize (optional) + rotate one head of length hd from src into dst
// (shared memory); `inv` is the head's 1/rms (ignored without weights);
// cs holds cos/sin of each pair's angle.
__device__ __forceinline__ void rope_head(const float* src, const float* w, float inv, float* dst, int hd, int inter,
                                          const float2* cs, int t0, int tstride) {
  int half = hd >> 1;
  for (int d = t0; d < half; d += tstride) {
    int i0 = inter ? 2 * d : d, i1 = inter ? 2 * d + 1 : d + half;
    float a = src[i0], b = src[i1];
    if (w) {
      a = (a * inv) * w[i0];
      b = (b * inv) * w[i1];
    }
    float co = cs[d].x, si = cs[d].y;
    dst[i0] = a * co - b * si;
    dst[i1] = a * si + b * co;
  }
}

// E elements (one lane's share of a head row) of the KV cache, held in
// registers in the cache's storage type until used: fp16 pairs or fp32 words.
template <int E, bool F32>
struct KvRow {
  uint32_t w[F32 ? E : E / 2];
};
template <int E, bool F32>
__device__ __forceinline__ void kv_zero(KvRow<E, F32>& r) {
#pragma unroll
  for (int i = 0; i < (F32 ? E : E / 2); i++) r.w[i] = 0u;
}
template <int E, bool F32>
__device__ __forceinline__ void kv_load(const void* base, size_t off, KvRow<E, F32>& r) {
  if (F32) {
    const uint32_t* p = (const uint32_t*)base + off;
    if (E == 2) {
      const uint2 v = *(const uint2*)p;
      r.w[0] = v.x; r.w[1] = v.y;
    } else {
#pragma unroll
      for (int i = 0; i < E / 4; i++) {
        const uint4 v = ((const uint4*)p)[i];
        r.w[4 * i] = v.x; r.w[4 * i + 1] = v.y; r.w[4 * i + 2] = v.z; r.w[4 * i + 3] = v.w;
      }
    }
  } else {
    const uint16_t* p = (const uint16_t*)base + off;
    if (E == 2) {
      r.w[0] = *(const uint32_t*)p;
    } else if (E == 4) {
      const uint2 v = *(const uint2*)p;
      r.w[0] = v.x; r.w[1] = v.y;
    } else {
      const uint4 v = *(const uint4*)p;
      r.w[0] = v.x; r.w[1] = v.y; r.w[2] = v.z; r.w[3] = v.w;
    }
  }
}
template <int E, bool F32>
__device__ __forceinline__ float kv_at(const KvRow<E, F32>& r, int e) {
  if (F32) return __uint_as_float(r.w[e]);
  const uint32_t w = r.w[e >> 1];
  return __half2float(__ushort_as_half((unsigned short)((e & 1) ? (w >> 16) : (w & 0xFFFFu))));
}
// a value as the cache stores it (what a later read of the cache returns)
template <bool F32>
__device__ __forceinline__ float kv_round(float x) {
  return F32 ? x : __half2float(__float2half_rn(x));
}

// Cache rows of positions t and t + wpg (zero rows past tend).
template <int E, bool F32>
__device__ __forceinline__ void kv_load_pair(const AttnPhase& P, size_t kvbase, int t, int tend, int wpg,
                                             KvRow<E, F32>& k0, KvRow<E, F32>& v0, KvRow<E, F32>& k1,
                                             KvRow<E, F32>& v1) {
  constexpr int hd = 32 * E;
  kv_zero(k0); kv_zero(v0); kv_zero(k1); kv_zero(v1);
  if (t < tend) { kv_load(P.kc, kvbase + (size_t)t * hd, k0); kv_load(P.vc, kvbase + (size_t)t * hd, v0); }
  if (t + wpg < tend) {
    kv_load(P.kc, kvbase + (size_t)(t + wpg) * hd, k1);
    kv_load(P.vc, kvbase + (size_t)(t + wpg) * hd, v1);
  }
}

// One online-softmax step over two positions of a warp (the second may be
// absent: score -inf and a zero row add nothing).
template <int E, bool F32>
__device__ __forceinline__ void softmax_pair(const float (&q)[E], const KvRow<E, F32>& k0, const KvRow<E, F32>& v0,
                                             const KvRow<E, F32>& k1, const KvRow<E, F32>& v1, bool has1,
                                             float scale, float& m, float& l, float (&acc)[E]) {
  float d0 = 0.f, d1 = 0.f;
#pragma unroll
  for (int e = 0; e < E; e++) {
    d0 += q[e] * kv_at(k0, e);
    d1 += q[e] * kv_at(k1, e);
  }
  const float s0 = warp_sum(d0) * scale;
  const float s1 = has1 ? warp_sum(d1) * scale : -INFINITY;
  const float mn = fmaxf(m, fmaxf(s0, s1));
  const float c = expf(m - mn), p0 = expf(s0 - mn), p1 = expf(s1 - mn);
  l = l * c + p0 + p1;
#pragma unroll
  for (int e = 0; e < E; e++) acc[e] = acc[e] * c + p0 * kv_at(v0, e) + p1 * kv_at(v1, e);
  m = mn;
}

// Merge of the S split partials (m, l, acc) of one kv head's G query heads:
// out = sum_s acc_s * exp(m_s - M) / sum_s l_s * exp(m_s - M), M = max_s m_s.
// Every load is issued in parallel: one round for the (m, l) pairs, one warp
// per head for the weights, then each output element's S accumulator values
// split over P adjacent lanes, eight loads in flight per lane.
template <int E>
__device__ __forceinline__ void attn_merge(const AttnPhase& P, SmemAt& s, int kvh, int S, uint32_t ep, int* err,
                                           int* abort_flag) {
  constexpr int hd = 32 * E;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = P.group, NE = G * hd;
  const float* pk = P.part + (size_t)kvh * P.smax * G * (hd + 2) * 2;   // tagged words: 2 floats each
  const uint32_t want = want_tag(ep, P.tout);
  const unsigned long long none = (unsigned long long)want << 32;
  float* sm_m = s.wacc;                 // [S * G] split maxima, then weights
  float* sm_l = s.wacc + 1024;          // [S * G] split sums
  float* sm_L = s.wacc + 2048;          // [G] merged sums
  int Pw = 1;                                        // lanes per element (power of two)
  while (Pw < 32 && 2 * Pw * NE <= CK_THREADS) Pw *= 2;
  const int part = tid & (Pw - 1), slots = CK_THREADS / Pw;
  const int passes = (NE + slots - 1) / slots;
  // the first eight accumulators of this lane's first element are requested
  // together with the split maxima and sums (one round trip, not two)
  unsigned long long x[8];
  {
    const int e = tid / Pw;
    const int gg = e < NE ? e / hd : 0, d = e % hd;
#pragma unroll
    for (int j = 0; j < 8; j++) {
      const int sp = part + j * Pw;
      x[j] = (e < NE && sp < S) ? ld_word(pk, ((size_t)sp * G + gg) * (hd + 2) + 2 + d, P.tout) : none;
    }
  }
  for (int i = tid; i < S * G; i += CK_THREADS) {   // one pass: S * G <= 64 * 8
    const size_t o = (size_t)i * (hd + 2);          // i = split * G + head
    unsigned long long ml[2] = {ld_word(pk, o, P.tout), ld_word(pk, o + 1, P.tout)};
    const uint32_t w2[2] = {want, want};
    settle(ml, w2, [&](int j) { return ld_word(pk, o + j, P.tout); }, err, abort_flag);
    sm_m[i] = word_float(ml[0]);
    sm_l[i] = word_float(ml[1]);
  }
  {   // the first accumulators settle in the same wait as the (m, l) pairs
    const int e = tid / Pw;
    const int gg = e < NE ? e / hd : 0, d = e % hd;
    const uint32_t w8[8] = {want, want, want, want, want, want, want, want};
    settle(x, w8, [&](int j) {
      return ld_word(pk, ((size_t)(part + j * Pw) * G + gg) * (hd + 2) + 2 + d, P.tout);
    }, err, abort_flag);
  }
  __syncthreads();
  for (int gg = warp; gg < G; gg += CK_WARPS) {
    float M = -INFINITY;
    for (int sp = lane; sp < S; sp += 32) M = fmaxf(M, sm_m[sp * G + gg]);
    M = warp_max(M);
    float L = 0.f;
    for (int sp = lane; sp < S; sp += 32) {
      const float f = expf(sm_m[sp * G + gg] - M);
      L += sm_l[sp * G + gg] * f;
      sm_m[sp * G + gg] = f;
    }
    L = warp_sum(L);
    if (lane == 0) sm_L[gg] = L;
  }
  __syncthreads();
  for (int ps = 0; ps < passes; ps++) {
    const int e = tid / Pw + ps * slots;
    const bool ok = e < NE;
    const int gg = ok ? e / hd : 0, d = e % hd;
    float A = 0.f;
    for (int sp0 = part; sp0 < S; sp0 += 8 * Pw) {
      if (ps > 0 || sp0 != part) {
#pragma unroll
        for (int j = 0; j < 8; j++) {
          const int sp = sp0 + j * Pw;
          x[j] = (ok && sp < S) ? ld_word(pk, ((size_t)sp * G + gg) * (hd + 2) + 2 + d, P.tout) : none;
        }
      }
      if (ps > 0 || sp0 != part) {   // the first group settled with the (m, l) pairs
        const uint32_t w8[8] = {want, want, want, want, want, want, want, want};
        settle(x, w8, [&](int j) {
          return ld_word(pk, ((size_t)(sp0 + j * Pw) * G + gg) * (hd + 2) + 2 + d, P.tout);
        }, err, abort_flag);
      }
#pragma unroll
      for (int j = 0; j < 8; j++) {
        const int sp = sp0 + j * Pw;
        if (ok && sp < S) A += word_float(x[j]) * sm_m[sp * G + gg];
      }
    }
    for (int o = 1; o < Pw; o <<= 1) A += __shfl_xor_sync(0xffffffffu, A, o);
    if (ok && part == 0) st_word(P.out, (size_t)(kvh * G + gg) * hd + d, A / sm_L[gg], P.tout, ep);
  }
}

template <int E, bool F32>
__device__ __forceinline__ void attn_unit(const AttnPhase& P, SmemAt& s, int kvh, int split, int pos,
                                          unsigned long long* tp, uint32_t ep, int* err, int* abort_flag) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  constexpr int hd = 32 * E;        // head_dim: one lane holds E elements of a row
  const int G = P.group;
  const int start = (P.window != 0 && pos + 1 > P.window) ? pos + 1 - P.window : 0;
  const int npos = pos - start + 1;
  int chunk = (npos + P.smax - 1) / P.smax;
  if (chunk < CK_MIN_SPLIT) chunk = CK_MIN_SPLIT;
  const int S = (npos + chunk - 1) / chunk;
  if (split >= S) return;
  const int t0 = start + split * chunk;
  const int t1 = min(t0 + chunk, pos + 1);
  const bool owner = split == S - 1;   // the split holding `pos` stores K/V there
  // positions read from the cache; the owner takes `pos` from shared memory
  const int tend = owner ? pos : t1;
  const int wpg = CK_WARPS / G;      // warps per q head (G <= 8)
  const int g = warp / wpg, sub = warp % wpg;

  // --- every global load of the unit issued in one round ---------------------
  stage_mark(tp, 0);
  const size_t kvbase = (size_t)kvh * P.ctx * hd + lane * E;
  int t = t0 + sub;
  // KV rows are in flight two position pairs ahead of the math (one pair
  // ahead for 256-wide rows, none for 256-wide fp32 rows: register budget);
  // the first pairs load under the q/k/v wait and the QK-norm / RoPE below
  constexpr int DEPTH = (E <= 4 && !(F32 && E == 4)) ? 2 : (F32 && E == 8) ? 0 : 1;
  KvRow<E, F32> ka, va, kb, vb, kc, vc, kd, vd;
  kv_zero(ka); kv_zero(va); kv_zero(kb); kv_zero(vb);
  kv_zero(kc); kv_zero(vc); kv_zero(kd); kv_zero(vd);
  if (g < G) {
    kv_load_pair<E, F32>(P, kvbase, t, tend, wpg, ka, va, kb, vb);
    if (DEPTH == 2) kv_load_pair<E, F32>(P, kvbase, t + 2 * wpg, tend, wpg, kc, vc, kd, vd);
  }
  float invf = 0.f, qv0 = 0.f, qv1 = 0.f, kk = 0.f, vv = 0.f, wq = 0.f, wk = 0.f;
  const uint32_t want = want_tag(ep, P.tqkv);
  const unsigned long long none = (unsigned long long)want << 32;
  const size_t q0 = (size_t)kvh * G * hd, kv0 = (size_t)kvh * hd;
  unsigned long long xw[4];   // q (two), k, v
  xw[0] = tid < G * hd ? ld_word(P.q, q0 + tid, P.tqkv) : none;
  xw[1] = tid + CK_THREADS < G * hd ? ld_word(P.q, q0 + tid + CK_THREADS, P.tqkv) : none;
  xw[2] = (owner && tid < hd) ? ld_word(P.k, kv0 + tid, P.tqkv) : none;
  xw[3] = (owner && tid < hd) ? ld_word(P.v, kv0 + tid, P.tqkv) : none;
  if (tid < (hd >> 1)) invf = P.inv_freq[tid];
  if (tid < hd) {
    if (owner && P.kw) wk = P.kw[tid];
    if (P.qw) wq = P.qw[tid];
  }
  const uint32_t wants[4] = {want, want, want, want};
  settle(xw, wants, [&](int j) {
    return j == 0 ? ld_word(P.q, q0 + tid, P.tqkv)
         : j == 1 ? ld_word(P.q, q0 + tid + CK_THREADS, P.tqkv)
         : j == 2 ? ld_word(P.k, kv0 + tid, P.tqkv) : ld_word(P.v, kv0 + tid, P.tqkv);
  }, err, abort_flag);
  qv0 = word_float(xw[0]);
  qv1 = word_float(xw[1]);
  kk = word_float(xw[2]);
  vv = word_float(xw[3]);
  if (tid < (hd >> 1)) {
    // angle = pos * theta^(-2d/hd) (rope_angle, :2885-2888); the power is the
    // per-layer table built at load time with the same powf
    float sn, cn;
    sincosf((float)pos * invf, &sn, &cn);
    s.cs[tid] = make_float2(cn, sn);
  }
  if (tid < G * hd) s.raw[tid] = qv0;
  if (tid + CK_THREADS < G * hd) s.raw[tid + CK_THREADS] = qv1;
  if (tid < hd) {
    if (owner) {
      s.kvw[0][tid] = kk;
      s.kvw[1][tid] = vv;
      if (P.kw) s.kvw[3][tid] = wk;
    }
    if (P.qw) s.kvw[2][tid] = wq;
  }
  __syncthreads();
  // --- per-head 1/rms of q (and k) for the QK-norm -----------------------
  if (P.qw) {
    for (int gg = warp; gg < G + (owner ? 1 : 0); gg += CK_WARPS) {
      const float* src = gg < G ? s.raw + gg * hd : s.kvw[0];
      float ss = 0.f;
      for (int d = lane; d < hd; d += 32) ss += src[d] * src[d];
      ss = warp_sum(ss);
      if (lane == 0) s.inv[gg] = rms_inv(ss, hd, P.eps);
    }
    __syncthreads();
  }
  // --- q: norm + rope into shared memory; owner: k/v into the cache --------
  for (int gg = 0; gg < G; gg++)
    rope_head(s.raw + gg * hd, P.qw ? s.kvw[2] : nullptr, P.qw ? s.inv[gg] : 1.f, s.qs + gg * hd, hd,
              P.interleaved, s.cs, tid, CK_THREADS);
  if (owner) {
    rope_head(s.kvw[0], P.kw ? s.kvw[3] : nullptr, P.kw ? s.inv[G] : 1.f, s.kst, hd, P.interleaved, s.cs, tid,
              CK_THREADS);
    __syncthreads();
    const size_t cb = ((size_t)kvh * P.ctx + pos) * hd;
    if (tid < hd) {
      const float kv = s.kst[tid], vv2 = s.kvw[1][tid];
      if (F32) {
        ((float*)P.kc)[cb + tid] = kv;
        ((float*)P.vc)[cb + tid] = vv2;
      } else {
        ((__half*)P.kc)[cb + tid] = __float2half_rn(kv);
        ((__half*)P.vc)[cb + tid] = __float2half_rn(vv2);
      }
    }
  }
  __syncthreads();
  stage_mark(tp, 1);

  // --- online softmax: warps split into G groups, one q head per group -----
  float q[E], acc[E], m = -INFINITY, l = 0.f;
#pragma unroll
  for (int e = 0; e < E; e++) {
    q[e] = g < G ? s.qs[g * hd + lane * E + e] : 0.f;
    acc[e] = 0.f;
  }
  if (g < G) {
    // two positions per step
    for (; t < tend; t += 2 * wpg) {
      KvRow<E, F32> nka, nva, nkb, nvb;
      if (DEPTH == 2) kv_load_pair<E, F32>(P, kvbase, t + 4 * wpg, tend, wpg, nka, nva, nkb, nvb);
      if (DEPTH == 1) kv_load_pair<E, F32>(P, kvbase, t + 2 * wpg, tend, wpg, nka, nva, nkb, nvb);
      softmax_pair<E, F32>(q, ka, va, kb, vb, t + wpg < tend, P.scale, m, l, acc);
      if (DEPTH == 2) {
        ka = kc; va = vc; kb = kd; vb = vd;
        kc = nka; vc = nva; kd = nkb; vd = nvb;
      } else if (DEPTH == 1) {
        ka = nka; va = nva; kb = nkb; vb = nvb;
      } else {
        kv_load_pair<E, F32>(P, kvbase, t + 2 * wpg, tend, wpg, ka, va, kb, vb);
      }
    }
    if (owner && sub == 0) {   // position pos, as the cache now holds it
      float d0 = 0.f;
#pragma unroll
      for (int e = 0; e < E; e++) d0 += q[e] * kv_round<F32>(s.kst[lane * E + e]);
      const float s0 = warp_sum(d0) * P.scale;
      const float mn = fmaxf(m, s0);
      const float c = expf(m - mn), p0 = expf(s0 - mn);
      l = l * c + p0;
#pragma unroll
      for (int e = 0; e < E; e++) acc[e] = acc[e] * c + p0 * kv_round<F32>(s.kvw[1][lane * E + e]);
      m = mn;
    }
  }
  // --- merge the warps of each head ------------------------------------------
  stage_mark(tp, 2);
  if (lane == 0) {
    s.wm[warp] = m;
    s.wl[warp] = l;
  }
#pragma unroll
  for (int e = 0; e < E; e++) s.wacc[warp * CK_HDMAX + lane * E + e] = acc[e];
  __syncthreads();
  // per head: M = max over its warps, each warp's weight exp(m_w - M), L
  if (tid < G) {
    float M = -INFINITY;
    for (int w = tid * wpg; w < tid * wpg + wpg; w++) M = fmaxf(M, s.wm[w]);
    float L = 0.f;
    for (int w = tid * wpg; w < tid * wpg + wpg; w++) {
      const float f = s.wm[w] == -INFINITY ? 0.f : expf(s.wm[w] - M);
      s.wf[w] = f;
      L += s.wl[w] * f;
    }
    s.hm[tid] = M;
    s.hl[tid] = L;
  }
  __syncthreads();
  if (S == 1) {   // one split covers the context: no partials, no merge
    for (int i = tid; i < G * hd; i += CK_THREADS) {
      const int gg = i / hd, d = i % hd;
      float A = 0.f;
      for (int w = gg * wpg; w < gg * wpg + wpg; w++) A += s.wacc[w * CK_HDMAX + d] * s.wf[w];
      st_word(P.out, (size_t)(kvh * G + gg) * hd + d, A / s.hl[gg], P.tout, ep);
    }
    stage_mark(tp, 3);
    return;
  }
  // partials (m, l, acc) of this split as tagged words
  float* part = P.part + ((size_t)kvh * P.smax + split) * G * (hd + 2) * 2;
  for (int i = tid; i < G * hd; i += CK_THREADS) {
    const int gg = i / hd, d = i % hd;
    float A = 0.f;
    for (int w = gg * wpg; w < gg * wpg + wpg; w++) A += s.wacc[w * CK_HDMAX + d] * s.wf[w];
    st_word(part, gg * (hd + 2) + 2 + d, A, P.tout, ep);
    if (d == 0) {
      st_word(part, gg * (hd + 2), s.hm[gg], P.tout, ep);
      st_word(part, gg * (hd + 2) + 1, s.hl[gg], P.tout, ep);
    }
  }
  stage_mark(tp, 4);
  // --- the split holding pos merges all splits of this kv head ---------------
  if (!owner) return;
  __syncthreads();
  attn_merge<E>(P, s, kvh, S, ep, err, abort_flag);
  stage_mark(tp, 6);
}

// Bulk prefetch into L2 (no shared memory): addr and bytes multiples of 16.
__device__ __forceinline__ void prefetch_l2(const void* addr, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(addr), "r"(bytes) : "memory");
}

// Issued one phase early (at the start of the layer's QKV phase): this CTA's
// attention unit's cache rows [t0, tend) of K and V move into L2 while the
// projections run, so the unit's first reads do not go to HBM.
// Megakernel instantiations with OT = 1, when every unit has a CTA of its own: the split holding `pos` (the one that merges, and so
// finishes last) of kv head h runs on CTA ncta - kvh + h and split s < S - 1
// on CTA s * kvh + h.  The phase after the attention leaves those top CTAs
// without rows, so none of its rows waits behind a merge.  False: this CTA
// has no unit.
__device__ __forceinline__ bool attn_unit_top(const AttnPhase& P, int S, int cta, int ncta, int& kvh, int& split) {
  if (cta >= ncta - P.kvh) {
    kvh = cta - (ncta - P.kvh);
    split = S - 1;
    return true;
  }
  kvh = cta % P.kvh;
  split = cta / P.kvh;
  return split < S - 1;
}

template <int AE, int OT>
__device__ __forceinline__ void attn_prefetch(const AttnPhase& P, int cta, int ncta, int pos) {
  if (threadIdx.x != 0) return;
  const int start = (P.window != 0 && pos + 1 > P.window) ? pos + 1 - P.window : 0;
  const int npos = pos - start + 1;
  int chunk = (npos + P.smax - 1) / P.smax;
  if (chunk < CK_MIN_SPLIT) chunk = CK_MIN_SPLIT;
  const int S = (npos + chunk - 1) / chunk;
  const size_t elem = P.kv_f32 ? 4 : 2;
  if constexpr (OT != 0) {
    int kvh, split;
    if (P.kvh * P.smax <= ncta) {
      if (!attn_unit_top(P, S, cta, ncta, kvh, split)) return;
      const int t0 = start + split * chunk;
      const int tend = split == S - 1 ? pos : min(t0 + chunk, pos + 1);
      if (tend <= t0) return;
      const size_t off = ((size_t)kvh * P.ctx + t0) * P.hd * elem;
      const uint32_t bytes = (uint32_t)((size_t)(tend - t0) * P.hd * elem);
      prefetch_l2((const uint8_t*)P.kc + off, bytes);
      prefetch_l2((const uint8_t*)P.vc + off, bytes);
      return;
    }
  }
  for (int u = cta; u < P.kvh * P.smax; u += ncta) {
    const int kvh = u % P.kvh, split = u / P.kvh;
    if (split >= S) continue;
    const int t0 = start + split * chunk;
    const int tend = split == S - 1 ? pos : min(t0 + chunk, pos + 1);
    if (tend <= t0) continue;
    const size_t off = ((size_t)kvh * P.ctx + t0) * P.hd * elem;
    const uint32_t bytes = (uint32_t)((size_t)(tend - t0) * P.hd * elem);
    prefetch_l2((const uint8_t*)P.kc + off, bytes);
    prefetch_l2((const uint8_t*)P.vc + off, bytes);
  }
}

// AE: 0 = head_dim and cache type dispatched at run time; 2 / 4 / 8 = only
// head_dim 32 * AE with an fp16 cache (the host guarantees it).
template <int AE = 0, int OT = 0>
__device__ __forceinline__ void phase_attn(const AttnPhase& P, Smem& sm, const CkDev& D, int cta, int ncta, int pos,
                                           unsigned long long* tp, uint32_t ep) {
  int* err = &D.st->err;
  int* ab = &D.st->abort_flag;
  if constexpr (OT != 0) {
    if (P.kvh * P.smax <= ncta) {
      const int start = (P.window != 0 && pos + 1 > P.window) ? pos + 1 - P.window : 0;
      const int npos = pos - start + 1;
      int chunk = (npos + P.smax - 1) / P.smax;
      if (chunk < CK_MIN_SPLIT) chunk = CK_MIN_SPLIT;
      const int S = (npos + chunk - 1) / chunk;
      int kvh, split;
      if (attn_unit_top(P, S, cta, ncta, kvh, split)) {
        if (P.kv_f32) {
          if (P.hd == 64) attn_unit<2, true>(P, sm.at, kvh, split, pos, tp, ep, err, ab);
          else if (P.hd == 128) attn_unit<4, true>(P, sm.at, kvh, split, pos, tp, ep, err, ab);
          else attn_unit<8, true>(P, sm.at, kvh, split, pos, tp, ep, err, ab);
        } else {
          if (P.hd == 64) attn_unit<2, false>(P, sm.at, kvh, split, pos, tp, ep, err, ab);
          else if (P.hd == 128) attn_unit<4, false>(P, sm.at, kvh, split, pos, tp, ep, err, ab);
          else attn_unit<8, false>(P, sm.at, kvh, split, pos, tp, ep, err, ab);
        }
        __syncthreads();
      }
      return;
    }
  }
  // split-major: the active split 0 units of every kv head land on
  // different CTAs even when the context needs one split only
  int units = P.kvh * P.smax;
  for (int u = cta; u < units; u += ncta) {
    int kvh = u % P.kvh, split = u / P.kvh;
    unsigned long long* up = (tp && u == cta) ? tp : nullptr;
    if constexpr (AE != 0) {
      attn_unit<(AE ? AE : 2), false>(P, sm.at, kvh, split, pos, up, ep, err, ab);
    } else if (P.kv_f32) {
      if (P.hd == 64) attn_unit<2, true>(P, sm.at, kvh, split, pos, up, ep, err, ab);
      else if (P.hd == 128) attn_unit<4, true>(P, sm.at, kvh, split, pos, up, ep, err, ab);
      else attn_unit<8, true>(P, sm.at, kvh, split, pos, up, ep, err, ab);
    } else {
      if (P.hd == 64) attn_unit<2, false>(P, sm.at, kvh, split, pos, up, ep, err, ab);
      else if (P.hd == 128) attn_unit<4, false>(P, sm.at, kvh, split, pos, up, ep, err, ab);
      else attn_unit<8, false>(P, sm.at, kvh, split, pos, up, ep, err, ab);
    }
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

__device__ __noinline__ void phase_topk_local(const CkDev& D, Smem& smu, int cta, int ncta);
template <int EXACT>
__device__ __forceinline__ void phase_argmax1(const CkDev& D, Smem& sm, int cta, int ncta) {
  const CkState* st = D.st;
  if (EXACT && st->exact && st->sampling && D.xval && ncta <= D.xgrid) {
    phase_topk_local(D, sm, cta, ncta);
    return;
  }
  const int groups = (D.vocab + 255) / 256;
  const bool pen = st->pen_d > 1.0;
  const float penalty = (float)st->pen_milli / 1000.0f;
  // one warp per 256-logit chunk, 8 logits per lane, every load issued
  // before the first comparison; the chunk's winner over its logits and
  // the sentinel (-3.402823e38, 0xffffffff) under `better`, a strict total
  // order, so the comparison order does not change the result
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int g = cta + warp * ncta; g < groups; g += ncta * CK_WARPS) {
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; j++) {
      const uint32_t i = (uint32_t)g * 256u + 32u * j + lane;
      v[j] = i < (uint32_t)D.vocab ? D.logits[i] : 0.f;
    }
    float bv = -3.402823e38f;
    uint32_t bi = 0xffffffffu;
#pragma unroll
    for (int j = 0; j < 8; j++) {
      const uint32_t i = (uint32_t)g * 256u + 32u * j + lane;
      if (i >= (uint32_t)D.vocab) continue;
      float x = v[j];
      if (pen && ((D.pen_mask[i >> 5] >> (i & 31)) & 1u)) x = x > 0.f ? x / penalty : x * penalty;
      if (better(x, i, bv, bi)) { bv = x; bi = i; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
    }
    if (lane == 0) {
      D.cand_val[g] = bv;
      D.cand_idx[g] = bi;
    }
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

// sampleFromCandidateBuffer (sampling.ts:23-76) on the device over a
// candidate list staged in s: val = -(value after the re-penalty of seen
// ids) or +inf (empty slot), idx = id, prob = the stable sort's tie-break
// (the candidate's place in the reference's list).  Stable descending sort,
// top-k, temperature softmax in fp64, top-p cutoff at the first cdf >= topP,
// Philox draw.  One CTA.
__device__ __forceinline__ void sample_core(const CkDev& D, SmemSm& s) {
  const CkState* st = D.st;
  const int tid = threadIdx.x;
  const int NP = CK_SAMPLE_MAX;
  __syncthreads();
  // Bitonic sort by (val, original order) ascending.  Warp w holds elements
  // e0 = 64 w + lane and e1 = e0 + 32 in registers: compare partners at
  // distance j <= 32 are in the same warp (j = 32: the same lane), so those
  // steps exchange by shuffles; each merge level's steps at j >= 64 come
  // first and go through shared memory, grouped between two barriers
  // (14 barriers instead of 55).  Pair (lower, upper) ends ascending when
  // (lower & kk) == 0, descending otherwise.
  const int lane = tid & 31, warp = tid >> 5;
  const int e0 = 64 * warp + lane, e1 = e0 + 32;
  double v0 = s.val[e0], v1 = s.val[e1], o0 = s.prob[e0], o1 = s.prob[e1];
  uint32_t x0 = s.idx[e0], x1 = s.idx[e1];
  auto cmpx = [&](double& v, double& o, uint32_t& x, int e, int j, int kk) {
    const double pv = __shfl_xor_sync(0xffffffffu, v, j), po = __shfl_xor_sync(0xffffffffu, o, j);
    const uint32_t px = __shfl_xor_sync(0xffffffffu, x, j);
    const bool mine_less = v < pv || (v == pv && o < po);
    const bool lower = (e & j) == 0, up = (e & kk) == 0;
    if (mine_less != (lower == up)) { v = pv; o = po; x = px; }
  };
  for (int kk = 2; kk <= NP; kk <<= 1) {
    int j = kk >> 1;
    if (j >= 64) {
      s.val[e0] = v0; s.val[e1] = v1; s.prob[e0] = o0; s.prob[e1] = o1; s.idx[e0] = x0; s.idx[e1] = x1;
      __syncthreads();
      for (; j >= 64; j >>= 1) {
#pragma unroll
        for (int h = 0; h < 2; h++) {
          const int i = h ? e1 : e0, p = i ^ j;
          if (p > i) {
            const bool up = (i & kk) == 0;
            const double a = s.val[i], b = s.val[p];
            const double oa = s.prob[i], ob = s.prob[p];
            const bool gt = (a > b) || (a == b && oa > ob);
            if (gt == up) {
              s.val[i] = b; s.val[p] = a;
              s.prob[i] = ob; s.prob[p] = oa;
              const uint32_t t = s.idx[i]; s.idx[i] = s.idx[p]; s.idx[p] = t;
            }
          }
        }
        __syncthreads();
      }
      v0 = s.val[e0]; v1 = s.val[e1]; o0 = s.prob[e0]; o1 = s.prob[e1]; x0 = s.idx[e0]; x1 = s.idx[e1];
    }
    for (; j > 0; j >>= 1) {
      if (j == 32) {   // e0 (lower) and e1 in this lane
        const bool up = (e0 & kk) == 0;
        const bool gt = v0 > v1 || (v0 == v1 && o0 > o1);
        if (gt == up) {
          const double tv = v0, to = o0;
          const uint32_t tx = x0;
          v0 = v1; o0 = o1; x0 = x1;
          v1 = tv; o1 = to; x1 = tx;
        }
      } else {
        cmpx(v0, o0, x0, e0, j, kk);
        cmpx(v1, o1, x1, e1, j, kk);
      }
    }
  }
  s.val[e0] = v0; s.val[e1] = v1; s.prob[e0] = o0; s.prob[e1] = o1; s.idx[e0] = x0; s.idx[e1] = x1;
  __syncthreads();
  // n: the finite candidates (they sort before the +inf sentinels), counted
  // by all threads; the k exponentials are independent, so every thread
  // takes some (same expression, same values); the fp64 sums, cdf and draw
  // below stay sequential in the reference's order
  static_assert(CK_SAMPLE_MAX == 2 * CK_THREADS, "two candidates per thread");
  const int n = __syncthreads_count(s.val[tid] != INFINITY) + __syncthreads_count(s.val[tid + CK_THREADS] != INFINITY);
  const int k = st->top_k > 0 ? min(st->top_k, n) : n;
  const bool draw = st->temperature > 0.0 && k > 0;
  if (draw) {
    const double T = st->temperature;
    const double maxv = -s.val[0];
    for (int i = tid; i < k; i += CK_THREADS) s.prob[i] = exp((-s.val[i] - maxv) / T);
  }
  __syncthreads();
  const double tp = fmin(fmax(st->top_p, 0.0), 1.0);
  if (tid == 0 && draw) {
    double total = 0.0;
    for (int i = 0; i < k; i++) total += s.prob[i];
    s.dtotal = total;
  }
  if (draw && tp < 1.0) {   // block-uniform: the cdf terms prob[i] / total, on every thread
    __syncthreads();
    const double total = s.dtotal;
    if (total > 0.0)
      for (int i = tid; i < k; i += CK_THREADS) s.val[i] = s.prob[i] / total;   // the sorted keys are done with
    __syncthreads();
  }
  if (tid == 0) {
    uint32_t choice = n > 0 ? s.idx[0] : 0u;
    if (draw) {
      const double total = s.dtotal;
      int cutoff = k;
      if (tp < 1.0 && total > 0.0) {
        double cdf = 0.0;
        for (int i = 0; i < k; i++) {
          cdf += s.val[i];
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

// One candidate as the sampler takes it: -(value with sampling.ts's
// re-penalty of seen ids), or +inf when it is dropped (non-finite).
__device__ __forceinline__ double sample_key(const CkDev& D, float fv, uint32_t ci, double rp) {
  if (!isfinite(fv) || ci == 0xffffffffu) return INFINITY;
  double dv = (double)fv;
  if (rp != 1.0 && ci < (uint32_t)D.vocab && ((D.pen_mask[ci >> 5] >> (ci & 31)) & 1u))
    dv = dv > 0 ? dv / rp : dv * rp;
  return -dv;        // ascending sort of -value == descending by value
}

// The reference's candidate buffer: the per-256 chunk maxima of argmax
// stage 1 (ARGMAX_STAGE1_WGSL :3645-3726), in chunk order.
__device__ __forceinline__ void phase_sample(const CkDev& D, Smem& smu, int cta) {
  const CkState* st = D.st;
  if (cta != 0 || !st->sampling) return;
  SmemSm& s = smu.sm;
  const int groups = (D.vocab + 255) / 256;
  const double rp = fmax(st->pen_d, 1e-6);
  for (int i = threadIdx.x; i < CK_SAMPLE_MAX; i += CK_THREADS) {
    const bool in = i < groups;
    s.val[i] = in ? sample_key(D, D.cand_val[i], D.cand_idx[i], rp) : INFINITY;
    s.idx[i] = in && isfinite(s.val[i]) ? D.cand_idx[i] : 0xffffffffu;
    s.prob[i] = (double)i;   // original order, the stable tie-break
  }
  sample_core(D, s);
}

// ---------------------------------------------------------------------------
// Exact sampler (CkState::exact): the candidate list is the K largest
// stage-1 values of the whole vocabulary (K = top-k when 1..1024, else 1024),
// ties going to the lower id, instead of the per-256 chunk maxima; the
// sampler then runs on it exactly as on the reference's list (ordered by id).
// Found by a block-level radix select twice: every CTA selects the top K of
// its slice of the vocabulary (any of the global top K is in its slice's),
// then one CTA selects the top K of those candidates.
//
// Keys: the float's bits turned order-preserving as unsigned (negative
// values inverted, positive ones with the sign bit set); NaN maps to 0, the
// smallest key, as it never wins the reference's argmax.
__device__ __forceinline__ uint32_t fkey(float v) {
  if (v != v) return 0u;
  const uint32_t u = __float_as_uint(v);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ int exact_k(const CkState* st) {
  return (st->top_k > 0 && st->top_k < CK_SAMPLE_MAX) ? st->top_k : CK_SAMPLE_MAX;
}

// Radix select over n keys key(i) (MSB first, 8 bits a pass): the K-th
// largest key T and how many keys equal T must be taken (need) so that the
// keys > T plus `need` keys == T make K.  Requires n > K.  Every thread gets
// the result.
template <typename KeyAt>
__device__ __forceinline__ void radix_select(int n, int K, KeyAt key, uint32_t& T, int& need, SmemSm& sm) {
  int* hist = sm.hist;
  uint32_t& s_prefix = sm.prefix;
  int& s_rem = sm.rem;
  const int tid = threadIdx.x;
  uint32_t prefix = 0u, mask = 0u;
  int rem = K;
  for (int pass = 0; pass < 4; pass++) {
    const int shift = 24 - 8 * pass;
    for (int b = tid; b < 256; b += CK_THREADS) hist[b] = 0;
    __syncthreads();
    for (int i = tid; i < n; i += CK_THREADS) {
      const uint32_t k = key(i);
      if ((k & mask) == prefix) atomicAdd(&hist[(k >> shift) & 255u], 1);
    }
    __syncthreads();
    if (tid == 0) {
      int cum = 0, sel = 0;
      for (int b = 255; b >= 0; b--) {
        if (cum + hist[b] >= rem) { sel = b; break; }
        cum += hist[b];
      }
      s_prefix = prefix | ((uint32_t)sel << shift);
      s_rem = rem - cum;
    }
    __syncthreads();
    prefix = s_prefix;
    rem = s_rem;
    mask |= 0xFFu << shift;
    __syncthreads();
  }
  T = prefix;
  need = rem;
}

// Write the selected keys of [0, n) in index order: every key > T, then the
// first `need` keys == T (lowest indices).  emit(i, pos) stores element i at
// output place pos; returns how many were written (K, or n when n <= K).
template <typename KeyAt, typename Emit>
__device__ __forceinline__ int radix_emit(int n, int K, KeyAt key, Emit emit, SmemSm& sm) {
  int* s_cnt = sm.cnt;
  int& s_base = sm.base;
  int& s_eqbase = sm.eqbase;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (n <= K) {
    for (int i = tid; i < n; i += CK_THREADS) emit(i, i);
    return n;
  }
  uint32_t T;
  int need;
  radix_select(n, K, key, T, need, sm);
  if (tid == 0) { s_base = 0; s_eqbase = 0; }
  __syncthreads();
  // chunks of CK_THREADS elements in order; within a chunk a block scan
  for (int c0 = 0; c0 < n; c0 += CK_THREADS) {
    const int i = c0 + tid;
    const uint32_t k = i < n ? key(i) : 0u;
    const bool gt = i < n && k > T, eq = i < n && k == T;
    const unsigned bg = __ballot_sync(0xffffffffu, gt), be = __ballot_sync(0xffffffffu, eq);
    if (lane == 0) s_cnt[warp] = (__popc(bg) << 16) | __popc(be);
    __syncthreads();
    int off_g = 0, off_e = 0, tot_g = 0, tot_e = 0;
    for (int w = 0; w < CK_WARPS; w++) {
      const int cg = s_cnt[w] >> 16, ce = s_cnt[w] & 0xFFFF;
      if (w < warp) { off_g += cg; off_e += ce; }
      tot_g += cg; tot_e += ce;
    }
    const unsigned lt = (1u << lane) - 1u;
    const int rg = s_base + off_g + __popc(bg & lt);
    if (gt) emit(i, rg);
    __syncthreads();
    if (tid == 0) { s_base += tot_g; s_eqbase += tot_e; }
    __syncthreads();
    (void)off_e;
  }
  // equal keys go after every greater key: their places are known once all
  // greater keys are counted, so a second sweep emits them
  const int ngt = s_base;
  if (tid == 0) s_eqbase = 0;
  __syncthreads();
  for (int c0 = 0; c0 < n; c0 += CK_THREADS) {
    const int i = c0 + tid;
    const bool eq = i < n && key(i) == T;
    const unsigned be = __ballot_sync(0xffffffffu, eq);
    if (lane == 0) s_cnt[warp] = __popc(be);
    __syncthreads();
    int off = 0, tot = 0;
    for (int w = 0; w < CK_WARPS; w++) {
      if (w < warp) off += s_cnt[w];
      tot += s_cnt[w];
    }
    const int re = s_eqbase + off + __popc(be & ((1u << lane) - 1u));
    if (eq && re < need) emit(i, ngt + re);
    __syncthreads();
    if (tid == 0) s_eqbase += tot;
    __syncthreads();
  }
  return K;
}

// Stage 1 of the exact sampler on this CTA: the top K of its slice of the
// penalized logits (the values ARGMAX_STAGE1_WGSL compares).
// Not inlined (runs only in exact mode): keeps the step kernels' code small.
__device__ __noinline__ void phase_topk_local(const CkDev& D, Smem& smu, int cta, int ncta) {
  const CkState* st = D.st;
  const bool pen = st->pen_d > 1.0;
  const float penalty = (float)st->pen_milli / 1000.0f;
  const int lo = (int)((long long)cta * D.vocab / ncta), hi = (int)((long long)(cta + 1) * D.vocab / ncta);
  const int K = exact_k(st);
  auto val = [&](int i) {
    const uint32_t id = (uint32_t)(lo + i);
    float v = D.logits[id];
    if (pen && ((D.pen_mask[id >> 5] >> (id & 31)) & 1u)) v = v > 0.f ? v / penalty : v * penalty;
    return v;
  };
  float* ov = D.xval + (size_t)cta * CK_SAMPLE_MAX;
  uint32_t* oi = D.xidx + (size_t)cta * CK_SAMPLE_MAX;
  const int cnt = radix_emit(hi - lo, K, [&](int i) { return fkey(val(i)); },
                             [&](int i, int p) { ov[p] = val(i); oi[p] = (uint32_t)(lo + i); }, smu.sm);
  if (threadIdx.x == 0) D.xcnt[cta] = cnt;
}

// Stage 2 (one CTA, after every CTA's stage 1): the top K of all candidates,
// ordered by id, then the sampler.
__device__ __noinline__ void phase_sample_exact(const CkDev& D, Smem& smu, int ncta) {
  const CkState* st = D.st;
  SmemSm& s = smu.sm;
  int* s_off = s.off;
  int& s_total = s.total;
  const int tid = threadIdx.x;
  const int K = exact_k(st);
  // prefix offsets of the CTAs' lists (CTA order = id order)
  if (tid == 0) {
    int t = 0;
    for (int c = 0; c < ncta && c < 1024; c++) { s_off[c] = t; t += D.xcnt[c]; }
    s_total = t;
  }
  __syncthreads();
  const int M = s_total;
  auto at = [&](int j, int& c, int& p) {   // j-th candidate overall -> (CTA, place)
    int lo = 0, hi = ncta - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (s_off[mid] <= j) lo = mid; else hi = mid - 1;
    }
    c = lo;
    p = j - s_off[lo];
  };
  // each CTA's list holds its keys > T_local before its keys == T_local, so
  // the id order within a list is restored by sorting the final list by id
  for (int i = tid; i < CK_SAMPLE_MAX; i += CK_THREADS) {
    s.val[i] = INFINITY;
    s.idx[i] = 0xffffffffu;
    s.prob[i] = 4294967296.0;
  }
  __syncthreads();
  const double rp = fmax(st->pen_d, 1e-6);
  radix_emit(M, K,
             [&](int j) { int c, p; at(j, c, p); return fkey(D.xval[(size_t)c * CK_SAMPLE_MAX + p]); },
             [&](int j, int pl) {
               int c, p;
               at(j, c, p);
               const float v = D.xval[(size_t)c * CK_SAMPLE_MAX + p];
               const uint32_t id = D.xidx[(size_t)c * CK_SAMPLE_MAX + p];
               s.val[pl] = sample_key(D, v, id, rp);
               s.idx[pl] = isfinite(s.val[pl]) ? id : 0xffffffffu;
               s.prob[pl] = (double)id;   // the reference's list order: by id
             }, s);
  sample_core(D, s);
}
// End of step: clear the penalty set, chain the produced id, advance pos.
__device__ __forceinline__ void phase_finish(int need_logits, const CkDev& D, int cta, uint32_t ep) {
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
    st->epoch = ep + 1;       // tags of the next step differ from this step's
  }
}

// argmax stage 2 -> sampling -> end of step, on CTA 0 in one phase.  `ncta`:
// the CTAs that ran stage 1 (the exact sampler's candidate lists).
template <int EXACT>
__device__ __forceinline__ void phase_select(int need_logits, const CkDev& D, Smem& sm, int cta, uint32_t ep,
                                             int ncta) {
  if (cta != 0) return;
  const CkState* st = D.st;
  if (EXACT && st->exact && st->sampling && D.xval && ncta <= D.xgrid) {
    phase_sample_exact(D, sm, ncta);
  } else {
    phase_argmax2(D, sm, 0);
    __syncthreads();
    phase_sample(D, sm, 0);
  }
  __syncthreads();
  phase_finish(need_logits, D, 0, ep);
}

// The LM head's prologue (RMS_NORM_WGSL over the last residual, or Gemma's
// post-FFN norm + residual add + final norm) on CTA 0, written as plain
// floats for the streaming head kernel.
__device__ __forceinline__ void phase_fnorm(const MvPhase& P, SmemMv& s, const CkDev& D, int cta, uint32_t ep) {
  if (cta != 0) return;
  build_x(P.pro, P.k, s, cta, ep, &D.st->err, &D.st->abort_flag);
  for (int i = threadIdx.x; i < P.k; i += CK_THREADS) D.xhead[i] = s.xf[i];
}

// ---------------------------------------------------------------------------
template <int EXACT, unsigned TM, int AE, int OT>
__device__ __forceinline__ void run_phase(const Phase* ph, int i, Smem& sm, Ring& R, const CkDev& D, int cta,
                                          int ncta, int pos, uint32_t ep) {
  const Phase& p = ph[i];
  unsigned long long* tp =
      !D.trace ? nullptr
      : (i == 2 && cta < 1024) ? D.trace + CK_TRACE_CTA_BASE + cta * 16 + 8
      : (cta == 0 && i < 512) ? D.trace + CK_TRACE_STAGE_BASE + i * 8 : nullptr;
  if (p.kind == PH_MATVEC && ph[i + 1].kind == PH_ATTN) attn_prefetch<AE, OT>(ph[i + 1].at, cta, ncta, pos);
  switch (p.kind) {
    case PH_EMBED: phase_embed(p.em, D, cta, ncta, pos, ep); break;
    case PH_MATVEC: phase_matvec<TM>(p.mv, sm, R, cta, &D.st->err, &D.st->abort_flag, tp, ep); break;
    case PH_ATTN: phase_attn<AE, OT>(p.at, sm, D, cta, ncta, pos, tp, ep); break;
    case PH_ARGMAX1: phase_argmax1<EXACT>(D, sm, cta, ncta); break;
    case PH_ARGMAX2: phase_argmax2(D, sm, cta); break;
    case PH_SAMPLE: phase_sample(D, sm, cta); break;
    case PH_FINISH: phase_finish(p.need_logits, D, cta, ep); break;
    case PH_SELECT: phase_select<EXACT>(p.need_logits, D, sm, cta, ep, ncta); break;
    case PH_FNORM: phase_fnorm(p.mv, sm.mv, D, cta, ep); break;
  }
}

// Dynamic shared memory: the tile ring (2 x CK_TILE_BYTES) + 2 mbarriers.

// One launch per phase (CUDA-graph mode): one kernel per phase kind so each
// gets its own register allocation.
__global__ void __launch_bounds__(CK_THREADS, 1) k_mv(const Phase* __restrict__ ph, CkDev D) {
  __shared__ Smem sm;
  unsigned long long* tr = (D.trace && threadIdx.x == 0 && blockIdx.x < 1024)
                               ? D.trace + CK_TRACE_MV_BASE + blockIdx.x * 8 : nullptr;
  if (tr) tr[0] = gtimer();
  Ring R;
  const Phase* sph = launch_start(R, ph, 1, blockIdx.x, &D.st->err, &D.st->abort_flag, D.l2_keep);
  if (!sph) return;
  if (tr) tr[1] = gtimer();
  unsigned long long* tp = (D.trace && blockIdx.x == 0 && sph->index < 512)
                               ? D.trace + CK_TRACE_STAGE_BASE + sph->index * 8 : nullptr;
  phase_matvec(sph->mv, sm, R, blockIdx.x, &D.st->err, &D.st->abort_flag, tp, D.st->epoch);
  if (tr) tr[2] = gtimer();
}
__global__ void __launch_bounds__(CK_THREADS, 1) k_attn(const Phase* __restrict__ ph, CkDev D) {
  __shared__ Smem sm;
  phase_attn(ph->at, sm, D, blockIdx.x, gridDim.x, D.st->pos, nullptr, D.st->epoch);
}
__global__ void __launch_bounds__(CK_THREADS, 1) k_misc(const Phase* __restrict__ ph, CkDev D) {
  __shared__ Smem sm;
  const Phase& p = *ph;
  // every CTA reads the epoch before CTA 0's step end can advance it: the
  // step-end phases run on a one-CTA grid
  const uint32_t ep = D.st->epoch;
  switch (p.kind) {
    case PH_EMBED: phase_embed(p.em, D, blockIdx.x, gridDim.x, D.st->pos, ep); break;
    case PH_ARGMAX1: phase_argmax1<1>(D, sm, blockIdx.x, gridDim.x); break;
    case PH_ARGMAX2: phase_argmax2(D, sm, blockIdx.x); break;
    case PH_SAMPLE: phase_sample(D, sm, blockIdx.x); break;
    case PH_FINISH: phase_finish(p.need_logits, D, blockIdx.x, ep); break;
    case PH_SELECT: phase_select<1>(p.need_logits, D, sm, blockIdx.x, ep, (ph - 1)->grid); break;
    case PH_FNORM: phase_fnorm(p.mv, sm.mv, D, blockIdx.x, ep); break;
  }
}

__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Grid-wide barrier for the cooperative megakernel.  Bounded: after ~2^21
// polls (seconds) the CTA flags CK_DERR_BARRIER + abort and returns false;
// every other CTA sees the abort flag and returns too.
__device__ __forceinline__ bool grid_sync(CkState* st, unsigned target) {
  __shared__ int s_ok;
  __syncthreads();
  if (threadIdx.x == 0) {
    // release: every write of this CTA before the __syncthreads above is
    // visible to a CTA whose acquire load sees the count
    asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(&st->bar) : "memory");
    int ok = 1;
    unsigned spins = 0;
    while (ld_acquire_u32(&st->bar) < target) {
      if (++spins > (1u << 23)) {
        atomicOr(&st->err, CK_DERR_BARRIER);
        atomicExch(&st->abort_flag, 1);
        ok = 0;
        break;
      }
      if ((spins & 255u) == 0 && *(volatile int*)&st->abort_flag) { ok = 0; break; }
    }
    s_ok = ok;
  }
  __syncthreads();
  return s_ok != 0;
}

// Whole step in one cooperative launch (megakernel mode).  Phases hand data
// over as tagged words, so a CTA moves to its next phase as soon as its own
// work is done; a grid barrier remains only where a phase is marked
// barrier_after (the LM head before argmax stage 1, stage 1 before select),
// whose outputs are plain.
// EXACT: the whole-vocabulary sampler is compiled in; TM / AE: the block
// types and the attention shape compiled in (CK_TM_ALL / 0: all, chosen at
// run time), see mega_kernel on the host; OT: the attention's mergers on the
// top CTAs (attn_unit_top).
template <int EXACT, unsigned TM, int AE, int OT = 0>
__global__ void __launch_bounds__(CK_THREADS, 1) k_mega(const Phase* __restrict__ ph, int nph, CkDev D) {
  __shared__ Smem sm;
  const int pos = D.st->pos;         // constant for the whole step (phase_finish runs last)
  const uint32_t ep = D.st->epoch;   // read before any CTA can reach the step end
  Ring R;
  const Phase* sph = launch_start(R, ph, nph, blockIdx.x, &D.st->err, &D.st->abort_flag, D.l2_keep);
  if (!sph) return;
  unsigned target = 0;
  const bool tr = D.trace && blockIdx.x == 0 && threadIdx.x == 0;
  // per-CTA stamps of phases 1..4: end of the phase and exit of its barrier
  unsigned long long* ct = (D.trace && threadIdx.x == 0 && blockIdx.x < 1024)
                               ? D.trace + CK_TRACE_CTA_BASE + blockIdx.x * 16 : nullptr;
#pragma unroll 1
  for (int i = 0; i < nph; i++) {
    if (tr && 2 * i + 1 < CK_TRACE_MV_BASE) D.trace[2 * i] = gtimer();
    run_phase<EXACT, TM, AE, OT>(sph, i, sm, R, D, blockIdx.x, gridDim.x, pos, ep);
    if (tr && 2 * i + 1 < CK_TRACE_MV_BASE) D.trace[2 * i + 1] = gtimer();
    if (ct && i >= 1 && i <= 4) ct[i - 1] = gtimer();
    if (!R.ok) return;
    if (i + 1 < nph && sph[i].barrier_after) {
      target += gridDim.x;
      if (!grid_sync(D.st, target)) return;
    }
    if (ct && i >= 1 && i <= 4) ct[i + 3] = gtimer();
  }
}
