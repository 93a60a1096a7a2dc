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
  unsigned long long* trace;  // optional globaltimer stamps (null = off)
};

__device__ __forceinline__ unsigned long long gtimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
// Trace layout: k_mega: [phase][2] (CTA 0: phase start / phase end);
// k_mv: [CK_TRACE_MV_BASE + cta * 8 + stage].
#define CK_TRACE_MV_BASE 4096
#define CK_TRACE_STAGE_BASE (CK_TRACE_MV_BASE + 8 * 1024)
#define CK_TRACE_SLOTS (CK_TRACE_STAGE_BASE + 8 * 512)
// sub-stage stamps of phase i on CTA 0: [CK_TRACE_STAGE_BASE + i * 8 + stage]
__device__ __forceinline__ void stage_mark(unsigned long long* tp, int stage) {
  if (tp && threadIdx.x == 0) tp[stage] = gtimer();
}

enum { PRO_COPY = 0, PRO_NORM = 1, PRO_SILU = 2, PRO_GELU = 3, PRO_GEMMA = 4 };
enum { PH_EMBED = 0, PH_MATVEC = 1, PH_ATTN = 2, PH_ARGMAX1 = 3, PH_ARGMAX2 = 4, PH_SAMPLE = 5, PH_FINISH = 6,
       PH_SELECT = 7 };

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
  const float* inv_freq;    // [head_dim/2] theta^(-2d/head_dim) of this layer
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

struct __align__(16) Phase {
  int kind;
  int grid;                 // CTAs for a standalone launch
  union {
    MvPhase mv;
    AttnPhase at;
    EmbedPhase em;
    int need_logits;        // PH_FINISH
  };
};
static_assert(sizeof(Phase) % 16 == 0, "phase descriptors are bulk-copied");

// ---------------------------------------------------------------------------
struct SmemMv {
  float xf[CK_KMAX];
  float wf[CK_KMAX];
  int8_t xh[CK_KMAX];
  int8_t xl[CK_KMAX];
  float sx[CK_KMAX / 32];
  int s16[CK_KMAX / 16];
  float red[CK_WARPS * 2];
};
struct SmemAt {
  float qs[CK_GMAX * CK_HDMAX];
  float raw[CK_GMAX * CK_HDMAX];   // q rows as produced by the projection
  float kvw[4][CK_HDMAX];          // k, v, q-norm weight, k-norm weight
  float wacc[CK_WARPS * CK_HDMAX];
  float wm[CK_WARPS];
  float wl[CK_WARPS];
  float2 cs[CK_HDMAX / 2];
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
  float* wf = s.wf;
  if (p.kind == PRO_COPY) {
    for (int i = tid; i < k; i += CK_THREADS) xf[i] = p.a[i];
  } else if (p.kind == PRO_NORM) {
    // activation and weight loads issued together; one reduction
    float ss = 0.f;
    for (int i = tid; i < k; i += CK_THREADS) {
      float v = p.a[i], w = p.w0[i];
      xf[i] = v;
      wf[i] = w;
      ss += v * v;
    }
    float inv = rms_inv(block_sum(ss, s.red), k, p.eps);
    for (int i = tid; i < k; i += CK_THREADS) xf[i] = (xf[i] * inv) * wf[i];
  } else if (p.kind == PRO_SILU) {
    for (int i = tid; i < k; i += CK_THREADS) {
      float g = p.a[i], u = p.b[i];
      xf[i] = (g / (1.0f + expf(-g))) * u;
    }
  } else if (p.kind == PRO_GELU) {
    for (int i = tid; i < k; i += CK_THREADS) {
      float g = p.a[i], u = p.b[i];
      xf[i] = gelu_tanh(g) * u;
    }
  } else {  // PRO_GEMMA: t = rmsnorm(a) * w1; h = clamp(rin + t); x = rmsnorm(h) * w0
    constexpr int PER = CK_KMAX / CK_THREADS;
    float rr[PER], ww[PER];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < PER; j++) {
      int i = tid + j * CK_THREADS;
      if (i < k) {
        float v = p.a[i];
        xf[i] = v;
        wf[i] = p.w1[i];
        rr[j] = p.rin[i];
        ww[j] = p.w0[i];
        ss += v * v;
      }
    }
    float inv = rms_inv(block_sum(ss, s.red), k, p.eps);
    float ss2 = 0.f;
#pragma unroll
    for (int j = 0; j < PER; j++) {
      int i = tid + j * CK_THREADS;
      if (i < k) {
        float t = (xf[i] * inv) * wf[i];
        float h = fminf(fmaxf(rr[j] + t, -65000.0f), 65000.0f);
        xf[i] = h;
        if (cta == 0) p.rout[i] = h;
        ss2 += h * h;
      }
    }
    float inv2 = rms_inv(block_sum(ss2, s.red), k, p.eps);
#pragma unroll
    for (int j = 0; j < PER; j++) {
      int i = tid + j * CK_THREADS;
      if (i < k) xf[i] = (xf[i] * inv2) * ww[j];
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

// ---------------------------------------------------------------------------
// Weight streaming: each CTA owns a contiguous row range of every matvec
// segment (rows are self-contained and 16-byte aligned in the device layout),
// packed into tiles of at most CK_TILE_BYTES.  One issuer thread copies tiles into a
// two-buffer shared-memory ring with cp.async.bulk (TMA bulk copy, no
// multicast) completing on an mbarrier; the ring runs ahead across phases, so
// the next matvec's weights are in flight while this CTA is in a grid barrier
// or an attention phase.  Consumers read the tile from shared memory.
#define CK_TILE_BYTES (64 * 1024)
#define CK_TILE_PIECES 4
#define CK_ISSUER (CK_THREADS - 32)   // lane 0 of the last warp copies tiles

struct Piece {
  int seg, r0, r1;
  uint32_t soff;
};
struct Tile {
  int phase, npc;
  uint32_t bytes;
  Piece pc[CK_TILE_PIECES];
};
struct Cursor {
  int phase, seg, row;
};

struct Ring {
  uint8_t* buf;            // 2 x CK_TILE_BYTES, 128-byte aligned
  uint64_t* full;          // 2 mbarriers
  const Phase* ph;
  int nph;
  Cursor issue;            // issuer thread: next tile to copy
  unsigned issued;         // issuer thread: tiles copied so far
  unsigned consumed;       // every thread: tiles consumed so far
  int ok;                  // 0 once a wait gave up
};

// Contiguous row range of a CTA (n * ncta < 2^31 for every model handled).
__device__ __forceinline__ void seg_range(const MvSeg& S, int cta, int ncta, int& lo, int& hi) {
  lo = (S.n * cta) / ncta;
  hi = (S.n * (cta + 1)) / ncta;
}

// Next tile from cursor `c` (phases [c.phase, last)), false when none.
// `last` bounds the search: nph for the issuer, phase + 1 for consumers.
__device__ bool next_tile(const Phase* ph, int last, int cta, int ncta, Cursor& c, Tile& t) {
  while (c.phase < last) {
    const Phase& p = ph[c.phase];
    if (p.kind != PH_MATVEC) {
      c.phase++; c.seg = 0; c.row = -1;
      continue;
    }
    const MvPhase& m = p.mv;
    t.phase = c.phase;
    t.npc = 0;
    t.bytes = 0;
    while (c.seg < m.nseg && t.npc < CK_TILE_PIECES) {
      int lo, hi;
      seg_range(m.seg[c.seg], cta, ncta, lo, hi);
      if (c.row < lo) c.row = lo;
      if (c.row >= hi) { c.seg++; c.row = -1; continue; }
      uint32_t rb = m.seg[c.seg].L.row_bytes;
      int fit = (int)((CK_TILE_BYTES - t.bytes) / rb);
      if (fit <= 0) break;
      int take = min(fit, hi - c.row);
      t.pc[t.npc].seg = c.seg;
      t.pc[t.npc].r0 = c.row;
      t.pc[t.npc].r1 = c.row + take;
      t.pc[t.npc].soff = t.bytes;
      t.npc++;
      t.bytes += (uint32_t)take * rb;
      c.row += take;
    }
    if (t.npc > 0) return true;
    c.phase++; c.seg = 0; c.row = -1;
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
// Same, marking the lines evict-first in L2: streamed weights are read once
// per token and should not push activations, norms or the KV cache out.
__device__ __forceinline__ void bulk_g2s_stream(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(pol)
      : "memory");
}

// issuer thread: copy the next tile (if any) into buffer issued & 1
__device__ void ring_issue(Ring& R, int cta, int ncta) {
  Tile t;
  if (!next_tile(R.ph, R.nph, cta, ncta, R.issue, t)) return;
  int b = R.issued & 1;
  uint64_t* bar = R.full + b;
  mbar_expect_tx(bar, t.bytes);
  const MvPhase& m = R.ph[t.phase].mv;
  for (int i = 0; i < t.npc; i++) {
    const MvSeg& S = m.seg[t.pc[i].seg];
    uint32_t rb = S.L.row_bytes;
    bulk_g2s_stream(R.buf + (size_t)b * CK_TILE_BYTES + t.pc[i].soff, S.w + (size_t)t.pc[i].r0 * rb,
                    (uint32_t)(t.pc[i].r1 - t.pc[i].r0) * rb, bar);
  }
  R.issued++;
}

// Shared-memory layout of the streaming kernels (dynamic part):
//   [tile buffer 0][tile buffer 1][3 mbarriers, 128 B][phase descriptors]
#define CK_DYN_BARS (2 * CK_TILE_BYTES)
#define CK_DYN_PHASES (2 * CK_TILE_BYTES + 128)
#define CK_PHASE_SMEM_MAX (48 * 1024)
#define CK_DYN_SMEM_MAX (CK_DYN_PHASES + CK_PHASE_SMEM_MAX)

// Start of a launch: init the barriers, stage the phase descriptors in shared
// memory with one bulk copy (every later descriptor read is a shared-memory
// read), then put the first two weight tiles in flight.  Returns the staged
// descriptors, or null when the wait gave up.
__device__ const Phase* launch_start(Ring& R, uint8_t* dyn, const Phase* gph, int nph, int cta, int ncta,
                                     int* err, int* abort_flag) {
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
  __syncthreads();
  unsigned spins = 0;
  while (!mbar_try_wait(bars + 2, 0)) {
    if (++spins > (1u << 20)) {
      atomicOr(err, CK_DERR_BARRIER);
      atomicExch(abort_flag, 1);
      return nullptr;
    }
  }
  R.buf = dyn;
  R.full = bars;
  R.ph = sph;
  R.nph = nph;
  R.issue.phase = 0; R.issue.seg = 0; R.issue.row = -1;
  R.issued = 0;
  R.consumed = 0;
  R.ok = 1;
  if (threadIdx.x == CK_ISSUER) {
    ring_issue(R, cta, ncta);
    ring_issue(R, cta, ncta);
  }
  return sph;
}

// Wait for tile `consumed` (bounded: ~seconds, then flags and gives up).
__device__ bool ring_wait(Ring& R, int* err, int* abort_flag) {
  uint64_t* bar = R.full + (R.consumed & 1);
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
__device__ __forceinline__ void ring_release(Ring& R, int cta, int ncta) {
  __syncthreads();
  R.consumed++;
  if (threadIdx.x == CK_ISSUER && R.issued < R.consumed + 2) ring_issue(R, cta, ncta);
}

// Rows of one tile piece, read from shared memory.  With one unit per lane
// (ONE) the lane's x unit stays in registers for the whole piece and a warp
// step handles two rows so their unpacks, dots and reductions overlap; with
// 2-3 units per lane the x units are re-read from shared memory per unit (the
// units of a row already overlap) to stay inside the register budget.  The
// block type is a runtime switch inside the unpack: compiling the row loop
// per type multiplies register pressure past the 128-register budget.
template <bool ONE>
__device__ __forceinline__ void mv_piece(const MvSeg& S, const uint8_t* base, int r0, int nrows, const SmemMv& s) {
  constexpr int R = ONE ? 2 : 1;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int U = S.L.U;
  const int T = S.L.type;
  const int upl = ONE ? 1 : (U + 31) >> 5;
  const uint32_t rb = S.L.row_bytes;
  float* __restrict__ out = S.out;
  const float* __restrict__ add = S.add;
  if (warp >= nrows) return;
  XUnit x0;
  if (ONE && lane < U) load_xunit(s, lane, x0);
  for (int r = warp; r < nrows; r += R * CK_WARPS) {
    float acc[R];
#pragma unroll
    for (int i = 0; i < R; i++) {
      acc[i] = 0.f;
      const int rr = r + i * CK_WARPS;
      if (rr < nrows) {
        const uint8_t* row = base + (size_t)rr * rb;
        if (ONE) {
          if (lane < U) {
            U8 u;
            unpack_unit<false>(T, row, S.L, lane, u);
            acc[i] += unit_dot8(u, x0);
          }
        } else {
#pragma unroll 1
          for (int j = 0; j < upl; j++) {
            int c = lane + 32 * j;
            if (c < U) {
              U8 u;
              unpack_unit<false>(T, row, S.L, c, u);
              XUnit xj;
              load_xunit(s, c, xj);
              acc[i] += unit_dot8(u, xj);
            }
          }
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
      for (int i = 0; i < R; i++) acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], o);
    float v = acc[0];
#pragma unroll
    for (int i = 1; i < R; i++)
      if (lane == i) v = acc[i];
    const int rr = r + lane * CK_WARPS;
    if (lane < R && rr < nrows) out[r0 + rr] = add ? add[r0 + rr] + v : v;
  }
}

__device__ __forceinline__ void mv_run(const MvPhase& P, int phase_idx, SmemMv& s, Ring& R, int cta, int ncta,
                                    int* err, int* abort_flag, unsigned long long* tp) {
  stage_mark(tp, 0);
  build_x(P.pro, P.k, s, cta);
  stage_mark(tp, 1);
  quant_x(P.k, s);
  stage_mark(tp, 2);
  int ntile = 0;
  const int upl = (P.k + 1023) >> 10;
  Cursor cur;
  cur.phase = phase_idx; cur.seg = 0; cur.row = -1;
  Tile t;
  while (next_tile(R.ph, phase_idx + 1, cta, ncta, cur, t)) {
    if (!ring_wait(R, err, abort_flag)) { R.ok = 0; return; }
    if (ntile == 0) stage_mark(tp, 3);
    const uint8_t* tb = R.buf + (size_t)(R.consumed & 1) * CK_TILE_BYTES;
    for (int i = 0; i < t.npc; i++) {
      const MvSeg& S = P.seg[t.pc[i].seg];
      const uint8_t* base = tb + t.pc[i].soff;
      int r0 = t.pc[i].r0, nrows = t.pc[i].r1 - t.pc[i].r0;
      if (upl <= 1) mv_piece<true>(S, base, r0, nrows, s);
      else mv_piece<false>(S, base, r0, nrows, s);
    }
    if (ntile == 0) stage_mark(tp, 4);
    ring_release(R, cta, ncta);
    if (ntile == 0) stage_mark(tp, 5);
    ntile++;
  }
  stage_mark(tp, 6);
}

__device__ __forceinline__ void phase_matvec(const MvPhase& P, int phase_idx, Smem& sm, Ring& R, int cta,
                                             int ncta, int* err, int* abort_flag, unsigned long long* tp = nullptr) {
  mv_run(P, phase_idx, sm.mv, R, cta, ncta, err, abort_flag, tp);
}

// ---------------------------------------------------------------------------
// Embedding (GGUF_*_EMBEDDING_WGSL, :2615-2866): row tokens[pos] of the
// (tied) table dequantized in WGSL order, times EMBEDDING_SCALE.  Also marks
// the repetition-penalty id set when this step computes logits.
__device__ __forceinline__ void phase_embed(const EmbedPhase& P, const CkDev& D, int cta, int ncta, int pos) {
  const CkState* st = D.st;
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

template <int E>
__device__ __forceinline__ void attn_unit(const AttnPhase& P, SmemAt& s, int kvh, int split, int pos,
                                          unsigned long long* tp) {
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

  // --- every input of this unit in one round of loads ----------------------
  stage_mark(tp, 0);
  for (int d = tid; d < (hd >> 1); d += CK_THREADS) {
    // angle = pos * theta^(-2d/hd) (rope_angle, :2885-2888); the power is the
    // per-layer table built at load time with the same powf
    float ang = (float)pos * P.inv_freq[d];
    float sn, cn;
    sincosf(ang, &sn, &cn);
    s.cs[d] = make_float2(cn, sn);
  }
  for (int i = tid; i < G * hd; i += CK_THREADS) s.raw[i] = P.q[(size_t)kvh * G * hd + i];
  for (int d = tid; d < hd; d += CK_THREADS) {
    if (owner) {
      s.kvw[0][d] = P.k[(size_t)kvh * hd + d];
      s.kvw[1][d] = P.v[(size_t)kvh * hd + d];
      if (P.kw) s.kvw[3][d] = P.kw[d];
    }
    if (P.qw) s.kvw[2][d] = P.qw[d];
  }
  __syncthreads();
  // --- per-head 1/rms of q (and k) for the QK-norm -----------------------
  if (P.qw) {
    for (int g = warp; g < G + (owner ? 1 : 0); g += CK_WARPS) {
      const float* src = g < G ? s.raw + g * hd : s.kvw[0];
      float ss = 0.f;
      for (int d = lane; d < hd; d += 32) ss += src[d] * src[d];
      ss = warp_sum(ss);
      if (lane == 0) s.inv[g] = rms_inv(ss, hd, P.eps);
    }
    __syncthreads();
  }
  // --- q: norm + rope into shared memory; owner: k/v into the cache --------
  for (int g = 0; g < G; g++)
    rope_head(s.raw + g * hd, P.qw ? s.kvw[2] : nullptr, P.qw ? s.inv[g] : 1.f, s.qs + g * hd, hd, P.interleaved,
              s.cs, tid, CK_THREADS);
  if (owner) {
    float* kst = s.wacc;  // scratch for the rotated k row
    rope_head(s.kvw[0], P.kw ? s.kvw[3] : nullptr, P.kw ? s.inv[G] : 1.f, kst, hd, P.interleaved, s.cs, tid,
              CK_THREADS);
    __syncthreads();
    size_t cb = ((size_t)kvh * P.ctx + pos) * hd;
    for (int d = tid; d < hd; d += CK_THREADS) {
      float kv = kst[d], vv = s.kvw[1][d];
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
  stage_mark(tp, 1);

  // --- online softmax: warps split into G groups, one q head per group -----
  const int wpg = CK_WARPS / G;      // warps per head (G <= 8)
  const int g = warp / wpg, sub = warp % wpg;
  float q[E], acc[E], m = -INFINITY, l = 0.f;
#pragma unroll
  for (int e = 0; e < E; e++) {
    q[e] = g < G ? s.qs[g * hd + lane * E + e] : 0.f;
    acc[e] = 0.f;
  }
  if (g < G) {
    const size_t base = (size_t)kvh * P.ctx * hd + lane * E;
    int t = t0 + sub;
    for (; t + wpg < t1; t += 2 * wpg) {   // two positions in flight
      float k0[E], v0[E], k1[E], v1[E];
      load_kv<E>(P.kc, P.kv_f32, base + (size_t)t * hd, k0);
      load_kv<E>(P.kc, P.kv_f32, base + (size_t)(t + wpg) * hd, k1);
      load_kv<E>(P.vc, P.kv_f32, base + (size_t)t * hd, v0);
      load_kv<E>(P.vc, P.kv_f32, base + (size_t)(t + wpg) * hd, v1);
      float d0 = 0.f, d1 = 0.f;
#pragma unroll
      for (int e = 0; e < E; e++) { d0 += q[e] * k0[e]; d1 += q[e] * k1[e]; }
      float s0 = warp_sum(d0) * P.scale, s1 = warp_sum(d1) * P.scale;
      float mn = fmaxf(m, fmaxf(s0, s1));
      float c = expf(m - mn), p0 = expf(s0 - mn), p1 = expf(s1 - mn);
      l = l * c + p0 + p1;
#pragma unroll
      for (int e = 0; e < E; e++) acc[e] = acc[e] * c + p0 * v0[e] + p1 * v1[e];
      m = mn;
    }
    if (t < t1) {
      float k0[E], v0[E];
      load_kv<E>(P.kc, P.kv_f32, base + (size_t)t * hd, k0);
      load_kv<E>(P.vc, P.kv_f32, base + (size_t)t * hd, v0);
      float d0 = 0.f;
#pragma unroll
      for (int e = 0; e < E; e++) d0 += q[e] * k0[e];
      float s0 = warp_sum(d0) * P.scale;
      float mn = fmaxf(m, s0);
      float c = expf(m - mn), p0 = expf(s0 - mn);
      l = l * c + p0;
#pragma unroll
      for (int e = 0; e < E; e++) acc[e] = acc[e] * c + p0 * v0[e];
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
  if (S == 1) {   // one split covers the context: no partials, no merge
    for (int i = tid; i < G * hd; i += CK_THREADS) {
      int gg = i / hd, d = i % hd;
      float M = -INFINITY;
      for (int w = gg * wpg; w < gg * wpg + wpg; w++) M = fmaxf(M, s.wm[w]);
      float L = 0.f, A = 0.f;
      for (int w = gg * wpg; w < gg * wpg + wpg; w++) {
        float wm = s.wm[w];
        if (wm == -INFINITY) continue;
        float f = expf(wm - M);
        L += s.wl[w] * f;
        A += s.wacc[w * CK_HDMAX + d] * f;
      }
      P.out[(size_t)(kvh * G + gg) * hd + d] = A / L;
    }
    stage_mark(tp, 3);
    return;
  }
  float* part = P.part + ((size_t)kvh * P.smax + split) * G * (hd + 2);
  for (int i = tid; i < G * hd; i += CK_THREADS) {
    int gg = i / hd, d = i % hd;
    float M = -INFINITY;
    for (int w = gg * wpg; w < gg * wpg + wpg; w++) M = fmaxf(M, s.wm[w]);
    float L = 0.f, A = 0.f;
    for (int w = gg * wpg; w < gg * wpg + wpg; w++) {
      float wm = s.wm[w];
      if (wm == -INFINITY) continue;
      float f = expf(wm - M);
      L += s.wl[w] * f;
      A += s.wacc[w * CK_HDMAX + d] * f;
    }
    part[gg * (hd + 2) + 2 + d] = A;
    if (d == 0) {
      part[gg * (hd + 2)] = M;
      part[gg * (hd + 2) + 1] = L;
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
    int gg = i / hd, d = i % hd;
    float M = -INFINITY;
    for (int sp = 0; sp < S; sp++) M = fmaxf(M, __ldcg(pk + ((size_t)sp * G + gg) * (hd + 2)));
    float L = 0.f, A = 0.f;
    for (int sp = 0; sp < S; sp++) {
      const float* pp = pk + ((size_t)sp * G + gg) * (hd + 2);
      float f = expf(__ldcg(pp) - M);
      L += __ldcg(pp + 1) * f;
      A += __ldcg(pp + 2 + d) * f;
    }
    P.out[(size_t)(kvh * G + gg) * hd + d] = A / L;
  }
  if (tid == 0) P.counter[kvh] = 0u;
}

__device__ __forceinline__ void phase_attn(const AttnPhase& P, Smem& sm, const CkDev& D, int cta, int ncta, int pos,
                                           unsigned long long* tp = nullptr) {
  // split-major: the active split 0 units of every kv head land on
  // different CTAs even when the context needs one split only
  int units = P.kvh * P.smax;
  for (int u = cta; u < units; u += ncta) {
    int kvh = u % P.kvh, split = u / P.kvh;
    unsigned long long* up = (tp && u == cta) ? tp : nullptr;
    if (P.hd == 64) attn_unit<2>(P, sm.at, kvh, split, pos, up);
    else if (P.hd == 128) attn_unit<4>(P, sm.at, kvh, split, pos, up);
    else attn_unit<8>(P, sm.at, kvh, split, pos, up);
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
    if (threadIdx.x < 256 && i < (uint32_t)D.vocab) {
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

// argmax stage 2 -> sampling -> end of step, on CTA 0 in one phase.
__device__ __forceinline__ void phase_select(int need_logits, const CkDev& D, Smem& sm, int cta) {
  if (cta != 0) return;
  phase_argmax2(D, sm, 0);
  __syncthreads();
  phase_sample(D, sm, 0);
  __syncthreads();
  phase_finish(need_logits, D, 0);
}

// ---------------------------------------------------------------------------
__device__ __forceinline__ void run_phase(const Phase* ph, int i, Smem& sm, Ring& R, const CkDev& D, int cta,
                                          int ncta, int pos) {
  const Phase& p = ph[i];
  unsigned long long* tp =
      (D.trace && cta == 0 && i < 512) ? D.trace + CK_TRACE_STAGE_BASE + i * 8 : nullptr;
  switch (p.kind) {
    case PH_EMBED: phase_embed(p.em, D, cta, ncta, pos); break;
    case PH_MATVEC: phase_matvec(p.mv, i, sm, R, cta, ncta, &D.st->err, &D.st->abort_flag, tp); break;
    case PH_ATTN: phase_attn(p.at, sm, D, cta, ncta, pos, tp); break;
    case PH_ARGMAX1: phase_argmax1(D, sm, cta, ncta); break;
    case PH_ARGMAX2: phase_argmax2(D, sm, cta); break;
    case PH_SAMPLE: phase_sample(D, sm, cta); break;
    case PH_FINISH: phase_finish(p.need_logits, D, cta); break;
    case PH_SELECT: phase_select(p.need_logits, D, sm, cta); break;
  }
}

// Dynamic shared memory: the tile ring (2 x CK_TILE_BYTES) + 2 mbarriers.

// One launch per phase (CUDA-graph mode): one kernel per phase kind so each
// gets its own register allocation.
__global__ void __launch_bounds__(CK_THREADS, 1) k_mv(const Phase* __restrict__ ph, CkDev D) {
  extern __shared__ __align__(128) uint8_t dyn[];
  __shared__ Smem sm;
  unsigned long long* tr = (D.trace && threadIdx.x == 0 && blockIdx.x < 1024)
                               ? D.trace + CK_TRACE_MV_BASE + blockIdx.x * 8 : nullptr;
  if (tr) tr[0] = gtimer();
  Ring R;
  const Phase* sph = launch_start(R, dyn, ph, 1, blockIdx.x, gridDim.x, &D.st->err, &D.st->abort_flag);
  if (!sph) return;
  if (tr) tr[1] = gtimer();
  phase_matvec(sph->mv, 0, sm, R, blockIdx.x, gridDim.x, &D.st->err, &D.st->abort_flag);
  if (tr) tr[2] = gtimer();
}
__global__ void __launch_bounds__(CK_THREADS, 1) k_attn(const Phase* __restrict__ ph, CkDev D) {
  __shared__ Smem sm;
  phase_attn(ph->at, sm, D, blockIdx.x, gridDim.x, D.st->pos);
}
__global__ void __launch_bounds__(CK_THREADS, 1) k_misc(const Phase* __restrict__ ph, CkDev D) {
  __shared__ Smem sm;
  const Phase& p = *ph;
  switch (p.kind) {
    case PH_EMBED: phase_embed(p.em, D, blockIdx.x, gridDim.x, D.st->pos); break;
    case PH_ARGMAX1: phase_argmax1(D, sm, blockIdx.x, gridDim.x); break;
    case PH_ARGMAX2: phase_argmax2(D, sm, blockIdx.x); break;
    case PH_SAMPLE: phase_sample(D, sm, blockIdx.x); break;
    case PH_FINISH: phase_finish(p.need_logits, D, blockIdx.x); break;
    case PH_SELECT: phase_select(p.need_logits, D, sm, blockIdx.x); break;
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
__device__ bool grid_sync(CkState* st, unsigned target) {
  __shared__ int s_ok;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    atomicAdd(&st->bar, 1u);
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

// Whole step in one cooperative launch (megakernel mode).
__global__ void __launch_bounds__(CK_THREADS, 1) k_mega(const Phase* __restrict__ ph, int nph, CkDev D) {
  extern __shared__ __align__(128) uint8_t dyn[];
  __shared__ Smem sm;
  const int pos = D.st->pos;   // constant for the whole step (phase_finish runs last)
  Ring R;
  const Phase* sph = launch_start(R, dyn, ph, nph, blockIdx.x, gridDim.x, &D.st->err, &D.st->abort_flag);
  if (!sph) return;
  unsigned target = 0;
  const bool tr = D.trace && blockIdx.x == 0 && threadIdx.x == 0;
  for (int i = 0; i < nph; i++) {
    if (tr && 2 * i + 1 < CK_TRACE_MV_BASE) D.trace[2 * i] = gtimer();
    run_phase(sph, i, sm, R, D, blockIdx.x, gridDim.x, pos);
    if (tr && 2 * i + 1 < CK_TRACE_MV_BASE) D.trace[2 * i + 1] = gtimer();
    if (!R.ok) return;
    if (i + 1 < nph) {
      target += gridDim.x;
      if (!grid_sync(D.st, target)) return;
    }
  }
}
