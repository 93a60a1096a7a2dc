// Streaming decode step: one token of LlamaWgslEngine.runToken
// (llama-wgsl-runtime.ts:1025-1150) in one persistent cooperative launch,
// laid out for the latency of a 148-SM B200 rather than for its bandwidth.
//
// At bs=1 a small decoder's weights stream from HBM in a fraction of the
// time the step's chain of dependent hand-offs takes (five per layer), so
// the kernel keeps the weights off that chain and makes each hand-off cheap:
//
// * Weights.  Warp 15 of every CTA is a producer: it walks the phases ahead
//   of the compute warps and copies the CTA's rows of every matvec into a
//   ring of SK_NSLOT shared-memory slots (cp.async.bulk into this CTA's
//   own shared memory, completing on the slot's mbarrier), limited only by free slots, so a
//   phase's weights are resident before its input exists.  The compute
//   warps release a slot through its "empty" mbarrier.
// * Hand-offs.  Every activation element is a 64-bit word, value low and
//   tag (step epoch << 10 | writer phase) high, stored in one single-copy-
//   atomic store; a consumer polls exactly the words it needs.  Producer CTA
//   c writes its rows into its own segment of 2^sh words (whole 128-byte
//   lines), so every line is written once per phase by one CTA.
// * Residual.  Every CTA keeps the whole residual vector in shared memory
//   and applies each sub-layer's output to it in the prologue of the phase
//   that reads it (residual add, gemma3's post-norm + clamp), so no phase
//   waits on a residual word after its dot products.
// * Work.  A tile's rows are spread over the 15 compute warps (several rows
//   per warp reduce their partial sums together; short tiles split rows
//   over warps), the dp4a unit dot of ck_layout.cuh on x quantized per
//   32-group (see XUnit).
// * End of step.  LM head -> grid barrier -> argmax stage 1 on every CTA;
//   the last CTA to finish runs stage 2, the sampler and the step end.  A
//   step without logits stops after the last layer's attention (its K/V are
//   the step's only lasting output).
#pragma once
#include "ck_ops.cuh"

#define SK_THREADS 512
#define SK_NCW 15                   // compute warps
#define SK_NCT (SK_NCW * 32)        // compute threads
#define SK_SLOT_BYTES (32 * 1024)
#define SK_NSLOT 5
#define SK_HMAX 2048                // residual elements kept per CTA
#define SK_RB 3                     // rows a warp reduces together
#define SK_GLU_MAX 256              // gate/up rows per CTA staged for the fused activation

// ---------------------------------------------------------------------------
// Row partition: CTA c of `grid` owns rows [c*n/grid, (c+1)*n/grid) of an
// n-row output, so with n >= grid every CTA produces in every matvec phase.
// That makes every phase's input a full fan-in of the phase before it, which
// is what keeps the reuse of each tagged buffer safe: no CTA can write a
// buffer's next contents before every CTA has finished reading the current
// ones (each writes only after its own prologue has read everything the
// previous phase produced, and that phase's writers had read theirs).
__host__ __device__ __forceinline__ int sk_row0(int c, int n, int grid) {
  return (int)(((long long)c * n) / grid);
}

// A row-partitioned vector of tagged words: element r, owned by CTA c,
// lives at word (c << sh) + r - row0(c); each CTA's segment of 2^sh words
// is a whole number of 128-byte lines.  c = ((r + 1) * grid - 1) / n and
// row0(c) = c * n / grid, both as multiply-shifts by ceil(2^40 / d), exact
// for numerators below 2^24.  grid = 1 is a flat vector.
struct PkVec {
  unsigned long long* p;
  int n, grid, sh, pad;
  unsigned long long mn, mg;   // ceil(2^40 / n), ceil(2^40 / grid)
};
__device__ __forceinline__ size_t pk_word(const PkVec& v, int r) {
  const unsigned long long x = (unsigned long long)(r + 1) * (unsigned)v.grid - 1ull;
  const unsigned long long c = (x * v.mn) >> 40;
  const unsigned long long r0 = ((c * (unsigned)v.n) * v.mg) >> 40;
  return (size_t)((c << v.sh) + (unsigned long long)r - r0);
}

enum { SK_MV = 1, SK_ATTN = 2, SK_HEAD = 3 };
enum { RES_NONE = 0, RES_EMBED = 1, RES_ADD = 2, RES_GEMMA = 3 };

struct SkSeg {
  const uint8_t* w;     // device-layout rows
  PkVec out;            // tagged output (not used by the head or a fused gate/up)
  Lay L;
  int n;
  int per;              // most rows a CTA owns: ceil(n / grid)
  int tile_rows;        // rows that fill an empty slot
  uint32_t soff;        // byte offset of this segment's rows in a packed tile
};

struct SkMv {
  PkVec in;             // the phase's input (tagged); not read with RES_EMBED
  int in_tag;           // writer phase + 1 of `in`
  int res;              // residual update applied in the prologue (RES_*)
  int norm;             // 1: x = rmsnorm(h) * wnorm, the RMS scale applied per output row
  const float* wnorm;
  const float* wpost;   // RES_GEMMA: post-norm weight of the sub-layer output
  float eps;
  int k, nseg, packed, epi;   // epi: EPI_SILU / EPI_GELU over segments 0 (gate), 1 (up)
  SkSeg seg[3];
  PkVec act;            // epi: act(gate) * up, rows partitioned like the gate
  float* logits;        // head: plain floats
  const uint8_t* emb;   // RES_EMBED: the (tied) embedding table
  Lay embL;
  float emb_scale;
};

struct SkAttn {
  PkVec q, k, v;        // projections (tagged words of the QKV phase)
  int in_tag;
  const float *qw, *kw;   // QK-norm weights (null when the model has none)
  void *kc, *vc;          // this layer's cache [kv_head][ctx][head_dim]
  const float* inv_freq;  // [head_dim/2]
  unsigned long long* out;    // [heads * head_dim] tagged words, flat
  unsigned long long* part;   // split partials [kvh][smax][G][hd + 2]
  int heads, kvh, hd, ctx, window, interleaved, kv_f32, smax, group;
  float eps, scale;
};

struct __align__(16) SkPhase {
  int kind;
  int index;            // position in the schedule
  int out_tag;          // index + 1: the tag of every word this phase writes
  int pad;
  union {
    SkMv mv;
    SkAttn at;
  };
};
static_assert(sizeof(SkPhase) % 16 == 0, "descriptors are bulk-copied");

// Host: tile shapes of an SkMv for a grid of `grid` CTAs.  A phase is packed
// when the largest share of every segment fits one slot together.
inline void sk_partition(SkMv& m, int grid) {
  uint32_t off = 0;
  for (int i = 0; i < m.nseg; i++) {
    SkSeg& s = m.seg[i];
    s.per = (s.n + grid - 1) / grid;
    s.tile_rows = (int)(SK_SLOT_BYTES / s.L.row_bytes);
    s.soff = off;
    off += (uint32_t)s.per * s.L.row_bytes;
  }
  m.packed = off <= SK_SLOT_BYTES ? 1 : 0;
  if (!m.packed)
    for (int i = 0; i < m.nseg; i++) m.seg[i].soff = 0;
}

// ---------------------------------------------------------------------------
struct SkSmemMv {
  float xf[CK_KMAX];
  alignas(16) int8_t xh[CK_KMAX];
  alignas(16) int8_t xl[CK_KMAX];
  float sx[CK_KMAX / 32];
  alignas(8) int s16[CK_KMAX / 16];
  float red[32];
  float rowacc[SK_NCW * SK_RB];     // per-warp partial sums when warps share rows
  float glu[2][SK_GLU_MAX];
};
union SkSmem {
  SkSmemMv mv;
  Smem o;          // attention (o.at) and the argmax / sampling phases
};

// Dynamic shared memory: [slots][full mbarriers][empty mbarriers][descriptor
// mbarriers][2 descriptor buffers]
#define SK_DYN_FULL (SK_NSLOT * SK_SLOT_BYTES)
#define SK_DYN_EMPTY (SK_DYN_FULL + 8 * SK_NSLOT)
#define SK_DYN_DBAR (SK_DYN_EMPTY + 8 * SK_NSLOT)
#define SK_DYN_DESC ((SK_DYN_DBAR + 16 + 127) & ~127)
#define SK_DYN_BYTES (SK_DYN_DESC + 2 * (int)sizeof(SkPhase))

__device__ __forceinline__ uint8_t* sk_slot(int s) { return dyn_smem() + (size_t)s * SK_SLOT_BYTES; }
__device__ __forceinline__ uint64_t* sk_full(int s) { return (uint64_t*)(dyn_smem() + SK_DYN_FULL) + s; }
__device__ __forceinline__ uint64_t* sk_empty(int s) { return (uint64_t*)(dyn_smem() + SK_DYN_EMPTY) + s; }
__device__ __forceinline__ uint64_t* sk_dbar(int b) { return (uint64_t*)(dyn_smem() + SK_DYN_DBAR) + b; }
__device__ __forceinline__ SkPhase* sk_desc(int b) { return (SkPhase*)(dyn_smem() + SK_DYN_DESC) + b; }

// barrier of the compute warps only (the producer warp never joins it)
__device__ __forceinline__ void sk_bar() { asm volatile("bar.sync 1, %0;" ::"n"(SK_NCT) : "memory"); }

// Bounded mbarrier wait: gives up after ~2^22 polls, or (heed_abort) once
// another CTA has given up, flagging the step; the caller carries on (a late
// or skipped wait only corrupts this step's values, which the host discards).
__device__ __forceinline__ void sk_wait(uint64_t* bar, uint32_t parity, int* err, int* abort_flag,
                                        bool heed_abort = true) {
  unsigned spins = 0;
  while (!mbar_try_wait(bar, parity)) {
    if (++spins > (1u << 22)) {
      atomicOr(err, CK_DERR_BARRIER);
      atomicExch(abort_flag, 1);
      return;
    }
    if (heed_abort && (spins & 1023u) == 0 && *(volatile int*)abort_flag) return;
  }
}

__device__ __forceinline__ float sk_block_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  sk_bar();
  if (l == 0) red[w] = v;
  sk_bar();
  float t = 0.f;
#pragma unroll
  for (int i = 0; i < SK_NCW; i++) t += red[i];
  return t;
}

// ---------------------------------------------------------------------------
// Tiles: the same walk in the producer and in the compute warps.
__device__ __forceinline__ void sk_seg_range(const SkSeg& S, int cta, int& lo, int& hi) {
  lo = sk_row0(cta, S.n, gridDim.x);
  hi = sk_row0(cta + 1, S.n, gridDim.x);
}
__device__ __forceinline__ bool sk_next_tile(const SkMv& m, int cta, int& seg, int& row, TileList& T) {
  tile_clear(T);
  if (m.packed) {
    if (seg != 0) return false;
    seg = 1;
#pragma unroll
    for (int i = 0; i < 3; i++) {
      if (i < m.nseg) {
        int lo, hi;
        sk_seg_range(m.seg[i], cta, lo, hi);
        if (hi > lo) tile_add(T, i, lo, hi - lo, m.seg[i].soff);
      }
    }
    return T.total > 0;
  }
  while (seg < m.nseg) {
    const SkSeg& S = m.seg[seg];
    int lo, hi;
    sk_seg_range(S, cta, lo, hi);
    if (row < lo) row = lo;
    if (row >= hi) { seg++; row = -1; continue; }
    const int take = min(S.tile_rows, hi - row);
    tile_add(T, seg, row, take, 0u);
    row += take;
    return true;
  }
  return false;
}

// Producer: copy one tile into slot ti % SK_NSLOT once the compute warps
// have released that slot's previous tile.
__device__ __forceinline__ void sk_issue_tile(const SkMv& m, const TileList& T, unsigned ti, int* err,
                                              int* abort_flag, int keep) {
  const int s = (int)(ti % SK_NSLOT);
  const unsigned use = ti / SK_NSLOT;
  if (use > 0) sk_wait(sk_empty(s), (use - 1) & 1u, err, abort_flag);
  uint32_t bytes = 0;
  for (int i = 0; i < T.n; i++) {
    const int rows = (i + 1 < T.n ? pick3(i + 1, 0, T.st1, T.st2) : T.total) - pick3(i, 0, T.st1, T.st2);
    bytes += (uint32_t)rows * m.seg[pick3(i, T.seg0, T.seg1, T.seg2)].L.row_bytes;
  }
  uint64_t* bar = sk_full(s);
  mbar_expect_tx(bar, bytes);
  uint8_t* dst = sk_slot(s);
  for (int i = 0; i < T.n; i++) {
    const int sg = pick3(i, T.seg0, T.seg1, T.seg2);
    const int r0 = pick3(i, T.r00, T.r01, T.r02);
    const int rows = (i + 1 < T.n ? pick3(i + 1, 0, T.st1, T.st2) : T.total) - pick3(i, 0, T.st1, T.st2);
    const SkSeg& S = m.seg[sg];
    bulk_g2s_stream(dst + pick3u(i, T.off0, T.off1, T.off2), S.w + (size_t)r0 * S.L.row_bytes,
                    (uint32_t)rows * S.L.row_bytes, bar, keep);
  }
}

// Bring this CTA's attention cache rows into L2 (no shared memory), one
// phase or more ahead of the attention phase.
__device__ __forceinline__ void sk_attn_prefetch(const SkAttn& P, int cta, int ncta, int pos) {
  const int start = (P.window != 0 && pos + 1 > P.window) ? pos + 1 - P.window : 0;
  const int npos = pos - start + 1;
  int chunk = (npos + P.smax - 1) / P.smax;
  if (chunk < CK_MIN_SPLIT) chunk = CK_MIN_SPLIT;
  const int S = (npos + chunk - 1) / chunk;
  const size_t elem = P.kv_f32 ? 4 : 2;
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

// ---------------------------------------------------------------------------
// Matvec prologue (compute threads): read the input words, apply the
// residual update to the CTA's copy of h, form x and quantize it.  Returns
// the RMS scale that multiplies every output row (1 without a norm).
//   RES_EMBED  h = embedding row of tokens[pos] * scale (GGUF_*_EMBEDDING_WGSL)
//   RES_ADD    h = h + in                              (ADD / ADD_RMS_NORM)
//   RES_GEMMA  h = clamp(h + rmsnorm(in) * wpost)      (gemma3 sandwich, :1050-1064)
//   norm       x = h * wnorm, scale rms_inv(h)         (RMS_NORM_WGSL :1910-1949)
template <int NPT>
__device__ float sk_prologue(const SkMv& P, SkSmemMv& s, float* hres, const CkDev& D, int pos, uint32_t ep,
                             int* err, int* abort_flag) {
  const int tid = threadIdx.x;
  const int k = P.k;
  const uint32_t want = want_tag(ep, P.in_tag);
  float v[NPT];
  if (P.res != RES_EMBED) {
    unsigned long long w[NPT];
    uint32_t wants[NPT];
#pragma unroll
    for (int j = 0; j < NPT; j++) {
      const int i = tid + j * SK_NCT;
      w[j] = i < k ? ld_word((const float*)P.in.p, pk_word(P.in, i), P.in_tag) : ((unsigned long long)want << 32);
      wants[j] = want;
    }
    settle(w, wants, [&](int j) {
      return ld_word((const float*)P.in.p, pk_word(P.in, tid + j * SK_NCT), P.in_tag);
    }, err, abort_flag);
#pragma unroll
    for (int j = 0; j < NPT; j++) v[j] = word_float(w[j]);
  } else {
    uint32_t token = D.tokens[pos];
    if (token >= (uint32_t)D.vocab) {
      if (blockIdx.x == 0 && tid == 0) atomicOr(&D.st->err, CK_DERR_TOKEN);
      token = 0;
    }
    const uint8_t* row = P.emb + (size_t)token * P.embL.row_bytes;
#pragma unroll
    for (int j = 0; j < NPT; j++) {
      const int i = tid + j * SK_NCT;
      v[j] = i < k ? __fmul_rn(dequant_at(row, P.embL, i), P.emb_scale) : 0.f;
    }
  }
  if (P.res == RES_GEMMA) {
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < NPT; j++) ss += v[j] * v[j];
    const float inv = rms_inv(sk_block_sum(ss, s.red), k, P.eps);
#pragma unroll
    for (int j = 0; j < NPT; j++) {
      const int i = tid + j * SK_NCT;
      if (i < k) {
        const float t = (v[j] * inv) * P.wpost[i];
        v[j] = fminf(fmaxf(hres[i] + t, -65000.0f), 65000.0f);
      }
    }
  } else if (P.res == RES_ADD) {
#pragma unroll
    for (int j = 0; j < NPT; j++) {
      const int i = tid + j * SK_NCT;
      if (i < k) v[j] = hres[i] + v[j];
    }
  }
  if (P.res != RES_NONE) {
#pragma unroll
    for (int j = 0; j < NPT; j++) {
      const int i = tid + j * SK_NCT;
      if (i < k) hres[i] = v[j];
    }
  }
  float scale = 1.0f;
  if (P.norm) {
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < NPT; j++) ss += v[j] * v[j];
    scale = rms_inv(sk_block_sum(ss, s.red), k, P.eps);
#pragma unroll
    for (int j = 0; j < NPT; j++) {
      const int i = tid + j * SK_NCT;
      if (i < k) v[j] = v[j] * P.wnorm[i];
    }
  }
#pragma unroll
  for (int j = 0; j < NPT; j++) {
    const int i = tid + j * SK_NCT;
    if (i < k) s.xf[i] = v[j];
  }
  sk_bar();
  // quantize per 32-group into X = hi * 256 + lo (XUnit): half a warp per
  // group, two elements per lane
  const int lane = tid & 31, half = (tid >> 4) & 1, warp = tid >> 5, hl = lane & 15;
  const int U = k >> 5;
  for (int gp = warp; 2 * gp < U; gp += SK_NCW) {
    const int g = 2 * gp + half;
    const bool ok = g < U;
    float2 xv = ok ? *(const float2*)(s.xf + 32 * g + 2 * hl) : make_float2(0.f, 0.f);
    float amax = fmaxf(fabsf(xv.x), fabsf(xv.y));
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const bool fin = amax <= 3.0e38f;
    const float step = amax * (1.0f / 32639.0f);
    const float inv = (step > 0.f && fin) ? 32639.0f / amax : 0.f;
    const int X0 = max(-32639, min(32639, __float2int_rn(xv.x * inv)));
    const int X1 = max(-32639, min(32639, __float2int_rn(xv.y * inv)));
    const int h0 = (X0 + 128) >> 8, h1 = (X1 + 128) >> 8;
    const int l0 = X0 - 256 * h0, l1 = X1 - 256 * h1;
    int sum = X0 + X1;
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (!ok) continue;
    *(short*)(s.xh + 32 * g + 2 * hl) = (short)((h0 & 0xFF) | (h1 << 8));
    *(short*)(s.xl + 32 * g + 2 * hl) = (short)((l0 & 0xFF) | (l1 << 8));
    if (hl == 0) s.sx[g] = fin ? step : __int_as_float(0x7fc00000);
    if (hl == 0) s.s16[2 * g] = sum;
    if (hl == 8) s.s16[2 * g + 1] = sum;
  }
  sk_bar();
  return scale;
}

__device__ __forceinline__ void sk_load_xunit(const SkSmemMv& s, int c, XUnit& x) {
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

// Where flat row t of a tile lives: segment, output row, bytes in the slot.
__device__ __forceinline__ void sk_tile_row(const SkMv& P, const TileList& T, int t, int& sg, int& orow,
                                            uint32_t& off) {
  const int pc = (t >= T.st1) + (t >= T.st2);
  sg = pick3(pc, T.seg0, T.seg1, T.seg2);
  const int local = t - pick3(pc, 0, T.st1, T.st2);
  orow = pick3(pc, T.r00, T.r01, T.r02) + local;
  off = pick3u(pc, T.off0, T.off1, T.off2) + (uint32_t)local * P.seg[sg].L.row_bytes;
}

__device__ __forceinline__ void sk_store_row(const SkMv& P, int sg, int orow, float v, SkSmemMv& s, int cta,
                                             int out_tag, uint32_t ep) {
  const SkSeg& S = P.seg[sg];
  if (P.logits) {
    P.logits[orow] = v;
  } else if (P.epi) {
    s.glu[sg][orow - sk_row0(cta, S.n, gridDim.x)] = v;
  } else {
    st_word((float*)S.out.p, pk_word(S.out, orow), v, out_tag, ep);
  }
}

// Dot products of one tile (in slot `tb`) with the quantized x.
__device__ __forceinline__ void sk_tile(const SkMv& P, const uint8_t* tb, const TileList& T, SkSmemMv& s,
                                        float xscale, int cta, int out_tag, uint32_t ep) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int U = P.k >> 5;
  const int total = T.total;
  if (total >= SK_NCW) {
    // whole rows per warp, up to SK_RB at a time
    const bool one = U <= 32;
    XUnit x0;
    if (one && lane < U) sk_load_xunit(s, lane, x0);
    for (int t0 = warp; t0 < total; t0 += SK_NCW * SK_RB) {
      float acc[SK_RB];
#pragma unroll
      for (int i = 0; i < SK_RB; i++) {
        acc[i] = 0.f;
        const int t = t0 + i * SK_NCW;
        if (t < total) {
          int sg, orow;
          uint32_t off;
          sk_tile_row(P, T, t, sg, orow, off);
          const SkSeg& S = P.seg[sg];
          if (one) {
            if (lane < U) {
              U8 u;
              unpack_unit<false>(S.L.type, tb + off, S.L, lane, u);
              acc[i] = unit_dot8(u, x0);
            }
          } else {
#pragma unroll 1
            for (int c = lane; c < U; c += 32) {
              U8 u;
              unpack_unit<false>(S.L.type, tb + off, S.L, c, u);
              XUnit xc;
              sk_load_xunit(s, c, xc);
              acc[i] += unit_dot8(u, xc);
            }
          }
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int i = 0; i < SK_RB; i++) acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], o);
#pragma unroll
      for (int i = 0; i < SK_RB; i++) {
        const int t = t0 + i * SK_NCW;
        if (lane == i && t < total) {
          int sg, orow;
          uint32_t off;
          sk_tile_row(P, T, t, sg, orow, off);
          sk_store_row(P, sg, orow, xscale * acc[i], s, cta, out_tag, ep);
        }
      }
    }
    return;
  }
  // fewer rows than warps: wpr warps share each row's units
  const int wpr = SK_NCW / total;
  const int t = warp / wpr, part = warp - t * wpr;
  float acc = 0.f;
  if (t < total) {
    int sg, orow;
    uint32_t off;
    sk_tile_row(P, T, t, sg, orow, off);
    const SkSeg& S = P.seg[sg];
#pragma unroll 1
    for (int c = part * 32 + lane; c < U; c += 32 * wpr) {
      U8 u;
      unpack_unit<false>(S.L.type, tb + off, S.L, c, u);
      XUnit xc;
      sk_load_xunit(s, c, xc);
      acc += unit_dot8(u, xc);
    }
  }
  acc = warp_sum(acc);
  if (lane == 0) s.rowacc[warp] = acc;
  sk_bar();
  if (warp == 0 && lane < total) {
    float a = 0.f;
    for (int p = 0; p < wpr; p++) a += s.rowacc[lane * wpr + p];
    int sg, orow;
    uint32_t off;
    sk_tile_row(P, T, lane, sg, orow, off);
    sk_store_row(P, sg, orow, xscale * a, s, cta, out_tag, ep);
  }
}

// One matvec phase on the compute warps; `ti` counts the tiles consumed.
__device__ void sk_matvec(const SkMv& P, SkSmemMv& s, float* hres, const CkDev& D, int cta, int pos, int out_tag,
                          uint32_t ep, unsigned& ti, unsigned long long* tp) {
  int* err = &D.st->err;
  int* ab = &D.st->abort_flag;
  int seg = 0, row = -1;
  TileList T;
  const bool rows = sk_next_tile(P, cta, seg, row, T);
  // a CTA with no rows still applies a residual update to its copy of h;
  // without one it reads nothing
  if (!rows && P.res == RES_NONE) return;
  stage_mark(tp, 0);
  float xscale;
  if (P.k <= 3 * SK_NCT) xscale = sk_prologue<3>(P, s, hres, D, pos, ep, err, ab);
  else if (P.k <= 5 * SK_NCT) xscale = sk_prologue<5>(P, s, hres, D, pos, ep, err, ab);
  else xscale = sk_prologue<7>(P, s, hres, D, pos, ep, err, ab);
  stage_mark(tp, 1);
  if (!rows) return;
  bool first = true;
  do {
    const int sl = (int)(ti % SK_NSLOT);
    sk_wait(sk_full(sl), (ti / SK_NSLOT) & 1u, err, ab);
    if (first) stage_mark(tp, 2);
    sk_tile(P, sk_slot(sl), T, s, xscale, cta, out_tag, ep);
    if (first) stage_mark(tp, 3);
    first = false;
    sk_bar();       // every compute thread is done with the slot
    if (threadIdx.x == 0) mbar_arrive(sk_empty(sl));
    ti++;
  } while (sk_next_tile(P, cta, seg, row, T));
  if (P.epi) {
    // fused SILU_MUL_WGSL (:3529-3547) / GELU_TANH_MUL_WGSL (:3568-3599) over
    // this CTA's gate/up rows (the barrier above published the staging rows)
    int lo, hi;
    sk_seg_range(P.seg[0], cta, lo, hi);
    for (int i = threadIdx.x; i < hi - lo; i += SK_NCT) {
      const float g = s.glu[0][i], u = s.glu[1][i];
      const float a = P.epi == EPI_SILU ? (g / (1.0f + expf(-g))) * u : gelu_tanh(g) * u;
      st_word((float*)P.act.p, pk_word(P.act, lo + i), a, out_tag, ep);
    }
  }
  stage_mark(tp, 4);
}

// ---------------------------------------------------------------------------
// Attention unit (split, kv head) on the compute warps: QK-norm + RoPE of q
// (and of k, by the split that holds `pos`, which also stores K/V there),
// online softmax over the split's positions, partials merged by the owner
// split.  Restates ROPE_STORE(_INTERLEAVED)_WGSL (:2868-2927, :3122-3184),
// QK_NORM_ROPE_STORE(_INTERLEAVED)_WGSL (:2929-3023, :3186-3283),
// ATTENTION_SCORE_WGSL (:3385-3437) and ATTENTION_VALUE_WGSL (:3439-3490).
template <int E>
__device__ __forceinline__ void sk_attn_merge(const SkAttn& P, SmemAt& s, int kvh, int S, int out_tag, uint32_t ep,
                                              int* err, int* abort_flag) {
  constexpr int hd = 32 * E;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = P.group, NE = G * hd;
  const float* pk = (const float*)(P.part + (size_t)kvh * P.smax * G * (hd + 2));
  const uint32_t want = want_tag(ep, out_tag);
  const unsigned long long none = (unsigned long long)want << 32;
  float* sm_m = s.wacc;
  float* sm_l = s.wacc + 1024;
  float* sm_L = s.wacc + 2048;
  int Pw = 1;
  while (Pw < 32 && 2 * Pw * NE <= SK_NCT) Pw *= 2;
  const int part = tid & (Pw - 1), slots = SK_NCT / Pw;
  const int passes = (NE + slots - 1) / slots;
  unsigned long long x[8];
  {
    const int e = tid / Pw;
    const int gg = e < NE ? e / hd : 0, d = e % hd;
#pragma unroll
    for (int j = 0; j < 8; j++) {
      const int sp = part + j * Pw;
      x[j] = (e < NE && sp < S) ? ld_word(pk, ((size_t)sp * G + gg) * (hd + 2) + 2 + d, out_tag) : none;
    }
  }
  for (int i = tid; i < S * G; i += SK_NCT) {
    const size_t o = (size_t)i * (hd + 2);
    unsigned long long ml[2] = {ld_word(pk, o, out_tag), ld_word(pk, o + 1, out_tag)};
    const uint32_t w2[2] = {want, want};
    settle(ml, w2, [&](int j) { return ld_word(pk, o + j, out_tag); }, err, abort_flag);
    sm_m[i] = word_float(ml[0]);
    sm_l[i] = word_float(ml[1]);
  }
  sk_bar();
  for (int gg = warp; gg < G; gg += SK_NCW) {
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
  sk_bar();
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
          x[j] = (ok && sp < S) ? ld_word(pk, ((size_t)sp * G + gg) * (hd + 2) + 2 + d, out_tag) : none;
        }
      }
      const uint32_t w8[8] = {want, want, want, want, want, want, want, want};
      settle(x, w8, [&](int j) {
        return ld_word(pk, ((size_t)(sp0 + j * Pw) * G + gg) * (hd + 2) + 2 + d, out_tag);
      }, err, abort_flag);
#pragma unroll
      for (int j = 0; j < 8; j++) {
        const int sp = sp0 + j * Pw;
        if (ok && sp < S) A += word_float(x[j]) * sm_m[sp * G + gg];
      }
    }
    for (int o = 1; o < Pw; o <<= 1) A += __shfl_xor_sync(0xffffffffu, A, o);
    if (ok && part == 0) st_word((float*)P.out, (size_t)(kvh * G + gg) * hd + d, A / sm_L[gg], out_tag, ep);
  }
}

template <int E, bool F32>
__device__ __forceinline__ void sk_attn_unit(const SkAttn& P, SmemAt& s, int kvh, int split, int pos, int out_tag,
                                             uint32_t ep, int* err, int* abort_flag) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  constexpr int hd = 32 * E;
  const int G = P.group;
  const int start = (P.window != 0 && pos + 1 > P.window) ? pos + 1 - P.window : 0;
  const int npos = pos - start + 1;
  int chunk = (npos + P.smax - 1) / P.smax;
  if (chunk < CK_MIN_SPLIT) chunk = CK_MIN_SPLIT;
  const int S = (npos + chunk - 1) / chunk;
  if (split >= S) return;
  const int t0 = start + split * chunk;
  const int t1 = min(t0 + chunk, pos + 1);
  const bool owner = split == S - 1;
  const int tend = owner ? pos : t1;
  const int wpg = SK_NCW / G;       // warps per q head
  const int g = warp / wpg, sub = warp % wpg;

  const size_t kvbase = (size_t)kvh * P.ctx * hd + lane * E;
  int t = t0 + sub;
  constexpr int DEPTH = (E <= 4 && !(F32 && E == 4)) ? 2 : (F32 && E == 8) ? 0 : 1;
  KvRow<E, F32> ka, va, kb, vb, kc, vc, kd, vd;
  kv_zero(ka); kv_zero(va); kv_zero(kb); kv_zero(vb);
  kv_zero(kc); kv_zero(vc); kv_zero(kd); kv_zero(vd);
  auto load_pair = [&](int tt, KvRow<E, F32>& k0, KvRow<E, F32>& v0, KvRow<E, F32>& k1, KvRow<E, F32>& v1) {
    kv_zero(k0); kv_zero(v0); kv_zero(k1); kv_zero(v1);
    if (tt < tend) { kv_load(P.kc, kvbase + (size_t)tt * hd, k0); kv_load(P.vc, kvbase + (size_t)tt * hd, v0); }
    if (tt + wpg < tend) {
      kv_load(P.kc, kvbase + (size_t)(tt + wpg) * hd, k1);
      kv_load(P.vc, kvbase + (size_t)(tt + wpg) * hd, v1);
    }
  };
  if (g < G) {
    load_pair(t, ka, va, kb, vb);
    if (DEPTH == 2) load_pair(t + 2 * wpg, kc, vc, kd, vd);
  }
  float invf = 0.f, kk = 0.f, vv = 0.f, wq = 0.f, wk = 0.f;
  const uint32_t want = want_tag(ep, P.in_tag);
  const unsigned long long none = (unsigned long long)want << 32;
  const int q0 = kvh * G * hd, kv0 = kvh * hd;
  constexpr int QPT = (CK_GMAX * CK_HDMAX + SK_NCT - 1) / SK_NCT;   // q words per thread (<= 5)
  unsigned long long xw[QPT + 2];
  uint32_t wants[QPT + 2];
#pragma unroll
  for (int j = 0; j < QPT; j++) {
    const int i = tid + j * SK_NCT;
    xw[j] = i < G * hd ? ld_word((const float*)P.q.p, pk_word(P.q, q0 + i), P.in_tag) : none;
    wants[j] = want;
  }
  xw[QPT] = (owner && tid < hd) ? ld_word((const float*)P.k.p, pk_word(P.k, kv0 + tid), P.in_tag) : none;
  xw[QPT + 1] = (owner && tid < hd) ? ld_word((const float*)P.v.p, pk_word(P.v, kv0 + tid), P.in_tag) : none;
  wants[QPT] = wants[QPT + 1] = want;
  if (tid < (hd >> 1)) invf = P.inv_freq[tid];
  if (tid < hd) {
    if (owner && P.kw) wk = P.kw[tid];
    if (P.qw) wq = P.qw[tid];
  }
  settle(xw, wants, [&](int j) {
    return j < QPT ? ld_word((const float*)P.q.p, pk_word(P.q, q0 + tid + j * SK_NCT), P.in_tag)
         : j == QPT ? ld_word((const float*)P.k.p, pk_word(P.k, kv0 + tid), P.in_tag)
                    : ld_word((const float*)P.v.p, pk_word(P.v, kv0 + tid), P.in_tag);
  }, err, abort_flag);
  kk = word_float(xw[QPT]);
  vv = word_float(xw[QPT + 1]);
  if (tid < (hd >> 1)) {
    float sn, cn;
    sincosf((float)pos * invf, &sn, &cn);
    s.cs[tid] = make_float2(cn, sn);
  }
#pragma unroll
  for (int j = 0; j < QPT; j++) {
    const int i = tid + j * SK_NCT;
    if (i < G * hd) s.raw[i] = word_float(xw[j]);
  }
  if (tid < hd) {
    if (owner) {
      s.kvw[0][tid] = kk;
      s.kvw[1][tid] = vv;
      if (P.kw) s.kvw[3][tid] = wk;
    }
    if (P.qw) s.kvw[2][tid] = wq;
  }
  sk_bar();
  if (P.qw) {
    for (int gg = warp; gg < G + (owner ? 1 : 0); gg += SK_NCW) {
      const float* src = gg < G ? s.raw + gg * hd : s.kvw[0];
      float ss = 0.f;
      for (int d = lane; d < hd; d += 32) ss += src[d] * src[d];
      ss = warp_sum(ss);
      if (lane == 0) s.inv[gg] = rms_inv(ss, hd, P.eps);
    }
    sk_bar();
  }
  for (int gg = 0; gg < G; gg++)
    rope_head(s.raw + gg * hd, P.qw ? s.kvw[2] : nullptr, P.qw ? s.inv[gg] : 1.f, s.qs + gg * hd, hd,
              P.interleaved, s.cs, tid, SK_NCT);
  if (owner) {
    rope_head(s.kvw[0], P.kw ? s.kvw[3] : nullptr, P.kw ? s.inv[G] : 1.f, s.kst, hd, P.interleaved, s.cs, tid,
              SK_NCT);
    sk_bar();
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
  sk_bar();

  float q[E], acc[E], m = -INFINITY, l = 0.f;
#pragma unroll
  for (int e = 0; e < E; e++) {
    q[e] = g < G ? s.qs[g * hd + lane * E + e] : 0.f;
    acc[e] = 0.f;
  }
  if (g < G) {
    for (; t < tend; t += 2 * wpg) {
      KvRow<E, F32> nka, nva, nkb, nvb;
      if (DEPTH == 2) load_pair(t + 4 * wpg, nka, nva, nkb, nvb);
      if (DEPTH == 1) load_pair(t + 2 * wpg, nka, nva, nkb, nvb);
      softmax_pair<E, F32>(q, ka, va, kb, vb, t + wpg < tend, P.scale, m, l, acc);
      if (DEPTH == 2) {
        ka = kc; va = vc; kb = kd; vb = vd;
        kc = nka; vc = nva; kd = nkb; vd = nvb;
      } else if (DEPTH == 1) {
        ka = nka; va = nva; kb = nkb; vb = nvb;
      } else {
        load_pair(t + 2 * wpg, ka, va, kb, vb);
      }
    }
    if (owner && sub == 0) {
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
  if (lane == 0) {
    s.wm[warp] = m;
    s.wl[warp] = l;
  }
#pragma unroll
  for (int e = 0; e < E; e++) s.wacc[warp * CK_HDMAX + lane * E + e] = acc[e];
  sk_bar();
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
  sk_bar();
  if (S == 1) {
    for (int i = tid; i < G * hd; i += SK_NCT) {
      const int gg = i / hd, d = i % hd;
      float A = 0.f;
      for (int w = gg * wpg; w < gg * wpg + wpg; w++) A += s.wacc[w * CK_HDMAX + d] * s.wf[w];
      st_word((float*)P.out, (size_t)(kvh * G + gg) * hd + d, A / s.hl[gg], out_tag, ep);
    }
    return;
  }
  float* part = (float*)(P.part + ((size_t)kvh * P.smax + split) * G * (hd + 2));
  for (int i = tid; i < G * hd; i += SK_NCT) {
    const int gg = i / hd, d = i % hd;
    float A = 0.f;
    for (int w = gg * wpg; w < gg * wpg + wpg; w++) A += s.wacc[w * CK_HDMAX + d] * s.wf[w];
    st_word(part, gg * (hd + 2) + 2 + d, A, out_tag, ep);
    if (d == 0) {
      st_word(part, gg * (hd + 2), s.hm[gg], out_tag, ep);
      st_word(part, gg * (hd + 2) + 1, s.hl[gg], out_tag, ep);
    }
  }
  if (!owner) return;
  sk_bar();
  sk_attn_merge<E>(P, s, kvh, S, out_tag, ep, err, abort_flag);
}

__device__ void sk_attn(const SkAttn& P, SmemAt& s, const CkDev& D, int cta, int ncta, int pos, int out_tag,
                        uint32_t ep) {
  int* err = &D.st->err;
  int* ab = &D.st->abort_flag;
  for (int u = cta; u < P.kvh * P.smax; u += ncta) {
    const int kvh = u % P.kvh, split = u / P.kvh;
    if (P.kv_f32) {
      if (P.hd == 64) sk_attn_unit<2, true>(P, s, kvh, split, pos, out_tag, ep, err, ab);
      else if (P.hd == 128) sk_attn_unit<4, true>(P, s, kvh, split, pos, out_tag, ep, err, ab);
      else sk_attn_unit<8, true>(P, s, kvh, split, pos, out_tag, ep, err, ab);
    } else {
      if (P.hd == 64) sk_attn_unit<2, false>(P, s, kvh, split, pos, out_tag, ep, err, ab);
      else if (P.hd == 128) sk_attn_unit<4, false>(P, s, kvh, split, pos, out_tag, ep, err, ab);
      else sk_attn_unit<8, false>(P, s, kvh, split, pos, out_tag, ep, err, ab);
    }
    sk_bar();
  }
}

// ---------------------------------------------------------------------------
// The step.  `logits`: the schedule ends with the LM head (argmax, sampling
// and step end follow); otherwise the step ends after the last phase.
__global__ void __launch_bounds__(SK_THREADS, 1) k_step(const SkPhase* __restrict__ ph, int nph, int logits, CkDev D) {
  __shared__ SkSmem sm;
  __shared__ float hres[SK_HMAX];
  __shared__ int s_last;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int cta = blockIdx.x, ncta = gridDim.x;
  CkState* st = D.st;
  const int pos = st->pos;
  const uint32_t ep = st->epoch;
  int* err = &st->err;
  int* ab = &st->abort_flag;
  if (tid == 0) {
    for (int i = 0; i < SK_NSLOT; i++) {
      mbar_init(sk_full(i), 1);
      mbar_init(sk_empty(i), 1);
    }
    mbar_init(sk_dbar(0), 1);
    mbar_init(sk_dbar(1), 1);
    mbar_fence_init();
  }
  __syncthreads();
  const bool trace0 = D.trace && cta == 0 && tid == 0;
  if (warp == SK_NCW) {
    // ---- producer: weights for every matvec tile of this CTA, in order ----
    if (lane == 0) {
      unsigned ti = 0;
      for (int i = 0; i < nph; i++) {
        const SkPhase& p = ph[i];
        if (p.kind == SK_ATTN) {
          sk_attn_prefetch(p.at, cta, ncta, pos);
          continue;
        }
        int seg = 0, row = -1;
        TileList T;
        while (sk_next_tile(p.mv, cta, seg, row, T)) sk_issue_tile(p.mv, T, ti++, err, ab, D.l2_keep);
      }
      // every issued copy lands before this CTA can exit, even after another
      // CTA gave up (copies from valid addresses always complete; bounded)
      for (unsigned j = ti > SK_NSLOT ? ti - SK_NSLOT : 0; j < ti; j++)
        sk_wait(sk_full((int)(j % SK_NSLOT)), (j / SK_NSLOT) & 1u, err, ab, false);
    }
    __syncwarp();
  } else {
    // ---- compute warps ----------------------------------------------------
    unsigned ti = 0;
    if (tid == 0) {
      mbar_expect_tx(sk_dbar(0), (uint32_t)sizeof(SkPhase));
      bulk_g2s(sk_desc(0), ph, (uint32_t)sizeof(SkPhase), sk_dbar(0));
    }
    for (int i = 0; i < nph; i++) {
      sk_wait(sk_dbar(i & 1), (i >> 1) & 1u, err, ab);
      if (tid == 0 && i + 1 < nph) {
        // the buffer was read (generic proxy) in phase i - 1: order those
        // reads before the bulk copy (async proxy) overwrites it
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        mbar_expect_tx(sk_dbar((i + 1) & 1), (uint32_t)sizeof(SkPhase));
        bulk_g2s(sk_desc((i + 1) & 1), ph + i + 1, (uint32_t)sizeof(SkPhase), sk_dbar((i + 1) & 1));
      }
      const SkPhase& p = *sk_desc(i & 1);
      if (trace0 && 2 * i + 1 < CK_TRACE_MV_BASE) D.trace[2 * i] = gtimer();
      unsigned long long* tp = (D.trace && cta == 0 && i < 512) ? D.trace + CK_TRACE_STAGE_BASE + i * 8 : nullptr;
      if (p.kind == SK_ATTN) {
        sk_attn(p.at, sm.o.at, D, cta, ncta, pos, p.out_tag, ep);
      } else {
        if (p.kind == SK_HEAD && st->pen_d != 1.0) {
          // the repetition-penalty id set of this step (argmax stage 1 reads it)
          const int cnt = st->pen_src == 0 ? pos + 1 : st->pen_count;
          const uint32_t* ids = st->pen_src == 0 ? D.tokens : D.pen_list;
          for (int j = cta * SK_NCT + tid; j < cnt; j += ncta * SK_NCT) {
            const uint32_t id = ids[j];
            if (id < (uint32_t)D.vocab) atomicOr(&D.pen_mask[id >> 5], 1u << (id & 31));
          }
        }
        sk_matvec(p.mv, sm.mv, hres, D, cta, pos, p.out_tag, ep, ti, tp);
      }
      sk_bar();   // the descriptor buffer and the scratch are free again
      if (trace0 && 2 * i + 1 < CK_TRACE_MV_BASE) D.trace[2 * i + 1] = gtimer();
    }
  }
  // ---- end of step: every warp again ----------------------------------------
  unsigned target = ncta;
  if (logits) {
    if (!grid_sync(st, target)) return;    // all logits stored
    phase_argmax1<1>(D, sm.o, cta, ncta);
    target += ncta;
  }
  __syncthreads();
  if (tid == 0) {
    unsigned old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(old) : "l"(&st->bar) : "memory");
    s_last = old == target - 1;
  }
  __syncthreads();
  if (!s_last) return;
  if (logits) phase_select<1>(1, D, sm.o, 0, ep, ncta);
  else phase_finish(0, D, 0, ep);
}
