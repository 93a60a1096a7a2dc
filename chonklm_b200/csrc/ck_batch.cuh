// Batched decode (continuous batching) over an engine's uploaded weights.
//
// The reference decodes one sequence, one token per runToken call
// (llama-wgsl-runtime.ts:242-314, :1025-1150).  Here a step advances every
// active sequence by one position at once: a sequence still reading its
// prompt feeds its next prompt token, every other sequence feeds its last
// generated id, so a step is T tokens of T different sequences and the
// arithmetic for each of them is the runToken restatement of the
// single-sequence path.  Sequences join and leave between steps.
//
// * KV cache: paged, fp16, blocks of CK_BLK positions from one pool per layer
//   ([layer][K|V][block][kv_head][CK_BLK][head_dim]), each sequence holding a
//   block table; its blocks are reserved when it joins.
// * Each matvec becomes a dequantizing GEMM over the step's tokens (k_bgemm):
//   a warp owns one weight row, unpacks its 32-weight units once and dots
//   them with every token of a token tile staged in shared memory; the
//   per-token partial sums of the 32 lanes are combined by a butterfly
//   reduce-scatter (31 shuffles for 32 tokens instead of 5 per token).
// * x is quantized per token and per 32-group exactly as in the
//   single-sequence prologue (k_bprep); attention is one CTA per
//   (token, kv head) over that token's sequence (k_battn).
// * The step's kernels read the active count T from device memory, so one
//   CUDA graph, captured at the first step, serves every T.
// Supported: llama / qwen3 architectures with an fp16 KV cache, greedy
// decoding.

#define CK_BLK 16        // positions per KV block

struct BStep {
  const uint32_t* tok;   // [max_seqs] token fed by active entry i
  const int* slot;       // [max_seqs] sequence slot of entry i
  const int* pos;        // [max_seqs] position of entry i
  const int* nact;       // [1] active entries this step
  const int* btab;       // [max_seqs][max_blocks] KV block of each CK_BLK positions
  int max_blocks;
};

struct BXq {             // per-token quantized x (layout of the single-sequence prologue)
  int8_t* xh;            // [max_seqs][k]
  int8_t* xl;
  float* sx;             // [max_seqs][k/32]
  int* s16;              // [max_seqs][k/16]
  float* xs;             // [max_seqs] output scale (RMS of NORM, else 1)
};

enum { BP_COPY = 0, BP_NORM = 1, BP_SILU = 2 };

struct BPrep {
  int kind;
  const float* a;        // [T][lda]
  const float* b;        // SILU: up [T][lda]
  const float* w;        // NORM: weight [k]
  float eps;
  int k, lda;
};

struct BSeg {
  const uint8_t* w;
  Lay L;
  int n;
  float* out;            // out[t * ldo + row]
  const float* add;      // residual: out = add + W x (may alias out)
  int ldo;
};

struct BGemm {
  BSeg seg[3];
  int nseg;
  int k;
  int tile0[4];          // first 16-row tile of each segment; tile0[nseg] = total
};

struct BAttn {
  const float *q, *k, *v;     // [T][heads*hd], [T][kv_heads*hd]
  const float *qw, *kw;       // QK-norm weights or null
  __half *kc, *vc;            // this layer's pools [block][kv_head][CK_BLK][hd]
  const float* inv_freq;      // [hd/2]
  float* out;                 // [T][heads*hd]
  int heads, kvh, hd, interleaved, window;
  float eps, scale;
};

// ---------------------------------------------------------------------------
// Embedding of every active entry's token (GGUF_*_EMBEDDING_WGSL, :2615-2866).
__global__ void __launch_bounds__(256) k_bembed(const uint8_t* w, Lay L, float scale, BStep st, float* x, int H,
                                                int vocab, int* err) {
  const int t = blockIdx.x;
  if (t >= *st.nact) return;
  uint32_t token = st.tok[t];
  if (token >= (uint32_t)vocab) {
    if (threadIdx.x == 0) atomicOr(err, CK_DERR_TOKEN);
    token = 0;
  }
  const uint8_t* row = w + (size_t)token * L.row_bytes;
  for (int i = threadIdx.x; i < H; i += blockDim.x) x[(size_t)t * H + i] = __fmul_rn(dequant_at(row, L, i), scale);
}

// Per-token prologue + quantization (one CTA per active entry): the forms of
// build_quant prologue kinds COPY / NORM / SILU of the single-sequence path,
// with every global load of the CTA issued before any math.
__global__ void __launch_bounds__(CK_THREADS) k_bprep(BPrep p, BStep st, BXq q) {
  constexpr int GPW = CK_KMAX / 32 / CK_WARPS;
  const int t = blockIdx.x;
  if (t >= *st.nact) return;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int k = p.k, U = k >> 5;
  const float* a = p.a + (size_t)t * p.lda;
  const float* b = p.kind == BP_SILU ? p.b + (size_t)t * p.lda : p.w;
  __shared__ float red[CK_WARPS];
  float va[GPW], vb[GPW];
#pragma unroll
  for (int j = 0; j < GPW; j++) {
    const int g = warp + j * CK_WARPS, i = 32 * g + lane;
    va[j] = g < U ? a[i] : 0.f;
    vb[j] = (g < U && p.kind != BP_COPY) ? b[i] : 0.f;
  }
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < GPW; j++) {
    const int g = warp + j * CK_WARPS;
    float v = va[j];
    if (p.kind == BP_NORM) { ss += va[j] * va[j]; v = va[j] * vb[j]; }
    else if (p.kind == BP_SILU) v = (va[j] / (1.0f + expf(-va[j]))) * vb[j];
    const float amax = warp_max(fabsf(v));
    const bool fin = amax <= 3.0e38f;
    const float step = amax * (1.0f / 32639.0f);
    const float inv = (step > 0.f && fin) ? 32639.0f / amax : 0.f;
    const int X = max(-32639, min(32639, __float2int_rn(v * inv)));
    const int h = (X + 128) >> 8;
    int sum = X;
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (g < U) {
      q.xh[(size_t)t * k + 32 * g + lane] = (int8_t)h;
      q.xl[(size_t)t * k + 32 * g + lane] = (int8_t)(X - 256 * h);
      if (lane == 0) q.sx[(size_t)t * U + g] = fin ? step : __int_as_float(0x7fc00000);
      if ((lane & 15) == 0) q.s16[(size_t)t * 2 * U + 2 * g + (lane >> 4)] = sum;
    }
  }
  if (p.kind == BP_NORM) {
    ss = warp_sum(ss);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    if (threadIdx.x == 0) {
      float tot = 0.f;
      for (int w = 0; w < CK_WARPS; w++) tot += red[w];
      q.xs[t] = rms_inv(tot, k, p.eps);
    }
  } else if (threadIdx.x == 0) {
    q.xs[t] = 1.0f;
  }
}

// Sum over the 32 lanes of each of N per-lane values, scattered: lane l ends
// with the total of value (l % N).  N = 32 takes 31 shuffles.
template <int N>
__device__ __forceinline__ float reduce_scatter(float (&v)[N]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int n = N; n > 1; n >>= 1) {
    const int o = n >> 1;
    const bool upper = (lane & o) != 0;
#pragma unroll
    for (int i = 0; i < o; i++) {
      const float send = upper ? v[i] : v[i + o];
      const float keep = upper ? v[i + o] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
    }
  }
  float r = v[0];
#pragma unroll
  for (int o = N; o < 32; o <<= 1) r += __shfl_xor_sync(0xffffffffu, r, o);
  return r;
}

__host__ __device__ inline int bgemm_tt(int k) { return k <= 1536 ? 32 : 16; }
__host__ __device__ inline size_t bgemm_smem(int k) {
  return (size_t)bgemm_tt(k) * (2 * (size_t)k + 4 * (size_t)(k / 32) + 4 * (size_t)(k / 16));
}

// Y = W X over the step's tokens for up to three weight matrices sharing x.
// CTA = 16 rows of one segment (a warp per row) x one tile of TT tokens
// (blockIdx.y): the tile's quantized x is staged in shared memory and every
// warp dots its row's units, unpacked once, with each token of the tile.
template <int TT>
__global__ void __launch_bounds__(CK_THREADS, 1) k_bgemm(BGemm G, BStep st, BXq q) {
  extern __shared__ __align__(16) uint8_t bsm[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int si = 0;
  while (si + 1 < G.nseg && (int)blockIdx.x >= G.tile0[si + 1]) si++;
  const BSeg& S = G.seg[si];
  const int row = ((int)blockIdx.x - G.tile0[si]) * CK_WARPS + warp;
  const bool has = row < S.n;
  const int k = G.k, U = k >> 5, upl = (U + 31) >> 5;
  U8 u[3];
  if (has) {
    const uint8_t* wrow = S.w + (size_t)row * S.L.row_bytes;
#pragma unroll
    for (int j = 0; j < 3; j++) {
      const int c = lane + 32 * j;
      if (j < upl && c < U) unpack_unit<true>(S.L.type, wrow, S.L, c, u[j]);
    }
  }
  int8_t* sxh = (int8_t*)bsm;
  int8_t* sxl = sxh + TT * k;
  float* ssx = (float*)(sxl + TT * k);
  int* ss16 = (int*)(ssx + TT * U);
  const int T = *st.nact;
  const int t0 = blockIdx.y * TT;
  if (t0 >= T) return;
  {
    const int nt = min(TT, T - t0);
    // stage the tile: xh, xl rows are contiguous per token and the tile's
    // tokens are consecutive, so each array is one contiguous span
    {
      const int4* gh = (const int4*)(q.xh + (size_t)t0 * k);
      const int4* gl = (const int4*)(q.xl + (size_t)t0 * k);
      const int nv = nt * k / 16;
      for (int i = threadIdx.x; i < nv; i += CK_THREADS) {
        ((int4*)sxh)[i] = gh[i];
        ((int4*)sxl)[i] = gl[i];
      }
      for (int i = threadIdx.x; i < nt * U; i += CK_THREADS) ssx[i] = q.sx[(size_t)t0 * U + i];
      for (int i = threadIdx.x; i < nt * 2 * U; i += CK_THREADS) ss16[i] = q.s16[(size_t)t0 * 2 * U + i];
    }
    __syncthreads();
    if (!has) return;
    float v[TT];
#pragma unroll
    for (int i = 0; i < TT; i++) {
      v[i] = 0.f;
      if (i < nt) {
#pragma unroll
        for (int j = 0; j < 3; j++) {
          const int c = lane + 32 * j;
          if (j < upl && c < U) {
            XUnit x;
            const int4* h = (const int4*)(sxh + i * k) + 2 * c;
            const int4* l = (const int4*)(sxl + i * k) + 2 * c;
            const int4 h0 = h[0], h1 = h[1], l0 = l[0], l1 = l[1];
            x.h[0] = h0.x; x.h[1] = h0.y; x.h[2] = h0.z; x.h[3] = h0.w;
            x.h[4] = h1.x; x.h[5] = h1.y; x.h[6] = h1.z; x.h[7] = h1.w;
            x.l[0] = l0.x; x.l[1] = l0.y; x.l[2] = l0.z; x.l[3] = l0.w;
            x.l[4] = l1.x; x.l[5] = l1.y; x.l[6] = l1.z; x.l[7] = l1.w;
            x.sx = ssx[i * U + c];
            x.sa = ss16[i * 2 * U + 2 * c];
            x.sb = ss16[i * 2 * U + 2 * c + 1];
            v[i] += unit_dot8(u[j], x);
          }
        }
      }
    }
    const float tot = reduce_scatter<TT>(v);
    const int i = lane % TT;
    if (lane < TT && i < nt) {
      const size_t o = (size_t)(t0 + i) * S.ldo + row;
      const float y = q.xs[t0 + i] * tot;
      S.out[o] = S.add ? S.add[o] + y : y;
    }
  }
}

// Attention for one (active entry, kv head): QK-norm + RoPE + K/V store at
// the entry's position in its sequence's blocks, then an online softmax over
// [start, pos] (the single-sequence attention unit with one split), one
// warp group per query head.
template <int E>
__global__ void __launch_bounds__(CK_THREADS, 1) k_battn(BAttn P, BStep st) {
  constexpr int hd = 32 * E;
  const int t = blockIdx.x / P.kvh, kvh = blockIdx.x % P.kvh;
  if (t >= *st.nact) return;
  __shared__ SmemAt s;
  __shared__ int sbt[256];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = P.heads / P.kvh, qd = P.heads * hd, kvd = P.kvh * hd;
  const int pos = st.pos[t];
  const int* bt = st.btab + (size_t)st.slot[t] * st.max_blocks;
  const int start = (P.window != 0 && pos + 1 > P.window) ? pos + 1 - P.window : 0;
  for (int i = tid; i <= (pos >> 4) && i < 256; i += CK_THREADS) sbt[i] = bt[i];
  for (int d = tid; d < (hd >> 1); d += CK_THREADS) {
    float sn, cn;
    sincosf((float)pos * P.inv_freq[d], &sn, &cn);
    s.cs[d] = make_float2(cn, sn);
  }
  const float* qsrc = P.q + (size_t)t * qd + (size_t)kvh * G * hd;
  for (int i = tid; i < G * hd; i += CK_THREADS) s.raw[i] = qsrc[i];
  for (int d = tid; d < hd; d += CK_THREADS) {
    s.kvw[0][d] = P.k[(size_t)t * kvd + (size_t)kvh * hd + d];
    s.kvw[1][d] = P.v[(size_t)t * kvd + (size_t)kvh * hd + d];
    if (P.kw) s.kvw[3][d] = P.kw[d];
    if (P.qw) s.kvw[2][d] = P.qw[d];
  }
  __syncthreads();
  if (P.qw) {
    for (int gg = warp; gg < G + 1; gg += CK_WARPS) {
      const float* src = gg < G ? s.raw + gg * hd : s.kvw[0];
      float ss = 0.f;
      for (int d = lane; d < hd; d += 32) ss += src[d] * src[d];
      ss = warp_sum(ss);
      if (lane == 0) s.inv[gg] = rms_inv(ss, hd, P.eps);
    }
    __syncthreads();
  }
  for (int gg = 0; gg < G; gg++)
    rope_head(s.raw + gg * hd, P.qw ? s.kvw[2] : nullptr, P.qw ? s.inv[gg] : 1.f, s.qs + gg * hd, hd, P.interleaved,
              s.cs, tid, CK_THREADS);
  rope_head(s.kvw[0], P.kw ? s.kvw[3] : nullptr, P.kw ? s.inv[G] : 1.f, s.kst, hd, P.interleaved, s.cs, tid,
            CK_THREADS);
  __syncthreads();
  {
    const size_t cb = (((size_t)sbt[pos >> 4] * P.kvh + kvh) * CK_BLK + (pos & (CK_BLK - 1))) * hd;
    for (int d = tid; d < hd; d += CK_THREADS) {
      P.kc[cb + d] = __float2half_rn(s.kst[d]);
      P.vc[cb + d] = __float2half_rn(s.kvw[1][d]);
    }
  }
  const int wpg = CK_WARPS / G;
  const int g = warp / wpg, sub = warp % wpg;
  float q[E], acc[E], m = -INFINITY, l = 0.f;
#pragma unroll
  for (int e = 0; e < E; e++) {
    q[e] = g < G ? s.qs[g * hd + lane * E + e] : 0.f;
    acc[e] = 0.f;
  }
  if (g < G) {
    auto off = [&](int p) {
      return (((size_t)sbt[p >> 4] * P.kvh + kvh) * CK_BLK + (p & (CK_BLK - 1))) * hd + lane * E;
    };
    // CH positions of the warp per round, all their rows requested before
    // the round's math (a round trip per round, not per position)
    constexpr int CH = E <= 4 ? 8 : 4;
    for (int p0 = start + sub; p0 < pos; p0 += CH * wpg) {
      KvRow<E, false> kr[CH], vr[CH];
#pragma unroll
      for (int j = 0; j < CH; j++) {
        const int p = p0 + j * wpg;
        kv_zero(kr[j]); kv_zero(vr[j]);
        if (p < pos) { kv_load(P.kc, off(p), kr[j]); kv_load(P.vc, off(p), vr[j]); }
      }
#pragma unroll
      for (int j = 0; j < CH; j += 2)   // positions grow with j: a pair past pos ends the round
        if (p0 + j * wpg < pos)
          softmax_pair<E, false>(q, kr[j], vr[j], kr[j + 1], vr[j + 1], p0 + (j + 1) * wpg < pos, P.scale, m, l,
                                 acc);
    }
    if (sub == 0) {   // position pos, as the cache now holds it
      float d0 = 0.f;
#pragma unroll
      for (int e = 0; e < E; e++) d0 += q[e] * kv_round<false>(s.kst[lane * E + e]);
      const float s0 = warp_sum(d0) * P.scale;
      const float mn = fmaxf(m, s0);
      const float c = expf(m - mn), p0 = expf(s0 - mn);
      l = l * c + p0;
#pragma unroll
      for (int e = 0; e < E; e++) acc[e] = acc[e] * c + p0 * kv_round<false>(s.kvw[1][lane * E + e]);
      m = mn;
    }
  }
  if (lane == 0) {
    s.wm[warp] = m;
    s.wl[warp] = l;
  }
#pragma unroll
  for (int e = 0; e < E; e++) s.wacc[warp * CK_HDMAX + lane * E + e] = acc[e];
  __syncthreads();
  if (tid < G) {
    float M = -INFINITY;
    for (int w = tid * wpg; w < tid * wpg + wpg; w++) M = fmaxf(M, s.wm[w]);
    float L = 0.f;
    for (int w = tid * wpg; w < tid * wpg + wpg; w++) {
      const float f = s.wm[w] == -INFINITY ? 0.f : expf(s.wm[w] - M);
      s.wf[w] = f;
      L += s.wl[w] * f;
    }
    s.hl[tid] = L;
  }
  __syncthreads();
  for (int i = tid; i < G * hd; i += CK_THREADS) {
    const int gg = i / hd, d = i % hd;
    float A = 0.f;
    for (int w = gg * wpg; w < gg * wpg + wpg; w++) A += s.wacc[w * CK_HDMAX + d] * s.wf[w];
    P.out[(size_t)t * qd + (size_t)(kvh * G + gg) * hd + d] = A / s.hl[gg];
  }
}

// Greedy id of every active entry: ARGMAX_STAGE1/2 rules (NaN never wins,
// ties go to the lower index) over its logits row.
__global__ void __launch_bounds__(CK_THREADS) k_bargmax(const float* logits, int V, BStep st, uint32_t* ids) {
  const int t = blockIdx.x;
  if (t >= *st.nact) return;
  __shared__ float sv[CK_WARPS];
  __shared__ uint32_t si[CK_WARPS];
  float v = -3.402823e38f;
  uint32_t idx = 0xffffffffu;
  const float* row = logits + (size_t)t * V;
  for (int i = threadIdx.x; i < V; i += CK_THREADS)
    if (better(row[i], (uint32_t)i, v, idx)) { v = row[i]; idx = (uint32_t)i; }
  block_argmax(v, idx, sv, si);
  if (threadIdx.x == 0) ids[t] = idx;
}

// ---------------------------------------------------------------------------
// Host side (compiled into the engine's translation unit: it reads the
// engine's uploaded weights and configuration).

struct BSeq {
  bool used = false;
  int id = -1;
  std::vector<uint32_t> prompt, gen, eos;
  int pos = 0;                // next position fed
  int max_new = 0;
  std::vector<int> blocks;    // reserved KV blocks
};

struct ck_batch {
  ck_engine* h = nullptr;
  int max_seqs = 0, max_blocks = 0, n_blocks = 0;
  cudaStream_t stream = nullptr;
  std::vector<void*> allocs;
  std::string err;
  __half* kv = nullptr;       // [layers][K|V][n_blocks][kv_heads][CK_BLK][head_dim]
  uint32_t* d_tok = nullptr;
  int *d_slot = nullptr, *d_pos = nullptr, *d_nact = nullptr, *d_btab = nullptr, *d_err = nullptr;
  uint32_t* d_ids = nullptr;
  float *x = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *ao = nullptr, *g = nullptr, *u = nullptr,
        *logits = nullptr;
  BXq xq{};
  uint8_t* pin = nullptr;     // pinned staging: tok | slot | pos | nact | ids | err
  std::vector<BSeq> seqs;     // one per slot
  std::vector<int> free_blocks;
  std::vector<int> btab;      // host copy of the block tables
  bool btab_dirty = true;
  std::map<int, std::vector<uint32_t>> finished;
  int next_id = 0;
  cudaGraphExec_t graph = nullptr;
  unsigned long long steps = 0, fed = 0, generated = 0;

  int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    err = buf;
    return code;
  }
};

#define CKB(b, call)                                                                                    \
  do {                                                                                                  \
    cudaError_t e_ = (call);                                                                            \
    if (e_ != cudaSuccess) return (b)->fail(CK_ECUDA, "%s: %s (%s:%d)", #call, cudaGetErrorString(e_), \
                                           __FILE__, __LINE__);                                          \
  } while (0)

namespace {

template <class T>
int balloc(ck_batch* b, T** p, size_t bytes) {
  void* q = nullptr;
  cudaError_t e = cudaMalloc(&q, bytes ? bytes : 16);
  if (e != cudaSuccess) return b->fail(CK_ENOMEM, "cudaMalloc(%zu): %s", bytes, cudaGetErrorString(e));
  b->allocs.push_back(q);
  *p = (T*)q;
  return CK_OK;
}

BStep bstep(const ck_batch* b) {
  BStep s;
  s.tok = b->d_tok;
  s.slot = b->d_slot;
  s.pos = b->d_pos;
  s.nact = b->d_nact;
  s.btab = b->d_btab;
  s.max_blocks = b->max_blocks;
  return s;
}

int bgemm_launch(ck_batch* b, cudaStream_t s, int k, std::initializer_list<BSeg> segs) {
  BGemm G;
  memset(&G, 0, sizeof G);
  G.k = k;
  int tiles = 0;
  for (const BSeg& x : segs) {
    G.tile0[G.nseg] = tiles;
    G.seg[G.nseg++] = x;
    tiles += (x.n + CK_WARPS - 1) / CK_WARPS;
  }
  G.tile0[G.nseg] = tiles;
  const size_t smem = bgemm_smem(k);
  const int tt = bgemm_tt(k);
  const dim3 grid(tiles, (b->max_seqs + tt - 1) / tt);   // token tiles past T return at once
  if (tt == 32) k_bgemm<32><<<grid, CK_THREADS, smem, s>>>(G, bstep(b), b->xq);
  else k_bgemm<16><<<grid, CK_THREADS, smem, s>>>(G, bstep(b), b->xq);
  return CK_OK;
}

BSeg bseg(const Weight& w, float* out, const float* add, int ldo) {
  BSeg s;
  s.w = w.dev;
  s.L = w.L;
  s.n = w.n;
  s.out = out;
  s.add = add;
  s.ldo = ldo;
  return s;
}

void bprep(ck_batch* b, cudaStream_t s, int kind, const float* a, const float* bb, const float* w, float eps, int k,
           int lda) {
  BPrep p;
  p.kind = kind; p.a = a; p.b = bb; p.w = w; p.eps = eps; p.k = k; p.lda = lda;
  k_bprep<<<b->max_seqs, CK_THREADS, 0, s>>>(p, bstep(b), b->xq);
}

// The whole step on stream s (captured once into a graph).
int batch_enqueue(ck_batch* b, cudaStream_t s) {
  ck_engine* h = b->h;
  const ck_model_cfg& c = h->cfg;
  const int H = c.hidden, hd = c.head_dim, qd = c.heads * hd, kvd = c.kv_heads * hd, I = c.intermediate;
  const size_t pool = (size_t)b->n_blocks * c.kv_heads * CK_BLK * hd;
  k_bembed<<<b->max_seqs, 256, 0, s>>>(h->emb.dev, h->emb.L, c.embedding_scale, bstep(b), b->x, H, c.vocab, b->d_err);
  for (int i = 0; i < c.layers; i++) {
    const LayerW& W = h->L[i];
    bprep(b, s, BP_NORM, b->x, nullptr, W.attn_norm, c.norm_eps, H, H);
    bgemm_launch(b, s, H, {bseg(W.q, b->q, nullptr, qd), bseg(W.k, b->k, nullptr, kvd), bseg(W.v, b->v, nullptr, kvd)});
    BAttn a;
    a.q = b->q; a.k = b->k; a.v = b->v;
    a.qw = c.qk_norm ? W.q_norm : nullptr;
    a.kw = c.qk_norm ? W.k_norm : nullptr;
    a.kc = b->kv + (size_t)(2 * i) * pool;
    a.vc = b->kv + (size_t)(2 * i + 1) * pool;
    a.inv_freq = h->inv_freq + (size_t)i * (hd / 2);
    a.out = b->ao;
    a.heads = c.heads; a.kvh = c.kv_heads; a.hd = hd; a.interleaved = c.rope_interleaved;
    a.window = (int)c.layer_window[i];
    a.eps = c.qk_norm_eps;
    a.scale = (float)(1.0 / sqrt((double)hd));   // ATTN_SCALE (:1711)
    const int grid = b->max_seqs * c.kv_heads;
    if (hd == 64) k_battn<2><<<grid, CK_THREADS, 0, s>>>(a, bstep(b));
    else if (hd == 128) k_battn<4><<<grid, CK_THREADS, 0, s>>>(a, bstep(b));
    else k_battn<8><<<grid, CK_THREADS, 0, s>>>(a, bstep(b));
    bprep(b, s, BP_COPY, b->ao, nullptr, nullptr, 0.f, qd, qd);
    bgemm_launch(b, s, qd, {bseg(W.o, b->x, b->x, H)});
    bprep(b, s, BP_NORM, b->x, nullptr, W.post_norm, c.norm_eps, H, H);
    bgemm_launch(b, s, H, {bseg(W.gate, b->g, nullptr, I), bseg(W.up, b->u, nullptr, I)});
    bprep(b, s, BP_SILU, b->g, b->u, nullptr, 0.f, I, I);
    bgemm_launch(b, s, I, {bseg(W.down, b->x, b->x, H)});
  }
  bprep(b, s, BP_NORM, b->x, nullptr, h->final_norm, c.norm_eps, H, H);
  bgemm_launch(b, s, H, {bseg(h->head, b->logits, nullptr, c.vocab)});
  k_bargmax<<<b->max_seqs, CK_THREADS, 0, s>>>(b->logits, c.vocab, bstep(b), b->d_ids);
  CKB(b, cudaGetLastError());
  return CK_OK;
}

}  // namespace

extern "C" {

int ck_batch_create(ck_engine* h, int max_seqs, int kv_blocks, ck_batch** out) {
  if (!h || !out) return set_global(CK_EINVAL, "ck_batch_create: bad argument");
  *out = nullptr;
  if (!h->finalized) return h->fail(CK_ESTATE, "engine not finalized");
  const ck_model_cfg& c = h->cfg;
  if (c.arch != CK_ARCH_LLAMA) return h->fail(CK_EINVAL, "batched decode supports the llama / qwen3 architectures");
  if (max_seqs < 1 || max_seqs > 1024) return h->fail(CK_EINVAL, "max_seqs %d outside [1, 1024]", max_seqs);
  const int max_blocks = (c.context_length + CK_BLK - 1) / CK_BLK;
  if (max_blocks > 256) return h->fail(CK_EINVAL, "batched decode handles contexts up to %d", 256 * CK_BLK);
  if (bgemm_smem(c.intermediate) > CK_DYN_SMEM_MAX || bgemm_smem(c.heads * c.head_dim) > CK_DYN_SMEM_MAX)
    return h->fail(CK_EINVAL, "batched decode: matmul input too wide");
  ck_batch* b = new ck_batch();
  b->h = h;
  b->max_seqs = max_seqs;
  b->max_blocks = max_blocks;
  b->n_blocks = kv_blocks > 0 ? kv_blocks : max_seqs * max_blocks;
  int rc = CK_OK;
  auto bail = [&](int code) {
    std::string m = b->err;
    for (void* p : b->allocs) cudaFree(p);
    if (b->pin) cudaFreeHost(b->pin);
    if (b->stream) cudaStreamDestroy(b->stream);
    delete b;
    return h->fail(code, "%s", m.c_str());
  };
  if (cudaSetDevice(h->device) != cudaSuccess) return bail(b->fail(CK_ECUDA, "cudaSetDevice"));
  if (cudaStreamCreateWithFlags(&b->stream, cudaStreamNonBlocking) != cudaSuccess)
    return bail(b->fail(CK_ECUDA, "stream"));
  const int H = c.hidden, qd = c.heads * c.head_dim, kvd = c.kv_heads * c.head_dim, I = c.intermediate;
  const size_t S = (size_t)max_seqs;
  const size_t kv_bytes = (size_t)c.layers * 2 * b->n_blocks * c.kv_heads * CK_BLK * c.head_dim * 2;
  if ((rc = balloc(b, &b->kv, kv_bytes)) || (rc = balloc(b, &b->d_tok, S * 4)) ||
      (rc = balloc(b, &b->d_slot, S * 4)) || (rc = balloc(b, &b->d_pos, S * 4)) ||
      (rc = balloc(b, &b->d_nact, 16)) || (rc = balloc(b, &b->d_btab, S * max_blocks * 4)) ||
      (rc = balloc(b, &b->d_err, 16)) || (rc = balloc(b, &b->d_ids, S * 4)) ||
      (rc = balloc(b, &b->x, S * H * 4)) || (rc = balloc(b, &b->q, S * qd * 4)) ||
      (rc = balloc(b, &b->k, S * kvd * 4)) || (rc = balloc(b, &b->v, S * kvd * 4)) ||
      (rc = balloc(b, &b->ao, S * qd * 4)) || (rc = balloc(b, &b->g, S * I * 4)) ||
      (rc = balloc(b, &b->u, S * I * 4)) || (rc = balloc(b, &b->logits, S * c.vocab * 4)) ||
      (rc = balloc(b, &b->xq.xh, S * CK_KMAX)) || (rc = balloc(b, &b->xq.xl, S * CK_KMAX)) ||
      (rc = balloc(b, &b->xq.sx, S * (CK_KMAX / 32) * 4)) || (rc = balloc(b, &b->xq.s16, S * (CK_KMAX / 16) * 4)) ||
      (rc = balloc(b, &b->xq.xs, S * 4)))
    return bail(rc);
  if (cudaMemset(b->d_err, 0, 16) != cudaSuccess || cudaMemset(b->d_nact, 0, 16) != cudaSuccess ||
      cudaMemset(b->d_btab, 0, S * max_blocks * 4) != cudaSuccess)
    return bail(b->fail(CK_ECUDA, "memset"));
  if (cudaMallocHost(&b->pin, S * 16 + 64) != cudaSuccess) return bail(b->fail(CK_ENOMEM, "pinned staging"));
  if (cudaFuncSetAttribute(k_bgemm<32>, cudaFuncAttributeMaxDynamicSharedMemorySize, CK_DYN_SMEM_MAX) != cudaSuccess ||
      cudaFuncSetAttribute(k_bgemm<16>, cudaFuncAttributeMaxDynamicSharedMemorySize, CK_DYN_SMEM_MAX) != cudaSuccess)
    return bail(b->fail(CK_ECUDA, "matmul shared memory"));
  b->seqs.resize(max_seqs);
  b->btab.assign(S * max_blocks, 0);
  for (int i = b->n_blocks - 1; i >= 0; i--) b->free_blocks.push_back(i);
  *out = b;
  return CK_OK;
}

int ck_batch_add_seq(ck_batch* b, const uint32_t* prompt, int n, int max_new, const uint32_t* eos_ids, int n_eos,
                     int* seq_id) {
  if (!b || !prompt || !seq_id || n < 1 || max_new < 1) return set_global(CK_EINVAL, "ck_batch_add_seq: bad argument");
  const ck_model_cfg& c = b->h->cfg;
  for (int i = 0; i < n; i++)
    if (prompt[i] >= (uint32_t)c.vocab) return b->fail(CK_EINVAL, "token id %u outside embedding table", prompt[i]);
  // generateLlamaWgsl caps the new tokens at the context left (:246)
  if (n >= c.context_length) return b->fail(CK_EINVAL, "Llama WGSL context exhausted at %d tokens", c.context_length);
  if (max_new > c.context_length - n) max_new = c.context_length - n;
  int slot = -1;
  for (int i = 0; i < b->max_seqs; i++)
    if (!b->seqs[i].used) { slot = i; break; }
  if (slot < 0) return b->fail(CK_EBUSY, "all %d sequence slots are in use", b->max_seqs);
  const int need = (n + max_new + CK_BLK - 1) / CK_BLK;
  if ((int)b->free_blocks.size() < need)
    return b->fail(CK_ENOMEM, "KV pool has %zu free blocks, the sequence needs %d", b->free_blocks.size(), need);
  BSeq& q = b->seqs[slot];
  q = BSeq();
  q.used = true;
  q.id = b->next_id++;
  q.prompt.assign(prompt, prompt + n);
  if (eos_ids && n_eos > 0) q.eos.assign(eos_ids, eos_ids + n_eos);
  q.max_new = max_new;
  for (int i = 0; i < need; i++) {
    q.blocks.push_back(b->free_blocks.back());
    b->free_blocks.pop_back();
    b->btab[(size_t)slot * b->max_blocks + i] = q.blocks.back();
  }
  b->btab_dirty = true;
  *seq_id = q.id;
  return CK_OK;
}

int ck_batch_step(ck_batch* b, int* n_active) {
  if (!b) return set_global(CK_EINVAL, "null batch");
  uint32_t* ptok = (uint32_t*)b->pin;
  int* pslot = (int*)(b->pin + (size_t)b->max_seqs * 4);
  int* ppos = (int*)(b->pin + (size_t)b->max_seqs * 8);
  uint32_t* pids = (uint32_t*)(b->pin + (size_t)b->max_seqs * 12);
  int* pn = (int*)(b->pin + (size_t)b->max_seqs * 16);
  int T = 0;
  for (int i = 0; i < b->max_seqs; i++) {
    const BSeq& q = b->seqs[i];
    if (!q.used) continue;
    const int L = (int)q.prompt.size();
    ptok[T] = q.pos < L ? q.prompt[q.pos] : q.gen[q.pos - L];
    pslot[T] = i;
    ppos[T] = q.pos;
    T++;
  }
  if (n_active) *n_active = T;
  if (T == 0) return CK_OK;
  pn[0] = T;
  cudaStream_t s = b->stream;
  CKB(b, cudaSetDevice(b->h->device));
  CKB(b, cudaMemcpyAsync(b->d_tok, ptok, (size_t)T * 4, cudaMemcpyHostToDevice, s));
  CKB(b, cudaMemcpyAsync(b->d_slot, pslot, (size_t)T * 4, cudaMemcpyHostToDevice, s));
  CKB(b, cudaMemcpyAsync(b->d_pos, ppos, (size_t)T * 4, cudaMemcpyHostToDevice, s));
  CKB(b, cudaMemcpyAsync(b->d_nact, pn, 4, cudaMemcpyHostToDevice, s));
  if (b->btab_dirty) {
    CKB(b, cudaMemcpyAsync(b->d_btab, b->btab.data(), b->btab.size() * 4, cudaMemcpyHostToDevice, s));
    CKB(b, cudaStreamSynchronize(s));   // the host table may change before the next step
    b->btab_dirty = false;
  }
  if (!b->graph) {
    cudaGraph_t g = nullptr;
    CKB(b, cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
    int rc = batch_enqueue(b, s);
    cudaError_t e = cudaStreamEndCapture(s, &g);
    if (rc) { if (g) cudaGraphDestroy(g); return rc; }
    CKB(b, e);
    e = cudaGraphInstantiate(&b->graph, g, 0);
    cudaGraphDestroy(g);
    CKB(b, e);
  }
  CKB(b, cudaGraphLaunch(b->graph, s));
  CKB(b, cudaMemcpyAsync(pids, b->d_ids, (size_t)T * 4, cudaMemcpyDeviceToHost, s));
  int* perr = pn + 1;
  CKB(b, cudaMemcpyAsync(perr, b->d_err, 4, cudaMemcpyDeviceToHost, s));
  CKB(b, cudaStreamSynchronize(s));
  if (*perr) {
    cudaMemset(b->d_err, 0, 4);
    return b->fail(CK_EDEVICE, "token id outside embedding table");
  }
  b->steps++;
  b->fed += T;
  for (int j = 0; j < T; j++) {
    BSeq& q = b->seqs[pslot[j]];
    const int L = (int)q.prompt.size();
    const bool produces = q.pos >= L - 1;   // prompt tokens before the last produce nothing
    q.pos++;
    if (!produces) continue;
    const uint32_t id = pids[j];
    q.gen.push_back(id);
    b->generated++;
    bool stop = (int)q.gen.size() >= q.max_new;
    for (uint32_t e : q.eos) stop = stop || e == id;
    if (stop) {
      b->finished[q.id] = q.gen;
      for (int blk : q.blocks) b->free_blocks.push_back(blk);
      q = BSeq();
    }
  }
  if (n_active) {
    int a = 0;
    for (const BSeq& q : b->seqs) a += q.used ? 1 : 0;
    *n_active = a;
  }
  return CK_OK;
}

int ck_batch_collect(ck_batch* b, int seq_id, uint32_t* out_ids, int cap, int* n_out, int* done) {
  if (!b || !n_out || !done) return set_global(CK_EINVAL, "ck_batch_collect: bad argument");
  auto it = b->finished.find(seq_id);
  const std::vector<uint32_t>* g = nullptr;
  if (it != b->finished.end()) {
    g = &it->second;
    *done = 1;
  } else {
    for (const BSeq& q : b->seqs)
      if (q.used && q.id == seq_id) g = &q.gen;
    if (!g) return b->fail(CK_EINVAL, "unknown sequence %d", seq_id);
    *done = 0;
  }
  const int n = (int)g->size();
  *n_out = n;
  if (out_ids) memcpy(out_ids, g->data(), (size_t)(n < cap ? n : cap) * 4);
  if (*done) b->finished.erase(it);
  return CK_OK;
}

int ck_batch_stats(ck_batch* b, uint64_t* steps, uint64_t* tokens_fed, uint64_t* tokens_generated) {
  if (!b) return set_global(CK_EINVAL, "null batch");
  if (steps) *steps = b->steps;
  if (tokens_fed) *tokens_fed = b->fed;
  if (tokens_generated) *tokens_generated = b->generated;
  return CK_OK;
}

const char* ck_batch_last_error(ck_batch* b) { return b ? b->err.c_str() : g_err.c_str(); }

int ck_batch_destroy(ck_batch* b) {
  if (!b) return CK_OK;
  cudaSetDevice(b->h->device);
  if (b->stream) cudaStreamSynchronize(b->stream);
  if (b->graph) cudaGraphExecDestroy(b->graph);
  for (void* p : b->allocs) cudaFree(p);
  if (b->pin) cudaFreeHost(b->pin);
  if (b->stream) cudaStreamDestroy(b->stream);
  delete b;
  return CK_OK;
}

}  // extern "C"
