// Prefill on the tensor cores: a prompt's tokens through the layers together.
//
// The reference feeds a prompt one id per runToken call
// (llama-wgsl-runtime.ts:281-288 inside generateLlamaWgsl, each call the
// whole graph of :1039-1124).  Here every prompt token but the last goes
// through the layers at once, up to a chunk of tokens at a time, on the
// batched path's kernels:
//
// * every matmul is the tcgen05 GEMM over the chunk's tokens (k_bgemm_tc on
//   the weights' operand tiles, the norm / SiLU prologue in k_bprep; the
//   attention kernels write the o projection's operand tiles themselves);
// * k_pkv applies the QK-norm and RoPE of each (token, kv head) and writes
//   the token's K and V rows into the engine's own cache at its position
//   (the ropeStore / qkNormRopeStore rows, :1467-1545), so that every row of
//   the chunk is in the cache before
// * k_pattn runs the causal attention of each (token, kv head) over
//   [start, position] (ATTENTION_SCORE / ATTENTION_VALUE, :3385-3490) from
//   the cache;
// * the last prompt token then takes the single-token step, which produces
//   the logits and the chosen id exactly as a decode step does.
//
// The matmuls keep ~22 significant bits of x and w (two fp16 parts each), so
// logits after a GEMM prefill agree with the token-by-token ones within the
// decode path's tolerance, not bit for bit; prompts shorter than the
// engine's threshold (ck_set_prefill_gemm) keep the token-by-token path.
// Supported: the llama / qwen3 graph (the same set as the batched decode).

#define PF_CHUNK_MAX 1024    // prompt tokens per pass through the layers

struct PfAttn {
  const float *q, *k, *v;     // [T][heads*hd], [T][kv_heads*hd] raw projections
  const float *qw, *kw;       // QK-norm weights or null
  void *kc, *vc;              // this layer's cache [kv_head][ctx][hd]
  const float* inv_freq;      // [hd/2]
  float* qr;                  // [T][heads*hd] q after norm + rope
  BXh xo;                     // the o projection's operand tiles: out written as x_hi / x_lo, scale 1
  int heads, kvh, hd, ctx, window, interleaved, pos0;
  float eps, scale;
};

__global__ void k_set_int(int* p, int v) { *p = v; }

// QK-norm + RoPE, one warp per (token, head row): the query heads into qr,
// the K rows (rounded as the cache stores them) and V rows into the cache at
// the token's position (the decode step's attention prologue).  Lane l holds
// dims l, l + 32, ...: the sum of squares runs in the decode prologue's
// order, a split-layout pair (d, d + hd/2) sits in one lane, an interleaved
// pair (2d, 2d + 1) in neighbouring lanes.
#define PKV_WARPS 8
template <int E, bool F32>
__global__ void __launch_bounds__(32 * PKV_WARPS) k_pkv(PfAttn P, const int* nact) {
  constexpr int hd = 32 * E;
  const int lane = threadIdx.x & 31;
  const int units = P.heads + 2 * P.kvh;                  // q heads, k heads, v heads
  const int gw = blockIdx.x * PKV_WARPS + (threadIdx.x >> 5);
  const int t = gw / units, u = gw % units;
  if (t >= *nact) return;
  const int qd = P.heads * hd, kvd = P.kvh * hd;
  const int pos = P.pos0 + t;
  const bool isq = u < P.heads, isk = !isq && u < P.heads + P.kvh;
  const int head = isq ? u : isk ? u - P.heads : u - P.heads - P.kvh;
  const float* src = isq ? P.q + (size_t)t * qd + (size_t)head * hd
                         : (isk ? P.k : P.v) + (size_t)t * kvd + (size_t)head * hd;
  float v[E];
#pragma unroll
  for (int e = 0; e < E; e++) v[e] = src[lane + 32 * e];
  if (isq || isk) {
    const float* w = isq ? P.qw : P.kw;
    if (w) {
      float ss = 0.f;
#pragma unroll
      for (int e = 0; e < E; e++) ss += v[e] * v[e];
      const float inv = rms_inv(warp_sum(ss), hd, P.eps);
#pragma unroll
      for (int e = 0; e < E; e++) v[e] = (v[e] * inv) * w[lane + 32 * e];
    }
    float o[E];
    if (P.interleaved) {
#pragma unroll
      for (int e = 0; e < E; e++) {
        const int d = lane + 32 * e;
        const float other = __shfl_xor_sync(0xffffffffu, v[e], 1);
        float sn, cn;
        sincosf((float)pos * P.inv_freq[d >> 1], &sn, &cn);
        o[e] = (d & 1) ? other * sn + v[e] * cn : v[e] * cn - other * sn;
      }
    } else {
#pragma unroll
      for (int e = 0; e < E / 2; e++) {
        float sn, cn;
        sincosf((float)pos * P.inv_freq[lane + 32 * e], &sn, &cn);
        const float a = v[e], b = v[e + E / 2];
        o[e] = a * cn - b * sn;
        o[e + E / 2] = a * sn + b * cn;
      }
    }
#pragma unroll
    for (int e = 0; e < E; e++) v[e] = o[e];
  }
  if (isq) {
    float* dst = P.qr + (size_t)t * qd + (size_t)head * hd;
#pragma unroll
    for (int e = 0; e < E; e++) dst[lane + 32 * e] = v[e];
  } else {
    const size_t cb = ((size_t)head * P.ctx + pos) * hd;
    void* cache = isk ? P.kc : P.vc;
#pragma unroll
    for (int e = 0; e < E; e++) {
      if (F32) ((float*)cache)[cb + lane + 32 * e] = v[e];
      else ((__half*)cache)[cb + lane + 32 * e] = __float2half_rn(v[e]);
    }
  }
}

// Causal attention of one (token, kv head) over [start, pos] from the cache:
// warps split into G groups (one query head each), CH positions of a warp
// requested per round, then the group's warps merged (the single-sequence
// attention unit with one split).
template <int E, bool F32>
__global__ void __launch_bounds__(CK_THREADS, 1) k_pattn(PfAttn P, const int* nact) {
  constexpr int hd = 32 * E;
  const int t = blockIdx.x / P.kvh, kvh = blockIdx.x % P.kvh;
  if (t >= *nact) return;
  __shared__ float wacc[CK_WARPS * CK_HDMAX];
  __shared__ float wm[CK_WARPS], wl[CK_WARPS], wf[CK_WARPS], hl[CK_GMAX];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = P.heads / P.kvh, qd = P.heads * hd;
  const int pos = P.pos0 + t;
  const int start = (P.window != 0 && pos + 1 > P.window) ? pos + 1 - P.window : 0;
  const int wpg = CK_WARPS / G;
  const int g = warp / wpg, sub = warp % wpg;
  float q[E], acc[E], m = -INFINITY, l = 0.f;
#pragma unroll
  for (int e = 0; e < E; e++) {
    q[e] = g < G ? P.qr[(size_t)t * qd + (size_t)(kvh * G + g) * hd + lane * E + e] : 0.f;
    acc[e] = 0.f;
  }
  if (g < G) {
    const size_t base = (size_t)kvh * P.ctx * hd + lane * E;
    constexpr int CH = E <= 4 ? 8 : 4;
    for (int p0 = start + sub; p0 <= pos; p0 += CH * wpg) {
      KvRow<E, F32> kr[CH], vr[CH];
#pragma unroll
      for (int j = 0; j < CH; j++) {
        const int p = p0 + j * wpg;
        kv_zero(kr[j]); kv_zero(vr[j]);
        if (p <= pos) { kv_load(P.kc, base + (size_t)p * hd, kr[j]); kv_load(P.vc, base + (size_t)p * hd, vr[j]); }
      }
#pragma unroll
      for (int j = 0; j < CH; j += 2)   // positions grow with j: a pair past pos ends the round
        if (p0 + j * wpg <= pos)
          softmax_pair<E, F32>(q, kr[j], vr[j], kr[j + 1], vr[j + 1], p0 + (j + 1) * wpg <= pos, P.scale, m, l, acc);
    }
  }
  if (lane == 0) {
    wm[warp] = m;
    wl[warp] = l;
  }
#pragma unroll
  for (int e = 0; e < E; e++) wacc[warp * CK_HDMAX + lane * E + e] = acc[e];
  __syncthreads();
  if (tid < G) {
    float M = -INFINITY;
    for (int w = tid * wpg; w < tid * wpg + wpg; w++) M = fmaxf(M, wm[w]);
    float L = 0.f;
    for (int w = tid * wpg; w < tid * wpg + wpg; w++) {
      const float f = wm[w] == -INFINITY ? 0.f : expf(wm[w] - M);
      wf[w] = f;
      L += wl[w] * f;
    }
    hl[tid] = L;
  }
  __syncthreads();
  const int nch = tc_nch(qd);
  for (int i = tid; i < G * hd; i += CK_THREADS) {
    const int gg = i / hd, d = i % hd;
    float A = 0.f;
    for (int w = gg * wpg; w < gg * wpg + wpg; w++) A += wacc[w * CK_HDMAX + d] * wf[w];
    const float o = A / hl[gg];
    const int col = (kvh * G + gg) * hd + d;
    const __half h = __float2half_rn(o);
    P.xo.xt[tc_index(t, col, nch, 0)] = h;
    P.xo.xt[tc_index(t, col, nch, 1)] = __float2half_rn(o - __half2float(h));
  }
  if (tid == 0 && kvh == 0) P.xo.xs[t] = 1.0f;
}

// Causal attention of a block of query rows on the tensor cores (fp16 cache).
//
// A CTA takes one kv head and FA_ROWS query rows (token-major: row r is head
// r % G of token qt0 + r / G).  Per chunk of FA_NP cache positions: S =
// Q K^T in tensor memory (Q as two fp16 parts, the cache's fp16 K exact), an
// online softmax over each row by the thread owning that accumulator lane
// (positions outside [start, pos] of the row's token weigh nothing), the
// output rows rescaled in tensor memory when the row maximum grows, P
// written to shared memory as fp16 and O += P V on the tensor cores.  The
// last chunk's O / l goes to out.  Operand tiles use the GEMM's K-major
// layout (kmaj_off); V is stored transposed (rows = dims, K = positions).
#define FA_ROWS 128
#define FA_NP 128
#define FA_THREADS 256

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,"
      "%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
      "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31]));
}
__device__ __forceinline__ void umma_f16(uint32_t tmem, uint64_t da, uint64_t db, uint32_t idesc, uint32_t acc) {
  asm volatile("{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
               " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem),
               "l"(da), "l"(db), "r"(idesc), "r"(acc));
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void proxy_fence_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

template <int HD>
constexpr int fa_smem() { return (HD / 64) * 3 * TC_TILE + 4 * TC_TILE + 64; }

template <int HD>
__global__ void __launch_bounds__(FA_THREADS, 1) k_fattn(PfAttn P, const int* nact, int* err) {
  constexpr int DC = HD / 64;
  extern __shared__ __align__(1024) uint8_t fsm[];
  uint8_t* sQ = fsm;                        // [DC][hi|lo]: rows = query rows, K = dims
  uint8_t* sK = sQ + DC * 2 * TC_TILE;      // [DC]: rows = positions, K = dims
  uint8_t* sV = sK + DC * TC_TILE;          // [2]: rows = dims, K = positions
  uint8_t* sP = sV + 2 * TC_TILE;           // [2]: rows = query rows, K = positions
  uint64_t* bar = (uint64_t*)(sP + 2 * TC_TILE);   // [0] S ready, [1] O updated, [2] all MMAs done
  __shared__ uint32_t s_tmem;
  __shared__ int s_ok;
  const int T = *nact;
  const int G = P.heads / P.kvh, Bt = FA_ROWS / G;
  const int kvh = blockIdx.y, qt0 = blockIdx.x * Bt;
  if (qt0 >= T) return;
  const int nq = min(Bt, T - qt0);
  const int tid = threadIdx.x, warp = tid >> 5;
  const int qd = P.heads * HD;
  const int pos_hi = P.pos0 + qt0 + nq - 1;
  const int pos_lo = P.pos0 + qt0;
  const int start_lo = (P.window != 0 && pos_lo + 1 > P.window) ? pos_lo + 1 - P.window : 0;
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                 "r"(256));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (tid == 0) {
    mbar_init(bar, 1);
    mbar_init(bar + 1, 1);
    mbar_init(bar + 2, 1);
    mbar_fence_init();
    s_ok = 1;
  }
  // Q rows as two fp16 parts
  for (int i = tid; i < FA_ROWS * (HD / 8); i += FA_THREADS) {
    const int r = i / (HD / 8), d0 = (i % (HD / 8)) * 8;
    float v[8];
    if (r < nq * G) {
      const float* src = P.qr + (size_t)(qt0 + r / G) * qd + (size_t)(kvh * G + r % G) * HD + d0;
      const float4 a = *(const float4*)src, b = *(const float4*)(src + 4);
      v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    } else {
#pragma unroll
      for (int e = 0; e < 8; e++) v[e] = 0.f;
    }
    __align__(16) __half hv[8], lv[8];
#pragma unroll
    for (int e = 0; e < 8; e++) {
      hv[e] = __float2half_rn(v[e]);
      lv[e] = __float2half_rn(v[e] - __half2float(hv[e]));
    }
    const uint32_t off = kmaj_off(r, d0 & 63);
    *(uint4*)(sQ + ((d0 >> 6) * 2) * TC_TILE + off) = *(const uint4*)hv;
    *(uint4*)(sQ + ((d0 >> 6) * 2 + 1) * TC_TILE + off) = *(const uint4*)lv;
  }
  asm volatile("tcgen05.fence::before_thread_sync;");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;");
  const uint32_t tmem = s_tmem, tS = tmem, tO = tmem + 128;
  // the row this thread works on: accumulator lane rl = 32 * (warp % 4) + lane,
  // column half warp / 4; both threads of a row keep its (m, l)
  const int rl = 32 * (warp & 3) + (tid & 31), half = warp >> 2;
  const bool rvalid = rl < nq * G;
  const int rpos = P.pos0 + qt0 + rl / G;
  const int rstart = (P.window != 0 && rpos + 1 > P.window) ? rpos + 1 - P.window : 0;
  const uint32_t lane_base = (uint32_t)(32 * (warp & 3)) << 16;
  const float sl2 = P.scale * 1.4426950408889634f;   // scores in log2 units: exp(x) = exp2(x log2 e)
  __shared__ float red[2][FA_ROWS];
  float m = -INFINITY, l = 0.f;
  const int c_first = start_lo / FA_NP, c_last = pos_hi / FA_NP;
  const uint32_t idS = (1u << 4) | ((uint32_t)(FA_NP >> 3) << 17) | ((uint32_t)(FA_ROWS >> 4) << 24);
  const uint32_t idO = (1u << 4) | ((uint32_t)(HD >> 3) << 17) | ((uint32_t)(FA_ROWS >> 4) << 24);
  bool ok = true;
  for (int ci = c_first; ci <= c_last; ci++) {
    const int j = ci - c_first, p0 = ci * FA_NP;
    if (j > 0 && !mbar_wait_bounded(bar + 1, (j - 1) & 1, err)) ok = false;   // K, V and P free again
    if (!__syncthreads_and(ok)) break;
    {
      // K: a 16-byte piece (8 dims of one position) per item, all of a
      // thread's loads issued before its stores.  A warp takes 8 positions x
      // 4 consecutive pieces: 64 contiguous bytes per position row read, and
      // its 16-byte stores spread over every bank (the 8 positions of a core
      // matrix are 16 bytes apart)
      constexpr int KI = FA_NP * (HD / 8) / FA_THREADS;
      uint4 kq[KI];
      auto kitem = [&](int u, int& pp, int& d0) {
        const int i = tid + u * FA_THREADS, ln = i & 31, w = i >> 5;
        pp = (w % (FA_NP / 8)) * 8 + (ln & 7);
        d0 = ((w / (FA_NP / 8)) * 4 + (ln >> 3)) * 8;
      };
#pragma unroll
      for (int u = 0; u < KI; u++) {
        int pp, d0;
        kitem(u, pp, d0);
        const int p = p0 + pp;
        kq[u] = make_uint4(0, 0, 0, 0);
        if (p >= start_lo && p <= pos_hi)   // rows outside every query's range stay zero
          kq[u] = *(const uint4*)((const __half*)P.kc + ((size_t)kvh * P.ctx + p) * HD + d0);
      }
#pragma unroll
      for (int u = 0; u < KI; u++) {
        int pp, d0;
        kitem(u, pp, d0);
        *(uint4*)(sK + (d0 >> 6) * TC_TILE + kmaj_off(pp, d0 & 63)) = kq[u];
      }
      // V transposed: an 8 x 8 block (8 positions x 8 dims) per item, turned
      // in registers into 8 rows of 8 positions, written in a lane-rotated
      // order (the 8 rows of a block share their bank offset)
      constexpr int VI = (FA_NP / 8) * (HD / 8);
      if (tid < VI) {
        const int pg = tid / (HD / 8), c = tid % (HD / 8);
        __align__(16) __half in[8][8];
#pragma unroll
        for (int r = 0; r < 8; r++) {
          const int p = p0 + 8 * pg + r;
          uint4 v = make_uint4(0, 0, 0, 0);
          if (p >= start_lo && p <= pos_hi)
            v = *(const uint4*)((const __half*)P.vc + ((size_t)kvh * P.ctx + p) * HD + 8 * c);
          *(uint4*)in[r] = v;
        }
        uint4 o[8];
#pragma unroll
        for (int e = 0; e < 8; e++) {
          __align__(16) __half out[8];
#pragma unroll
          for (int r = 0; r < 8; r++) out[r] = in[r][e];
          o[e] = *(const uint4*)out;
        }
        uint8_t* vt = sV + ((8 * pg) >> 6) * TC_TILE;
#pragma unroll
        for (int e0 = 0; e0 < 8; e0++) {
          const int e = (e0 + tid) & 7;
          uint4 v = o[0];
#pragma unroll
          for (int q = 1; q < 8; q++)
            if (e == q) v = o[q];   // selects, not an indexed (local memory) array
          *(uint4*)(vt + kmaj_off(8 * c + e, (8 * pg) & 63)) = v;
        }
      }
    }
    proxy_fence_smem();
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;");
    if (tid == 0) {
#pragma unroll
      for (int c = 0; c < DC; c++)
#pragma unroll
        for (int kk = 0; kk < 4; kk++) {
          const uint64_t db = umma_desc(smem_u32(sK + c * TC_TILE + kk * 4096), 128, 256);
          umma_f16(tS, umma_desc(smem_u32(sQ + (2 * c) * TC_TILE + kk * 4096), 128, 256), db, idS,
                   (c > 0 || kk > 0) ? 1u : 0u);
          umma_f16(tS, umma_desc(smem_u32(sQ + (2 * c + 1) * TC_TILE + kk * 4096), 128, 256), db, idS, 1u);
        }
      umma_commit(bar);
    }
    {
      // two threads per row: warp w reads accumulator lanes 32*(w%4).. and
      // columns 64*(w/4)..+63 of S (held in registers), the row's maximum
      // and sum combined through shared memory; scores in log2 units
      if (!mbar_wait_bounded(bar, j & 1, err)) ok = false;
      asm volatile("tcgen05.fence::after_thread_sync;");
      uint32_t r0[32], r1[32];
      tmem_ld32(tS + lane_base + 64 * half, r0);
      tmem_ld32(tS + lane_base + 64 * half + 32, r1);
      // this row's positions inside the chunk: [vlo, vhi] relative to p0
      const int vlo = max(rstart - p0, 64 * half), vhi = min(rpos - p0, 64 * half + 63);
      float mx = -INFINITY;
#pragma unroll
      for (int e = 0; e < 32; e++) {
        const int c0 = 64 * half + e, c1 = c0 + 32;
        if (rvalid && c0 >= vlo && c0 <= vhi) mx = fmaxf(mx, __uint_as_float(r0[e]) * sl2);
        if (rvalid && c1 >= vlo && c1 <= vhi) mx = fmaxf(mx, __uint_as_float(r1[e]) * sl2);
      }
      red[half][rl] = mx;
      __syncthreads();
      const float mn = fmaxf(m, fmaxf(red[0][rl], red[1][rl]));
      float sum = 0.f;
#pragma unroll
      for (int e8 = 0; e8 < 64; e8 += 8) {
        __align__(16) __half pv[8];
#pragma unroll
        for (int e = 0; e < 8; e++) {
          const int ce = e8 + e, cc = 64 * half + ce;
          const float sv = __uint_as_float(ce < 32 ? r0[ce] : r1[ce - 32]);
          const float pr = (rvalid && cc >= vlo && cc <= vhi) ? exp2f(sv * sl2 - mn) : 0.f;
          sum += pr;
          pv[e] = __float2half_rn(pr);
        }
        *(uint4*)(sP + half * TC_TILE + kmaj_off(rl, e8)) = *(const uint4*)pv;
      }
      const float c = m == -INFINITY ? 0.f : exp2f(m - mn);
      if (j > 0 && __any_sync(0xffffffffu, c != 1.f)) {   // O rows hold earlier chunks: rescale in place
        uint32_t r[32];
        for (int db = half * (HD / 2); db < (half + 1) * (HD / 2); db += 32) {
          tmem_ld32(tO + lane_base + db, r);
#pragma unroll
          for (int e = 0; e < 32; e++) r[e] = __float_as_uint(__uint_as_float(r[e]) * c);
          tmem_st32(tO + lane_base + db, r);
        }
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
      }
      __syncthreads();   // red[] read by both threads of the row before it is reused
      red[half][rl] = sum;
      __syncthreads();
      l = l * c + red[0][rl] + red[1][rl];
      m = mn;
    }
    proxy_fence_smem();
    asm volatile("tcgen05.fence::before_thread_sync;");
    if (!__syncthreads_and(ok)) break;
    asm volatile("tcgen05.fence::after_thread_sync;");
    if (tid == 0) {
#pragma unroll
      for (int pc = 0; pc < 2; pc++)
#pragma unroll
        for (int kk = 0; kk < 4; kk++)
          umma_f16(tO, umma_desc(smem_u32(sP + pc * TC_TILE + kk * 4096), 128, 256),
                   umma_desc(smem_u32(sV + pc * TC_TILE + kk * 4096), 128, 256), idO,
                   (j > 0 || pc > 0 || kk > 0) ? 1u : 0u);
      umma_commit(bar + 1);
    }
  }
  // one more commit: arrives once every MMA issued above has completed (also
  // after an early exit, before shared and tensor memory are released)
  if (tid == 0) umma_commit(bar + 2);
  if (!mbar_wait_bounded(bar + 2, 0, err)) ok = false;
  asm volatile("tcgen05.fence::after_thread_sync;");
  if (!ok) s_ok = 0;
  __syncthreads();
  if (s_ok) {
    // O / l straight into the o projection's operand tiles (8 dims = one
    // 16-byte row of a core matrix per store)
    uint32_t r[32];
    const int tok = qt0 + rl / G, col0 = (kvh * G + rl % G) * HD, nch = tc_nch(qd);
    const float inv = 1.f / l;
    for (int db = half * (HD / 2); db < (half + 1) * (HD / 2); db += 32) {
      tmem_ld32(tO + lane_base + db, r);
      if (rvalid) {
#pragma unroll
        for (int e8 = 0; e8 < 32; e8 += 8) {
          __align__(16) __half hv[8], lv[8];
#pragma unroll
          for (int e = 0; e < 8; e++) {
            const float o = __uint_as_float(r[e8 + e]) * inv;
            hv[e] = __float2half_rn(o);
            lv[e] = __float2half_rn(o - __half2float(hv[e]));
          }
          *(uint4*)(P.xo.xt + tc_index(tok, col0 + db + e8, nch, 0)) = *(const uint4*)hv;
          *(uint4*)(P.xo.xt + tc_index(tok, col0 + db + e8, nch, 1)) = *(const uint4*)lv;
        }
      }
    }
    if (tid == 0 && kvh == 0)
      for (int t = 0; t < nq; t++) P.xo.xs[qt0 + t] = 1.0f;
  }
  asm volatile("tcgen05.fence::before_thread_sync;");
  __syncthreads();
  if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(256));
}

// ---------------------------------------------------------------------------
// Host side.

struct ck_prefill_state {
  std::vector<void*> allocs;
  std::vector<__half*> wt;    // operand tiles: layer-major q k v o gate up down
  int chunk = 0;              // tokens per pass (<= PF_CHUNK_MAX)
  int* d_nact = nullptr;
  int* d_err = nullptr;
  float *x = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *qr = nullptr, *g = nullptr, *u = nullptr;
  BXh xh{};                   // attention output / SiLU product tiles
  BXh xn{};                   // normed residual-stream tiles (written by the o / down epilogues)
  float* ssq = nullptr;       // [token][row tile of hidden] sums of squares of the residual stream
  bool glu = false;           // gate / up interleaved (SiLU in the gate/up GEMM's epilogue)
};

namespace {

template <class T>
int palloc(ck_engine* h, ck_prefill_state* p, T** out, size_t bytes) {
  void* q = nullptr;
  cudaError_t e = cudaMalloc(&q, bytes ? bytes : 16);
  if (e != cudaSuccess) return h->fail(CK_ENOMEM, "prefill cudaMalloc(%zu): %s", bytes, cudaGetErrorString(e));
  p->allocs.push_back(q);
  *out = (T*)q;
  return CK_OK;
}

// The GEMM prefill handles the engine's model.
bool pf_supported(const ck_engine* h) {
  const ck_model_cfg& c = h->cfg;
  const int hd = c.head_dim;
  return c.arch == CK_ARCH_LLAMA && c.hidden % 32 == 0 && c.intermediate % 32 == 0 && c.hidden <= CK_KMAX &&
         c.intermediate <= CK_KMAX && c.heads * hd <= CK_KMAX && (hd == 64 || hd == 128 || hd == 256) &&
         c.heads % c.kv_heads == 0 && c.heads / c.kv_heads <= CK_WARPS && c.heads / c.kv_heads <= CK_GMAX;
}

// Buffers and operand tiles, made at the first GEMM prefill and kept.
int pf_ensure(ck_engine* h) {
  if (h->pf) return CK_OK;
  const ck_model_cfg& c = h->cfg;
  ck_prefill_state* p = new ck_prefill_state();
  auto bail = [&](int rc) {
    for (void* a : p->allocs) cudaFree(a);
    delete p;
    return rc;
  };
  const size_t T = PF_CHUNK_MAX;
  const int H = c.hidden, qd = c.heads * c.head_dim, kvd = c.kv_heads * c.head_dim, I = c.intermediate;
  int rc;
  if ((rc = palloc(h, p, &p->d_nact, 16)) || (rc = palloc(h, p, &p->d_err, 16)) ||
      (rc = palloc(h, p, &p->x, T * H * 4)) || (rc = palloc(h, p, &p->q, T * qd * 4)) ||
      (rc = palloc(h, p, &p->k, T * kvd * 4)) || (rc = palloc(h, p, &p->v, T * kvd * 4)) ||
      (rc = palloc(h, p, &p->qr, T * qd * 4)) ||
      (rc = palloc(h, p, &p->g, T * I * 4)) || (rc = palloc(h, p, &p->u, T * I * 4)) ||
      (rc = palloc(h, p, &p->xh.xt, tc_bytes((int)T, CK_KMAX))) || (rc = palloc(h, p, &p->xh.xs, T * 4)) ||
      (rc = palloc(h, p, &p->xn.xt, tc_bytes((int)T, CK_KMAX))) || (rc = palloc(h, p, &p->xn.xs, T * 4)) ||
      (rc = palloc(h, p, &p->ssq, T * ((H + TC_ROWS - 1) / TC_ROWS) * 4)))
    return bail(rc);
  p->glu = I % (TC_ROWS / 2) == 0;
  for (int i = 0; i < c.layers; i++) {
    const LayerW& W = h->L[i];
    int role = 0;
    for (const Weight* w : {&W.q, &W.k, &W.v, &W.o, &W.gate, &W.up, &W.down}) {
      __half* t = nullptr;
      const int kk = w->L.k;
      if (p->glu && role == 5) {   // held by the gate's interleaved tiles
        p->wt.push_back(nullptr);
        role++;
        continue;
      }
      if (p->glu && role == 4) {
        if ((rc = palloc(h, p, &t, tc_bytes(2 * w->n, kk)))) return bail(rc);
        k_tc_format<<<dim3(2 * w->n / TC_ROWS, tc_nch(kk)), 256, 0, h->stream>>>(w->dev, w->L, w->n, kk, t,
                                                                               W.up.dev, W.up.L);
      } else {
        if ((rc = palloc(h, p, &t, tc_bytes(w->n, kk)))) return bail(rc);
        k_tc_format<<<dim3((w->n + TC_ROWS - 1) / TC_ROWS, tc_nch(kk)), 256, 0, h->stream>>>(w->dev, w->L, w->n,
                                                                                            kk, t);
      }
      p->wt.push_back(t);
      role++;
    }
  }
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) e = cudaMemsetAsync(p->d_err, 0, 16, h->stream);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(k_bgemm_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, TC_SMEM);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(k_fattn<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, fa_smem<64>());
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(k_fattn<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, fa_smem<128>());
  if (e == cudaSuccess) e = cudaStreamSynchronize(h->stream);
  if (e != cudaSuccess) return bail(h->fail(CK_ECUDA, "prefill setup: %s", cudaGetErrorString(e)));
  tc_max_clusters(1);
  p->chunk = h->pf_chunk > 0 && h->pf_chunk <= PF_CHUNK_MAX ? h->pf_chunk : PF_CHUNK_MAX;
  h->pf = p;
  return CK_OK;
}

// K/V rows into the cache, then the attention: on the tensor cores for an
// fp16 cache with head_dim 64 or 128, else one CTA per (token, kv head).
template <int E>
void pf_attn_launch(const PfAttn& a, bool f32, int T, const int* nact, int* err, cudaStream_t s) {
  constexpr int hd = 32 * E;
  const int grid = T * a.kvh;
  const int pkv_grid = (T * (a.heads + 2 * a.kvh) + PKV_WARPS - 1) / PKV_WARPS;
  if (f32) {
    k_pkv<E, true><<<pkv_grid, 32 * PKV_WARPS, 0, s>>>(a, nact);
    k_pattn<E, true><<<grid, CK_THREADS, 0, s>>>(a, nact);
    return;
  }
  k_pkv<E, false><<<pkv_grid, 32 * PKV_WARPS, 0, s>>>(a, nact);
  if (hd == 64 || hd == 128) {
    const int bt = FA_ROWS / (a.heads / a.kvh);
    k_fattn<hd == 64 ? 64 : 128><<<dim3((T + bt - 1) / bt, a.kvh), FA_THREADS, fa_smem<hd == 64 ? 64 : 128>(), s>>>(
        a, nact, err);
  } else {
    k_pattn<E, false><<<grid, CK_THREADS, 0, s>>>(a, nact);
  }
}

// Tokens D.tokens[h->pos .. h->pos + n) through every layer, their K/V rows
// written into the cache; no logits.  h->pos is not advanced here.
int prefill_gemm(ck_engine* h, int n) {
  int rc = pf_ensure(h);
  if (rc) return rc;
  ck_prefill_state* p = h->pf;
  const ck_model_cfg& c = h->cfg;
  const int H = c.hidden, hd = c.head_dim, qd = c.heads * hd, kvd = c.kv_heads * hd, I = c.intermediate;
  const size_t per = (size_t)c.kv_heads * c.context_length * hd * elem_kv(c);
  const bool f32 = c.kv_dtype == CK_KV_F32;
  cudaStream_t s = h->stream;
  for (int c0 = 0; c0 < n; c0 += p->chunk) {
    const int T = n - c0 < p->chunk ? n - c0 : p->chunk;
    const int p0 = h->pos + c0, ttiles = (T + TC_NT - 1) / TC_NT;
    k_set_int<<<1, 1, 0, s>>>(p->d_nact, T);
    BStep st;
    memset(&st, 0, sizeof st);
    st.tok = h->D.tokens + p0;
    st.nact = p->d_nact;
    const int htiles = (H + TC_ROWS - 1) / TC_ROWS;
    auto prep = [&](int kind, const float* a, const float* bb, const float* w, int k, BXh x) {
      BPrep pp;
      pp.kind = kind; pp.a = a; pp.b = bb; pp.w = w; pp.eps = c.norm_eps; pp.k = k; pp.lda = k;
      k_bprep<<<T, CK_THREADS, 0, s>>>(pp, st, x);
    };
    // x: operand tiles read; nw: also write the next norm's tiles into xn
    // (residual-stream GEMMs); norm_in: prologue scale from those sums;
    // glu_xt: gate/up over interleaved tiles, silu(gate) * up into glu_xt
    auto gemm = [&](int k, std::initializer_list<BSeg> segs, BXh x, const float* nw, bool norm_in,
                    __half* glu_xt) {
      BGemm G;
      memset(&G, 0, sizeof G);
      G.k = k;
      if (nw) { G.nw = nw; G.nxt = p->xn.xt; G.nssq = p->ssq; G.ntiles = htiles; }
      if (norm_in) { G.ssq_in = p->ssq; G.ssq_tiles = htiles; G.eps = c.norm_eps; }
      G.glu_xt = glu_xt;
      G.glu_k = I;
      int tiles = 0;
      for (const BSeg& x : segs) {
        G.tile0[G.nseg] = tiles;
        G.seg[G.nseg++] = x;
        tiles += (x.n + TC_ROWS - 1) / TC_ROWS;
      }
      G.tile0[G.nseg] = tiles;
      return tc_launch(G, st, x, p->d_err, ttiles, s);
    };
    k_bembed<<<T, 256, 0, s>>>(h->emb.dev, h->emb.L, c.embedding_scale, st, p->x, H, c.vocab, p->d_err);
    // only layer 0's attention norm is a prologue; the o and down GEMMs write
    // the next norm's operand tiles in their epilogue
    prep(BP_NORM, p->x, nullptr, h->L[0].attn_norm, H, p->xn);
    for (int i = 0; i < c.layers; i++) {
      const LayerW& W = h->L[i];
      __half* const* wt = &p->wt[(size_t)7 * i];
      CKC(h, gemm(H, {bseg(W.q, wt[0], p->q, nullptr, qd), bseg(W.k, wt[1], p->k, nullptr, kvd),
                      bseg(W.v, wt[2], p->v, nullptr, kvd)}, p->xn, nullptr, i > 0, nullptr));
      PfAttn a;
      a.q = p->q; a.k = p->k; a.v = p->v;
      a.qw = c.qk_norm ? W.q_norm : nullptr;
      a.kw = c.qk_norm ? W.k_norm : nullptr;
      a.kc = h->kv + (size_t)(2 * i) * per;
      a.vc = h->kv + (size_t)(2 * i + 1) * per;
      a.inv_freq = h->inv_freq + (size_t)i * (hd / 2);
      a.qr = p->qr;
      a.xo = p->xh;
      a.heads = c.heads; a.kvh = c.kv_heads; a.hd = hd; a.ctx = c.context_length;
      a.window = (int)c.layer_window[i];
      a.interleaved = c.rope_interleaved;
      a.pos0 = p0;
      a.eps = c.qk_norm_eps;
      a.scale = (float)(1.0 / sqrt((double)hd));   // ATTN_SCALE (:1711)
      if (hd == 64) pf_attn_launch<2>(a, f32, T, p->d_nact, p->d_err, s);
      else if (hd == 128) pf_attn_launch<4>(a, f32, T, p->d_nact, p->d_err, s);
      else pf_attn_launch<8>(a, f32, T, p->d_nact, p->d_err, s);
      CKC(h, gemm(qd, {bseg(W.o, wt[3], p->x, p->x, H)}, p->xh, W.post_norm, false, nullptr));
      if (p->glu) {
        BSeg gu = bseg(W.gate, wt[4], nullptr, nullptr, 0);
        gu.n = 2 * I;
        CKC(h, gemm(H, {gu}, p->xn, nullptr, true, p->xh.xt));
      } else {
        CKC(h, gemm(H, {bseg(W.gate, wt[4], p->g, nullptr, I), bseg(W.up, wt[5], p->u, nullptr, I)}, p->xn, nullptr,
                    true, nullptr));
        prep(BP_SILU, p->g, p->u, nullptr, I, p->xh);
      }
      // the last layer's output only feeds the single-token step (its own norm)
      const float* next_norm = i + 1 < c.layers ? h->L[i + 1].attn_norm : nullptr;
      CKC(h, gemm(I, {bseg(W.down, wt[6], p->x, p->x, H)}, p->xh, next_norm, false, nullptr));
    }
    CKC(h, cudaGetLastError());
  }
  int* e = (int*)(h->pinned + 512);
  CKC(h, d2h(h, e, p->d_err, 4));
  CKC(h, cudaStreamSynchronize(h->stream));
  if (*e) {
    cudaMemsetAsync(p->d_err, 0, 16, h->stream);
    cudaStreamSynchronize(h->stream);
    return h->fail(CK_EDEVICE, "prefill: device wait timed out (bits 0x%x)", *e);
  }
  return CK_OK;
}

}  // namespace

void pf_free(ck_engine* h) {
  if (!h->pf) return;
  for (void* a : h->pf->allocs) cudaFree(a);
  delete h->pf;
  h->pf = nullptr;
}

extern "C" int ck_set_prefill_gemm(ck_engine* h, int min_tokens, int chunk) {
  if (!h) return set_global(CK_EINVAL, "null engine");
  if (min_tokens < 0 || chunk < 0 || chunk > PF_CHUNK_MAX)
    return h->fail(CK_EINVAL, "ck_set_prefill_gemm: min_tokens %d, chunk %d (at most %d)", min_tokens, chunk,
                   PF_CHUNK_MAX);
  h->pf_min = min_tokens;
  h->pf_chunk = chunk;
  if (h->pf) h->pf->chunk = chunk > 0 ? chunk : PF_CHUNK_MAX;
  return CK_OK;
}
