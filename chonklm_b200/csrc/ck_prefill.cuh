// Prefill on the tensor cores: a prompt's tokens through the layers together.
//
// The reference feeds a prompt one id per runToken call
// (llama-wgsl-runtime.ts:281-288 inside generateLlamaWgsl, each call the
// whole graph of :1039-1124).  Here every prompt token but the last goes
// through the layers at once, up to a chunk of tokens at a time, on the
// batched path's kernels:
//
// * every matmul is the tcgen05 GEMM over the chunk's tokens (k_bgemm_tc on
//   the weights' operand tiles, the norm / copy / SiLU prologue in k_bprep);
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
  float* out;                 // [T][heads*hd]
  int heads, kvh, hd, ctx, window, interleaved, pos0;
  float eps, scale;
};

__global__ void k_set_int(int* p, int v) { *p = v; }

// QK-norm + RoPE of one (token, kv head): the G query heads into qr, the K
// and V rows into the cache at the token's position (the decode step's
// attention prologue, one token per CTA).
template <int E, bool F32>
__global__ void __launch_bounds__(CK_THREADS) k_pkv(PfAttn P, const int* nact) {
  constexpr int hd = 32 * E;
  const int t = blockIdx.x / P.kvh, kvh = blockIdx.x % P.kvh;
  if (t >= *nact) return;
  __shared__ SmemAt s;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = P.heads / P.kvh, qd = P.heads * hd, kvd = P.kvh * hd;
  const int pos = P.pos0 + t;
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
  float* qdst = P.qr + (size_t)t * qd + (size_t)kvh * G * hd;
  for (int i = tid; i < G * hd; i += CK_THREADS) qdst[i] = s.qs[i];
  const size_t cb = ((size_t)kvh * P.ctx + pos) * hd;
  for (int d = tid; d < hd; d += CK_THREADS) {
    if (F32) {
      ((float*)P.kc)[cb + d] = s.kst[d];
      ((float*)P.vc)[cb + d] = s.kvw[1][d];
    } else {
      ((__half*)P.kc)[cb + d] = __float2half_rn(s.kst[d]);
      ((__half*)P.vc)[cb + d] = __float2half_rn(s.kvw[1][d]);
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
  for (int i = tid; i < G * hd; i += CK_THREADS) {
    const int gg = i / hd, d = i % hd;
    float A = 0.f;
    for (int w = gg * wpg; w < gg * wpg + wpg; w++) A += wacc[w * CK_HDMAX + d] * wf[w];
    P.out[(size_t)t * qd + (size_t)(kvh * G + gg) * hd + d] = A / hl[gg];
  }
}

// ---------------------------------------------------------------------------
// Host side.

struct ck_prefill_state {
  std::vector<void*> allocs;
  std::vector<__half*> wt;    // operand tiles: layer-major q k v o gate up down
  int chunk = 0;              // tokens per pass (<= PF_CHUNK_MAX)
  int* d_nact = nullptr;
  int* d_err = nullptr;
  float *x = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *qr = nullptr, *ao = nullptr, *g = nullptr,
        *u = nullptr;
  BXh xh{};
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
      (rc = palloc(h, p, &p->qr, T * qd * 4)) || (rc = palloc(h, p, &p->ao, T * qd * 4)) ||
      (rc = palloc(h, p, &p->g, T * I * 4)) || (rc = palloc(h, p, &p->u, T * I * 4)) ||
      (rc = palloc(h, p, &p->xh.xt, tc_bytes((int)T, CK_KMAX))) || (rc = palloc(h, p, &p->xh.xs, T * 4)))
    return bail(rc);
  for (int i = 0; i < c.layers; i++) {
    const LayerW& W = h->L[i];
    for (const Weight* w : {&W.q, &W.k, &W.v, &W.o, &W.gate, &W.up, &W.down}) {
      __half* t = nullptr;
      const int kk = w->L.k;
      if ((rc = palloc(h, p, &t, tc_bytes(w->n, kk)))) return bail(rc);
      k_tc_format<<<dim3((w->n + TC_ROWS - 1) / TC_ROWS, tc_nch(kk)), 256, 0, h->stream>>>(w->dev, w->L, w->n, kk, t);
      p->wt.push_back(t);
    }
  }
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) e = cudaMemsetAsync(p->d_err, 0, 16, h->stream);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(k_bgemm_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, TC_SMEM);
  if (e == cudaSuccess) e = cudaStreamSynchronize(h->stream);
  if (e != cudaSuccess) return bail(h->fail(CK_ECUDA, "prefill setup: %s", cudaGetErrorString(e)));
  tc_max_clusters(1);
  p->chunk = h->pf_chunk > 0 && h->pf_chunk <= PF_CHUNK_MAX ? h->pf_chunk : PF_CHUNK_MAX;
  h->pf = p;
  return CK_OK;
}

template <int E>
void pf_attn_launch(const PfAttn& a, bool f32, int grid, const int* nact, cudaStream_t s) {
  if (f32) {
    k_pkv<E, true><<<grid, CK_THREADS, 0, s>>>(a, nact);
    k_pattn<E, true><<<grid, CK_THREADS, 0, s>>>(a, nact);
  } else {
    k_pkv<E, false><<<grid, CK_THREADS, 0, s>>>(a, nact);
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
    auto prep = [&](int kind, const float* a, const float* bb, const float* w, int k) {
      BPrep pp;
      pp.kind = kind; pp.a = a; pp.b = bb; pp.w = w; pp.eps = c.norm_eps; pp.k = k; pp.lda = k;
      k_bprep<<<T, CK_THREADS, 0, s>>>(pp, st, p->xh);
    };
    auto gemm = [&](int k, std::initializer_list<BSeg> segs) {
      BGemm G;
      memset(&G, 0, sizeof G);
      G.k = k;
      int tiles = 0;
      for (const BSeg& x : segs) {
        G.tile0[G.nseg] = tiles;
        G.seg[G.nseg++] = x;
        tiles += (x.n + TC_ROWS - 1) / TC_ROWS;
      }
      G.tile0[G.nseg] = tiles;
      return tc_launch(G, st, p->xh, p->d_err, ttiles, s);
    };
    k_bembed<<<T, 256, 0, s>>>(h->emb.dev, h->emb.L, c.embedding_scale, st, p->x, H, c.vocab, p->d_err);
    for (int i = 0; i < c.layers; i++) {
      const LayerW& W = h->L[i];
      __half* const* wt = &p->wt[(size_t)7 * i];
      prep(BP_NORM, p->x, nullptr, W.attn_norm, H);
      CKC(h, gemm(H, {bseg(W.q, wt[0], p->q, nullptr, qd), bseg(W.k, wt[1], p->k, nullptr, kvd),
                      bseg(W.v, wt[2], p->v, nullptr, kvd)}));
      PfAttn a;
      a.q = p->q; a.k = p->k; a.v = p->v;
      a.qw = c.qk_norm ? W.q_norm : nullptr;
      a.kw = c.qk_norm ? W.k_norm : nullptr;
      a.kc = h->kv + (size_t)(2 * i) * per;
      a.vc = h->kv + (size_t)(2 * i + 1) * per;
      a.inv_freq = h->inv_freq + (size_t)i * (hd / 2);
      a.qr = p->qr;
      a.out = p->ao;
      a.heads = c.heads; a.kvh = c.kv_heads; a.hd = hd; a.ctx = c.context_length;
      a.window = (int)c.layer_window[i];
      a.interleaved = c.rope_interleaved;
      a.pos0 = p0;
      a.eps = c.qk_norm_eps;
      a.scale = (float)(1.0 / sqrt((double)hd));   // ATTN_SCALE (:1711)
      const int grid = T * c.kv_heads;
      if (hd == 64) pf_attn_launch<2>(a, f32, grid, p->d_nact, s);
      else if (hd == 128) pf_attn_launch<4>(a, f32, grid, p->d_nact, s);
      else pf_attn_launch<8>(a, f32, grid, p->d_nact, s);
      prep(BP_COPY, p->ao, nullptr, nullptr, qd);
      CKC(h, gemm(qd, {bseg(W.o, wt[3], p->x, p->x, H)}));
      prep(BP_NORM, p->x, nullptr, W.post_norm, H);
      CKC(h, gemm(H, {bseg(W.gate, wt[4], p->g, nullptr, I), bseg(W.up, wt[5], p->u, nullptr, I)}));
      prep(BP_SILU, p->g, p->u, nullptr, I);
      CKC(h, gemm(I, {bseg(W.down, wt[6], p->x, p->x, H)}));
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
