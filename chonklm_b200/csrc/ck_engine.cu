// chonk_b200 engine: device buffers, phase schedule, CUDA graphs and the C ABI.
//
// Host-side twin of LlamaWgslEngine (llama-wgsl-runtime.ts:619-1220): it owns
// every device buffer (weights, KV cache, scratch) and frees them in
// ck_destroy, as `dispose` does (:1152-1215).
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/chonk_b200.h"
#include "ck_ops.cuh"
#include "ck_step.cuh"
#include "ck_gemv.cuh"

namespace {

thread_local std::string g_err;

int set_global(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_err = buf;
  return code;
}

struct Weight {
  Lay L;
  int n = 0;
  uint8_t* dev = nullptr;
  bool present = false;
};

struct LayerW {
  Weight q, k, v, o, gate, up, down;
  float *attn_norm = nullptr, *post_norm = nullptr, *pre_ffn = nullptr, *post_ffn = nullptr;
  float *q_norm = nullptr, *k_norm = nullptr;
};

size_t elem_kv(const ck_model_cfg& c) { return c.kv_dtype == CK_KV_F32 ? 4 : 2; }

}  // namespace

struct ck_prefill_state;   // tensor-core prefill buffers (ck_prefill.cuh)

// Weights (device layout) up to this size are kept in the 126 MB L2 across tokens.
#define CK_L2_RESIDENT_BYTES (112.0 * 1024 * 1024)

struct ck_engine {
  ck_model_cfg cfg;
  int device = 0;
  int sms = 0;
  cudaStream_t own = nullptr, stream = nullptr;
  std::string err;
  bool finalized = false;
  int mode = 0;  // 0 megakernel, 1 graph of per-phase kernels, 2 streaming step (k_step)

  std::vector<LayerW> L;
  Weight emb, head;
  float* final_norm = nullptr;
  std::vector<void*> allocs;

  // device state
  CkState* st = nullptr;
  CkDev D;
  // inter-phase activations: 8-byte tagged words (value + tag, see ck_ops.cuh)
  float *resA = nullptr, *resB = nullptr, *tmp = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *attn = nullptr,
        *g = nullptr, *u = nullptr;
  float* part = nullptr;
  uint32_t epoch_steps = 1;       // mirror of CkState::epoch
  std::vector<std::pair<void*, size_t>> tagged_bufs;
  float* inv_freq = nullptr;  // [layers][head_dim/2] RoPE inverse frequencies
  uint8_t* kv = nullptr;
  size_t kv_bytes = 0;
  int smax = 1;

  // schedules
  std::vector<Phase> ph_logits, ph_prefill;
  Phase *d_logits = nullptr, *d_prefill = nullptr;     // per-phase launches (mode 1)
  Phase *dm_logits = nullptr, *dm_prefill = nullptr;   // same phases partitioned for the megakernel grid
  int mega_grid = 0;
  cudaGraphExec_t gx_logits[3] = {nullptr, nullptr, nullptr}, gx_prefill[3] = {nullptr, nullptr, nullptr};
  // streaming step (mode 2): schedules and its tagged vectors (ck_step.cuh)
  bool sk_ok = false;
  std::vector<SkPhase> sk_logits, sk_prefill;
  SkPhase *dsk_logits = nullptr, *dsk_prefill = nullptr;
  unsigned long long *pk_sub = nullptr, *pk_q = nullptr, *pk_k = nullptr, *pk_v = nullptr, *pk_att = nullptr,
                     *pk_act = nullptr, *pk_part = nullptr;

  CkDev Dlaunch;            // CkDev passed to kernels (trace pointer only when tracing)
  bool trace_on = false;
  // host mirrors
  int pos = 0;
  unsigned long long io_h2d = 0, io_d2h = 0;  // bytes copied by step calls
  CkState shadow;
  uint8_t* pinned = nullptr;  // staging for small copies
  // tensor-core prefill: prompts of at least pf_min tokens (0: never), pf_chunk
  // tokens per pass (0: the largest)
  ck_prefill_state* pf = nullptr;
  int pf_min = 64, pf_chunk = 0;
  int sampler_exact = 0;      // ck_set_sampler
  const void* mega_fn = nullptr;   // the k_mega instantiation for this model (mega_kernel)

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

#define CKC(h, call)                                                                                    \
  do {                                                                                                  \
    cudaError_t e_ = (call);                                                                            \
    if (e_ != cudaSuccess) return (h)->fail(CK_ECUDA, "%s: %s (%s:%d)", #call, cudaGetErrorString(e_), \
                                           __FILE__, __LINE__);                                          \
  } while (0)

#define CKG(call)                                                                                       \
  do {                                                                                                  \
    cudaError_t e_ = (call);                                                                            \
    if (e_ != cudaSuccess) return set_global(CK_ECUDA, "%s: %s", #call, cudaGetErrorString(e_));       \
  } while (0)

namespace {

// Host<->device copies of the step calls, counted for the e2e report.
cudaError_t h2d(ck_engine* h, void* dst, const void* src, size_t n) {
  h->io_h2d += n;
  return cudaMemcpyAsync(dst, src, n, cudaMemcpyHostToDevice, h->stream);
}
cudaError_t d2h(ck_engine* h, void* dst, const void* src, size_t n) {
  h->io_d2h += n;
  return cudaMemcpyAsync(dst, src, n, cudaMemcpyDeviceToHost, h->stream);
}

template <class T>
int dalloc(ck_engine* h, T** p, size_t bytes) {
  void* q = nullptr;
  cudaError_t e = cudaMalloc(&q, bytes ? bytes : 16);
  if (e != cudaSuccess) return h->fail(CK_ENOMEM, "cudaMalloc(%zu): %s", bytes, cudaGetErrorString(e));
  h->allocs.push_back(q);
  *p = (T*)q;
  return CK_OK;
}

// Raw GGUF blocks (host) -> device streaming layout.
int upload_quant(ck_engine* h, Weight& w, int type, int k, int n, const void* bytes, size_t nbytes,
                 const char* name) {
  if (!ck_type_ok(type))
    return h->fail(CK_EINVAL, "Llama WGSL tensor %s is not a supported GGUF quantized tensor (type %d)", name, type);
  if (k % ck_block_weights(type) != 0)
    return h->fail(CK_EINVAL, "GGML tensor type %d requires %d-element rows, %s has %d", type,
                   ck_block_weights(type), name, k);
  size_t raw = (size_t)n * (k / ck_block_weights(type)) * ck_block_bytes(type);
  if (nbytes != raw) return h->fail(CK_EINVAL, "%s: %zu bytes, expected %zu", name, nbytes, raw);
  Lay L = make_lay(type, k);
  uint8_t* tmp = nullptr;
  CKC(h, cudaMalloc(&tmp, raw));
  cudaError_t e = cudaMemcpyAsync(tmp, bytes, raw, cudaMemcpyHostToDevice, h->own);
  if (e != cudaSuccess) { cudaFree(tmp); return h->fail(CK_ECUDA, "upload %s: %s", name, cudaGetErrorString(e)); }
  uint8_t* dst = nullptr;
  int rc = dalloc(h, &dst, (size_t)L.row_bytes * n);
  if (rc) { cudaFree(tmp); return rc; }
  cudaMemsetAsync(dst, 0, (size_t)L.row_bytes * n, h->own);
  long long total = (long long)n * L.nb;
  k_relayout<<<(unsigned)((total + 255) / 256), 256, 0, h->own>>>(tmp, dst, L, n);
  e = cudaStreamSynchronize(h->own);
  cudaFree(tmp);
  if (e != cudaSuccess) return h->fail(CK_ECUDA, "relayout %s: %s", name, cudaGetErrorString(e));
  w.L = L;
  w.n = n;
  w.dev = dst;
  w.present = true;
  return CK_OK;
}

float f16_bits_to_f32(uint16_t b) {
  // exact, subnormals kept (f16ToF32, llama-wgsl-runtime.ts:1837-1844)
  int s = (b >> 15) & 1, e = (b >> 10) & 0x1f, f = b & 0x3ff;
  float v;
  if (e == 0) v = ldexpf((float)f, -24);
  else if (e == 31) v = f ? NAN : INFINITY;
  else v = ldexpf((float)(1024 + f), e - 25);
  return s ? -v : v;
}

int upload_norm(ck_engine* h, float** dst, int type, int n_expected, int64_t ne, const void* bytes, size_t nbytes,
                const char* name) {
  if (type != CK_GGML_F32 && type != CK_GGML_F16)
    return h->fail(CK_EINVAL, "Llama WGSL tensor %s is %d, expected float32/float16", name, type);
  if (ne != n_expected) return h->fail(CK_EINVAL, "%s: %lld elements, expected %d", name, (long long)ne, n_expected);
  if (nbytes != (size_t)ne * (type == CK_GGML_F32 ? 4 : 2))
    return h->fail(CK_EINVAL, "%s: %zu bytes for %lld elements", name, nbytes, (long long)ne);
  std::vector<float> f(ne);
  if (type == CK_GGML_F32) memcpy(f.data(), bytes, nbytes);
  else {
    const uint16_t* p = (const uint16_t*)bytes;
    for (int64_t i = 0; i < ne; i++) f[i] = f16_bits_to_f32(p[i]);
  }
  if (!*dst) {
    int rc = dalloc(h, dst, (size_t)ne * 4);
    if (rc) return rc;
  }
  CKC(h, cudaMemcpy(*dst, f.data(), (size_t)ne * 4, cudaMemcpyHostToDevice));
  return CK_OK;
}

Pro pro_norm(const float* a, const float* w, float eps) {
  Pro p{};
  p.kind = PRO_NORM; p.a = a; p.w0 = w; p.eps = eps;
  return p;
}
Pro pro_gemma(const float* sub, const float* wpost, const float* rin, float* rout, const float* wpre, float eps) {
  Pro p{};
  p.kind = PRO_GEMMA; p.a = sub; p.w1 = wpost; p.rin = rin; p.rout = rout; p.w0 = wpre; p.eps = eps;
  return p;
}
MvSeg seg(const Weight& w, float* out, const float* add) {
  MvSeg s{};
  s.w = w.dev; s.out = out; s.add = add; s.L = w.L; s.n = w.n;
  return s;
}

Phase mk_mv(ck_engine* h, const Pro& pro, int k, std::initializer_list<MvSeg> segs) {
  Phase p;
  memset(&p, 0, sizeof p);
  p.kind = PH_MATVEC;
  p.mv.pro = pro;
  p.mv.k = k;
  p.mv.nseg = 0;
  for (const MvSeg& s : segs) p.mv.seg[p.mv.nseg++] = s;
  // one CTA per SM: each streams a contiguous row range through its tile ring
  int rows = 0;
  for (int i = 0; i < p.mv.nseg; i++) rows = rows > p.mv.seg[i].n ? rows : p.mv.seg[i].n;
  p.grid = rows < h->sms ? (rows < 1 ? 1 : rows) : h->sms;
  set_partition(p, p.grid);
  return p;
}

// The down projection's prologue.  When every CTA's share of the gate/up
// rows fits the staging rows, the gate/up phase applies the activation to its
// own rows (act(gate) * up into h->g) and down copies that; otherwise down
// applies it to the whole vector in its prologue.
Pro glu_input(ck_engine* h, Phase& gateup, int epi) {
  const int n = gateup.mv.seg[0].n;
  const int grid = n < h->sms ? n : h->sms;    // the smallest grid either mode launches
  Pro p{};
  if ((n + grid - 1) / grid <= CK_GLU_MAX && gateup.mv.seg[1].n == n) {
    gateup.mv.epi = epi;
    gateup.mv.glu_out = h->g;
    p.kind = PRO_COPY;
    p.a = h->g;
  } else {
    p.kind = epi == EPI_SILU ? PRO_SILU : PRO_GELU;
    p.a = h->g;
    p.b = h->u;
  }
  return p;
}

// Inter-phase activations are tagged words; weights and logits are plain.
bool tagged_buffer(const ck_engine* h, const void* p) {
  return p && (p == h->resA || p == h->resB || p == h->tmp || p == h->q || p == h->k || p == h->v || p == h->attn ||
               p == h->g || p == h->u);
}

// Walk a schedule in order: a read of a tagged buffer expects the tag of its
// latest writer (phase index + 1), a write carries the writer's own tag.
void assign_tags(ck_engine* h, std::vector<Phase>& ph) {
  std::map<const void*, int> last;
  auto rd = [&](const void* p) {
    if (!tagged_buffer(h, p)) return 0;
    auto it = last.find(p);
    return it == last.end() ? 0 : it->second;
  };
  auto wr = [&](const void* p, int me) {
    if (!tagged_buffer(h, p)) return 0;
    last[p] = me;
    return me;
  };
  for (size_t i = 0; i < ph.size(); i++) {
    Phase& p = ph[i];
    const int me = (int)i + 1;
    if (p.kind == PH_EMBED) {
      p.em.tout = wr(p.em.out, me);
    } else if (p.kind == PH_MATVEC || p.kind == PH_FNORM) {
      Pro& r = p.mv.pro;
      r.ta = rd(r.a);
      r.tb = (r.kind == PRO_SILU || r.kind == PRO_GELU) ? rd(r.b) : 0;
      r.trin = r.kind == PRO_GEMMA ? rd(r.rin) : 0;
      for (int s = 0; s < p.mv.nseg; s++) p.mv.seg[s].tadd = rd(p.mv.seg[s].add);
      if (r.kind == PRO_GEMMA) r.trout = wr(r.rout, me);
      if (p.mv.epi) p.mv.tglu = wr(p.mv.glu_out, me);
      else
        for (int s = 0; s < p.mv.nseg; s++) p.mv.seg[s].tout = wr(p.mv.seg[s].out, me);
    } else if (p.kind == PH_ATTN) {
      p.at.tqkv = rd(p.at.q);
      p.at.tout = wr(p.at.out, me);
    }
  }
}

void build_schedule(ck_engine* h, bool logits, std::vector<Phase>& out) {
  const ck_model_cfg& c = h->cfg;
  const int H = c.hidden, hd = c.head_dim, qd = c.heads * hd;
  const bool gemma = c.arch == CK_ARCH_GEMMA3;
  out.clear();
  Phase p;
  memset(&p, 0, sizeof p);
  p.kind = PH_EMBED;
  p.grid = (H + CK_THREADS - 1) / CK_THREADS;
  if (p.grid < 8) p.grid = 8;
  p.em.w = h->emb.dev;
  p.em.L = h->emb.L;
  p.em.out = h->resA;
  p.em.scale = c.embedding_scale;
  p.em.need_logits = logits ? 1 : 0;
  out.push_back(p);

  float* cur = h->resA;    // residual before the layer's first add
  float* other = h->resB;
  for (int i = 0; i < c.layers; i++) {
    const LayerW& W = h->L[i];
    Pro pq = (!gemma || i == 0) ? pro_norm(cur, W.attn_norm, c.norm_eps)
                                : pro_gemma(h->tmp, h->L[i - 1].post_ffn, cur, other, W.attn_norm, c.norm_eps);
    if (gemma && i > 0) std::swap(cur, other);
    out.push_back(mk_mv(h, pq, H, {seg(W.q, h->q, nullptr), seg(W.k, h->k, nullptr), seg(W.v, h->v, nullptr)}));

    Phase a;
    memset(&a, 0, sizeof a);
    a.kind = PH_ATTN;
    a.at.q = h->q; a.at.k = h->k; a.at.v = h->v;
    a.at.qw = c.qk_norm ? W.q_norm : nullptr;
    a.at.kw = c.qk_norm ? W.k_norm : nullptr;
    size_t per = (size_t)c.kv_heads * c.context_length * hd * elem_kv(c);
    a.at.inv_freq = h->inv_freq + (size_t)i * (hd / 2);
    a.at.kc = h->kv + (size_t)(2 * i) * per;
    a.at.vc = h->kv + (size_t)(2 * i + 1) * per;
    a.at.out = h->attn;
    a.at.part = h->part;
    a.at.heads = c.heads; a.at.kvh = c.kv_heads; a.at.hd = hd; a.at.ctx = c.context_length;
    a.at.group = c.heads / c.kv_heads;
    a.at.window = (int)c.layer_window[i];
    a.at.interleaved = c.rope_interleaved;
    a.at.kv_f32 = c.kv_dtype == CK_KV_F32;
    a.at.smax = h->smax;
    a.at.theta = c.layer_rope_theta[i];
    a.at.eps = c.qk_norm_eps;
    a.at.scale = (float)(1.0 / sqrt((double)hd));  // ATTN_SCALE constant (:1711)
    a.grid = c.kv_heads * h->smax;  // units are split-major: unit = split * kv_heads + head
    out.push_back(a);

    Pro pc{};
    pc.kind = PRO_COPY;
    pc.a = h->attn;
    if (!gemma) {
      // o_proj + residual add; addRmsNorm's norm moves into the gate/up prologue
      out.push_back(mk_mv(h, pc, qd, {seg(W.o, cur, cur)}));
      out.push_back(mk_mv(h, pro_norm(cur, W.post_norm, c.norm_eps), H,
                          {seg(W.gate, h->g, nullptr), seg(W.up, h->u, nullptr)}));
      out.push_back(mk_mv(h, glu_input(h, out.back(), EPI_SILU), c.intermediate, {seg(W.down, cur, cur)}));
    } else {
      out.push_back(mk_mv(h, pc, qd, {seg(W.o, h->tmp, nullptr)}));
      out.push_back(mk_mv(h, pro_gemma(h->tmp, W.post_norm, cur, other, W.pre_ffn, c.norm_eps), H,
                          {seg(W.gate, h->g, nullptr), seg(W.up, h->u, nullptr)}));
      std::swap(cur, other);
      out.push_back(mk_mv(h, glu_input(h, out.back(), EPI_GELU), c.intermediate, {seg(W.down, h->tmp, nullptr)}));
    }
  }
  if (logits) {
    Pro pf = !gemma ? pro_norm(cur, h->final_norm, c.norm_eps)
                    : pro_gemma(h->tmp, h->L[c.layers - 1].post_ffn, cur, other, h->final_norm, c.norm_eps);
    // the final norm on one CTA, then the LM head as its own launch of the
    // streaming matvec kernel (k_gemv: dedicated copy warp, 96 KB slots,
    // block type fixed at compile time), plain floats in and out
    Phase fn = mk_mv(h, pf, H, {seg(h->head, h->D.logits, nullptr)});
    fn.kind = PH_FNORM;
    fn.mv.nseg = 0;
    fn.grid = 1;
    out.push_back(fn);
    Phase hp;
    memset(&hp, 0, sizeof hp);
    hp.kind = PH_HEAD;
    hp.grid = h->sms;
    out.push_back(hp);
    Phase a1;
    memset(&a1, 0, sizeof a1);
    a1.kind = PH_ARGMAX1;
    a1.barrier_after = 1;           // select reads every chunk's candidate
    // one CTA per SM, one warp per 256-logit chunk: a CTA of its own per
    // chunk kept 15 of its 16 warps idle and took several waves
    a1.grid = (c.vocab + 255) / 256;
    if (a1.grid > h->sms) a1.grid = h->sms;
    out.push_back(a1);
  }
  Phase f;
  memset(&f, 0, sizeof f);
  f.kind = logits ? PH_SELECT : PH_FINISH;   // select = argmax stage 2 + sampling + finish
  f.grid = 1;
  f.need_logits = logits ? 1 : 0;
  out.push_back(f);
  for (size_t i = 0; i < out.size(); i++) out[i].index = (int)i;
  assign_tags(h, out);
}

// ---- streaming step (mode 2) -------------------------------------------------
// Words of a row-partitioned tagged vector of n elements over `grid` CTAs:
// CTA c's rows start its own segment of 2^sh words (at least 16 words, one
// 128-byte line).  grid 1: a flat vector.
int pk_sh(int per) {
  int sh = 4;
  while ((1 << sh) < per) sh++;
  return sh;
}
unsigned long long magic40(int d) { return ((1ull << 40) + (unsigned long long)d - 1) / (unsigned long long)d; }
PkVec make_pk(unsigned long long* p, int n, int grid) {
  PkVec v;
  memset(&v, 0, sizeof v);
  v.p = p; v.n = n; v.grid = grid; v.sh = pk_sh((n + grid - 1) / grid);
  v.mn = magic40(n);
  v.mg = magic40(grid);
  return v;
}
size_t pk_words(int n, int grid) { return (size_t)grid << pk_sh((n + grid - 1) / grid); }

bool sk_supported(const ck_engine* h) {
  const ck_model_cfg& c = h->cfg;
  const int G = c.heads / c.kv_heads, I = c.intermediate, grid = h->sms;
  // every CTA must own rows of every matvec phase (see sk_row0)
  const bool fanin = c.hidden >= grid && I >= grid && c.heads * c.head_dim >= grid;
  return fanin && c.hidden <= SK_HMAX && c.hidden <= CK_KMAX && I <= CK_KMAX && c.heads * c.head_dim <= CK_KMAX &&
         G <= CK_GMAX && (c.head_dim == 64 || c.head_dim == 128 || c.head_dim == 256) &&
         (I + grid - 1) / grid <= SK_GLU_MAX && c.vocab < (1 << 20);
}

SkPhase sk_mv(const ck_engine* h, int k, std::initializer_list<std::pair<const Weight*, PkVec>> segs) {
  SkPhase p;
  memset(&p, 0, sizeof p);
  p.kind = SK_MV;
  p.mv.k = k;
  p.mv.eps = h->cfg.norm_eps;
  for (const auto& sg : segs) {
    SkSeg& S = p.mv.seg[p.mv.nseg++];
    S.w = sg.first->dev; S.L = sg.first->L; S.n = sg.first->n; S.out = sg.second;
  }
  sk_partition(p.mv, h->sms);
  return p;
}

// The step as streaming phases (see ck_step.cuh): per layer QKV, attention,
// o, gate/up (+ activation), down; the LM head last.  Residual updates and
// norms sit in the prologue of the phase that reads a sub-layer's output.
void build_sk_schedule(ck_engine* h, bool logits, std::vector<SkPhase>& out) {
  const ck_model_cfg& c = h->cfg;
  const int H = c.hidden, hd = c.head_dim, qd = c.heads * hd, kvd = c.kv_heads * hd, I = c.intermediate;
  const int grid = h->sms;
  const bool gemma = c.arch == CK_ARCH_GEMMA3;
  const PkVec sub = make_pk(h->pk_sub, H, grid);
  const PkVec q = make_pk(h->pk_q, qd, grid), k = make_pk(h->pk_k, kvd, grid), v = make_pk(h->pk_v, kvd, grid);
  const PkVec att = make_pk(h->pk_att, qd, 1);    // flat: written by the attention owners
  const PkVec act = make_pk(h->pk_act, I, grid);
  PkVec none;
  memset(&none, 0, sizeof none);
  out.clear();
  auto push = [&](SkPhase p) {
    p.index = (int)out.size();
    p.out_tag = p.index + 1;
    out.push_back(p);
    return p.out_tag;
  };
  int sub_tag = 0;
  for (int i = 0; i < c.layers; i++) {
    const LayerW& W = h->L[i];
    SkPhase a = sk_mv(h, H, {{&W.q, q}, {&W.k, k}, {&W.v, v}});
    a.mv.in = sub;
    a.mv.in_tag = sub_tag;
    a.mv.norm = 1;
    a.mv.wnorm = W.attn_norm;
    if (i == 0) {
      a.mv.res = RES_EMBED;
      a.mv.emb = h->emb.dev;
      a.mv.embL = h->emb.L;
      a.mv.emb_scale = c.embedding_scale;
    } else if (gemma) {
      a.mv.res = RES_GEMMA;
      a.mv.wpost = h->L[i - 1].post_ffn;
    } else {
      a.mv.res = RES_ADD;
    }
    const int qkv_tag = push(a);

    SkPhase t;
    memset(&t, 0, sizeof t);
    t.kind = SK_ATTN;
    t.at.q = q; t.at.k = k; t.at.v = v;
    t.at.in_tag = qkv_tag;
    t.at.qw = c.qk_norm ? W.q_norm : nullptr;
    t.at.kw = c.qk_norm ? W.k_norm : nullptr;
    const size_t per_layer = (size_t)c.kv_heads * c.context_length * hd * elem_kv(c);
    t.at.kc = h->kv + (size_t)(2 * i) * per_layer;
    t.at.vc = h->kv + (size_t)(2 * i + 1) * per_layer;
    t.at.inv_freq = h->inv_freq + (size_t)i * (hd / 2);
    t.at.out = h->pk_att;
    t.at.part = h->pk_part;
    t.at.heads = c.heads; t.at.kvh = c.kv_heads; t.at.hd = hd; t.at.ctx = c.context_length;
    t.at.group = c.heads / c.kv_heads;
    t.at.window = (int)c.layer_window[i];
    t.at.interleaved = c.rope_interleaved;
    t.at.kv_f32 = c.kv_dtype == CK_KV_F32;
    t.at.smax = h->smax;
    t.at.eps = c.qk_norm_eps;
    t.at.scale = (float)(1.0 / sqrt((double)hd));  // ATTN_SCALE constant (:1711)
    const int att_tag = push(t);
    // without logits nothing reads the last layer past its K/V store
    if (!logits && i == c.layers - 1) break;

    SkPhase o = sk_mv(h, qd, {{&W.o, sub}});
    o.mv.in = att;
    o.mv.in_tag = att_tag;
    const int o_tag = push(o);

    SkPhase gu = sk_mv(h, H, {{&W.gate, none}, {&W.up, none}});
    gu.mv.in = sub;
    gu.mv.in_tag = o_tag;
    gu.mv.norm = 1;
    if (gemma) {
      gu.mv.res = RES_GEMMA;
      gu.mv.wpost = W.post_norm;
      gu.mv.wnorm = W.pre_ffn;
      gu.mv.epi = EPI_GELU;
    } else {
      gu.mv.res = RES_ADD;
      gu.mv.wnorm = W.post_norm;
      gu.mv.epi = EPI_SILU;
    }
    gu.mv.act = act;
    const int gu_tag = push(gu);

    SkPhase d = sk_mv(h, I, {{&W.down, sub}});
    d.mv.in = act;
    d.mv.in_tag = gu_tag;
    sub_tag = push(d);
  }
  if (logits) {
    SkPhase hp = sk_mv(h, H, {{&h->head, none}});
    hp.kind = SK_HEAD;
    hp.mv.in = sub;
    hp.mv.in_tag = sub_tag;
    hp.mv.norm = 1;
    hp.mv.wnorm = h->final_norm;
    hp.mv.logits = h->D.logits;
    if (gemma) {
      hp.mv.res = RES_GEMMA;
      hp.mv.wpost = h->L[c.layers - 1].post_ffn;
    } else {
      hp.mv.res = RES_ADD;
    }
    push(hp);
  }
}

int sk_setup(ck_engine* h) {
  const ck_model_cfg& c = h->cfg;
  if (!sk_supported(h)) return CK_OK;   // the other modes serve this model
  const int grid = h->sms, G = c.heads / c.kv_heads, hd = c.head_dim;
  const size_t words[6] = {pk_words(c.hidden, grid), pk_words(c.heads * hd, grid), pk_words(c.kv_heads * hd, grid),
                           pk_words(c.kv_heads * hd, grid), (size_t)c.heads * hd, pk_words(c.intermediate, grid)};
  unsigned long long** bufs[6] = {&h->pk_sub, &h->pk_q, &h->pk_k, &h->pk_v, &h->pk_att, &h->pk_act};
  int rc;
  for (int i = 0; i < 6; i++) {
    if ((rc = dalloc(h, bufs[i], words[i] * 8))) return rc;
    CKC(h, cudaMemset(*bufs[i], 0, words[i] * 8));
    h->tagged_bufs.push_back({*bufs[i], words[i] * 8});
  }
  const size_t part = (size_t)c.kv_heads * h->smax * G * (hd + 2) * 8;
  if ((rc = dalloc(h, &h->pk_part, part))) return rc;
  CKC(h, cudaMemset(h->pk_part, 0, part));
  h->tagged_bufs.push_back({h->pk_part, part});
  build_sk_schedule(h, true, h->sk_logits);
  build_sk_schedule(h, false, h->sk_prefill);
  for (int l = 0; l < 2; l++) {
    std::vector<SkPhase>& v = l ? h->sk_logits : h->sk_prefill;
    SkPhase** dst = l ? &h->dsk_logits : &h->dsk_prefill;
    if ((rc = dalloc(h, dst, v.size() * sizeof(SkPhase)))) return rc;
    CKC(h, cudaMemcpy(*dst, v.data(), v.size() * sizeof(SkPhase), cudaMemcpyHostToDevice));
  }
  CKC(h, cudaFuncSetAttribute(k_step, cudaFuncAttributeMaxDynamicSharedMemorySize, SK_DYN_BYTES));
  int per_sm = 0;
  CKC(h, cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_step, SK_THREADS, SK_DYN_BYTES));
  if (per_sm < 1) return CK_OK;
  h->sk_ok = true;
  return CK_OK;
}

// A k_mega instantiation compiled for the headline model family (Qwen3
// Q4_K_M: Q4_K and Q6_K weights, head_dim 128, fp16 cache): it only leaves
// out code for the types and head sizes the model does not have, so its
// results are the generic kernel's bit for bit, and it decodes ~2 % faster
// (906 vs 922 us per token).  Compiled the same way, the SmolLM2, Gemma-3
// and Q8_0 families measured 0.5-4 % slower than the generic kernel, so they
// run the generic one.
#define CK_TM_KQ (CK_TM(GT_Q4_K) | CK_TM(GT_Q6_K))
struct MegaVariant {
  unsigned tm;
  int ae;
  const void* fn;
};
const MegaVariant kMegaVariants[] = {
    {CK_TM_KQ, 4, (const void*)k_mega<0, CK_TM_KQ, 4>},
};
const void* const kMegaGeneric = (const void*)k_mega<0, CK_TM_ALL, 0>;
// The generic kernel with the attention's mergers on the top kv_heads CTAs
// (attn_unit_top) and the phase after the attention on the CTAs below them:
// for head_dim 64 (the SmolLM2 family), where it decodes 6-10 % faster.  As
// a run-time switch inside the generic kernel the same code cost the other
// families 0.5-3 %, so it is an instantiation of its own.
const void* const kMegaOwnTop = (const void*)k_mega<0, CK_TM_ALL, 0, 1>;

unsigned model_type_mask(const ck_engine* h) {
  unsigned m = CK_TM(h->head.L.type);
  for (int i = 0; i < h->cfg.layers; i++) {
    const LayerW& W = h->L[i];
    for (const Weight* w : {&W.q, &W.k, &W.v, &W.o, &W.gate, &W.up, &W.down})
      if (w->present) m |= CK_TM(w->L.type);
  }
  return m;
}

const void* mega_kernel(const ck_engine* h) {
  const char* g = getenv("CK_MEGA_GENERIC");
  if (g && atoi(g) != 0) return kMegaGeneric;
  const ck_model_cfg& c = h->cfg;
  const int ae = c.kv_dtype != CK_KV_F16 ? 0 : c.head_dim == 64 ? 2 : c.head_dim == 128 ? 4 : c.head_dim == 256 ? 8 : 0;
  const unsigned m = model_type_mask(h);
  for (const MegaVariant& v : kMegaVariants)
    if (v.ae == ae && (m & ~v.tm) == 0) return v.fn;
  if (c.head_dim == 64 && h->mega_grid > 2 * c.kv_heads) return kMegaOwnTop;
  return kMegaGeneric;
}

// The LM head of a logits step: D.xhead (the final norm's output) -> D.logits.
void head_launch(ck_engine* h, cudaStream_t s) {
  const Weight& w = h->head;
  gv_kernel(w.L.type)<<<h->sms, GV_THREADS, GV_DYN_BYTES, s>>>(w.dev, w.L, w.n, h->D.xhead, h->D.logits, &h->st->err);
}

int enqueue_phases(ck_engine* h, bool logits, int mode, cudaStream_t s) {
  const std::vector<Phase>& ph = logits ? h->ph_logits : h->ph_prefill;
  if (mode == 2) {
    CKC(h, cudaMemsetAsync(&h->st->bar, 0, sizeof(uint32_t), s));
    const SkPhase* dph = logits ? h->dsk_logits : h->dsk_prefill;
    int nph = (int)(logits ? h->sk_logits.size() : h->sk_prefill.size());
    int lg = logits ? 1 : 0;
    void* args[] = {(void*)&dph, (void*)&nph, (void*)&lg, (void*)&h->Dlaunch};
    CKC(h, cudaLaunchCooperativeKernel((const void*)k_step, dim3(h->sms), dim3(SK_THREADS), args, SK_DYN_BYTES, s));
    return CK_OK;
  }
  if (mode == 1) {
    const Phase* dph = logits ? h->d_logits : h->d_prefill;
    for (size_t i = 0; i < ph.size(); i++) {
      if (ph[i].kind == PH_HEAD) head_launch(h, s);
      else if (ph[i].kind == PH_MATVEC) k_mv<<<ph[i].grid, CK_THREADS, CK_DYN_PHASES + sizeof(Phase), s>>>(dph + i, h->Dlaunch);
      else if (ph[i].kind == PH_ATTN) k_attn<<<ph[i].grid, CK_THREADS, 0, s>>>(dph + i, h->Dlaunch);
      else k_misc<<<ph[i].grid, CK_THREADS, 0, s>>>(dph + i, h->Dlaunch);
    }
    CKC(h, cudaGetLastError());
    return CK_OK;
  }
  CKC(h, cudaMemsetAsync(&h->st->bar, 0, sizeof(uint32_t), s));
  // the megakernel runs every phase up to the LM head; the head (k_gemv),
  // argmax stage 1 and select follow as their own launches
  const Phase* dph = logits ? h->dm_logits : h->dm_prefill;
  int nph = (int)ph.size();
  for (int i = 0; i < (int)ph.size(); i++)
    if (ph[i].kind == PH_HEAD) { nph = i; break; }
  void* args[] = {(void*)&dph, (void*)&nph, (void*)&h->Dlaunch};
  size_t dyn = CK_DYN_PHASES + (size_t)nph * sizeof(Phase);
  CKC(h, cudaLaunchCooperativeKernel(h->mega_fn, dim3(h->mega_grid), dim3(CK_THREADS), args, dyn, s));
  for (size_t i = nph; i < ph.size(); i++) {
    if (ph[i].kind == PH_HEAD) head_launch(h, s);
    else k_misc<<<ph[i].grid, CK_THREADS, 0, s>>>(dph + i, h->Dlaunch);
  }
  CKC(h, cudaGetLastError());
  return CK_OK;
}

int capture(ck_engine* h, bool logits, int mode, cudaGraphExec_t* out) {
  cudaStream_t s = h->own;
  cudaGraph_t g = nullptr;
  CKC(h, cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
  int rc = enqueue_phases(h, logits, mode, s);
  cudaError_t e = cudaStreamEndCapture(s, &g);
  if (rc) { if (g) cudaGraphDestroy(g); return rc; }
  if (e != cudaSuccess) return h->fail(CK_ECUDA, "graph capture: %s", cudaGetErrorString(e));
  e = cudaGraphInstantiate(out, g, 0);
  cudaGraphDestroy(g);
  if (e != cudaSuccess) return h->fail(CK_ECUDA, "graph instantiate: %s", cudaGetErrorString(e));
  return CK_OK;
}

// Clear every tagged buffer and restart the
// device step counter at 1, so no stored tag can match a later step: at
// set-up, after a step gave up part-way, and before the 22-bit step field
// of the tags would wrap.
int epoch_restart(ck_engine* h) {
  CKC(h, cudaStreamSynchronize(h->stream));
  for (auto& b : h->tagged_bufs) CKC(h, cudaMemset(b.first, 0, b.second));
  const uint32_t one = 1;
  CKC(h, cudaMemcpy(&h->st->epoch, &one, 4, cudaMemcpyHostToDevice));
  h->epoch_steps = 1;
  return CK_OK;
}

int launch_step(ck_engine* h, bool logits) {
  if (h->epoch_steps >= (1u << 22) - 2) {
    int rc = epoch_restart(h);
    if (rc) return rc;
  }
  h->epoch_steps++;
  cudaGraphExec_t gx = logits ? h->gx_logits[h->mode] : h->gx_prefill[h->mode];
  if (gx) {
    CKC(h, cudaGraphLaunch(gx, h->stream));
    return CK_OK;
  }
  return enqueue_phases(h, logits, h->mode, h->stream);
}

// Host option block -> device (sampling.ts SamplingOptions + penalty plumbing
// of LlamaWgslEngine.argmax, llama-wgsl-runtime.ts:1647-1665).
int set_params(ck_engine* h, const ck_sampling* s, int chain, uint64_t draw_override, bool use_override) {
  CkState& p = h->shadow;
  double temp = s ? s->temperature : 0.0, top_p = s ? s->top_p : 1.0, pen = s ? s->repetition_penalty : 1.0;
  int top_k = s ? s->top_k : 0;
  p.temperature = temp;
  p.top_p = top_p;
  p.top_k = top_k < 0 ? 0 : top_k;
  p.pen_d = pen;
  p.pen_milli = (uint32_t)floor(pen * 1000.0 + 0.5);
  p.sampling = (temp > 0.0 || top_p < 1.0 || p.top_k > 0) ? 1 : 0;
  p.chain = chain;
  p.seed = s ? s->philox_seed : 0ull;
  p.exact = h->sampler_exact;
  p.draw = use_override ? (uint32_t)draw_override : (s ? (uint32_t)s->philox_offset : 0u);
  p.abort_flag = 0;
  p.bar = 0;
  p.pen_src = 0;
  p.pen_count = 0;
  if (s && s->penalized_ids) {
    int n = s->n_penalized;
    if (n < 0) n = 0;
    // penalizedTokenIds.slice(-contextLength) (:1651-1653)
    int keep = n > h->cfg.context_length ? h->cfg.context_length : n;
    const uint32_t* ids = s->penalized_ids + (n - keep);
    p.pen_src = 1;
    p.pen_count = keep;
    if (keep > 0) CKC(h, h2d(h, h->D.pen_list, ids, (size_t)keep * 4));
  }
  size_t off = offsetof(CkState, draw);
  memcpy(h->pinned, (const uint8_t*)&p + off, sizeof(CkState) - off);
  CKC(h, h2d(h, (uint8_t*)h->st + off, h->pinned, sizeof(CkState) - off));
  return CK_OK;
}

int check_device(ck_engine* h) {
  int* e = (int*)(h->pinned + 256);
  CKC(h, d2h(h, e, &h->st->err, 4));
  CKC(h, cudaStreamSynchronize(h->stream));
  if (*e) {
    int bits = *e;
    cudaMemsetAsync(&h->st->err, 0, 4, h->stream);
    cudaMemsetAsync(&h->st->abort_flag, 0, 4, h->stream);
    cudaStreamSynchronize(h->stream);
    if (bits & ~CK_DERR_TOKEN) epoch_restart(h);   // a step gave up part-way
    if (bits & CK_DERR_TOKEN) return h->fail(CK_EDEVICE, "token id outside embedding table");
    if (bits & CK_DERR_BARRIER) return h->fail(CK_EDEVICE, "device grid barrier timed out");
    return h->fail(CK_EDEVICE, "device error bits 0x%x", bits);
  }
  return CK_OK;
}

int set_pos_dev(ck_engine* h, int pos) {
  int* p = (int*)(h->pinned + 320);
  *p = pos;
  CKC(h, h2d(h, &h->st->pos, p, 4));
  CKC(h, cudaStreamSynchronize(h->stream));
  h->pos = pos;
  return CK_OK;
}

}  // namespace

// ============================================================================
extern "C" {

const char* ck_global_error(void) { return g_err.c_str(); }

void ck_abi_info(int* sizeof_cfg, int* sizeof_sampling) {
  if (sizeof_cfg) *sizeof_cfg = (int)sizeof(ck_model_cfg);
  if (sizeof_sampling) *sizeof_sampling = (int)sizeof(ck_sampling);
}
const char* ck_last_error(ck_engine* h) { return h ? h->err.c_str() : g_err.c_str(); }

int ck_create(const ck_model_cfg* cfg, int device, ck_engine** out) {
  if (!cfg || !out) return set_global(CK_EINVAL, "ck_create: null argument");
  const ck_model_cfg& c = *cfg;
  if (c.arch != CK_ARCH_LLAMA && c.arch != CK_ARCH_GEMMA3) return set_global(CK_EINVAL, "unsupported arch %d", c.arch);
  if (c.layers <= 0 || c.layers > CK_MAX_LAYERS) return set_global(CK_EINVAL, "layers %d out of range", c.layers);
  if (c.hidden <= 0 || c.hidden % 32 || c.hidden > CK_KMAX) return set_global(CK_EINVAL, "hidden %d unsupported", c.hidden);
  if (c.intermediate <= 0 || c.intermediate % 32 || c.intermediate > CK_KMAX)
    return set_global(CK_EINVAL, "intermediate %d unsupported", c.intermediate);
  if (c.head_dim != 64 && c.head_dim != 128 && c.head_dim != 256)
    return set_global(CK_EINVAL, "head_dim %d unsupported (64/128/256)", c.head_dim);
  if (c.heads <= 0 || c.kv_heads <= 0 || c.heads % c.kv_heads)
    return set_global(CK_EINVAL, "heads %d / kv_heads %d invalid", c.heads, c.kv_heads);
  int G = c.heads / c.kv_heads;
  if (G > CK_GMAX || G * c.head_dim > 1024)
    return set_global(CK_EINVAL, "GQA group %d x head_dim %d unsupported", G, c.head_dim);
  if (c.heads * c.head_dim > CK_KMAX) return set_global(CK_EINVAL, "q dim too large");
  if (c.vocab <= 0 || (c.vocab + 255) / 256 > CK_SAMPLE_MAX) return set_global(CK_EINVAL, "vocab %d unsupported", c.vocab);
  if (c.context_length <= 0) return set_global(CK_EINVAL, "context_length %d", c.context_length);
  CKG(cudaSetDevice(device));
  ck_engine* h = new ck_engine();
  h->cfg = c;
  h->device = device;
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) { delete h; return set_global(CK_ECUDA, "no device"); }
  h->sms = prop.multiProcessorCount;
  if (cudaStreamCreateWithFlags(&h->own, cudaStreamNonBlocking) != cudaSuccess) {
    delete h;
    return set_global(CK_ECUDA, "stream create failed");
  }
  h->stream = h->own;
  h->L.resize(c.layers);
  memset(&h->shadow, 0, sizeof h->shadow);
  if (cudaHostAlloc((void**)&h->pinned, 4096, cudaHostAllocDefault) != cudaSuccess) {
    cudaStreamDestroy(h->own);
    delete h;
    return set_global(CK_ECUDA, "pinned alloc failed");
  }
  const char* m = getenv("CK_MODE");
  if (m && atoi(m) == 1) h->mode = 1;
  *out = h;
  return CK_OK;
}

int ck_upload_tensor(ck_engine* h, const char* name, int ggml_type, const int64_t* shape, int ndim, const void* bytes,
                     size_t nbytes) {
  if (!h || !name || !shape || ndim < 1 || !bytes) return set_global(CK_EINVAL, "ck_upload_tensor: bad argument");
  if (h->finalized) return h->fail(CK_ESTATE, "ck_upload_tensor after ck_finalize");
  CKC(h, cudaSetDevice(h->device));
  const ck_model_cfg& c = h->cfg;
  int64_t ne0 = shape[0], ne1 = ndim > 1 ? shape[1] : 1;
  for (int i = 2; i < ndim; i++) ne1 *= shape[i];
  std::string s(name);
  const int H = c.hidden, qd = c.heads * c.head_dim, kvd = c.kv_heads * c.head_dim, I = c.intermediate;
  auto quant = [&](Weight& w, int k, int n) -> int {
    if (ne0 != k || ne1 != n)
      return h->fail(CK_EINVAL, "%s: shape [%lld, %lld], expected [%d, %d]", name, (long long)ne0, (long long)ne1, k, n);
    return upload_quant(h, w, ggml_type, k, n, bytes, nbytes, name);
  };
  if (s == "token_embd.weight") return quant(h->emb, H, c.vocab);
  if (s == "output.weight") return quant(h->head, H, c.vocab);
  if (s == "output_norm.weight") return upload_norm(h, &h->final_norm, ggml_type, H, ne0 * ne1, bytes, nbytes, name);
  int layer = -1, used = 0;
  char rest[128];
  if (sscanf(name, "blk.%d.%127s%n", &layer, rest, &used) == 2 && layer >= 0 && layer < c.layers) {
    LayerW& W = h->L[layer];
    std::string r(rest);
    bool gemma = c.arch == CK_ARCH_GEMMA3;
    if (r == "attn_q.weight") return quant(W.q, H, qd);
    if (r == "attn_k.weight") return quant(W.k, H, kvd);
    if (r == "attn_v.weight") return quant(W.v, H, kvd);
    if (r == "attn_output.weight") return quant(W.o, qd, H);
    if (r == "ffn_gate.weight") return quant(W.gate, H, I);
    if (r == "ffn_up.weight") return quant(W.up, H, I);
    if (r == "ffn_down.weight") return quant(W.down, I, H);
    if (r == "attn_norm.weight") return upload_norm(h, &W.attn_norm, ggml_type, H, ne0 * ne1, bytes, nbytes, name);
    if (r == "attn_q_norm.weight")
      return upload_norm(h, &W.q_norm, ggml_type, c.head_dim, ne0 * ne1, bytes, nbytes, name);
    if (r == "attn_k_norm.weight")
      return upload_norm(h, &W.k_norm, ggml_type, c.head_dim, ne0 * ne1, bytes, nbytes, name);
    // post_attention_layernorm alias: ffn_norm (llama) / post_attention_norm (gemma3), :346-352
    if (!gemma && r == "ffn_norm.weight")
      return upload_norm(h, &W.post_norm, ggml_type, H, ne0 * ne1, bytes, nbytes, name);
    if (gemma && r == "post_attention_norm.weight")
      return upload_norm(h, &W.post_norm, ggml_type, H, ne0 * ne1, bytes, nbytes, name);
    if (gemma && r == "ffn_norm.weight")
      return upload_norm(h, &W.pre_ffn, ggml_type, H, ne0 * ne1, bytes, nbytes, name);
    if (gemma && r == "post_ffw_norm.weight")
      return upload_norm(h, &W.post_ffn, ggml_type, H, ne0 * ne1, bytes, nbytes, name);
  }
  return CK_OK;  // tensors the decode step does not read are ignored
}

int ck_finalize(ck_engine* h) {
  if (!h) return set_global(CK_EINVAL, "null engine");
  if (h->finalized) return CK_OK;
  CKC(h, cudaSetDevice(h->device));
  const ck_model_cfg& c = h->cfg;
  bool gemma = c.arch == CK_ARCH_GEMMA3;
  if (!h->emb.present) return h->fail(CK_EINVAL, "Llama WGSL manifest missing tensor token_embd.weight");
  if (!h->final_norm) return h->fail(CK_EINVAL, "Llama WGSL manifest missing tensor output_norm.weight");
  if (!h->head.present) h->head = h->emb;  // tied LM head (:345)
  for (int i = 0; i < c.layers; i++) {
    LayerW& W = h->L[i];
    if (!W.q.present || !W.k.present || !W.v.present)
      return h->fail(CK_EINVAL, "Llama WGSL layer %d is missing attention projection weights", i);
    if (!W.o.present) return h->fail(CK_EINVAL, "layer %d is missing attn_output.weight", i);
    if (!W.gate.present || !W.up.present || !W.down.present)
      return h->fail(CK_EINVAL, "Llama WGSL layer %d is missing MLP projection weights", i);
    if (!W.attn_norm || !W.post_norm) return h->fail(CK_EINVAL, "layer %d is missing norm weights", i);
    if (gemma && (!W.pre_ffn || !W.post_ffn || !W.q_norm || !W.k_norm))
      return h->fail(CK_EINVAL, "Gemma WGSL layer is missing required weights");
    if (c.qk_norm && (!W.q_norm || !W.k_norm)) return h->fail(CK_EINVAL, "layer %d is missing q/k norm", i);
  }
  int rc;
  const int H = c.hidden, hd = c.head_dim;
  int G = c.heads / c.kv_heads;
  // at most one attention unit per CTA: a CTA that ran two units in turn
  // would finish last and hold up the merge
  h->smax = h->sms / c.kv_heads;
  if (h->smax > 64) h->smax = 64;
  {
    // The split holding pos merges the splits' partials with 8 loads in
    // flight per lane and Pw lanes per output element: when one pass covers
    // every element, up to 8 * Pw splits cost one round trip and more cost
    // two, so the split count stops there (Qwen3: 16 instead of 18).
    const int NE = (c.heads / c.kv_heads) * c.head_dim;
    int pw = 1;
    while (pw < 32 && 2 * pw * NE <= CK_THREADS) pw *= 2;
    if (pw * NE <= CK_THREADS && h->smax > 8 * pw) h->smax = 8 * pw;
    const char* se = getenv("CK_SMAX");
    if (se && atoi(se) > 0) h->smax = atoi(se);
  }
  if (h->smax < 1) h->smax = 1;
  if ((rc = dalloc(h, &h->st, sizeof(CkState)))) return rc;
  CKC(h, cudaMemset(h->st, 0, sizeof(CkState)));
  memset(&h->D, 0, sizeof h->D);
  h->D.st = h->st;
  h->D.vocab = c.vocab;
  h->D.ctx = c.context_length;
  if ((rc = dalloc(h, &h->D.tokens, (size_t)c.context_length * 4))) return rc;
  if ((rc = dalloc(h, &h->D.pen_list, (size_t)c.context_length * 4))) return rc;
  if ((rc = dalloc(h, &h->D.pen_mask, (size_t)((c.vocab + 31) / 32) * 4))) return rc;
  if ((rc = dalloc(h, &h->D.logits, (size_t)c.vocab * 4))) return rc;
  if ((rc = dalloc(h, &h->D.xhead, (size_t)c.hidden * 4))) return rc;
  int groups = (c.vocab + 255) / 256;
  if ((rc = dalloc(h, &h->D.cand_val, (size_t)groups * 4))) return rc;
  if ((rc = dalloc(h, &h->D.cand_idx, (size_t)groups * 4))) return rc;
  // exact sampler: per-CTA candidate lists for the widest stage-1 grid
  h->D.xgrid = h->sms * 4;
  if ((rc = dalloc(h, &h->D.xval, (size_t)h->D.xgrid * CK_SAMPLE_MAX * 4))) return rc;
  if ((rc = dalloc(h, &h->D.xidx, (size_t)h->D.xgrid * CK_SAMPLE_MAX * 4))) return rc;
  if ((rc = dalloc(h, &h->D.xcnt, (size_t)h->D.xgrid * 4))) return rc;
  CKC(h, cudaMemset(h->D.tokens, 0, (size_t)c.context_length * 4));
  CKC(h, cudaMemset(h->D.pen_mask, 0, (size_t)((c.vocab + 31) / 32) * 4));
  // tagged activations: 8 bytes per element, cleared so no tag matches a step
  const size_t tagged_elems[9] = {(size_t)H, (size_t)H, (size_t)H, (size_t)c.heads * hd, (size_t)c.kv_heads * hd,
                                  (size_t)c.kv_heads * hd, (size_t)c.heads * hd, (size_t)c.intermediate,
                                  (size_t)c.intermediate};
  float** tagged[9] = {&h->resA, &h->resB, &h->tmp, &h->q, &h->k, &h->v, &h->attn, &h->g, &h->u};
  for (int i = 0; i < 9; i++) {
    if ((rc = dalloc(h, tagged[i], tagged_elems[i] * 8))) return rc;
    CKC(h, cudaMemset(*tagged[i], 0, tagged_elems[i] * 8));
    h->tagged_bufs.push_back({*tagged[i], tagged_elems[i] * 8});
  }
  // attention split partials, tagged words
  const size_t part_bytes = (size_t)c.kv_heads * h->smax * G * (hd + 2) * 8;
  if ((rc = dalloc(h, &h->part, part_bytes))) return rc;
  CKC(h, cudaMemset(h->part, 0, part_bytes));
  h->tagged_bufs.push_back({h->part, part_bytes});
  if ((rc = dalloc(h, &h->inv_freq, (size_t)c.layers * (hd / 2) * 4))) return rc;
  for (int i = 0; i < c.layers; i++)
    k_inv_freq<<<1, 128>>>(h->inv_freq + (size_t)i * (hd / 2), c.layer_rope_theta[i], hd);
  CKC(h, cudaGetLastError());
  h->kv_bytes = (size_t)c.layers * 2 * c.kv_heads * c.context_length * hd * elem_kv(c);
  if ((rc = dalloc(h, &h->kv, h->kv_bytes))) return rc;
  CKC(h, cudaMemset(h->kv, 0, h->kv_bytes));

  if ((rc = epoch_restart(h))) return rc;
  {
    // every weight read per token (layers + LM head, device layout) fits L2
    // with room for the KV cache and activations: stream them evict-last so
    // they stay resident across tokens (CK_L2_KEEP=0/1 overrides)
    double wb = 0, kb = 0;
    ck_step_bytes(h, &wb, &kb);
    h->D.l2_keep = wb <= CK_L2_RESIDENT_BYTES ? 1 : 0;
    const char* keep = getenv("CK_L2_KEEP");
    if (keep) h->D.l2_keep = atoi(keep) ? 1 : 0;
  }
  h->Dlaunch = h->D;
  build_schedule(h, true, h->ph_logits);
  build_schedule(h, false, h->ph_prefill);
  if ((rc = dalloc(h, &h->d_logits, h->ph_logits.size() * sizeof(Phase)))) return rc;
  if ((rc = dalloc(h, &h->d_prefill, h->ph_prefill.size() * sizeof(Phase)))) return rc;
  CKC(h, cudaMemcpy(h->d_logits, h->ph_logits.data(), h->ph_logits.size() * sizeof(Phase), cudaMemcpyHostToDevice));
  CKC(h, cudaMemcpy(h->d_prefill, h->ph_prefill.data(), h->ph_prefill.size() * sizeof(Phase),
                    cudaMemcpyHostToDevice));
  if (h->ph_logits.size() * sizeof(Phase) > CK_PHASE_SMEM_MAX)
    return h->fail(CK_EINVAL, "%zu decode phases exceed the %d-byte descriptor stage", h->ph_logits.size(),
                   CK_PHASE_SMEM_MAX);
  CKC(h, cudaFuncSetAttribute(kMegaGeneric, cudaFuncAttributeMaxDynamicSharedMemorySize, CK_DYN_SMEM_MAX));
  CKC(h, cudaFuncSetAttribute(kMegaOwnTop, cudaFuncAttributeMaxDynamicSharedMemorySize, CK_DYN_SMEM_MAX));
  if (!gv_kernel(h->head.L.type)) return h->fail(CK_EINVAL, "LM head block type %d unsupported", h->head.L.type);
  CKC(h, cudaFuncSetAttribute((const void*)gv_kernel(h->head.L.type), cudaFuncAttributeMaxDynamicSharedMemorySize,
                              GV_DYN_BYTES));
  for (const MegaVariant& v : kMegaVariants)
    CKC(h, cudaFuncSetAttribute(v.fn, cudaFuncAttributeMaxDynamicSharedMemorySize, CK_DYN_SMEM_MAX));
  CKC(h, cudaFuncSetAttribute(k_mv, cudaFuncAttributeMaxDynamicSharedMemorySize, CK_DYN_SMEM_MAX));
  int per_sm = 0;
  CKC(h, cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kMegaGeneric, CK_THREADS,
                                                       CK_DYN_PHASES + h->ph_logits.size() * sizeof(Phase)));
  int want = 1;
  const char* w = getenv("CK_MEGA_CTAS_PER_SM");
  if (w) want = atoi(w);
  if (want < 1) want = 1;
  if (per_sm < 1) return h->fail(CK_ECUDA, "megakernel does not fit on an SM");
  h->mega_grid = h->sms * (want < per_sm ? want : per_sm);
  h->mega_fn = mega_kernel(h);
  for (int l = 0; l < 2; l++) {
    std::vector<Phase> mp = l ? h->ph_logits : h->ph_prefill;
    // kMegaOwnTop: the phase after an attention phase has its rows on the
    // CTAs below the attention's mergers only
    const bool own_top = h->mega_fn == kMegaOwnTop && h->cfg.kv_heads * h->smax <= h->mega_grid;
    for (size_t j = 0; j < mp.size(); j++) {
      Phase& p = mp[j];
      const bool below = own_top && j > 0 && mp[j - 1].kind == PH_ATTN;
      set_partition(p, below ? h->mega_grid - h->cfg.kv_heads : h->mega_grid);
    }
    Phase** dst = l ? &h->dm_logits : &h->dm_prefill;
    if ((rc = dalloc(h, dst, mp.size() * sizeof(Phase)))) return rc;
    CKC(h, cudaMemcpy(*dst, mp.data(), mp.size() * sizeof(Phase), cudaMemcpyHostToDevice));
  }
  if ((rc = sk_setup(h))) return rc;
  const char* menv = getenv("CK_MODE");
  if (h->sk_ok && menv && atoi(menv) == 2) h->mode = 2;
  for (int m = 0; m < 3; m++) {
    if (m == 2 && !h->sk_ok) continue;
    if ((rc = capture(h, true, m, &h->gx_logits[m]))) {
      cudaGetLastError();
      h->gx_logits[m] = nullptr;  // fall back to direct launches
    }
    if ((rc = capture(h, false, m, &h->gx_prefill[m]))) {
      cudaGetLastError();
      h->gx_prefill[m] = nullptr;
    }
  }
  h->err.clear();
  CKC(h, cudaDeviceSynchronize());
  h->finalized = true;
  h->pos = 0;
  return CK_OK;
}

int ck_set_stream(ck_engine* h, void* stream) {
  if (!h) return set_global(CK_EINVAL, "null engine");
  h->stream = stream ? (cudaStream_t)stream : h->own;
  return CK_OK;
}

int ck_set_sampler(ck_engine* h, int exact) {
  if (!h) return set_global(CK_EINVAL, "null engine");
  h->sampler_exact = exact ? 1 : 0;
  return CK_OK;
}

int ck_set_mode(ck_engine* h, int mode) {
  if (!h) return set_global(CK_EINVAL, "null engine");
  if (mode != 0 && mode != 1 && mode != 2) return h->fail(CK_EINVAL, "mode %d", mode);
  if (mode == 2 && !h->sk_ok) return h->fail(CK_EINVAL, "the streaming step does not support this model's shapes");
  h->mode = mode;
  return CK_OK;
}

static int pre_step(ck_engine* h) {
  if (!h) return set_global(CK_EINVAL, "null engine");
  if (!h->finalized) return h->fail(CK_ESTATE, "engine not finalized");
  if (h->pos >= h->cfg.context_length)
    return h->fail(CK_ECONTEXT, "Llama WGSL context exhausted at %d tokens", h->cfg.context_length);
  CKC(h, cudaSetDevice(h->device));
  return CK_OK;
}

int ck_run_token(ck_engine* h, uint32_t token, int need_logits, const ck_sampling* s, uint32_t* out_id) {
  int rc = pre_step(h);
  if (rc) return rc;
  if (token >= (uint32_t)h->cfg.vocab) return h->fail(CK_EINVAL, "token id %u outside embedding table", token);
  if ((rc = set_params(h, s, 0, 0, false))) return rc;
  uint32_t* tk = (uint32_t*)(h->pinned + 384);
  *tk = token;
  CKC(h, h2d(h, h->D.tokens + h->pos, tk, 4));
  if ((rc = launch_step(h, need_logits != 0))) return rc;
  uint32_t* res = (uint32_t*)(h->pinned + 448);
  if (need_logits) CKC(h, d2h(h, res, &h->st->next_token, 4));
  if ((rc = check_device(h))) return rc;
  h->pos += 1;
  if (out_id) *out_id = need_logits ? *res : 0u;
  return CK_OK;
}

}  // extern "C"
namespace {   // tensor-core prefill (ck_prefill.cuh)
bool pf_supported(const ck_engine* h);
int prefill_gemm(ck_engine* h, int n);
}  // namespace
extern "C" {

int ck_prefill(ck_engine* h, const uint32_t* tokens, int n, int need_logits_last, const ck_sampling* s,
               uint32_t* out_id) {
  int rc = pre_step(h);
  if (rc) return rc;
  if (n <= 0 || !tokens) return h->fail(CK_EINVAL, "ck_prefill: empty prompt");
  if (h->pos + n > h->cfg.context_length)
    return h->fail(CK_ECONTEXT, "Llama WGSL context exhausted at %d tokens", h->cfg.context_length);
  for (int i = 0; i < n; i++)
    if (tokens[i] >= (uint32_t)h->cfg.vocab) return h->fail(CK_EINVAL, "token id %u outside embedding table", tokens[i]);
  if ((rc = set_params(h, s, 0, 0, false))) return rc;
  CKC(h, h2d(h, h->D.tokens + h->pos, tokens, (size_t)n * 4));
  int first = 0;   // tokens before this one went through the tensor-core prefill
  if (h->pf_min > 0 && n - 1 >= h->pf_min && pf_supported(h)) {
    if ((rc = prefill_gemm(h, n - 1))) return rc;
    if ((rc = set_pos_dev(h, h->pos + n - 1))) return rc;
    h->pos -= n - 1;   // advanced with the last token below
    first = n - 1;
  }
  for (int i = first; i < n; i++)
    if ((rc = launch_step(h, need_logits_last && i == n - 1))) return rc;
  uint32_t* res = (uint32_t*)(h->pinned + 448);
  if (need_logits_last) CKC(h, d2h(h, res, &h->st->next_token, 4));
  if ((rc = check_device(h))) return rc;
  h->pos += n;
  if (out_id) *out_id = need_logits_last ? *res : 0u;
  return CK_OK;
}

int ck_decode(ck_engine* h, uint32_t first, int max_new, const ck_sampling* s, const uint32_t* eos_ids, int n_eos,
              uint32_t* out_ids, int* n_out) {
  if (!h) return set_global(CK_EINVAL, "null engine");
  if (!h->finalized) return h->fail(CK_ESTATE, "engine not finalized");
  if (!out_ids || !n_out) return h->fail(CK_EINVAL, "ck_decode: null output");
  *n_out = 0;
  if (max_new <= 0) return CK_OK;
  auto is_eos = [&](uint32_t id) {
    for (int i = 0; i < n_eos; i++) if (eos_ids[i] == id) return true;
    return false;
  };
  out_ids[0] = first;
  int produced = 1;
  if (is_eos(first) || max_new == 1) { *n_out = 1; return CK_OK; }
  int rc = pre_step(h);
  if (rc) return rc;
  if (first >= (uint32_t)h->cfg.vocab) return h->fail(CK_EINVAL, "token id %u outside embedding table", first);
  uint64_t draw0 = s ? s->philox_offset : 0;
  if ((rc = set_params(h, s, 1, draw0, true))) return rc;
  uint32_t* tk = (uint32_t*)(h->pinned + 384);
  *tk = first;
  CKC(h, h2d(h, h->D.tokens + h->pos, tk, 4));
  const int CH = 16;
  uint32_t* back = (uint32_t*)(h->pinned + 1024);
  bool done = false;
  while (!done) {
    int remaining = max_new - produced;
    int room = h->cfg.context_length - h->pos;
    int steps = remaining < CH ? remaining : CH;
    if (steps > room) steps = room;
    if (steps <= 0) break;
    for (int i = 0; i < steps; i++)
      if ((rc = launch_step(h, true))) return rc;
    // ids produced by these steps: tokens[pos+1 .. pos+steps] (the last one
    // may sit at ctx, which is not stored: read it from next_token instead)
    int stored = steps;
    if (h->pos + steps >= h->cfg.context_length) stored = h->cfg.context_length - 1 - h->pos;
    if (stored > 0)
      CKC(h, d2h(h, back, h->D.tokens + h->pos + 1, (size_t)stored * 4));
    CKC(h, d2h(h, back + stored, &h->st->next_token, 4));
    if ((rc = check_device(h))) return rc;
    if (stored < steps) back[steps - 1] = back[stored];
    int used = steps;
    for (int i = 0; i < steps; i++) {
      out_ids[produced++] = back[i];
      if (is_eos(back[i]) || produced >= max_new) { used = i + 1; done = true; break; }
    }
    if (used < steps) {  // ran past an EOS: rewind the position (KV beyond is dead)
      if ((rc = set_pos_dev(h, h->pos + used))) return rc;
    } else {
      h->pos += steps;
    }
    if (h->pos >= h->cfg.context_length) break;
  }
  *n_out = produced;
  return CK_OK;
}

int ck_enqueue_decode_steps(ck_engine* h, int n) {
  int rc = pre_step(h);
  if (rc) return rc;
  if (h->pos + n > h->cfg.context_length) return h->fail(CK_ECONTEXT, "context exhausted");
  // greedy, chained: each step's id becomes the next step's input
  if ((rc = set_params(h, nullptr, 1, 0, true))) return rc;
  for (int i = 0; i < n; i++)
    if ((rc = launch_step(h, true))) return rc;
  h->pos += n;
  return CK_OK;
}

int ck_enqueue_decode_steps_sampled(ck_engine* h, int n, const ck_sampling* s) {
  int rc = pre_step(h);
  if (rc) return rc;
  if (h->pos + n > h->cfg.context_length) return h->fail(CK_ECONTEXT, "context exhausted");
  // chained like ck_decode: each step samples with `s` (draws from its
  // philox_offset on) and feeds its id to the next step
  if ((rc = set_params(h, s, 1, s ? s->philox_offset : 0, true))) return rc;
  for (int i = 0; i < n; i++)
    if ((rc = launch_step(h, true))) return rc;
  h->pos += n;
  return CK_OK;
}

int ck_sync(ck_engine* h) {
  if (!h) return set_global(CK_EINVAL, "null engine");
  return check_device(h);
}

int ck_get_logits(ck_engine* h, float* out, size_t n) {
  if (!h || !out) return set_global(CK_EINVAL, "bad argument");
  if (n > (size_t)h->cfg.vocab) n = h->cfg.vocab;
  CKC(h, cudaStreamSynchronize(h->stream));
  CKC(h, cudaMemcpy(out, h->D.logits, n * 4, cudaMemcpyDeviceToHost));
  return CK_OK;
}

int ck_get_candidates(ck_engine* h, float* val, uint32_t* idx, size_t n) {
  if (!h || !val || !idx) return set_global(CK_EINVAL, "bad argument");
  size_t g = (size_t)(h->cfg.vocab + 255) / 256;
  if (n > g) n = g;
  CKC(h, cudaStreamSynchronize(h->stream));
  CKC(h, cudaMemcpy(val, h->D.cand_val, n * 4, cudaMemcpyDeviceToHost));
  CKC(h, cudaMemcpy(idx, h->D.cand_idx, n * 4, cudaMemcpyDeviceToHost));
  return CK_OK;
}

int ck_reset(ck_engine* h) {
  if (!h) return set_global(CK_EINVAL, "null engine");
  if (!h->finalized) return h->fail(CK_ESTATE, "engine not finalized");
  CKC(h, cudaSetDevice(h->device));
  CKC(h, cudaMemsetAsync(h->kv, 0, h->kv_bytes, h->stream));  // clearBuffer (:1014-1017)
  return set_pos_dev(h, 0);
}

int ck_position(ck_engine* h, int* pos) {
  if (!h || !pos) return set_global(CK_EINVAL, "bad argument");
  *pos = h->pos;
  return CK_OK;
}

int ck_truncate(ck_engine* h, int pos) {
  if (!h) return set_global(CK_EINVAL, "null engine");
  if (pos < 0 || pos > h->pos) return h->fail(CK_EINVAL, "truncate to %d outside [0, %d]", pos, h->pos);
  return set_pos_dev(h, pos);
}

int ck_step_bytes(ck_engine* h, double* weight_bytes, double* kv_bytes) {
  if (!h || !weight_bytes || !kv_bytes) return set_global(CK_EINVAL, "bad argument");
  const ck_model_cfg& c = h->cfg;
  double wb = 0;
  auto add = [&](const Weight& w) { wb += (double)w.L.row_bytes * w.n; };
  for (const LayerW& W : h->L) {
    add(W.q); add(W.k); add(W.v); add(W.o); add(W.gate); add(W.up); add(W.down);
  }
  add(h->head);
  double kb = 0;
  for (int i = 0; i < c.layers; i++) {
    int p = h->pos;
    int start = (c.layer_window[i] && p + 1 > (int)c.layer_window[i]) ? p + 1 - (int)c.layer_window[i] : 0;
    kb += 2.0 * c.kv_heads * (double)(p - start + 1) * c.head_dim * elem_kv(c);
  }
  *weight_bytes = wb;
  *kv_bytes = kb;
  return CK_OK;
}

int ck_trace(ck_engine* h, int enable) {
  if (!h) return set_global(CK_EINVAL, "null engine");
  if (!h->finalized) return h->fail(CK_ESTATE, "engine not finalized");
  if (enable && !h->D.trace) {
    int rc = dalloc(h, &h->D.trace, CK_TRACE_SLOTS * sizeof(unsigned long long));
    if (rc) return rc;
    CKC(h, cudaMemset(h->D.trace, 0, CK_TRACE_SLOTS * sizeof(unsigned long long)));
  }
  h->trace_on = enable != 0;
  CkDev D = h->D;
  if (!enable) D.trace = nullptr;
  h->Dlaunch = D;
  // graphs hold the kernel arguments: rebuild them with the new CkDev
  for (int m = 0; m < 3; m++) {
    if (h->gx_logits[m]) { cudaGraphExecDestroy(h->gx_logits[m]); h->gx_logits[m] = nullptr; }
    if (h->gx_prefill[m]) { cudaGraphExecDestroy(h->gx_prefill[m]); h->gx_prefill[m] = nullptr; }
    if (m == 2 && !h->sk_ok) continue;
    if (capture(h, true, m, &h->gx_logits[m])) { cudaGetLastError(); h->gx_logits[m] = nullptr; }
    if (capture(h, false, m, &h->gx_prefill[m])) { cudaGetLastError(); h->gx_prefill[m] = nullptr; }
  }
  h->err.clear();
  return CK_OK;
}

int ck_trace_read(ck_engine* h, uint64_t* out, size_t n) {
  if (!h || !out) return set_global(CK_EINVAL, "bad argument");
  if (!h->D.trace) return h->fail(CK_ESTATE, "tracing is off");
  if (n > CK_TRACE_SLOTS) n = CK_TRACE_SLOTS;
  CKC(h, cudaStreamSynchronize(h->stream));
  CKC(h, cudaMemcpy(out, h->D.trace, n * 8, cudaMemcpyDeviceToHost));
  return CK_OK;
}

int ck_io_bytes(ck_engine* h, uint64_t* h2d_bytes, uint64_t* d2h_bytes) {
  if (!h || !h2d_bytes || !d2h_bytes) return set_global(CK_EINVAL, "bad argument");
  *h2d_bytes = h->io_h2d;
  *d2h_bytes = h->io_d2h;
  return CK_OK;
}

void pf_free(ck_engine* h);

int ck_destroy(ck_engine* h) {
  if (!h) return CK_OK;
  cudaSetDevice(h->device);
  cudaStreamSynchronize(h->own);
  pf_free(h);
  for (int m = 0; m < 3; m++) {
    if (h->gx_logits[m]) cudaGraphExecDestroy(h->gx_logits[m]);
    if (h->gx_prefill[m]) cudaGraphExecDestroy(h->gx_prefill[m]);
  }
  for (void* p : h->allocs) cudaFree(p);
  if (h->pinned) cudaFreeHost(h->pinned);
  if (h->own) cudaStreamDestroy(h->own);
  delete h;
  return CK_OK;
}

// ---- parity / measurement helpers --------------------------------------------
namespace {
int prep_weight(ck_engine* h, int type, const void* bytes, size_t nbytes, int k, int n, Weight& w) {
  return upload_quant(h, w, type, k, n, bytes, nbytes, "tensor");
}

int make_tmp(int device, ck_engine** out) {
  CKG(cudaSetDevice(device));
  ck_engine* h = new ck_engine();
  h->device = device;
  cudaDeviceProp prop;
  CKG(cudaGetDeviceProperties(&prop, device));
  h->sms = prop.multiProcessorCount;
  CKG(cudaStreamCreateWithFlags(&h->own, cudaStreamNonBlocking));
  h->stream = h->own;
  CKG(cudaFuncSetAttribute(k_mv, cudaFuncAttributeMaxDynamicSharedMemorySize, CK_DYN_SMEM_MAX));
  int rc = dalloc(h, &h->st, sizeof(CkState));
  if (rc) return set_global(rc, "%s", h->err.c_str());
  CKG(cudaMemset(h->st, 0, sizeof(CkState)));
  memset(&h->D, 0, sizeof h->D);
  h->D.st = h->st;
  *out = h;
  return CK_OK;
}

void free_tmp(ck_engine* h) {
  cudaStreamSynchronize(h->own);
  for (void* p : h->allocs) cudaFree(p);
  cudaStreamDestroy(h->own);
  delete h;
}
}  // namespace

int ck_dequant(int ggml_type, const void* bytes, size_t nbytes, int k, int n, float* out, int device) {
  if (!bytes || !out || k <= 0 || n <= 0) return set_global(CK_EINVAL, "ck_dequant: bad argument");
  ck_engine* h;
  int rc = make_tmp(device, &h);
  if (rc) return rc;
  Weight w;
  if ((rc = prep_weight(h, ggml_type, bytes, nbytes, k, n, w))) {
    std::string m = h->err;
    free_tmp(h);
    return set_global(rc, "%s", m.c_str());
  }
  float* d = nullptr;
  if ((rc = dalloc(h, &d, (size_t)k * n * 4))) { free_tmp(h); return set_global(rc, "alloc"); }
  long long total = (long long)k * n;
  k_dequant<<<(unsigned)((total + 255) / 256), 256, 0, h->own>>>(w.dev, w.L, n, d);
  cudaError_t e = cudaMemcpyAsync(out, d, (size_t)total * 4, cudaMemcpyDeviceToHost, h->own);
  if (e == cudaSuccess) e = cudaStreamSynchronize(h->own);
  free_tmp(h);
  if (e != cudaSuccess) return set_global(CK_ECUDA, "ck_dequant: %s", cudaGetErrorString(e));
  return CK_OK;
}

// The streaming matvec (ck_gemv.cuh) over a whole device-layout weight.
static cudaError_t gv_launch(ck_engine* h, const Weight& w, const float* dx, float* dy, cudaStream_t s) {
  GvKernel fn = gv_kernel(w.L.type);
  if (!fn) return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute((const void*)fn, cudaFuncAttributeMaxDynamicSharedMemorySize, GV_DYN_BYTES);
  if (e != cudaSuccess) return e;
  fn<<<h->sms, GV_THREADS, GV_DYN_BYTES, s>>>(w.dev, w.L, w.n, dx, dy, &h->st->err);
  return cudaGetLastError();
}

static int matvec_setup(ck_engine* h, int type, const void* bytes, size_t nbytes, int k, int n, Weight& w, float** x,
                        float** y, Phase** dph, Phase& ph) {
  int rc;
  if (k > CK_KMAX || k % 32) return h->fail(CK_EINVAL, "k %d unsupported", k);
  if ((rc = prep_weight(h, type, bytes, nbytes, k, n, w))) return rc;
  if ((rc = dalloc(h, x, (size_t)k * 4))) return rc;
  if ((rc = dalloc(h, y, (size_t)n * 4))) return rc;
  Pro p{};
  p.kind = PRO_COPY;
  p.a = *x;
  ph = mk_mv(h, p, k, {seg(w, *y, nullptr)});
  if ((rc = dalloc(h, dph, sizeof(Phase)))) return rc;
  CKC(h, cudaMemcpy(*dph, &ph, sizeof(Phase), cudaMemcpyHostToDevice));
  return CK_OK;
}

int ck_matvec(int ggml_type, const void* bytes, size_t nbytes, int k, int n, const float* x, float* y, int device) {
  if (!bytes || !x || !y) return set_global(CK_EINVAL, "ck_matvec: bad argument");
  ck_engine* h;
  int rc = make_tmp(device, &h);
  if (rc) return rc;
  Weight w;
  float *dx, *dy;
  Phase* dph;
  Phase ph;
  if ((rc = matvec_setup(h, ggml_type, bytes, nbytes, k, n, w, &dx, &dy, &dph, ph))) {
    std::string m = h->err;
    free_tmp(h);
    return set_global(rc, "%s", m.c_str());
  }
  cudaMemcpyAsync(dx, x, (size_t)k * 4, cudaMemcpyHostToDevice, h->own);
  cudaError_t e = gv_launch(h, w, dx, dy, h->own);
  if (e == cudaSuccess) e = cudaMemcpyAsync(y, dy, (size_t)n * 4, cudaMemcpyDeviceToHost, h->own);
  if (e == cudaSuccess) e = cudaStreamSynchronize(h->own);
  free_tmp(h);
  if (e != cudaSuccess) return set_global(CK_ECUDA, "ck_matvec: %s", cudaGetErrorString(e));
  return CK_OK;
}

int ck_bench_matvec(int ggml_type, const void* bytes, size_t nbytes, int k, int n, int reps, double* us_per,
                    int device) {
  if (!bytes || !us_per || reps <= 0) return set_global(CK_EINVAL, "ck_bench_matvec: bad argument");
  ck_engine* h;
  int rc = make_tmp(device, &h);
  if (rc) return rc;
  Weight w;
  float *dx, *dy;
  Phase* dph;
  Phase ph;
  if ((rc = matvec_setup(h, ggml_type, bytes, nbytes, k, n, w, &dx, &dy, &dph, ph))) {
    std::string m = h->err;
    free_tmp(h);
    return set_global(rc, "%s", m.c_str());
  }
  cudaMemsetAsync(dx, 0, (size_t)k * 4, h->own);
  // Rotate over enough weight copies to exceed L2 so every launch streams
  // from HBM.
  size_t wbytes = (size_t)w.L.row_bytes * n;
  int copies = (int)((256ull << 20) / (wbytes ? wbytes : 1)) + 1;
  if (copies > 64) copies = 64;
  std::vector<Weight> ws;
  ws.push_back(w);
  for (int c = 1; c < copies; c++) {
    Weight wc = w;
    if (dalloc(h, &wc.dev, wbytes)) break;
    cudaMemcpyAsync(wc.dev, w.dev, wbytes, cudaMemcpyDeviceToDevice, h->own);
    ws.push_back(wc);
  }
  (void)dph; (void)ph;
  cudaError_t e = cudaSuccess;
  for (int i = 0; i < 3 && e == cudaSuccess; i++) e = gv_launch(h, ws[i % ws.size()], dx, dy, h->own);
  cudaEvent_t a, b;
  cudaEventCreate(&a);
  cudaEventCreate(&b);
  cudaEventRecord(a, h->own);
  for (int i = 0; i < reps && e == cudaSuccess; i++) e = gv_launch(h, ws[i % ws.size()], dx, dy, h->own);
  cudaEventRecord(b, h->own);
  if (e == cudaSuccess) e = cudaEventSynchronize(b);
  float ms = 0.f;
  if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, a, b);
  cudaEventDestroy(a);
  cudaEventDestroy(b);
  free_tmp(h);
  if (e != cudaSuccess) return set_global(CK_ECUDA, "ck_bench_matvec: %s", cudaGetErrorString(e));
  *us_per = (double)ms * 1000.0 / reps;
  return CK_OK;
}

}  // extern "C"

// ---- matvec without device allocation -------------------------------------
// For callers that cannot allocate device memory of their own: hosts whose
// device memory is owned by another caching allocator (a framework pool that
// already holds the device's memory, so a raw cudaMalloc would fail or bypass
// its accounting), and latency-bound serving loops where cudaMalloc/cudaFree
// would synchronise the device and stall every other stream.  The caller
// passes its own device buffers; this entry point's scratch -- the step state,
// the phase descriptor and the device-layout copy of the weights -- lives in
// the one static array below, which every GPU that loads this library holds
// until the process exits.  Every call shares it and it keeps the last call's
// contents, so calls that overlap on the GPU (other threads, other streams)
// race; the state words that must start at zero are cleared on every call.
#define CK_NOALLOC_STATE_BYTES 256
#define CK_NOALLOC_PHASE_BYTES 4096
#define CK_NOALLOC_WEIGHT_BYTES (16u << 20)   // largest device-layout weight: 16 MiB
#define CK_NOALLOC_SCRATCH_BYTES (CK_NOALLOC_STATE_BYTES + CK_NOALLOC_PHASE_BYTES + CK_NOALLOC_WEIGHT_BYTES)
static __device__ __align__(256) uint8_t g_noalloc_scratch[CK_NOALLOC_SCRATCH_BYTES];
static_assert(sizeof(CkState) <= CK_NOALLOC_STATE_BYTES, "state slot");
static_assert(sizeof(Phase) <= CK_NOALLOC_PHASE_BYTES, "phase slot");

#define CK_NOALLOC_MAX_DEVICES 64
// Per-device set-up, done once under std::call_once: the array's device
// address (cudaGetSymbolAddress with that device current), the kernel's
// shared-memory attribute and the SM count.  A device reset invalidates the
// address; the entry point is not meant to be used across cudaDeviceReset.
struct NoallocDev {
  uint8_t* base;
  int sms;
  cudaError_t rc;
};
static NoallocDev g_noalloc_dev[CK_NOALLOC_MAX_DEVICES];
static std::once_flag g_noalloc_once[CK_NOALLOC_MAX_DEVICES];

static void noalloc_setup(int dev) {
  NoallocDev& d = g_noalloc_dev[dev];
  void* p = nullptr;
  d.rc = cudaGetSymbolAddress(&p, g_noalloc_scratch);
  if (d.rc == cudaSuccess) d.rc = cudaFuncSetAttribute(k_mv, cudaFuncAttributeMaxDynamicSharedMemorySize, CK_DYN_SMEM_MAX);
  if (d.rc == cudaSuccess) d.rc = cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev);
  d.base = d.rc == cudaSuccess ? (uint8_t*)p : nullptr;
}

extern "C" int ck_matvec_noalloc(int ggml_type, const void* w_dev, size_t nbytes, int k, int n, const float* x_dev,
                                 float* y_dev, void* stream) {
  if (!w_dev || !x_dev || !y_dev || k <= 0 || n <= 0) return set_global(CK_EINVAL, "ck_matvec_noalloc: bad argument");
  if (!ck_type_ok(ggml_type)) return set_global(CK_EINVAL, "ck_matvec_noalloc: unsupported GGML type %d", ggml_type);
  if (k % ck_block_weights(ggml_type) || k > CK_KMAX)
    return set_global(CK_EINVAL, "ck_matvec_noalloc: row length %d unsupported for type %d", k, ggml_type);
  size_t raw = (size_t)n * (k / ck_block_weights(ggml_type)) * ck_block_bytes(ggml_type);
  if (nbytes != raw) return set_global(CK_EINVAL, "ck_matvec_noalloc: %zu bytes, expected %zu", nbytes, raw);
  Lay L = make_lay(ggml_type, k);
  size_t need = (size_t)L.row_bytes * n;
  if (need > CK_NOALLOC_WEIGHT_BYTES)
    return set_global(CK_EINVAL, "ck_matvec_noalloc: %d x %d weights need %zu device bytes, the static scratch holds %u",
                      n, k, need, CK_NOALLOC_WEIGHT_BYTES);
  int dev = 0;
  CKG(cudaGetDevice(&dev));
  if (dev < 0 || dev >= CK_NOALLOC_MAX_DEVICES) return set_global(CK_EINVAL, "ck_matvec_noalloc: device %d", dev);
  // one-time set-up on this device (current here), so the first call on a
  // device should come before any stream capture; threads that make their
  // first calls at the same time wait for the one that runs it
  std::call_once(g_noalloc_once[dev], noalloc_setup, dev);
  const NoallocDev& nd = g_noalloc_dev[dev];
  if (nd.rc != cudaSuccess)
    return set_global(CK_ECUDA, "ck_matvec_noalloc: device %d set-up: %s", dev, cudaGetErrorString(nd.rc));
  uint8_t* base = nd.base;
  CkState* st = (CkState*)base;
  Phase* dph = (Phase*)(base + CK_NOALLOC_STATE_BYTES);
  uint8_t* wl = base + CK_NOALLOC_STATE_BYTES + CK_NOALLOC_PHASE_BYTES;
  cudaStream_t s = (cudaStream_t)stream;

  Phase ph;
  memset(&ph, 0, sizeof ph);
  ph.kind = PH_MATVEC;
  ph.mv.pro.kind = PRO_COPY;
  ph.mv.pro.a = x_dev;
  ph.mv.k = k;
  ph.mv.nseg = 1;
  ph.mv.seg[0].w = wl;
  ph.mv.seg[0].out = y_dev;
  ph.mv.seg[0].add = nullptr;
  ph.mv.seg[0].L = L;
  ph.mv.seg[0].n = n;
  int grid = n < nd.sms ? n : nd.sms;
  set_partition(ph, grid);
  CkDev D;
  memset(&D, 0, sizeof D);
  D.st = st;

  CKG(cudaMemsetAsync(st, 0, sizeof(CkState), s));          // error and abort words start at zero
  CKG(cudaMemcpyAsync(dph, &ph, sizeof(Phase), cudaMemcpyHostToDevice, s));
  long long total = (long long)n * L.nb;
  k_relayout<<<(unsigned)((total + 255) / 256), 256, 0, s>>>((const uint8_t*)w_dev, wl, L, n);
  CKG(cudaGetLastError());
  k_mv<<<grid, CK_THREADS, CK_DYN_PHASES + sizeof(Phase), s>>>(dph, D);
  CKG(cudaGetLastError());
  int derr = 0;
  CKG(cudaMemcpyAsync(&derr, &st->err, sizeof(int), cudaMemcpyDeviceToHost, s));
  CKG(cudaStreamSynchronize(s));
  if (derr) return set_global(CK_EDEVICE, "ck_matvec_noalloc: device error bits 0x%x", derr);
  return CK_OK;
}

// Batched decode: kernels and scheduler over this engine's weights.
#include "ck_batch.cuh"
#include "ck_prefill.cuh"
