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
// * Each matvec becomes a tensor-core GEMM over the step's tokens
//   (k_bgemm_tc, below) on the weights' fp16 operand tiles, made once per
//   batch; x reaches a GEMM as operand tiles too: written by the per-token
//   prologue (k_bprep: layer 0's RMS norm, the SiLU gate), by attention (one
//   CTA per token and kv head over that token's sequence, k_battn) for the o
//   projection, and by the o / down GEMMs' epilogue for the next RMS norm.
// * The step's kernels are launched with programmatic dependent launch: each
//   may start while its predecessor runs and waits before touching shared
//   data (pdl_wait).
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

struct BXh {             // per-token matmul input x = hi + lo (two fp16 parts)
  __half* xt;            // operand tiles of the step's tokens (tc_index layout)
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
  const uint8_t* w;      // device-layout weight rows (the single-sequence matvec's copy)
  const __half* wt;      // the same weights as fp16 operand tiles (tc_format)
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
  int tile0[4];          // first 128-row tile of each segment; tile0[nseg] = total
  int splits;            // K slices per row tile (the cluster size, <= 8 and <= the K chunks)
  // epilogue of a residual-stream GEMM (one segment): also write the next RMS
  // norm's operand tiles, out * nw, and each row tile's sum of squares of out
  // per token (nssq[token][row tile], ntiles row tiles); off when nw is null
  const float* nw;
  __half* nxt;
  float* nssq;
  int ntiles;
  // prologue scale of each token from those partial sums:
  // 1 / sqrt(sum / k + eps) (RMS_NORM_WGSL); xh.xs when ssq_in is null
  const float* ssq_in;
  int ssq_tiles;
  float eps;
  // gate/up GEMM over interleaved tiles (k_tc_format with a second weight):
  // instead of its outputs, write silu(gate) * up for the 64 features of each
  // row tile as the down projection's operand tiles (K = glu_k); off when null
  __half* glu_xt;
  int glu_k;
};

// SILU_MUL_WGSL (llama-wgsl-runtime.ts:3529-3547), split into the two fp16
// parts of an operand tile
__device__ __forceinline__ void glu_parts(float g, float u, __half& hi, __half& lo) {
  const float v = (g / (1.0f + expf(-g))) * u;
  hi = __float2half_rn(v);
  lo = __float2half_rn(v - __half2float(hi));
}

struct BAttn {
  const float *q, *k, *v;     // [T][heads*hd], [T][kv_heads*hd]
  const float *qw, *kw;       // QK-norm weights or null
  __half *kc, *vc;            // this layer's pools [block][kv_head][CK_BLK][hd]
  const float* inv_freq;      // [hd/2]
  BXh xo;                     // the o projection's operand tiles: out written as x_hi / x_lo, scale 1
  int heads, kvh, hd, interleaved, window;
  float eps, scale;
};

// Programmatic dependent launch: the step's kernels are launched with
// programmatic stream serialization, so a kernel's CTAs may start while its
// predecessor is still running.  Each kernel waits (griddepcontrol.wait:
// the predecessor grid has completed and its writes are visible) before it
// reads or writes anything the step's kernels share, then lets its own
// successor launch.  Without the launch attribute both are no-ops.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---------------------------------------------------------------------------
// Embedding of every active entry's token (GGUF_*_EMBEDDING_WGSL, :2615-2866).
__global__ void __launch_bounds__(256) k_bembed(const uint8_t* w, Lay L, float scale, BStep st, float* x, int H,
                                                int vocab, int* err) {
  const int t = blockIdx.x;
  if (t >= *st.nact) return;
  pdl_wait();
  pdl_launch();
  uint32_t token = st.tok[t];
  if (token >= (uint32_t)vocab) {
    if (threadIdx.x == 0) atomicOr(err, CK_DERR_TOKEN);
    token = 0;
  }
  const uint8_t* row = w + (size_t)token * L.row_bytes;
  for (int i = threadIdx.x; i < H; i += blockDim.x) x[(size_t)t * H + i] = __fmul_rn(dequant_at(row, L, i), scale);
}

// ---------------------------------------------------------------------------
// Tensor-core GEMM (tcgen05) for the batched matmuls.
//
// Operands are fp16 "operand tiles": 128 rows x 64 columns in the K-major
// canonical shared-memory layout (8-row x 16-byte core matrices; the two
// 16-byte K halves of a 16-wide step 128 bytes apart, 8-row groups 256 bytes
// apart, 16-wide steps 4 KB apart), 16 KB each, stored [row tile][K chunk]
// [hi|lo] so a CTA moves every tile with one bulk copy.  A value v is kept
// as two fp16 parts hi = fp16(v), lo = fp16(v - hi) (~22 significant bits):
// the weights are dequantized into tiles once, when a batch is created
// (k_tc_format: 4 bytes per weight), and the prologue kernel writes x the
// same way.  D[128 weight rows x N tokens] accumulates in tensor memory
// (fp32): one thread keeps TC_STAGES chunks of four tiles in flight
// (cp.async.bulk completing on the stage's mbarrier), issues three MMAs per
// 16-wide step (w_hi x_hi + w_hi x_lo + w_lo x_hi; fp16 alone measured
// 3.8e-4 relative error per dot, bf16 3.3e-3) and commits them to the
// stage's release barrier; the accumulator is read back (tcgen05.ld, 32 rows
// per warp quarter) for the epilogue (prologue scale, residual add).
#define TC_ROWS 128
#define TC_NT 128            // tokens per CTA tile (columns of the accumulator)
#define TC_KC 64             // K per chunk
#define TC_THREADS 256
#define TC_STAGES 3
#define TC_TILE 16384        // bytes of one operand tile
#define TC_SMEM (TC_STAGES * 4 * TC_TILE + 128)

__host__ __device__ inline int tc_nch(int k) { return (k + TC_KC - 1) / TC_KC; }
__host__ __device__ inline size_t tc_bytes(int rows, int k) {
  return (size_t)((rows + TC_ROWS - 1) / TC_ROWS) * tc_nch(k) * 2 * TC_TILE;
}
// byte offset of (row, k) inside one tile
__device__ __forceinline__ uint32_t kmaj_off(int row, int k) {
  return (uint32_t)((k >> 4) * TC_ROWS * 32 + (row >> 3) * 256 + ((k >> 3) & 1) * 128 + (row & 7) * 16 + (k & 7) * 2);
}
// half-element index of (row r, column e) in a tiled matrix, part 0 = hi, 1 = lo
__device__ __forceinline__ size_t tc_index(int r, int e, int nch, int part) {
  const size_t tile = ((size_t)(r >> 7) * nch + (e >> 6)) * 2 + part;
  return tile * (TC_TILE / 2) + kmaj_off(r & 127, e & 63) / 2;
}
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);   // version 1, no swizzle
}
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, int* err) {
  unsigned spins = 0;
  while (!mbar_try_wait(bar, parity)) {
    if (++spins > (1u << 22)) {
      atomicOr(err, CK_DERR_BARRIER);
      return false;
    }
  }
  return true;
}

// Dequantize n x k weights into operand tiles (grid: row tiles x K chunks;
// a thread per 32-weight unit of the chunk).  Rows past n and columns past k
// are zero.
// With a second weight (w2: the up projection of a gate weight w), tile row r
// of each 128-row tile holds gate row 64 m + r for r < 64 and up row
// 64 m + r - 64 for r >= 64 (m = the tile): a GEMM over these tiles has a
// gate value and its up value in the same tile (n = rows of each weight).
__global__ void __launch_bounds__(256) k_tc_format(const uint8_t* w, Lay L, int n, int k, __half* out,
                                                   const uint8_t* w2 = nullptr, Lay L2 = Lay()) {
  const int row = blockIdx.x * TC_ROWS + (threadIdx.x >> 1), uu = threadIdx.x & 1;
  const int c = blockIdx.y, unit = c * 2 + uu, nch = gridDim.y;
  const bool second = w2 && (row & (TC_ROWS - 1)) >= TC_ROWS / 2;
  const int src = w2 ? (row / TC_ROWS) * (TC_ROWS / 2) + (row & (TC_ROWS / 2 - 1)) : row;
  const uint8_t* ws = second ? w2 : w;
  const Lay& Ls = second ? L2 : L;
  float wv[32];
  if (src < n && unit < (k >> 5)) {
    U8 u;
    unpack_unit<true>(Ls.type, ws + (size_t)src * Ls.row_bytes, Ls, unit, u);
#pragma unroll
    for (int i = 0; i < 32; i++) {
      // byte codes are signed (Q8_0 stores int8; the other types' codes are < 64)
      const int code = (int)(int8_t)((u.q[i >> 2] >> (8 * (i & 3))) & 0xFF);
      wv[i] = (i < 16 ? u.a0 : u.a1) * (float)(code + u.ko) + u.b;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 32; i++) wv[i] = 0.f;
  }
#pragma unroll
  for (int cc = 0; cc < 4; cc++) {
    __align__(16) __half hv[8], lv[8];
#pragma unroll
    for (int e = 0; e < 8; e++) {
      const float x = wv[8 * cc + e];
      hv[e] = __float2half_rn(x);
      lv[e] = __float2half_rn(x - __half2float(hv[e]));
    }
    const int col = c * TC_KC + 32 * uu + 8 * cc;
    *(int4*)(out + tc_index(row, col, nch, 0)) = *(const int4*)hv;
    *(int4*)(out + tc_index(row, col, nch, 1)) = *(const int4*)lv;
  }
}

// Per-token prologue (one CTA per active entry): the COPY / NORM / SILU forms
// of the single-sequence prologue, x written as two fp16 parts into the
// operand tiles of the tensor-core GEMM.  NORM's RMS scale is applied to the matmul output, as in
// the single-sequence path.
__global__ void __launch_bounds__(CK_THREADS) k_bprep(BPrep p, BStep st, BXh q) {
  constexpr int PER = CK_KMAX / CK_THREADS;
  const int t = blockIdx.x;
  if (t >= *st.nact) return;
  pdl_wait();
  pdl_launch();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int k = p.k, nch = tc_nch(k);
  const float* a = p.a + (size_t)t * p.lda;
  const float* b = p.kind == BP_SILU ? p.b + (size_t)t * p.lda : p.w;
  __shared__ float red[CK_WARPS];
  float va[PER], vb[PER];
#pragma unroll
  for (int j = 0; j < PER; j++) {
    const int i = tid + j * CK_THREADS;
    va[j] = i < k ? a[i] : 0.f;
    vb[j] = (i < k && p.kind != BP_COPY) ? b[i] : 0.f;
  }
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < PER; j++) {
    const int i = tid + j * CK_THREADS;
    float v = va[j];
    if (p.kind == BP_NORM) { ss += va[j] * va[j]; v = va[j] * vb[j]; }
    else if (p.kind == BP_SILU) v = (va[j] / (1.0f + expf(-va[j]))) * vb[j];
    if (i < k) {
      const __half h = __float2half_rn(v);
      q.xt[tc_index(t, i, nch, 0)] = h;
      q.xt[tc_index(t, i, nch, 1)] = __float2half_rn(v - __half2float(h));
    }
  }
  // columns past k in the last chunk meet zero weights: keep them finite
  for (int i = k + tid; i < nch * TC_KC; i += CK_THREADS) {
    q.xt[tc_index(t, i, nch, 0)] = __float2half_rn(0.f);
    q.xt[tc_index(t, i, nch, 1)] = __float2half_rn(0.f);
  }
  if (p.kind == BP_NORM) {
    ss = warp_sum(ss);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    if (tid == 0) {
      float tot = 0.f;
      for (int w = 0; w < CK_WARPS; w++) tot += red[w];
      q.xs[t] = rms_inv(tot, k, p.eps);
    }
  } else if (tid == 0) {
    q.xs[t] = 1.0f;
  }
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ float4 ld_dsmem4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr));
  return v;
}

// One CTA = one 128-row tile x one 128-token tile x one K slice.  A row
// tile's G.splits K slices form one thread-block cluster (cluster rank =
// slice): each slice accumulates its chunks in its own tensor memory, copies
// the accumulator to shared memory, and after a cluster barrier every CTA
// sums one column range of the tile over all slices in rank order (read
// through distributed shared memory, so the result does not depend on
// timing) and writes it with the epilogue.
__global__ void __launch_bounds__(TC_THREADS, 1) k_bgemm_tc(BGemm G, BStep st, BXh xh, int* err) {
  extern __shared__ __align__(1024) uint8_t tsm[];
  __shared__ uint32_t s_tmem;
  __shared__ int s_ok;
  __shared__ float s_xs[TC_NT];
  __shared__ float s_red[4][TC_NT];             // norm epilogue: per-warp-quarter sums of squares
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int T = *st.nact;
  const int t0 = blockIdx.y * TC_NT;
  if (t0 >= T) return;                          // the whole cluster (same blockIdx.y), before any TMEM is held
  const int nt = min(TC_NT, T - t0);
  const int N = (nt + 15) & ~15;                // MMA N: a multiple of 16
  const int S = G.splits, ks = (int)blockIdx.x % S, tile = (int)blockIdx.x / S;
  // the row tile's segment: its fields read into registers with constant
  // parameter indices (a dynamically indexed parameter is read through a
  // generic address, again after every asm statement that clobbers memory)
  const int si = (G.nseg > 1 && tile >= G.tile0[1]) + (G.nseg > 2 && tile >= G.tile0[2]);
  const __half* s_wt;
  const float* s_add;
  float* s_out;
  int s_n, s_ldo;
#define TC_PICK(I) \
  { s_wt = G.seg[I].wt; s_add = G.seg[I].add; s_out = G.seg[I].out; s_n = G.seg[I].n; s_ldo = G.seg[I].ldo; }
  if (si == 0) TC_PICK(0) else if (si == 1) TC_PICK(1) else TC_PICK(2)
#undef TC_PICK
  const int rt = tile - G.tile0[si], r0 = rt * TC_ROWS;
  const int nch = tc_nch(G.k);
  const int c_lo = ks * nch / S, c_hi = (ks + 1) * nch / S;   // splits <= chunks: never empty
  uint64_t* full = (uint64_t*)(tsm + TC_STAGES * 4 * TC_TILE);
  uint64_t* empty = full + TC_STAGES;
  uint64_t* done = empty + TC_STAGES;
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                 "r"(TC_NT));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (tid == 0) {
    for (int i = 0; i < 2 * TC_STAGES + 1; i++) mbar_init(full + i, 1);
    mbar_fence_init();
  }
  asm volatile("tcgen05.fence::before_thread_sync;");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;");
  const uint32_t tmem = s_tmem;
  bool ok = true;
  // instruction descriptor: fp32 D, fp16 A and B, both K-major, M = 128, N
  const uint32_t idesc = (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(TC_ROWS >> 4) << 24);
  const uint8_t* a_src = (const uint8_t*)s_wt + (size_t)rt * nch * 2 * TC_TILE;
  const uint8_t* b_src = (const uint8_t*)xh.xt + (size_t)blockIdx.y * nch * 2 * TC_TILE;
  // chunk c's four tiles complete on its stage's barrier: the weight pair
  // (with the stage's expect_tx) and the token pair may be issued apart
  auto issue_a = [&](int c) {
    const int sg = (c - c_lo) % TC_STAGES;
    uint8_t* dst = tsm + sg * 4 * TC_TILE;
    mbar_expect_tx(full + sg, 4 * TC_TILE);
    bulk_g2s(dst, a_src + (size_t)c * 2 * TC_TILE, TC_TILE, full + sg);
    bulk_g2s(dst + TC_TILE, a_src + ((size_t)c * 2 + 1) * TC_TILE, TC_TILE, full + sg);
  };
  auto issue_b = [&](int c) {
    const int sg = (c - c_lo) % TC_STAGES;
    uint8_t* dst = tsm + sg * 4 * TC_TILE;
    bulk_g2s(dst + 2 * TC_TILE, b_src + (size_t)c * 2 * TC_TILE, TC_TILE, full + sg);
    bulk_g2s(dst + 3 * TC_TILE, b_src + ((size_t)c * 2 + 1) * TC_TILE, TC_TILE, full + sg);
  };
  int issued = c_lo;
  // the weights are read-only: their first stages load while the previous
  // kernel may still run; the token tiles wait for it
  if (tid == 0)
    for (; issued < c_lo + TC_STAGES && issued < c_hi; issued++) issue_a(issued);
  pdl_wait();
  pdl_launch();
  if (tid == 0) {
    for (int c = c_lo; c < issued; c++) issue_b(c);
    int c = c_lo;
    for (; c < c_hi; c++) {
      const int j = c - c_lo, sg = j % TC_STAGES;
      if (!mbar_wait_bounded(full + sg, (j / TC_STAGES) & 1, err)) { ok = false; break; }
      asm volatile("tcgen05.fence::after_thread_sync;");
      const uint32_t base = smem_u32(tsm + sg * 4 * TC_TILE);
#pragma unroll
      for (int kk = 0; kk < TC_KC / 16; kk++) {
        const uint64_t da_hi = umma_desc(base + kk * TC_ROWS * 32, 128, 256);
        const uint64_t da_lo = umma_desc(base + TC_TILE + kk * TC_ROWS * 32, 128, 256);
        const uint64_t db_hi = umma_desc(base + 2 * TC_TILE + kk * TC_ROWS * 32, 128, 256);
        const uint64_t db_lo = umma_desc(base + 3 * TC_TILE + kk * TC_ROWS * 32, 128, 256);
        const uint32_t acc0 = (j > 0 || kk > 0) ? 1u : 0u;
        asm volatile("{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
                     " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n"
                     ::"r"(tmem), "l"(da_hi), "l"(db_hi), "r"(idesc), "r"(acc0));
        asm volatile("{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
                     " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n"
                     ::"r"(tmem), "l"(da_hi), "l"(db_lo), "r"(idesc), "r"(1u));
        asm volatile("{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
                     " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n"
                     ::"r"(tmem), "l"(da_lo), "l"(db_hi), "r"(idesc), "r"(1u));
      }
      asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                       smem_u32(empty + sg))
                   : "memory");
      // refill the previous chunk's stage (its MMAs ran ahead of this
      // chunk's, which stay queued on the tensor pipe meanwhile)
      if (j >= 1 && issued < c_hi) {
        const int pj = j - 1;
        if (!mbar_wait_bounded(empty + pj % TC_STAGES, (pj / TC_STAGES) & 1, err)) { ok = false; c++; break; }
        issue_a(issued);
        issue_b(issued++);
      }
    }
    if (!ok) {   // copies still in flight must land before the CTA's shared memory is reused
      for (int i = c; i < issued; i++) mbar_wait_bounded(full + (i - c_lo) % TC_STAGES, ((i - c_lo) / TC_STAGES) & 1, err);
    }
    // one more commit: arrives once every MMA issued above has completed
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(done))
                 : "memory");
  }
  // while thread 0 runs the K loop: the tokens' output scales (the row
  // tiles' partial sums in tile order, or the prologue's scale)
  if (tid >= TC_THREADS - TC_NT) {
    const int n = tid - (TC_THREADS - TC_NT);
    float v = 0.f;
    if (n < nt) {
      if (G.ssq_in) {
        float sum = 0.f;
        for (int q = 0; q < G.ssq_tiles; q++) sum += G.ssq_in[(size_t)(t0 + n) * G.ssq_tiles + q];
        v = rms_inv(sum, G.k, G.eps);
      } else {
        v = xh.xs[t0 + n];
      }
    }
    s_xs[n] = v;
  }
  __syncthreads();
  if (!mbar_wait_bounded(done, 0, err)) ok = false;
  asm volatile("tcgen05.fence::after_thread_sync;");
  if (tid == 0) s_ok = ok ? 1 : 0;
  __syncthreads();
  // warp w holds accumulator lanes (rows) 32*(w%4).. and half the columns
  const int q4 = warp & 3, half = warp >> 2, rl = 32 * q4 + lane, row = r0 + rl;
  const int cend = min((half + 1) * (TC_NT / 2), nt);
  if (S == 1) {
    // straight from the accumulator: 16 columns (tokens) per tcgen05.ld
    for (int col = half * (TC_NT / 2); col < cend; col += 16) {
      uint32_t r[16];
      const uint32_t taddr = tmem + ((uint32_t)(32 * q4) << 16) + (uint32_t)col;
      asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
                   : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                     "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
                     "=r"(r[15])
                   : "r"(taddr));
      const int m = min(16, cend - col);
      float av[16];
      if (s_add && row < s_n) {   // every residual value before any store (out may alias add)
        const float* ap = s_add + (size_t)(t0 + col) * s_ldo + row;
#pragma unroll
        for (int j = 0; j < 16; j++) av[j] = j < m ? ap[(size_t)j * s_ldo] : 0.f;
      } else {
#pragma unroll
        for (int j = 0; j < 16; j++) av[j] = 0.f;
      }
      asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
      float yv[16];
#pragma unroll
      for (int j = 0; j < 16; j++) yv[j] = (row < s_n && j < m) ? av[j] + s_xs[col + j] * __uint_as_float(r[j]) : 0.f;
      if (G.glu_xt) {   // gate / up values to shared memory (the drained stage buffers), [column][row]
        float* ex = (float*)tsm;
#pragma unroll
        for (int j = 0; j < 16; j++) ex[(col + j) * TC_ROWS + rl] = yv[j];
      } else if (s_ok && row < s_n) {
        float* op = s_out + (size_t)(t0 + col) * s_ldo + row;
#pragma unroll
        for (int j = 0; j < 16; j++)
          if (j < m) op[(size_t)j * s_ldo] = yv[j];
      }
      if (G.nw) {   // the next norm's operand tiles and this warp's 32 rows' sums of squares per token
        const int nchn = tc_nch(s_n);
        if (row < s_n) {
          const float wn = G.nw[row];
#pragma unroll
          for (int j = 0; j < 16; j++) {
            if (j < m) {
              const float v = yv[j] * wn;
              const __half h = __float2half_rn(v);
              G.nxt[tc_index(t0 + col + j, row, nchn, 0)] = h;
              G.nxt[tc_index(t0 + col + j, row, nchn, 1)] = __float2half_rn(v - __half2float(h));
            }
          }
        }
#pragma unroll
        for (int j = 0; j < 16; j++) {
          const float sq = warp_sum(yv[j] * yv[j]);
          if (lane == 0) s_red[q4][col + j] = sq;
        }
      }
    }
    if (G.nw) {
      __syncthreads();
      if (tid < nt)
        G.nssq[(size_t)(t0 + tid) * G.ntiles + rt] = ((s_red[0][tid] + s_red[1][tid]) + s_red[2][tid]) + s_red[3][tid];
    }
    if (G.glu_xt) {
      // silu(gate) * up of this tile's 64 features (feature 64 rt + f), 8
      // consecutive features of one token per item: 16-byte tile stores
      __syncthreads();
      const float* ex = (const float*)tsm;
      const int nchg = tc_nch(G.glu_k);
      for (int it = tid; it < 8 * nt; it += TC_THREADS) {
        const int cc = it >> 3, f0 = (it & 7) * 8;
        __align__(16) __half hv[8], lv[8];
#pragma unroll
        for (int e = 0; e < 8; e++)
          glu_parts(ex[cc * TC_ROWS + f0 + e], ex[cc * TC_ROWS + TC_ROWS / 2 + f0 + e], hv[e], lv[e]);
        if (s_ok) {
          *(uint4*)(G.glu_xt + tc_index(t0 + cc, (TC_ROWS / 2) * rt + f0, nchg, 0)) = *(const uint4*)hv;
          *(uint4*)(G.glu_xt + tc_index(t0 + cc, (TC_ROWS / 2) * rt + f0, nchg, 1)) = *(const uint4*)lv;
        }
      }
    }
  } else {
    // accumulator -> ex[column][row] (fp32, over the drained stage buffers)
    float* ex = (float*)tsm;
    for (int col = half * (TC_NT / 2); col < cend; col += 16) {
      uint32_t r[16];
      const uint32_t taddr = tmem + ((uint32_t)(32 * q4) << 16) + (uint32_t)col;
      asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
                   : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                     "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
                     "=r"(r[15])
                   : "r"(taddr));
      asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
      float* ep = ex + col * TC_ROWS + rl;
#pragma unroll
      for (int j = 0; j < 16; j++) ep[j * TC_ROWS] = s_ok ? __uint_as_float(r[j]) : 0.f;   // past nt: never read
    }
    // this CTA's columns [cb, ce) of the tile, summed over the slices in
    // rank order through distributed shared memory (16-byte loads); thread:
    // rows 4*(tid % 32) .. +3, columns cb + tid / 32, + 8, ...; two column
    // passes' loads in flight per round
    const int cb = ks * nt / S, ce = (ks + 1) * nt / S;
    const int rr = 4 * (tid & 31), orow = r0 + rr, cs = tid >> 5;
    const bool vec = (s_ldo & 3) == 0 && orow + 3 < s_n;
    uint32_t rbase[8];
    const uint32_t lbase = smem_u32(ex) + (uint32_t)rr * 4u;
#pragma unroll
    for (int q = 0; q < 8; q++) {
      rbase[q] = lbase;
      if (q < S) asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(rbase[q]) : "r"(lbase), "r"(q));
    }
    cluster_sync_all();
    for (int c0 = cb + cs; c0 < ce; c0 += 16) {
      const int c1 = c0 + 8;   // second column of the round (valid if < ce)
      float4 v[2][8];
#pragma unroll
      for (int q = 0; q < 8; q++) {
        if (q < S) {   // uniform over the CTA
          v[0][q] = ld_dsmem4(rbase[q] + (uint32_t)(c0 * TC_ROWS * 4));
          v[1][q] = ld_dsmem4(rbase[q] + (uint32_t)(min(c1, TC_NT - 1) * TC_ROWS * 4));
        }
      }
#pragma unroll
      for (int h = 0; h < 2; h++) {
        const int c = h ? c1 : c0;
        if (c >= ce) continue;   // uniform over the warp (one column per warp)
        float4 acc = v[h][0];
#pragma unroll
        for (int q = 1; q < 8; q++)
          if (q < S) { acc.x += v[h][q].x; acc.y += v[h][q].y; acc.z += v[h][q].z; acc.w += v[h][q].w; }
        const float xs = s_xs[c];
        float* op = s_out + (size_t)(t0 + c) * s_ldo + orow;
        const float* ap = (s_add && orow < s_n) ? s_add + (size_t)(t0 + c) * s_ldo + orow : nullptr;
        float y[4] = {xs * acc.x, xs * acc.y, xs * acc.z, xs * acc.w};
        if (G.glu_xt) {   // lanes 0-15 hold gate rows 0-63, lanes 16-31 the matching up rows
          __align__(8) __half hv[4], lv[4];
#pragma unroll
          for (int i = 0; i < 4; i++) {
            const float up = __shfl_xor_sync(0xffffffffu, y[i], 16);
            glu_parts(y[i], up, hv[i], lv[i]);
          }
          if ((tid & 31) < 16) {
            const int f = (TC_ROWS / 2) * rt + rr, nchg = tc_nch(G.glu_k);
            *(uint2*)(G.glu_xt + tc_index(t0 + c, f, nchg, 0)) = *(const uint2*)hv;
            *(uint2*)(G.glu_xt + tc_index(t0 + c, f, nchg, 1)) = *(const uint2*)lv;
          }
          continue;
        }
        if (vec) {
          if (ap) {
            const float4 a4 = *(const float4*)ap;
            y[0] += a4.x; y[1] += a4.y; y[2] += a4.z; y[3] += a4.w;
          }
          *(float4*)op = make_float4(y[0], y[1], y[2], y[3]);
        } else {
#pragma unroll
          for (int i = 0; i < 4; i++) {
            if (orow + i < s_n) {
              y[i] = (ap ? ap[i] : 0.f) + y[i];
              op[i] = y[i];
            }
          }
        }
        if (G.nw) {   // the next norm's operand tiles; the column's sum of squares over all 128 rows
          const int nchn = tc_nch(s_n);
          float sq = 0.f;
          __align__(8) __half hv[4], lv[4];
#pragma unroll
          for (int i = 0; i < 4; i++) {
            const bool in = orow + i < s_n;
            const float yi = in ? y[i] : 0.f;
            sq += yi * yi;
            const float vn = in ? yi * G.nw[orow + i] : 0.f;
            hv[i] = __float2half_rn(vn);
            lv[i] = __float2half_rn(vn - __half2float(hv[i]));
          }
          if (orow + 3 < s_n) {   // 4 consecutive K = 8 bytes of one 16-byte core-matrix row
            *(uint2*)(G.nxt + tc_index(t0 + c, orow, nchn, 0)) = *(const uint2*)hv;
            *(uint2*)(G.nxt + tc_index(t0 + c, orow, nchn, 1)) = *(const uint2*)lv;
          } else {
#pragma unroll
            for (int i = 0; i < 4; i++) {
              if (orow + i < s_n) {
                G.nxt[tc_index(t0 + c, orow + i, nchn, 0)] = hv[i];
                G.nxt[tc_index(t0 + c, orow + i, nchn, 1)] = lv[i];
              }
            }
          }
          sq = warp_sum(sq);
          if ((tid & 31) == 0) G.nssq[(size_t)(t0 + c) * G.ntiles + rt] = sq;
        }
      }
    }
    cluster_sync_all();   // no CTA leaves while another still reads its shared memory
  }
  asm volatile("tcgen05.fence::before_thread_sync;");
  __syncthreads();
  if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TC_NT));
}

// Prologue of the batched attention for one (active entry t, kv head):
// block table to shared memory, QK-norm + RoPE of the G query heads (into
// s.qs) and of the new K row (s.kst), and the K/V rows stored into the
// entry's block at its position.
template <int E, int NT = CK_THREADS>
__device__ __forceinline__ void battn_prologue(const BAttn& P, const BStep& st, SmemAt& s, int* sbt, int t, int kvh,
                                               int pos) {
  constexpr int hd = 32 * E;
  constexpr int NW = NT / 32;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = P.heads / P.kvh, qd = P.heads * hd, kvd = P.kvh * hd;
  const int* bt = st.btab + (size_t)st.slot[t] * st.max_blocks;
  for (int i = tid; i <= (pos >> 4) && i < 256; i += NT) sbt[i] = bt[i];
  for (int d = tid; d < (hd >> 1); d += NT) {
    float sn, cn;
    sincosf((float)pos * P.inv_freq[d], &sn, &cn);
    s.cs[d] = make_float2(cn, sn);
  }
  const float* qsrc = P.q + (size_t)t * qd + (size_t)kvh * G * hd;
  for (int i = tid; i < G * hd; i += NT) s.raw[i] = qsrc[i];
  for (int d = tid; d < hd; d += NT) {
    s.kvw[0][d] = P.k[(size_t)t * kvd + (size_t)kvh * hd + d];
    s.kvw[1][d] = P.v[(size_t)t * kvd + (size_t)kvh * hd + d];
    if (P.kw) s.kvw[3][d] = P.kw[d];
    if (P.qw) s.kvw[2][d] = P.qw[d];
  }
  __syncthreads();
  if (P.qw) {
    for (int gg = warp; gg < G + 1; gg += NW) {
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
              s.cs, tid, NT);
  rope_head(s.kvw[0], P.kw ? s.kvw[3] : nullptr, P.kw ? s.inv[G] : 1.f, s.kst, hd, P.interleaved, s.cs, tid,
            NT);
  __syncthreads();
  const size_t cb = (((size_t)sbt[pos >> 4] * P.kvh + kvh) * CK_BLK + (pos & (CK_BLK - 1))) * hd;
  for (int d = tid; d < hd; d += NT) {
    P.kc[cb + d] = __float2half_rn(s.kst[d]);
    P.vc[cb + d] = __float2half_rn(s.kvw[1][d]);
  }
}

// Attention for one (active entry, kv head): the prologue above, then an
// online softmax over [start, pos] (the single-sequence attention unit with
// one split), one warp group per query head.
template <int E>
__global__ void __launch_bounds__(CK_THREADS, 1) k_battn(BAttn P, BStep st) {
  constexpr int hd = 32 * E;
  const int t = blockIdx.x / P.kvh, kvh = blockIdx.x % P.kvh;
  if (t >= *st.nact) return;
  pdl_wait();
  pdl_launch();
  __shared__ SmemAt s;
  __shared__ int sbt[256];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = P.heads / P.kvh, qd = P.heads * hd;
  const int pos = st.pos[t];
  const int start = (P.window != 0 && pos + 1 > P.window) ? pos + 1 - P.window : 0;
  battn_prologue<E>(P, st, s, sbt, t, kvh, pos);
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
    // the round's math (a round trip per round, not per position); deeper
    // rounds (16 positions at head_dim 64) measured slower: more registers,
    // one CTA per SM instead of two
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
  // the output goes straight into the o projection's operand tiles (the
  // prologue's split: x_hi = fp16(x), x_lo = fp16(x - x_hi))
  const int nch = tc_nch(qd);
  for (int i = tid; i < G * hd; i += CK_THREADS) {
    const int gg = i / hd, d = i % hd;
    float A = 0.f;
    for (int w = gg * wpg; w < gg * wpg + wpg; w++) A += s.wacc[w * CK_HDMAX + d] * s.wf[w];
    const float o = A / s.hl[gg];
    const int col = (kvh * G + gg) * hd + d;
    const __half h = __float2half_rn(o);
    P.xo.xt[tc_index(t, col, nch, 0)] = h;
    P.xo.xt[tc_index(t, col, nch, 1)] = __float2half_rn(o - __half2float(h));
  }
  if (tid == 0 && kvh == 0) P.xo.xs[t] = 1.0f;
}

// Attention for one (active entry, kv head) with the G query heads of the
// group handled together: every warp takes positions start + warp, + 16, ...
// for all G heads (each K/V row is loaded once for the group, 16 positions in
// flight per round across the CTA), keeping one online softmax per head; the
// warps' partials are then merged per head.  Same prologue and output as
// k_battn.  Used for head_dim 64 (E = 2), where it fits two CTAs per SM.
template <int E, int G, int NT = CK_THREADS>
__global__ void __launch_bounds__(NT, 2 * CK_THREADS / NT) k_battn_g(BAttn P, BStep st) {
  constexpr int NW = NT / 32;
  constexpr int hd = 32 * E;
  static_assert(G * hd <= CK_HDMAX, "the warps' partials live in SmemAt::wacc");
  const int t = blockIdx.x / P.kvh, kvh = blockIdx.x % P.kvh;
  if (t >= *st.nact) return;
  pdl_wait();
  pdl_launch();
  __shared__ SmemAt s;
  __shared__ int sbt[256];
  __shared__ float wm[NW * G], wl[NW * G], wf[NW * G], hl[G];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int qd = P.heads * hd;
  const int pos = st.pos[t];
  const int start = (P.window != 0 && pos + 1 > P.window) ? pos + 1 - P.window : 0;
  battn_prologue<E, NT>(P, st, s, sbt, t, kvh, pos);
  float q[G][E], acc[G][E], m[G], l[G];
#pragma unroll
  for (int g = 0; g < G; g++) {
    m[g] = -INFINITY;
    l[g] = 0.f;
#pragma unroll
    for (int e = 0; e < E; e++) {
      q[g][e] = s.qs[g * hd + lane * E + e];
      acc[g][e] = 0.f;
    }
  }
  auto off = [&](int p) {
    return (((size_t)sbt[p >> 4] * P.kvh + kvh) * CK_BLK + (p & (CK_BLK - 1))) * hd + lane * E;
  };
  constexpr int CH = E <= 4 ? 8 : 4;   // positions of a warp per round
  for (int p0 = start + warp; p0 < pos; p0 += CH * NW) {
    KvRow<E, false> kr[CH], vr[CH];
#pragma unroll
    for (int j = 0; j < CH; j++) {
      const int p = p0 + j * NW;
      kv_zero(kr[j]); kv_zero(vr[j]);
      if (p < pos) { kv_load(P.kc, off(p), kr[j]); kv_load(P.vc, off(p), vr[j]); }
    }
#pragma unroll
    for (int j = 0; j < CH; j += 2) {   // positions grow with j: a pair past pos ends the round
      if (p0 + j * NW < pos) {
        const bool has1 = p0 + (j + 1) * NW < pos;
#pragma unroll
        for (int g = 0; g < G; g++)
          softmax_pair<E, false>(q[g], kr[j], vr[j], kr[j + 1], vr[j + 1], has1, P.scale, m[g], l[g], acc[g]);
      }
    }
  }
  if (warp == 0) {   // position pos, as the cache now holds it
#pragma unroll
    for (int g = 0; g < G; g++) {
      float d0 = 0.f;
#pragma unroll
      for (int e = 0; e < E; e++) d0 += q[g][e] * kv_round<false>(s.kst[lane * E + e]);
      const float s0 = warp_sum(d0) * P.scale;
      const float mn = fmaxf(m[g], s0);
      const float c = expf(m[g] - mn), p0 = expf(s0 - mn);
      l[g] = l[g] * c + p0;
#pragma unroll
      for (int e = 0; e < E; e++) acc[g][e] = acc[g][e] * c + p0 * kv_round<false>(s.kvw[1][lane * E + e]);
      m[g] = mn;
    }
  }
#pragma unroll
  for (int g = 0; g < G; g++) {
    if (lane == 0) {
      wm[warp * G + g] = m[g];
      wl[warp * G + g] = l[g];
    }
#pragma unroll
    for (int e = 0; e < E; e++) s.wacc[warp * (G * hd) + g * hd + lane * E + e] = acc[g][e];
  }
  __syncthreads();
  if (tid < G) {   // per head: the warps' weights exp(m_w - M) and the merged sum
    float M = -INFINITY;
    for (int w = 0; w < NW; w++) M = fmaxf(M, wm[w * G + tid]);
    float L = 0.f;
    for (int w = 0; w < NW; w++) {
      const float f = wm[w * G + tid] == -INFINITY ? 0.f : expf(wm[w * G + tid] - M);
      wf[w * G + tid] = f;
      L += wl[w * G + tid] * f;
    }
    hl[tid] = L;
  }
  __syncthreads();
  const int nch = tc_nch(qd);
  for (int i = tid; i < G * hd; i += NT) {
    const int gg = i / hd, d = i % hd;
    float A = 0.f;
    for (int w = 0; w < NW; w++) A += s.wacc[w * (G * hd) + gg * hd + d] * wf[w * G + gg];
    const float o = A / hl[gg];
    const int col = (kvh * G + gg) * hd + d;
    const __half h = __float2half_rn(o);
    P.xo.xt[tc_index(t, col, nch, 0)] = h;
    P.xo.xt[tc_index(t, col, nch, 1)] = __float2half_rn(o - __half2float(h));
  }
  if (tid == 0 && kvh == 0) P.xo.xs[t] = 1.0f;
}

// Greedy id of every active entry: ARGMAX_STAGE1/2 rules (NaN never wins,
// ties go to the lower index) over its logits row.
__global__ void __launch_bounds__(CK_THREADS) k_bargmax(const float* logits, int V, BStep st, uint32_t* ids) {
  const int t = blockIdx.x;
  if (t >= *st.nact) return;
  pdl_wait();
  pdl_launch();
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
  int battn_nt = 256;         // threads of a head_dim-64 attention CTA (CK_BATTN_THREADS=512: the wider form)
  cudaStream_t stream = nullptr;
  std::vector<void*> allocs;
  std::string err;
  __half* kv = nullptr;       // [layers][K|V][n_blocks][kv_heads][CK_BLK][head_dim]
  uint32_t* d_tok = nullptr;
  int *d_slot = nullptr, *d_pos = nullptr, *d_nact = nullptr, *d_btab = nullptr, *d_err = nullptr;
  uint32_t* d_ids = nullptr;
  float *x = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *g = nullptr, *u = nullptr, *logits = nullptr;
  BXh xh{};                   // operand tiles of the attention output / SiLU product (scale 1)
  BXh xn{};                   // operand tiles of the normed residual stream (scale from ssq or the prologue)
  float* ssq = nullptr;       // [max_seqs][row tiles of hidden] sums of squares of the residual stream
  bool glu = false;           // gate / up interleaved into one tile set (SiLU in the GEMM epilogue)
  std::vector<__half*> wt;    // operand tiles per weight: layer-major q k v o gate up down, then the head
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

// K slices per row tile (the cluster size): the largest size, at most 8 (the
// portable cluster size) and at most one slice per K chunk, whose clusters
// all fit on the device at once (cudaOccupancyMaxActiveClusters); 1 when the
// row tiles alone fill it.
int tc_max_clusters(int s) {
  static int cache[64][9];
  static bool init[64];
  static std::mutex mu;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 0;
  std::lock_guard<std::mutex> lock(mu);
  if (!init[dev]) {
    for (int c = 1; c <= 8; c++) {
      cudaLaunchConfig_t cfg;
      memset(&cfg, 0, sizeof cfg);
      cfg.gridDim = dim3(c, 1, 1);
      cfg.blockDim = dim3(TC_THREADS);
      cfg.dynamicSmemBytes = TC_SMEM;
      cudaLaunchAttribute at[1];
      at[0].id = cudaLaunchAttributeClusterDimension;
      at[0].val.clusterDim.x = c;
      at[0].val.clusterDim.y = 1;
      at[0].val.clusterDim.z = 1;
      cfg.attrs = at;
      cfg.numAttrs = 1;
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(&n, k_bgemm_tc, &cfg) != cudaSuccess) {
        cudaGetLastError();
        n = 0;
      }
      cache[dev][c] = n;
    }
    init[dev] = true;
  }
  return cache[dev][s];
}

int tc_splits(int units, int nch) {
  // a cluster waits for its longest slice: among the sizes whose clusters all
  // fit at once, the one with the shortest longest slice, the smallest such
  // (fewer partial tiles to sum)
  int best = 1, best_len = nch;
  for (int s = 2; s <= 8 && s <= nch; s++) {
    if (units > tc_max_clusters(s)) continue;
    const int len = (nch + s - 1) / s;
    if (len < best_len) { best = s; best_len = len; }
  }
  return best;
}

// pdl: launch with programmatic stream serialization (the kernel may start
// while its predecessor runs; it waits before touching shared data)
cudaError_t tc_launch(BGemm& G, BStep st, BXh xh, int* err, int ttiles, cudaStream_t s, bool pdl = false) {
  const int tiles = G.tile0[G.nseg];
  G.splits = tc_splits(tiles * ttiles, tc_nch(G.k));
  cudaLaunchConfig_t cfg;
  memset(&cfg, 0, sizeof cfg);
  cfg.gridDim = dim3(tiles * G.splits, ttiles);
  cfg.blockDim = dim3(TC_THREADS);
  cfg.dynamicSmemBytes = TC_SMEM;
  cfg.stream = s;
  cudaLaunchAttribute at[2];
  int na = 0;
  if (G.splits > 1) {
    at[na].id = cudaLaunchAttributeClusterDimension;
    at[na].val.clusterDim.x = G.splits;
    at[na].val.clusterDim.y = 1;
    at[na].val.clusterDim.z = 1;
    na++;
  }
  if (pdl) {
    at[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[na].val.programmaticStreamSerializationAllowed = 1;
    na++;
  }
  cfg.attrs = at;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, k_bgemm_tc, G, st, xh, err);
}

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*k)(KArgs...), dim3 grid, dim3 block, cudaStream_t s, Args... args) {
  cudaLaunchConfig_t cfg;
  memset(&cfg, 0, sizeof cfg);
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k, args...);
}

// x: the operand tiles to read.  nw: the residual-stream GEMMs (o, down) also
// write the next RMS norm's operand tiles (x * nw) into xn with their row
// tiles' sums of squares; norm_in: the GEMM's prologue scale comes from
// those sums (the GEMMs that read xn after such an epilogue).
int bgemm_launch(ck_batch* b, cudaStream_t s, int k, std::initializer_list<BSeg> segs, BXh x,
                 const float* nw = nullptr, bool norm_in = false, __half* glu_xt = nullptr) {
  BGemm G;
  memset(&G, 0, sizeof G);
  G.k = k;
  G.glu_xt = glu_xt;
  G.glu_k = b->h->cfg.intermediate;
  const int htiles = (b->h->cfg.hidden + TC_ROWS - 1) / TC_ROWS;
  if (nw) {
    G.nw = nw;
    G.nxt = b->xn.xt;
    G.nssq = b->ssq;
    G.ntiles = htiles;
  }
  if (norm_in) {
    G.ssq_in = b->ssq;
    G.ssq_tiles = htiles;
    G.eps = b->h->cfg.norm_eps;
  }
  int tiles = 0;
  for (const BSeg& x : segs) {
    G.tile0[G.nseg] = tiles;
    G.seg[G.nseg++] = x;
    tiles += (x.n + TC_ROWS - 1) / TC_ROWS;
  }
  G.tile0[G.nseg] = tiles;
  // token tiles past T return at once
  CKB(b, tc_launch(G, bstep(b), x, b->d_err, (b->max_seqs + TC_NT - 1) / TC_NT, s, true));
  return CK_OK;
}

BSeg bseg(const Weight& w, const __half* wt, float* out, const float* add, int ldo) {
  BSeg s;
  s.w = w.dev;
  s.wt = wt;
  s.L = w.L;
  s.n = w.n;
  s.out = out;
  s.add = add;
  s.ldo = ldo;
  return s;
}

void bprep(ck_batch* b, cudaStream_t s, int kind, const float* a, const float* bb, const float* w, float eps, int k,
           int lda, BXh x) {
  BPrep p;
  p.kind = kind; p.a = a; p.b = bb; p.w = w; p.eps = eps; p.k = k; p.lda = lda;
  launch_pdl(k_bprep, dim3(b->max_seqs), dim3(CK_THREADS), s, p, bstep(b), x);
}

// The whole step on stream s (captured once into a graph).
int batch_enqueue(ck_batch* b, cudaStream_t s) {
  ck_engine* h = b->h;
  const ck_model_cfg& c = h->cfg;
  const int H = c.hidden, hd = c.head_dim, qd = c.heads * hd, kvd = c.kv_heads * hd, I = c.intermediate;
  const size_t pool = (size_t)b->n_blocks * c.kv_heads * CK_BLK * hd;
  CKB(b, launch_pdl(k_bembed, dim3(b->max_seqs), dim3(256), s, (const uint8_t*)h->emb.dev, h->emb.L,
                    c.embedding_scale, bstep(b), b->x, H, c.vocab, b->d_err));
  // The RMS norms after the first: the o and down GEMMs (which produce the
  // residual stream) write the next norm's operand tiles and partial sums of
  // squares in their epilogue, so only layer 0's attention norm is a prologue.
  bprep(b, s, BP_NORM, b->x, nullptr, h->L[0].attn_norm, c.norm_eps, H, H, b->xn);
  for (int i = 0; i < c.layers; i++) {
    const LayerW& W = h->L[i];
    __half* const* wt = &b->wt[(size_t)7 * i];
    int rc = bgemm_launch(b, s, H, {bseg(W.q, wt[0], b->q, nullptr, qd), bseg(W.k, wt[1], b->k, nullptr, kvd),
                                    bseg(W.v, wt[2], b->v, nullptr, kvd)}, b->xn, nullptr, i > 0);
    if (rc) return rc;
    BAttn a;
    a.q = b->q; a.k = b->k; a.v = b->v;
    a.qw = c.qk_norm ? W.q_norm : nullptr;
    a.kw = c.qk_norm ? W.k_norm : nullptr;
    a.kc = b->kv + (size_t)(2 * i) * pool;
    a.vc = b->kv + (size_t)(2 * i + 1) * pool;
    a.inv_freq = h->inv_freq + (size_t)i * (hd / 2);
    a.xo = b->xh;
    a.heads = c.heads; a.kvh = c.kv_heads; a.hd = hd; a.interleaved = c.rope_interleaved;
    a.window = (int)c.layer_window[i];
    a.eps = c.qk_norm_eps;
    a.scale = (float)(1.0 / sqrt((double)hd));   // ATTN_SCALE (:1711)
    const int grid = b->max_seqs * c.kv_heads, G = c.heads / c.kv_heads;
    if (hd == 64 && G == 3 && b->battn_nt == 256)
      CKB(b, launch_pdl(k_battn_g<2, 3, 256>, dim3(grid), dim3(256), s, a, bstep(b)));
    else if (hd == 64 && G == 2 && b->battn_nt == 256)
      CKB(b, launch_pdl(k_battn_g<2, 2, 256>, dim3(grid), dim3(256), s, a, bstep(b)));
    else if (hd == 64 && G == 3) CKB(b, launch_pdl(k_battn_g<2, 3>, dim3(grid), dim3(CK_THREADS), s, a, bstep(b)));
    else if (hd == 64 && G == 2) CKB(b, launch_pdl(k_battn_g<2, 2>, dim3(grid), dim3(CK_THREADS), s, a, bstep(b)));
    else if (hd == 64) CKB(b, launch_pdl(k_battn<2>, dim3(grid), dim3(CK_THREADS), s, a, bstep(b)));
    else if (hd == 128) CKB(b, launch_pdl(k_battn<4>, dim3(grid), dim3(CK_THREADS), s, a, bstep(b)));
    else CKB(b, launch_pdl(k_battn<8>, dim3(grid), dim3(CK_THREADS), s, a, bstep(b)));
    if ((rc = bgemm_launch(b, s, qd, {bseg(W.o, wt[3], b->x, b->x, H)}, b->xh, W.post_norm))) return rc;
    if (b->glu) {   // silu(gate) * up straight into the down projection's tiles (xh.xs stays 1)
      BSeg gu = bseg(W.gate, wt[4], nullptr, nullptr, 0);
      gu.n = 2 * I;
      rc = bgemm_launch(b, s, H, {gu}, b->xn, nullptr, true, b->xh.xt);
      if (rc) return rc;
    } else {
      rc = bgemm_launch(b, s, H, {bseg(W.gate, wt[4], b->g, nullptr, I), bseg(W.up, wt[5], b->u, nullptr, I)}, b->xn,
                        nullptr, true);
      if (rc) return rc;
      bprep(b, s, BP_SILU, b->g, b->u, nullptr, 0.f, I, I, b->xh);
    }
    const float* next_norm = i + 1 < c.layers ? h->L[i + 1].attn_norm : h->final_norm;
    if ((rc = bgemm_launch(b, s, I, {bseg(W.down, wt[6], b->x, b->x, H)}, b->xh, next_norm))) return rc;
  }
  int rc = bgemm_launch(b, s, H, {bseg(h->head, b->wt[(size_t)7 * c.layers], b->logits, nullptr, c.vocab)}, b->xn,
                        nullptr, true);
  if (rc) return rc;
  CKB(b, launch_pdl(k_bargmax, dim3(b->max_seqs), dim3(CK_THREADS), s, (const float*)b->logits, c.vocab, bstep(b),
                    b->d_ids));
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
  if (c.hidden % 32 || c.intermediate % 32 || c.hidden > CK_KMAX || c.intermediate > CK_KMAX)
    return h->fail(CK_EINVAL, "batched decode: matmul widths must be multiples of 32 up to %d", CK_KMAX);
  ck_batch* b = new ck_batch();
  b->h = h;
  b->max_seqs = max_seqs;
  b->max_blocks = max_blocks;
  b->n_blocks = kv_blocks > 0 ? kv_blocks : max_seqs * max_blocks;
  if (const char* e = getenv("CK_BATTN_THREADS")) b->battn_nt = atoi(e) == 512 ? 512 : 256;
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
      (rc = balloc(b, &b->g, S * I * 4)) ||
      (rc = balloc(b, &b->u, S * I * 4)) || (rc = balloc(b, &b->logits, S * c.vocab * 4)) ||
      (rc = balloc(b, &b->xh.xt, tc_bytes(max_seqs, CK_KMAX))) || (rc = balloc(b, &b->xh.xs, S * 4)) ||
      (rc = balloc(b, &b->xn.xt, tc_bytes(max_seqs, CK_KMAX))) || (rc = balloc(b, &b->xn.xs, S * 4)) ||
      (rc = balloc(b, &b->ssq, S * ((c.hidden + TC_ROWS - 1) / TC_ROWS) * 4)))
    return bail(rc);
  // every weight as operand tiles (dequantized once: 4 bytes per weight)
  {
    std::vector<const Weight*> ws;
    for (int i = 0; i < c.layers; i++) {
      const LayerW& W = h->L[i];
      for (const Weight* w : {&W.q, &W.k, &W.v, &W.o, &W.gate, &W.up, &W.down}) ws.push_back(w);
    }
    ws.push_back(&h->head);
    // gate and up as one interleaved tile set when the intermediate size is a
    // multiple of 64: the gate/up GEMM then applies SiLU in its epilogue
    b->glu = c.intermediate % (TC_ROWS / 2) == 0;
    for (size_t j = 0; j < ws.size(); j++) {
      const Weight* w = ws[j];
      const int role = j < (size_t)7 * c.layers ? (int)(j % 7) : -1;   // 4 gate, 5 up
      __half* t = nullptr;
      const int kk = w->L.k;
      if (b->glu && role == 5) {   // held by the gate's tiles
        b->wt.push_back(nullptr);
        continue;
      }
      if (b->glu && role == 4) {
        const Weight* up = ws[j + 1];
        if ((rc = balloc(b, &t, tc_bytes(2 * w->n, kk)))) return bail(rc);
        k_tc_format<<<dim3(2 * w->n / TC_ROWS, tc_nch(kk)), 256, 0, b->stream>>>(w->dev, w->L, w->n, kk, t, up->dev,
                                                                               up->L);
      } else {
        if ((rc = balloc(b, &t, tc_bytes(w->n, kk)))) return bail(rc);
        k_tc_format<<<dim3((w->n + TC_ROWS - 1) / TC_ROWS, tc_nch(kk)), 256, 0, b->stream>>>(w->dev, w->L, w->n, kk,
                                                                                           t);
      }
      b->wt.push_back(t);
    }
    if (cudaGetLastError() != cudaSuccess || cudaStreamSynchronize(b->stream) != cudaSuccess)
      return bail(b->fail(CK_ECUDA, "weight tiles"));
  }
  if (cudaMemset(b->d_err, 0, 16) != cudaSuccess || cudaMemset(b->d_nact, 0, 16) != cudaSuccess ||
      cudaMemset(b->d_btab, 0, S * max_blocks * 4) != cudaSuccess)
    return bail(b->fail(CK_ECUDA, "memset"));
  if (cudaMallocHost(&b->pin, S * 16 + 64) != cudaSuccess) return bail(b->fail(CK_ENOMEM, "pinned staging"));
  if (cudaFuncSetAttribute(k_bgemm_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, TC_SMEM) != cudaSuccess)
    return bail(b->fail(CK_ECUDA, "matmul shared memory"));
  tc_max_clusters(1);   // the occupancy table, before the step graph is captured
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
    const int bits = *perr;
    cudaMemset(b->d_err, 0, 4);
    if (bits & CK_DERR_TOKEN) return b->fail(CK_EDEVICE, "token id outside embedding table");
    return b->fail(CK_EDEVICE, "batched step: a device wait timed out (bits 0x%x)", bits);
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

// Y[T x n] = X[T x k] W^T through the batched path's prologue and
// tensor-core GEMM (parity helper: x host fp32 [T][k], y host fp32 [T][n]).
int ck_matmul(int ggml_type, const void* bytes, size_t nbytes, int k, int n, const float* x, int T, float* y,
              int device) {
  if (!bytes || !x || !y || T < 1 || T > 1024 || k % 32 || k > CK_KMAX)
    return set_global(CK_EINVAL, "ck_matmul: bad argument");
  ck_engine* h;
  int rc = make_tmp(device, &h);
  if (rc) return rc;
  Weight w;
  float *dx = nullptr, *dy = nullptr, *xs = nullptr;
  __half *wt = nullptr, *xt = nullptr;
  int *nact = nullptr, *err = nullptr;
  auto done = [&](int code) {
    std::string m = h->err;
    free_tmp(h);
    return code ? set_global(code, "ck_matmul: %s", m.c_str()) : CK_OK;
  };
  if ((rc = prep_weight(h, ggml_type, bytes, nbytes, k, n, w)) || (rc = dalloc(h, &dx, (size_t)T * k * 4)) ||
      (rc = dalloc(h, &dy, (size_t)T * n * 4)) || (rc = dalloc(h, &xs, (size_t)T * 4)) ||
      (rc = dalloc(h, &wt, tc_bytes(n, k))) || (rc = dalloc(h, &xt, tc_bytes(T, k))) ||
      (rc = dalloc(h, &nact, 16)) || (rc = dalloc(h, &err, 16)))
    return done(rc);
  cudaMemcpy(dx, x, (size_t)T * k * 4, cudaMemcpyHostToDevice);
  cudaMemcpy(nact, &T, 4, cudaMemcpyHostToDevice);
  cudaMemset(err, 0, 16);
  k_tc_format<<<dim3((n + TC_ROWS - 1) / TC_ROWS, tc_nch(k)), 256, 0, h->own>>>(w.dev, w.L, n, k, wt);
  BStep st;
  memset(&st, 0, sizeof st);
  st.nact = nact;
  BXh xh;
  xh.xt = xt;
  xh.xs = xs;
  BPrep p;
  p.kind = BP_COPY; p.a = dx; p.b = nullptr; p.w = nullptr; p.eps = 0.f; p.k = k; p.lda = k;
  k_bprep<<<T, CK_THREADS, 0, h->own>>>(p, st, xh);
  BGemm G;
  memset(&G, 0, sizeof G);
  G.k = k;
  G.nseg = 1;
  G.seg[0] = bseg(w, wt, dy, nullptr, n);
  G.tile0[1] = (n + TC_ROWS - 1) / TC_ROWS;
  cudaFuncSetAttribute(k_bgemm_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, TC_SMEM);
  cudaError_t e = tc_launch(G, st, xh, err, (T + TC_NT - 1) / TC_NT, h->own);
  int herr = 0;
  if (e == cudaSuccess) e = cudaMemcpyAsync(y, dy, (size_t)T * n * 4, cudaMemcpyDeviceToHost, h->own);
  if (e == cudaSuccess) e = cudaMemcpyAsync(&herr, err, 4, cudaMemcpyDeviceToHost, h->own);
  if (e == cudaSuccess) e = cudaStreamSynchronize(h->own);
  if (e != cudaSuccess) return done(h->fail(CK_ECUDA, "%s", cudaGetErrorString(e)));
  if (herr) return done(h->fail(CK_EDEVICE, "device wait timed out"));
  return done(CK_OK);
}

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
