// Streaming matvec y = W x over one large weight matrix of a single GGUF
// block type: the LM head (GGUF_Q6_K_MATVEC_WGSL / GGUF_Q8_0_MATVEC_WGSL,
// llama-wgsl-runtime.ts:2291-2613, the 151936-row tied head of Qwen3) and
// any matrix large enough to be bandwidth bound.
//
// One CTA of 20 warps per SM; CTA c owns rows [c*n/grid, (c+1)*n/grid).
// The last warp copies the CTA's rows, a slot at a time, into a ring of
// GV_NSLOT shared-memory slots (cp.async.bulk into this CTA's own shared
// memory, completing on the slot's mbarrier, L2 evict-first); the other 19
// warps take each slot's rows GV_RB at a time per warp (20 warps measured
// 2-5 % faster than 16; a third 64 KB slot in place of two 96 KB ones was
// slower).
// Each kernel instance is compiled for one block type, so a unit's decode is
// straight-line code, and x (quantized per 32 elements into X = hi * 256 +
// lo, as XUnit describes) sits in shared memory in 16-byte chunks that the
// lanes of a warp read without bank conflicts.
#pragma once
#include "ck_ops.cuh"

#ifndef GV_THREADS
#define GV_THREADS 640
#endif
#define GV_NCW (GV_THREADS / 32 - 1)   // compute warps (the last warp copies)
#define GV_NCT (GV_NCW * 32)
#ifndef GV_SLOT_BYTES
#define GV_SLOT_BYTES (96 * 1024)
#endif
#ifndef GV_NSLOT
#define GV_NSLOT 2
#endif
#ifndef GV_RB
#define GV_RB 4                   // rows a warp reduces together
#endif
#define GV_DYN_BYTES (GV_NSLOT * GV_SLOT_BYTES + 16 * GV_NSLOT)

// x of one unit in registers
struct GvX {
  int4 h0, h1, l0, l1;   // hi / lo bytes of X, elements 0..15 and 16..31
  float sx, sf;          // step and (float)(sa + sb)
  int sa, sb;            // sum of X over elements 0..15 and 16..31
};
struct GvSmem {
  int4 xq[4][CK_KMAX / 32];   // hi 0..15, hi 16..31, lo 0..15, lo 16..31 of unit c at [.][c]
  float4 xs[CK_KMAX / 32];    // {step, (float)(sa + sb), sa, sb}
};
__device__ __forceinline__ void gv_x(const GvSmem& s, int c, GvX& x) {
  x.h0 = s.xq[0][c]; x.h1 = s.xq[1][c]; x.l0 = s.xq[2][c]; x.l1 = s.xq[3][c];
  const float4 v = s.xs[c];
  x.sx = v.x; x.sf = v.y; x.sa = __float_as_int(v.z); x.sb = __float_as_int(v.w);
}

__device__ __forceinline__ int gv_dp_all(const int (&q)[8], const GvX& x) {
  int h0 = __dp4a(q[0], x.h0.x, 0), h1 = __dp4a(q[1], x.h0.y, 0);
  int l0 = __dp4a(q[0], x.l0.x, 0), l1 = __dp4a(q[1], x.l0.y, 0);
  h0 = __dp4a(q[2], x.h0.z, h0); h1 = __dp4a(q[3], x.h0.w, h1);
  l0 = __dp4a(q[2], x.l0.z, l0); l1 = __dp4a(q[3], x.l0.w, l1);
  h0 = __dp4a(q[4], x.h1.x, h0); h1 = __dp4a(q[5], x.h1.y, h1);
  l0 = __dp4a(q[4], x.l1.x, l0); l1 = __dp4a(q[5], x.l1.y, l1);
  h0 = __dp4a(q[6], x.h1.z, h0); h1 = __dp4a(q[7], x.h1.w, h1);
  l0 = __dp4a(q[6], x.l1.z, l0); l1 = __dp4a(q[7], x.l1.w, l1);
  return (h0 + h1) * 256 + (l0 + l1);
}
__device__ __forceinline__ void gv_dp_halves(const int (&q)[8], const GvX& x, int& da, int& db) {
  int ha = __dp4a(q[0], x.h0.x, 0), la = __dp4a(q[0], x.l0.x, 0);
  int hb = __dp4a(q[4], x.h1.x, 0), lb = __dp4a(q[4], x.l1.x, 0);
  ha = __dp4a(q[1], x.h0.y, ha); la = __dp4a(q[1], x.l0.y, la);
  hb = __dp4a(q[5], x.h1.y, hb); lb = __dp4a(q[5], x.l1.y, lb);
  ha = __dp4a(q[2], x.h0.z, ha); la = __dp4a(q[2], x.l0.z, la);
  hb = __dp4a(q[6], x.h1.z, hb); lb = __dp4a(q[6], x.l1.z, lb);
  ha = __dp4a(q[3], x.h0.w, ha); la = __dp4a(q[3], x.l0.w, la);
  hb = __dp4a(q[7], x.h1.w, hb); lb = __dp4a(q[7], x.l1.w, lb);
  da = ha * 256 + la;
  db = hb * 256 + lb;
}

// sum_i x_i w_i over unit c of a row of block type TYPE (weights as the WGSL
// dequantizers give them, see unpack_unit).  sum_i X_i q_i and sum_i X_i are
// exact integers below 2^24, so a unit costs one or two conversions.
template <int TYPE>
__device__ __forceinline__ float gv_unit(const uint8_t* row, const Lay& L, int c, const GvX& x) {
  if (TYPE == GT_Q4_K) {
    const uint4 w = *(const uint4*)(row + L.off_q + 16 * c);
    const uint4 hd = *(const uint4*)(row + L.off_sc + 16 * (c >> 3));
    int q[8];
    q[0] = (int)(w.x & 0x0F0F0F0Fu); q[4] = (int)((w.x >> 4) & 0x0F0F0F0Fu);
    q[1] = (int)(w.y & 0x0F0F0F0Fu); q[5] = (int)((w.y >> 4) & 0x0F0F0F0Fu);
    q[2] = (int)(w.z & 0x0F0F0F0Fu); q[6] = (int)((w.z >> 4) & 0x0F0F0F0Fu);
    q[3] = (int)(w.w & 0x0F0F0F0Fu); q[7] = (int)((w.w >> 4) & 0x0F0F0F0Fu);
    const int D = gv_dp_all(q, x);
    // scale_min_k4 (llama-wgsl-runtime.ts:2387-2394) over the packed bytes
    // q0..3 (header word y), q4..7 (z), q8..11 (w), without a branch
    const int sub = c & 7;
    const uint32_t s4 = 8 * (sub & 3);
    const uint32_t by = (hd.y >> s4) & 0xFFu, bz = (hd.z >> s4) & 0xFFu, bw = (hd.w >> s4) & 0xFFu;
    const uint32_t sc = sub < 4 ? (by & 63u) : ((bw & 15u) | ((by >> 6) << 4));
    const uint32_t m = sub < 4 ? (bz & 63u) : ((bw >> 4) | ((bz >> 6) << 4));
    const float d = h2f_u16(hd.x), dmin = h2f_u16(hd.x >> 16);
    return x.sx * ((d * (float)sc) * (float)D - (dmin * (float)m) * x.sf);
  } else if (TYPE == GT_Q6_K) {
    const uint4 w = *(const uint4*)(row + L.off_q + 16 * c);
    const uint2 h = *(const uint2*)(row + L.off_q2 + 8 * c);
    const int sb = c >> 3, sub = c & 7;
    const uint32_t dd = *(const unsigned short*)(row + L.off_d + 2 * sb);
    const uint32_t scp = *(const unsigned short*)(row + L.off_sc + 16 * sb + 2 * sub);
    const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
    int q[8];
#pragma unroll
    for (int t = 0; t < 4; t++) {
      const uint32_t H = (t & 1) ? h.y : h.x;
      const int sh = (t >> 1) * 4;
      q[t] = (int)((ww[t] & 0x0F0F0F0Fu) | (((H >> sh) << 4) & 0x30303030u));
      q[4 + t] = (int)(((ww[t] >> 4) & 0x0F0F0F0Fu) | (((H >> (sh + 2)) << 4) & 0x30303030u));
    }
    int da, db;
    gv_dp_halves(q, x, da, db);
    const float d = h2f_u16(dd);
    return x.sx * ((d * (float)(int)(int8_t)(scp & 0xFFu)) * (float)(da - 32 * x.sa) +
                   (d * (float)(int)(int8_t)(scp >> 8)) * (float)(db - 32 * x.sb));
  } else if (TYPE == GT_Q8_0) {
    const uint4 w0 = *(const uint4*)(row + L.off_q + 32 * c), w1 = *(const uint4*)(row + L.off_q + 32 * c + 16);
    const int q[8] = {(int)w0.x, (int)w0.y, (int)w0.z, (int)w0.w, (int)w1.x, (int)w1.y, (int)w1.z, (int)w1.w};
    const float d = h2f_u16(*(const unsigned short*)(row + L.off_d + 2 * c));
    return x.sx * (d * (float)gv_dp_all(q, x));
  } else {   // Q5_0 / Q5_1
    const uint4 w = *(const uint4*)(row + L.off_q + 16 * c);
    const uint32_t qh = *(const uint32_t*)(row + L.off_qh + 4 * c);
    const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
    int q[8];
#pragma unroll
    for (int t = 0; t < 4; t++) {
      q[t] = (int)((ww[t] & 0x0F0F0F0Fu) | ((qh << (4 - t)) & 0x10101010u));
      q[4 + t] = (int)(((ww[t] >> 4) & 0x0F0F0F0Fu) | ((qh >> t) & 0x10101010u));
    }
    const int D = gv_dp_all(q, x);
    const float d = h2f_u16(*(const unsigned short*)(row + L.off_d + 2 * c));
    if (TYPE == GT_Q5_0) return x.sx * (d * (float)(D - 16 * (x.sa + x.sb)));
    const float m = h2f_u16(*(const unsigned short*)(row + L.off_m + 2 * c));
    return x.sx * (d * (float)D + m * x.sf);
  }
}

__device__ __forceinline__ void gv_bar() { asm volatile("bar.sync 1, %0;" ::"n"(GV_NCT) : "memory"); }

// Bounded mbarrier wait (flags the run and carries on when it gives up).
__device__ __forceinline__ void gv_wait(uint64_t* bar, uint32_t parity, int* err) {
  unsigned spins = 0;
  while (!mbar_try_wait(bar, parity)) {
    if (++spins > (1u << 22)) {
      if (err) atomicOr(err, CK_DERR_BARRIER);
      return;
    }
  }
}

// Quantize x[0..k) per 32-element unit into s (compute warps).
__device__ __forceinline__ void gv_quant_x(const float* __restrict__ x, int k, GvSmem& s) {
  const int tid = threadIdx.x, lane = tid & 31, half = (tid >> 4) & 1, warp = tid >> 5, hl = lane & 15;
  const int U = k >> 5;
  for (int gp = warp; 2 * gp < U; gp += GV_NCW) {
    const int g = 2 * gp + half;
    const bool ok = g < U;
    const float2 xv = ok ? __ldg((const float2*)(x + 32 * g + 2 * hl)) : make_float2(0.f, 0.f);
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
    const int tot = sum + __shfl_xor_sync(0xffffffffu, sum, 8);
    if (!ok) continue;
    ((short*)&s.xq[hl >> 3][g])[hl & 7] = (short)((h0 & 0xFF) | (h1 << 8));
    ((short*)&s.xq[2 + (hl >> 3)][g])[hl & 7] = (short)((l0 & 0xFF) | (l1 << 8));
    if (hl == 0) {
      s.xs[g].x = fin ? step : __int_as_float(0x7fc00000);
      s.xs[g].y = (float)tot;
      s.xs[g].z = __int_as_float(sum);
    }
    if (hl == 8) s.xs[g].w = __int_as_float(sum);
  }
}

// Q4_K rows of 32 units: lane (half h, j) takes units 2j and 2j + 1 of row
// 2 p + h (they share their super-block header and its d, dmin); the 16
// lanes of a row reduce in four shuffle levels.  GV_RB row pairs per warp at
// a time.
__device__ __forceinline__ float gv_q4k_pair(const uint8_t* row, const Lay& L, int c, const GvX& xa,
                                             const GvX& xb) {
  const uint4 hd = *(const uint4*)(row + L.off_sc + 16 * (c >> 3));
  const float d = h2f_u16(hd.x), dmin = h2f_u16(hd.x >> 16);
  float r = 0.f;
#pragma unroll
  for (int u = 0; u < 2; u++) {
    const GvX& x = u ? xb : xa;
    const uint4 w = *(const uint4*)(row + L.off_q + 16 * (c + u));
    int q[8];
    q[0] = (int)(w.x & 0x0F0F0F0Fu); q[4] = (int)((w.x >> 4) & 0x0F0F0F0Fu);
    q[1] = (int)(w.y & 0x0F0F0F0Fu); q[5] = (int)((w.y >> 4) & 0x0F0F0F0Fu);
    q[2] = (int)(w.z & 0x0F0F0F0Fu); q[6] = (int)((w.z >> 4) & 0x0F0F0F0Fu);
    q[3] = (int)(w.w & 0x0F0F0F0Fu); q[7] = (int)((w.w >> 4) & 0x0F0F0F0Fu);
    const int D = gv_dp_all(q, x);
    const int sub = (c + u) & 7;
    const uint32_t s4 = 8 * (sub & 3);
    const uint32_t by = (hd.y >> s4) & 0xFFu, bz = (hd.z >> s4) & 0xFFu, bw = (hd.w >> s4) & 0xFFu;
    const uint32_t sc = sub < 4 ? (by & 63u) : ((bw & 15u) | ((by >> 6) << 4));
    const uint32_t m = sub < 4 ? (bz & 63u) : ((bw >> 4) | ((bz >> 6) << 4));
    r += x.sx * ((d * (float)sc) * (float)D - (dmin * (float)m) * x.sf);
  }
  return r;
}
__device__ __forceinline__ void gv_tile_q4k_pairs(const uint8_t* tb, const Lay& L, int rows, int r0,
                                                  const GvX& xa, const GvX& xb, float* __restrict__ y) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int h = lane >> 4, j = lane & 15;
  const int pairs = (rows + 1) >> 1;
  for (int p0 = warp; p0 < pairs; p0 += GV_NCW * GV_RB) {
    float acc[GV_RB];
#pragma unroll
    for (int i = 0; i < GV_RB; i++) {
      const int t = 2 * (p0 + i * GV_NCW) + h;
      acc[i] = t < rows ? gv_q4k_pair(tb + (uint32_t)t * L.row_bytes, L, 2 * j, xa, xb) : 0.f;
    }
#pragma unroll
    for (int o = 8; o > 0; o >>= 1)
#pragma unroll
      for (int i = 0; i < GV_RB; i++) acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], o);
#pragma unroll
    for (int i = 0; i < GV_RB; i++) {
      const int t = 2 * (p0 + i * GV_NCW) + h;
      if (j == i && t < rows) y[r0 + t] = acc[i];
    }
  }
}

// The rows of one slot: flat rows t = warp + 15 i (t < rows), GV_RB per warp
// at a time; k <= 1024: lane = unit with x in registers, else lanes cover
// units lane + 32 j.
template <int TYPE>
__device__ __forceinline__ void gv_tile(const uint8_t* tb, const Lay& L, int rows, int r0, const GvSmem& s,
                                        const GvX& x0, float* __restrict__ y) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int U = L.U;
  for (int t0 = warp; t0 < rows; t0 += GV_NCW * GV_RB) {
    float acc[GV_RB];
#pragma unroll
    for (int i = 0; i < GV_RB; i++) {
      const int t = t0 + i * GV_NCW;
      acc[i] = 0.f;
      if (t < rows) {
        const uint8_t* row = tb + (uint32_t)t * L.row_bytes;
        if (U <= 32) {
          if (lane < U) acc[i] = gv_unit<TYPE>(row, L, lane, x0);
        } else {
#pragma unroll 1
          for (int c = lane; c < U; c += 32) {
            GvX xc;
            gv_x(s, c, xc);
            acc[i] += gv_unit<TYPE>(row, L, c, xc);
          }
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
      for (int i = 0; i < GV_RB; i++) acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], o);
#pragma unroll
    for (int i = 0; i < GV_RB; i++) {
      const int t = t0 + i * GV_NCW;
      if (lane == i && t < rows) y[r0 + t] = acc[i];
    }
  }
}

// y[0..n) = W x, W in the device layout L (n rows), x fp32[L.k].  err: device
// error word (a wait gave up), may be null.
template <int TYPE>
__global__ void __launch_bounds__(GV_THREADS, 1) k_gemv(const uint8_t* __restrict__ W, Lay L, int n,
                                                        const float* __restrict__ x, float* __restrict__ y, int* err) {
  __shared__ GvSmem s;
  uint8_t* dyn = dyn_smem();
  uint64_t* full = (uint64_t*)(dyn + GV_NSLOT * GV_SLOT_BYTES);
  uint64_t* empty = full + GV_NSLOT;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int lo = (int)((long long)blockIdx.x * n / gridDim.x);
  const int hi = (int)((long long)(blockIdx.x + 1) * n / gridDim.x);
  const int tile_rows = (int)(GV_SLOT_BYTES / L.row_bytes);
  const int ntiles = (hi - lo + tile_rows - 1) / tile_rows;
  if (tid == 0) {
    for (int i = 0; i < GV_NSLOT; i++) {
      mbar_init(full + i, 1);
      mbar_init(empty + i, GV_NCW);   // one arrival per compute warp
    }
    mbar_fence_init();
  }
  __syncthreads();
  if (warp == GV_NCW) {
    if (lane == 0) {
      for (int t = 0; t < ntiles; t++) {
        const int sl = t % GV_NSLOT;
        if (t >= GV_NSLOT) gv_wait(empty + sl, ((t / GV_NSLOT) - 1) & 1u, err);
        const int r = lo + t * tile_rows;
        const int rows = min(tile_rows, hi - r);
        const uint32_t bytes = (uint32_t)rows * L.row_bytes;
        mbar_expect_tx(full + sl, bytes);
        bulk_g2s_stream(dyn + (size_t)sl * GV_SLOT_BYTES, W + (size_t)r * L.row_bytes, bytes, full + sl);
      }
      // every copy lands before the CTA exits
      for (int t = ntiles > GV_NSLOT ? ntiles - GV_NSLOT : 0; t < ntiles; t++)
        gv_wait(full + (t % GV_NSLOT), (t / GV_NSLOT) & 1u, err);
    }
    return;
  }
  gv_quant_x(x, L.k, s);
  gv_bar();
  const bool pairs = TYPE == GT_Q4_K && L.U == 32;
  GvX x0, x1;
  if (pairs) {
    gv_x(s, 2 * (lane & 15), x0);
    gv_x(s, 2 * (lane & 15) + 1, x1);
  } else if (L.U <= 32 && lane < L.U) {
    gv_x(s, lane, x0);
  }
  for (int t = 0; t < ntiles; t++) {
    const int sl = t % GV_NSLOT;
    gv_wait(full + sl, (t / GV_NSLOT) & 1u, err);
    const int r = lo + t * tile_rows;
    if (pairs) gv_tile_q4k_pairs(dyn + (size_t)sl * GV_SLOT_BYTES, L, min(tile_rows, hi - r), r, x0, x1, y);
    else gv_tile<TYPE>(dyn + (size_t)sl * GV_SLOT_BYTES, L, min(tile_rows, hi - r), r, s, x0, y);
    // this warp is done with the slot (its loads have been consumed): it
    // hands it back on its own and moves on; the copy warp refills the slot
    // once every compute warp has arrived
    __syncwarp();
    if (lane == 0) mbar_arrive(empty + sl);
  }
}

// Host: the kernel instance for a block type.
typedef void (*GvKernel)(const uint8_t*, Lay, int, const float*, float*, int*);
inline GvKernel gv_kernel(int type) {
  switch (type) {
    case GT_Q4_K: return k_gemv<GT_Q4_K>;
    case GT_Q6_K: return k_gemv<GT_Q6_K>;
    case GT_Q8_0: return k_gemv<GT_Q8_0>;
    case GT_Q5_0: return k_gemv<GT_Q5_0>;
    case GT_Q5_1: return k_gemv<GT_Q5_1>;
  }
  return nullptr;
}
