// Device weight layout for GGUF quantized tensors, and the per-unit decoders.
//
// The reference uploads GGUF block bytes unchanged and reads them one byte at
// a time through u32 words (byte_at, llama-wgsl-runtime.ts:2219-2223).  On the
// B200 the same blocks are re-laid once at upload so that every per-lane load
// is a 16-byte aligned vector and every 32-weight "unit" is contiguous:
//
//   row = [metadata arrays][units]          (every array 16-byte aligned)
//
//   Q4_K : hdr[nsb] x16 B (fp16 d, fp16 dmin, 12 B packed 6-bit scale/min, the
//          GGUF header verbatim) | units[8*nsb] x16 B: unit s of a super-block
//          holds sub-block s (32 weights), byte i = q[i] | q[16+i] << 4.
//   Q6_K : sc[nsb] x16 B (int8 scale per 16 weights) | d[nsb] fp16 |
//          ql units[8*nsb] x16 B (low nibbles, same packing as Q4_K) |
//          qh units[8*nsb] x8 B (high 2 bits, see q6_hbits below).
//   Q8_0 : d[nb] fp16 | units[nb] x32 B int8.
//   Q5_0 : d[nb] fp16 | qh'[nb] u32 (bit-permuted, see q5_hperm) | units x16 B.
//   Q5_1 : d[nb] fp16 | m[nb] fp16 | qh'[nb] u32 | units x16 B.
//
// The re-layout is lossless: the same fp16 scales and integer codes, so the
// dequantized values (dequant_at, WGSL operation order) are bit-identical to
// the WGSL dequantizers' (:2234-2245, :2280-2289, :2321-2327, :2396-2410,
// :2560-2580).  Total bytes equal the GGUF's up to 16-byte padding of the small
// metadata arrays.
#pragma once
#include <cuda_fp16.h>
#include <stdint.h>

#define GT_F32 0
#define GT_F16 1
#define GT_Q5_0 6
#define GT_Q5_1 7
#define GT_Q8_0 8
#define GT_Q4_K 12
#define GT_Q6_K 14

struct Lay {
  uint16_t type;
  uint16_t k;         // weights per row (<= 4096)
  uint16_t nb;        // blocks (32) or super-blocks (256) per row
  uint16_t U;         // 32-weight units per row (k / 32)
  uint32_t row_bytes;
  uint16_t off_d, off_m, off_sc, off_qh, off_q, off_q2;   // byte offsets inside a row
};

__host__ __device__ inline uint32_t ck_r16(uint32_t x) { return (x + 15u) & ~15u; }

__host__ __device__ inline bool ck_type_ok(int t) {
  return t == GT_Q4_K || t == GT_Q6_K || t == GT_Q8_0 || t == GT_Q5_0 || t == GT_Q5_1;
}
__host__ __device__ inline int ck_block_weights(int t) { return (t == GT_Q4_K || t == GT_Q6_K) ? 256 : 32; }
__host__ __device__ inline int ck_block_bytes(int t) {
  switch (t) {
    case GT_Q4_K: return 144;
    case GT_Q6_K: return 210;
    case GT_Q8_0: return 34;
    case GT_Q5_0: return 22;
    case GT_Q5_1: return 24;
  }
  return 0;
}

__host__ __device__ inline Lay make_lay(int type, int k) {
  Lay L;
  L.type = (uint16_t)type; L.k = (uint16_t)k; L.U = (uint16_t)(k / 32);
  L.off_d = L.off_m = L.off_sc = L.off_qh = L.off_q = L.off_q2 = 0;
  uint32_t nb = (uint32_t)(k / ck_block_weights(type));
  L.nb = (uint16_t)nb;
  switch (type) {
    case GT_Q4_K:
      L.off_sc = 0;
      L.off_q = (uint16_t)(16 * nb);
      L.row_bytes = L.off_q + 128 * nb;
      break;
    case GT_Q6_K:
      L.off_sc = 0;
      L.off_d = (uint16_t)(16 * nb);
      L.off_q = (uint16_t)(L.off_d + ck_r16(2 * nb));
      L.off_q2 = (uint16_t)(L.off_q + 128 * nb);
      L.row_bytes = L.off_q2 + 64 * nb;
      break;
    case GT_Q8_0:
      L.off_d = 0;
      L.off_q = (uint16_t)ck_r16(2 * nb);
      L.row_bytes = L.off_q + 32 * nb;
      break;
    case GT_Q5_0:
      L.off_d = 0;
      L.off_qh = (uint16_t)ck_r16(2 * nb);
      L.off_q = (uint16_t)(L.off_qh + ck_r16(4 * nb));
      L.row_bytes = L.off_q + 16 * nb;
      break;
    case GT_Q5_1:
      L.off_d = 0;
      L.off_m = (uint16_t)ck_r16(2 * nb);
      L.off_qh = (uint16_t)(L.off_m + ck_r16(2 * nb));
      L.off_q = (uint16_t)(L.off_qh + ck_r16(4 * nb));
      L.row_bytes = L.off_q + 16 * nb;
      break;
    default:
      L.row_bytes = 0;
  }
  return L;
}

// ---------------------------------------------------------------------------
// Re-layout kernel: one thread per (row, GGUF block).

// 6-bit code (0..63) of weight w (0..255) of a raw Q6_K super-block:
// ql/qh addressing of GGUF_Q6_K_MATVEC_WGSL (:2560-2580).
__device__ inline uint32_t raw_q6(const uint8_t* sb, int w) {
  int half = w >> 7, local = w & 127, lane = local & 31, quarter = local >> 5;
  uint32_t ql = sb[half * 64 + lane + ((quarter & 1) ? 32 : 0)];
  uint32_t lo = quarter < 2 ? (ql & 15u) : (ql >> 4);
  uint32_t qh = (sb[128 + half * 32 + lane] >> (quarter * 2)) & 3u;
  return lo | (qh << 4);
}

// High 2 bits of a 32-weight Q6_K unit, packed so that for ql word t (bytes b
// = weights 4t+b and 16+4t+b) word H[t & 1], shifted by (t >> 1) * 4, holds
// the low-group bits at bit 0..1 and the high-group bits at 2..3 of each byte.
__device__ inline void q6_hbits(const uint32_t q[32], uint32_t H[2]) {
  H[0] = H[1] = 0;
  for (int tp = 0; tp < 2; tp++)
    for (int b = 0; b < 4; b++) {
      uint32_t v = ((q[4 * tp + b] >> 4) & 3u) | (((q[16 + 4 * tp + b] >> 4) & 3u) << 2) |
                   (((q[4 * (tp + 2) + b] >> 4) & 3u) << 4) | (((q[16 + 4 * (tp + 2) + b] >> 4) & 3u) << 6);
      H[tp] |= v << (8 * b);
    }
}

// Q5 high-bit permutation: bit (8b + t) <- weight 4t+b, bit (8b + 4 + t) <-
// weight 16+4t+b (t, b in 0..3), so ql word t's fifth bits are one shift and
// one mask away.
__device__ inline uint32_t q5_hperm(uint32_t qh) {
  uint32_t o = 0;
  for (int t = 0; t < 4; t++)
    for (int b = 0; b < 4; b++) {
      o |= ((qh >> (4 * t + b)) & 1u) << (8 * b + t);
      o |= ((qh >> (16 + 4 * t + b)) & 1u) << (8 * b + 4 + t);
    }
  return o;
}

__global__ void k_relayout(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst, Lay L, int n) {
  long long gid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  long long total = (long long)n * L.nb;
  if (gid >= total) return;
  int row = (int)(gid / L.nb), b = (int)(gid % L.nb);
  size_t raw_row = (size_t)L.nb * ck_block_bytes(L.type);
  const uint8_t* s = src + (size_t)row * raw_row + (size_t)b * ck_block_bytes(L.type);
  uint8_t* d = dst + (size_t)row * L.row_bytes;
  switch (L.type) {
    case GT_Q4_K: {
      for (int i = 0; i < 16; i++) d[L.off_sc + 16 * b + i] = s[i];
      const uint8_t* qs = s + 16;
      for (int sub = 0; sub < 8; sub++) {
        int g = sub >> 1, nib = sub & 1;
        uint8_t* u = d + L.off_q + (8 * b + sub) * 16;
        for (int i = 0; i < 16; i++) {
          uint32_t lo = (qs[32 * g + i] >> (4 * nib)) & 15u;
          uint32_t hi = (qs[32 * g + 16 + i] >> (4 * nib)) & 15u;
          u[i] = (uint8_t)(lo | (hi << 4));
        }
      }
      break;
    }
    case GT_Q6_K: {
      for (int i = 0; i < 16; i++) d[L.off_sc + 16 * b + i] = s[192 + i];
      d[L.off_d + 2 * b] = s[208];
      d[L.off_d + 2 * b + 1] = s[209];
      for (int sub = 0; sub < 8; sub++) {
        uint32_t q[32];
        for (int j = 0; j < 32; j++) q[j] = raw_q6(s, 32 * sub + j);
        uint8_t* u = d + L.off_q + (8 * b + sub) * 16;
        for (int i = 0; i < 16; i++) u[i] = (uint8_t)((q[i] & 15u) | ((q[16 + i] & 15u) << 4));
        uint32_t H[2];
        q6_hbits(q, H);
        uint8_t* h = d + L.off_q2 + (8 * b + sub) * 8;
        for (int i = 0; i < 4; i++) { h[i] = (uint8_t)(H[0] >> (8 * i)); h[4 + i] = (uint8_t)(H[1] >> (8 * i)); }
      }
      break;
    }
    case GT_Q8_0:
      d[L.off_d + 2 * b] = s[0];
      d[L.off_d + 2 * b + 1] = s[1];
      for (int i = 0; i < 32; i++) d[L.off_q + 32 * b + i] = s[2 + i];
      break;
    case GT_Q5_0:
    case GT_Q5_1: {
      int is1 = L.type == GT_Q5_1;
      d[L.off_d + 2 * b] = s[0];
      d[L.off_d + 2 * b + 1] = s[1];
      if (is1) { d[L.off_m + 2 * b] = s[2]; d[L.off_m + 2 * b + 1] = s[3]; }
      const uint8_t* qhp = s + (is1 ? 4 : 2);
      uint32_t qh = (uint32_t)qhp[0] | ((uint32_t)qhp[1] << 8) | ((uint32_t)qhp[2] << 16) | ((uint32_t)qhp[3] << 24);
      uint32_t p = q5_hperm(qh);
      for (int i = 0; i < 4; i++) d[L.off_qh + 4 * b + i] = (uint8_t)(p >> (8 * i));
      const uint8_t* qs = s + (is1 ? 8 : 6);
      for (int i = 0; i < 16; i++) d[L.off_q + 16 * b + i] = qs[i];
      break;
    }
  }
}

// ---------------------------------------------------------------------------
// Exact dequantization from the device layout (WGSL operation order, each
// product/difference rounded separately: no FMA contraction).

__device__ __forceinline__ float ld_f16(const uint8_t* p) {
  return __half2float(__ushort_as_half(*(const unsigned short*)p));
}

// scale_min_k4 (llama-wgsl-runtime.ts:2387-2394) over the 12 packed bytes.
__device__ __forceinline__ void scale_min_k4(const uint8_t* q, int j, uint32_t& sc, uint32_t& m) {
  if (j < 4) {
    sc = q[j] & 63u;
    m = q[j + 4] & 63u;
  } else {
    sc = (q[j + 4] & 15u) | ((q[j - 4] >> 6) << 4);
    m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
  }
}

__device__ inline float dequant_at(const uint8_t* row, const Lay& L, int col) {
  switch (L.type) {
    case GT_Q4_K: {
      int sb = col >> 8, within = col & 255, sub = within >> 5, j = within & 31;
      const uint8_t* hdr = row + L.off_sc + 16 * sb;
      float d = ld_f16(hdr), dmin = ld_f16(hdr + 2);
      uint32_t sc, m;
      scale_min_k4(hdr + 4, sub, sc, m);
      uint32_t byte = row[L.off_q + (8 * sb + sub) * 16 + (j & 15)];
      uint32_t q = j < 16 ? (byte & 15u) : (byte >> 4);
      return __fsub_rn(__fmul_rn(__fmul_rn(d, (float)sc), (float)q), __fmul_rn(dmin, (float)m));
    }
    case GT_Q6_K: {
      int sb = col >> 8, within = col & 255, sub = within >> 5, j = within & 31;
      uint32_t byte = row[L.off_q + (8 * sb + sub) * 16 + (j & 15)];
      uint32_t lo = j < 16 ? (byte & 15u) : (byte >> 4);
      int jj = j & 15, t = jj >> 2, b = jj & 3;
      uint32_t H = *(const uint32_t*)(row + L.off_q2 + (8 * sb + sub) * 8 + 4 * (t & 1));
      int sh = (t >> 1) * 4 + (j < 16 ? 0 : 2);
      uint32_t hi = (H >> (8 * b + sh)) & 3u;
      int q = (int)(lo | (hi << 4)) - 32;
      int sc = (int)(int8_t)row[L.off_sc + 16 * sb + (within >> 4)];
      float d = ld_f16(row + L.off_d + 2 * sb);
      return __fmul_rn(__fmul_rn(d, (float)sc), (float)q);
    }
    case GT_Q8_0: {
      int b = col >> 5, j = col & 31;
      int q = (int)(int8_t)row[L.off_q + 32 * b + j];
      return __fmul_rn((float)q, ld_f16(row + L.off_d + 2 * b));
    }
    case GT_Q5_0:
    case GT_Q5_1: {
      int b = col >> 5, j = col & 31;
      uint32_t byte = row[L.off_q + 16 * b + (j & 15)];
      uint32_t lo = j < 16 ? (byte & 15u) : (byte >> 4);
      uint32_t qh = *(const uint32_t*)(row + L.off_qh + 4 * b);
      int jj = j & 15, t = jj >> 2, bb = jj & 3;
      uint32_t hb = (qh >> (8 * bb + t + (j < 16 ? 0 : 4))) & 1u;
      uint32_t q = lo | (hb << 4);
      float d = ld_f16(row + L.off_d + 2 * b);
      if (L.type == GT_Q5_0) return __fmul_rn(d, (float)((int)q - 16));
      return __fadd_rn(__fmul_rn(d, (float)q), ld_f16(row + L.off_m + 2 * b));
    }
  }
  return 0.f;
}

__global__ void k_dequant(const uint8_t* __restrict__ w, Lay L, int n, float* __restrict__ out) {
  long long gid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (gid >= (long long)n * L.k) return;
  int row = (int)(gid / L.k), col = (int)(gid % L.k);
  out[gid] = dequant_at(w + (size_t)row * L.row_bytes, L, col);
}

// ---------------------------------------------------------------------------
// Integer unit dot products for the matvec.
//
// The activation x is quantized per 32-element group into a 16-bit integer
// X = hi * 256 + lo (hi, lo int8; |X| <= 32639) with a float step sx, so
// sum_i x_i q_i = sx * (256 * dp4a(hi, q) + dp4a(lo, q)) is evaluated exactly
// in int32; the only approximation is x's 16-bit grid (relative 1.5e-5 of the
// group's max), far inside the 1e-3 logits tolerance.  Per unit a lane holds:
struct XUnit {
  int h[8];     // hi bytes of X for the unit's 32 weights, 4 per word, in order
  int l[8];     // lo bytes
  float sx;     // group step
  int sa, sb;   // sum of X over weights 0..15 and 16..31
};

template <bool G>
__device__ __forceinline__ uint4 ld16(const uint8_t* p) { return G ? __ldg((const uint4*)p) : *(const uint4*)p; }
template <bool G>
__device__ __forceinline__ uint2 ld8(const uint8_t* p) { return G ? __ldg((const uint2*)p) : *(const uint2*)p; }
template <bool G>
__device__ __forceinline__ uint32_t ld4(const uint8_t* p) {
  return G ? __ldg((const unsigned int*)p) : *(const unsigned int*)p;
}
template <bool G>
__device__ __forceinline__ uint32_t ld2(const uint8_t* p) {
  return G ? (uint32_t)__ldg((const unsigned short*)p) : (uint32_t) * (const unsigned short*)p;
}

// Normalized unit: every block type decodes to the same form, so the dp4a
// dot product is shared code and only the unpack differs per type.
//   q[0..3]: byte codes of weights 0..15 (4 per word, in order), q[4..7]: 16..31
//   contribution = sx * (a0 * (dlo + ko*sa) + a1 * (dhi + ko*sb) + b * (sa + sb))
// with dlo/dhi the integer dots of X with the codes of each half.
//   Q4_K  a0 = a1 = d*sc, ko = 0, b = -dmin*m      (w = d*sc*q - dmin*m)
//   Q6_K  a0 = d*sc0, a1 = d*sc1, ko = -32, b = 0   (w = d*sc*(q - 32))
//   Q8_0  a0 = a1 = d, ko = 0, b = 0                (w = q*d)
//   Q5_0  a0 = a1 = d, ko = -16, b = 0              (w = d*(q - 16))
//   Q5_1  a0 = a1 = d, ko = 0, b = m                (w = d*q + m)
struct U8 {
  int q[8];
  float a0, a1, b;
  int ko;
};

__device__ __forceinline__ float h2f_u16(uint32_t b) { return __half2float(__ushort_as_half((unsigned short)(b & 0xFFFFu))); }

// Sets of block types as bit masks (bit t = GGML type t).  A kernel compiled
// for a set only decodes the types in it: ck_fold_type maps a type to itself
// when it is in the set and to the set's first type otherwise (the host
// picks such a kernel only for models whose types are all in the set), so
// the compiler keeps only the set's arms of a switch over the result.
#define CK_TM(t) (1u << (t))
#define CK_TM_ALL (CK_TM(GT_Q4_K) | CK_TM(GT_Q6_K) | CK_TM(GT_Q8_0) | CK_TM(GT_Q5_0) | CK_TM(GT_Q5_1))
template <unsigned TM>
__device__ __forceinline__ int ck_fold_type(int type) {
  if (TM == CK_TM_ALL) return type;
  int r = (TM & CK_TM(GT_Q4_K)) ? GT_Q4_K
        : (TM & CK_TM(GT_Q6_K)) ? GT_Q6_K
        : (TM & CK_TM(GT_Q8_0)) ? GT_Q8_0
        : (TM & CK_TM(GT_Q5_0)) ? GT_Q5_0 : GT_Q5_1;
  if ((TM & CK_TM(GT_Q6_K)) && type == GT_Q6_K) r = GT_Q6_K;
  if ((TM & CK_TM(GT_Q8_0)) && type == GT_Q8_0) r = GT_Q8_0;
  if ((TM & CK_TM(GT_Q5_0)) && type == GT_Q5_0) r = GT_Q5_0;
  if ((TM & CK_TM(GT_Q5_1)) && type == GT_Q5_1) r = GT_Q5_1;
  return r;
}

template <bool G, unsigned TM = CK_TM_ALL>
__device__ __forceinline__ void unpack_unit(int type, const uint8_t* row, const Lay& L, int c, U8& u) {
  switch (ck_fold_type<TM>(type)) {  // folds away when `type` is a compile-time constant
    case GT_Q4_K: {
      uint4 w = ld16<G>(row + L.off_q + 16 * c);
      uint4 hd = ld16<G>(row + L.off_sc + 16 * (c >> 3));
      uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int t = 0; t < 4; t++) {
        u.q[t] = (int)(ww[t] & 0x0F0F0F0Fu);
        u.q[4 + t] = (int)((ww[t] >> 4) & 0x0F0F0F0Fu);
      }
      int sub = c & 7;
      uint32_t sc, m;
      // scale_min_k4 (llama-wgsl-runtime.ts:2387-2394): packed bytes q0..3 in
      // header word y, q4..7 in z, q8..11 in w
      if (sub < 4) {
        sc = (hd.y >> (8 * sub)) & 63u;
        m = (hd.z >> (8 * sub)) & 63u;
      } else {
        uint32_t s4 = 8 * (sub - 4);
        uint32_t qj4 = (hd.w >> s4) & 0xFFu, qjm4 = (hd.y >> s4) & 0xFFu, qj = (hd.z >> s4) & 0xFFu;
        sc = (qj4 & 15u) | ((qjm4 >> 6) << 4);
        m = (qj4 >> 4) | ((qj >> 6) << 4);
      }
      float d = h2f_u16(hd.x), dmin = h2f_u16(hd.x >> 16);
      u.a0 = u.a1 = d * (float)sc;
      u.b = -(dmin * (float)m);
      u.ko = 0;
      break;
    }
    case GT_Q6_K: {
      uint4 w = ld16<G>(row + L.off_q + 16 * c);
      uint2 h = ld8<G>(row + L.off_q2 + 8 * c);
      int sb = c >> 3, sub = c & 7;
      uint32_t dd = ld2<G>(row + L.off_d + 2 * sb), scp = ld2<G>(row + L.off_sc + 16 * sb + 2 * sub);
      uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int t = 0; t < 4; t++) {
        uint32_t H = (t & 1) ? h.y : h.x;
        int sh = (t >> 1) * 4;
        u.q[t] = (int)((ww[t] & 0x0F0F0F0Fu) | (((H >> sh) << 4) & 0x30303030u));
        u.q[4 + t] = (int)(((ww[t] >> 4) & 0x0F0F0F0Fu) | (((H >> (sh + 2)) << 4) & 0x30303030u));
      }
      float d = h2f_u16(dd);
      u.a0 = d * (float)(int)(int8_t)(scp & 0xFFu);
      u.a1 = d * (float)(int)(int8_t)(scp >> 8);
      u.b = 0.f;
      u.ko = -32;
      break;
    }
    case GT_Q8_0: {
      uint4 w0 = ld16<G>(row + L.off_q + 32 * c), w1 = ld16<G>(row + L.off_q + 32 * c + 16);
      u.q[0] = (int)w0.x; u.q[1] = (int)w0.y; u.q[2] = (int)w0.z; u.q[3] = (int)w0.w;
      u.q[4] = (int)w1.x; u.q[5] = (int)w1.y; u.q[6] = (int)w1.z; u.q[7] = (int)w1.w;
      u.a0 = u.a1 = h2f_u16(ld2<G>(row + L.off_d + 2 * c));
      u.b = 0.f;
      u.ko = 0;
      break;
    }
    default: {  // Q5_0, Q5_1
      uint4 w = ld16<G>(row + L.off_q + 16 * c);
      uint32_t qh = ld4<G>(row + L.off_qh + 4 * c);
      uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int t = 0; t < 4; t++) {
        u.q[t] = (int)((ww[t] & 0x0F0F0F0Fu) | ((qh << (4 - t)) & 0x10101010u));
        u.q[4 + t] = (int)(((ww[t] >> 4) & 0x0F0F0F0Fu) | ((qh >> t) & 0x10101010u));
      }
      float d = h2f_u16(ld2<G>(row + L.off_d + 2 * c));
      u.a0 = u.a1 = d;
      if (type == GT_Q5_1) {
        u.b = h2f_u16(ld2<G>(row + L.off_m + 2 * c));
        u.ko = 0;
      } else {
        u.b = 0.f;
        u.ko = -16;
      }
      break;
    }
  }
}

__device__ __forceinline__ float unit_dot8(const U8& u, const XUnit& x) {
  int hl = 0, ll = 0, hh = 0, lh = 0;
#pragma unroll
  for (int t = 0; t < 4; t++) {
    hl = __dp4a(u.q[t], x.h[t], hl);
    ll = __dp4a(u.q[t], x.l[t], ll);
    hh = __dp4a(u.q[4 + t], x.h[4 + t], hh);
    lh = __dp4a(u.q[4 + t], x.l[4 + t], lh);
  }
  int dlo = hl * 256 + ll + u.ko * x.sa;
  int dhi = hh * 256 + lh + u.ko * x.sb;
  return x.sx * (u.a0 * (float)dlo + u.a1 * (float)dhi + u.b * (float)(x.sa + x.sb));
}
