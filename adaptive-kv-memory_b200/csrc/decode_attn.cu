// Mixed-tier decode attention: FP16 hot window + packed warm block records.
//
// softmax(q . [K_warm; K_hot]^T * sm_scale) . [V_warm; V_hot] for one query
// token per (batch row, query head), GQA-batched: one CTA owns one
// (batch row, KV head, <= 8 query heads) and a contiguous range of 32-token
// blocks (split-K over the sequence); an LSE combine merges the splits.
//
// Warm CTAs: one producer warp streams whole block records HBM -> SMEM with
// 1-D bulk TMA (cp.async.bulk + mbarrier ring); consumer warps each take whole
// blocks and dequantise them in registers exactly like the reference
// (akv/affine_quantizer.py:112-124, :178-189: fp16(fp16(code*scale) + zero),
// outlier channels replaced by their fp16 originals), so the contraction sees
// the same fp16 K/V values the reference attends over.  Packed codes become
// fp16 with the "1024 + code" magic (one LOP3 per pair); one HFMA2 then gives
// fp16(code*scale) with a single rounding and one HADD2 adds the zero point.
// The contraction runs on mma.sync m16n8k16 (f16 in, f32 accumulate): tokens
// are M for q.K^T, head_dim is M for P.V, and the (<= 8) query heads of the KV
// head are N.  movmatrix transposes P between the two; P enters the second MMA
// as an fp16 hi + lo pair so the probabilities keep ~22 bits.
//
// Hot CTAs read the FP16 window with 128-bit loads and use the same MMA
// layout with natural channel order.
#include <cuda_runtime.h>

#include <algorithm>

#include "common.cuh"

namespace akv {

constexpr int kHeadDim = 128;
constexpr int kConsumerWarps = 4;
constexpr int kDecodeThreads = (kConsumerWarps + 1) * 32;
constexpr int kStages = 8;
constexpr int kMaxDecodeOutliers = 8;
constexpr float kLog2e = 1.4426950408889634f;

struct DecodeParams {
  const __half* q;
  int64_t q_sb, q_sh;
  const __half* hk;
  const __half* hv;
  int64_t h_sb, h_sh, h_sn;
  int n_hot;
  const int32_t* hot_len;
  const uint8_t* warm;
  int64_t w_sb, w_sh;
  akv_warm_layout L;
  int n_warm_blocks;
  const int32_t* warm_len;
  int B, Hq, Hkv, g, n_hg;
  float scale_log2;
  int warm_splits, hot_splits, wbps, hbps, splits;
  float* ws;  // split partials: row (b*Hq + hq)*splits + split holds (acc[D], m, l)
  int* status;
};

// ------------------------------------------------------------------ exact fp16 dequantisation
// x holds (1024 + M*c_a, 1024 + M*c_b) as fp16 (the LOP3 magic).  Fast form:
// fp16(c*s) = fma(x, s/M, -1024*s/M) with one rounding, exact when s/M and
// 1024*s/M are representable; then + zero.  Safe form for any scale:
// c = fma(x, 1/M, -1024/M) (exact), fp16(c*s), + zero.
AKV_DEV bool scale_is_fast(float s) { return s == 0.f || (s >= 0.015625f && s <= 63.9f); }

template <int M>
AKV_DEV uint32_t dq_fast(uint32_t x, __half2 s_over_m, __half2 neg1024s_over_m, __half2 z) {
  return h2_as_u32(__hadd2_rn(__hfma2(u32_as_h2(x), s_over_m, neg1024s_over_m), z));
}

template <int M>
AKV_DEV uint32_t dq_safe(uint32_t x, __half2 s, __half2 z) {
  return h2_as_u32(__hadd2_rn(__hmul2_rn(u32_as_h2(fix_magic<M>(x)), s), z));
}

template <int M>
AKV_DEV __half2 over_m(__half2 s) { return __hmul2(s, __float2half2_rn(1.0f / M)); }
template <int M>
AKV_DEV __half2 neg1024_over_m(__half2 s) { return __hmul2(s, __float2half2_rn(-1024.0f / M)); }

// ------------------------------------------------------------------ K codes -> A fragments
// Thread (g8, q4) holds, for one token row, the 32 codes of channel chunk q4
// as 16 half2 "pairs"; pair i feeds k-step i/2, low (i even) or high k slots.
// The channel order inside a chunk is permuted per bit width (kPairs*), with
// the magic multiplier of each pair in kMult*; the query fragment uses the
// same permutation.
struct PairIdx {
  int a, b;
};

__device__ constexpr PairIdx kPairs4[16] = {{1, 5},   {0, 4},   {3, 7},   {2, 6},   {9, 13},  {8, 12},
                                            {11, 15}, {10, 14}, {17, 21}, {16, 20}, {19, 23}, {18, 22},
                                            {25, 29}, {24, 28}, {27, 31}, {26, 30}};
__device__ constexpr PairIdx kPairs2[16] = {{3, 11},  {2, 10},  {1, 9},   {0, 8},   {7, 15},  {6, 14},
                                            {5, 13},  {4, 12},  {19, 27}, {18, 26}, {17, 25}, {16, 24},
                                            {23, 31}, {22, 30}, {21, 29}, {20, 28}};
__device__ constexpr PairIdx kPairs3[16] = {{7, 15},  {6, 14},  {5, 13},  {4, 12},  {3, 11},  {2, 10},
                                            {1, 9},   {0, 8},   {23, 31}, {22, 30}, {21, 29}, {20, 28},
                                            {19, 27}, {18, 26}, {17, 25}, {16, 24}};
__device__ constexpr int kMult4[16] = {1, 16, 1, 16, 1, 16, 1, 16, 1, 16, 1, 16, 1, 16, 1, 16};
__device__ constexpr int kMult2[16] = {1, 4, 16, 64, 256, 4, 16, 64, 1, 4, 16, 64, 256, 4, 16, 64};
__device__ constexpr int kMult3[16] = {1, 8, 64, 1, 8, 1, 8, 64, 1, 8, 64, 1, 8, 1, 8, 64};

// Lookups used only with compile-time indices (template recursion below), so
// every pair permutation and magic multiplier is a constant in the code.
template <int KB>
AKV_DEV constexpr PairIdx kpair(int i) {
  return KB == 4 ? kPairs4[i] : (KB == 2 ? kPairs2[i] : kPairs3[i]);
}
template <int BITS>
AKV_DEV constexpr int kmult(int i) {
  return BITS == 4 ? kMult4[i] : (BITS == 2 ? kMult2[i] : kMult3[i]);
}

// 3-bit: two big-endian 24-bit groups (low 24 bits of wa, wb) -> 8 magic pairs
// ordered c7, c6, c5, c4, c3, c2, c1, c0 (pair = (code of wa, code of wb)),
// multipliers 1, 8, 64, 1, 8, 1, 8, 64.
AKV_DEV void raw3_pair(uint32_t wa, uint32_t wb, uint32_t* e) {
  const uint32_t y = prmt(wa, wb, 0x5410);
  e[0] = lop_magic<0x00070007u>(y);
  e[1] = lop_magic<0x00380038u>(y);
  e[2] = lop_magic<0x01C001C0u>(y);
  const uint32_t y9 = y >> 9;
  e[3] = lop_magic<0x00070007u>(y9);
  e[4] = lop_magic<0x00380038u>(y9);
  const uint32_t z = prmt(wa >> 15, wb >> 15, 0x5410);
  e[5] = lop_magic<0x00070007u>(z);
  e[6] = lop_magic<0x00380038u>(z);
  e[7] = lop_magic<0x01C001C0u>(z);
}

template <int KB>
AKV_DEV void k_row_raw(const uint8_t* row, int q4, uint32_t (&e)[16]) {
  if constexpr (KB == 4) {
    const uint4 w = lds_v4(row + 16 * q4);
    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const uint32_t x = ws[k], y = ws[k] >> 8;
      e[4 * k + 0] = lop_magic<0x000F000Fu>(x);
      e[4 * k + 1] = lop_magic<0x00F000F0u>(x);
      e[4 * k + 2] = lop_magic<0x000F000Fu>(y);
      e[4 * k + 3] = lop_magic<0x00F000F0u>(y);
    }
  } else if constexpr (KB == 2) {
    const uint2 w = lds_v2(row + 8 * q4);
    const uint32_t ws[2] = {w.x, w.y};
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const uint32_t x = ws[k], y = ws[k] >> 8;
      e[8 * k + 0] = lop_magic<0x00030003u>(x);
      e[8 * k + 1] = lop_magic<0x000C000Cu>(x);
      e[8 * k + 2] = lop_magic<0x00300030u>(x);
      e[8 * k + 3] = lop_magic<0x00C000C0u>(x);
      e[8 * k + 4] = lop_magic<0x03000300u>(x);
      e[8 * k + 5] = lop_magic<0x000C000Cu>(y);
      e[8 * k + 6] = lop_magic<0x00300030u>(y);
      e[8 * k + 7] = lop_magic<0x00C000C0u>(y);
    }
  } else {
    const uint8_t* p = row + 12 * q4;
    const uint32_t w0 = lds_u32(p), w1 = lds_u32(p + 4), w2 = lds_u32(p + 8);
    const uint32_t g0 = prmt(w0, 0u, 0x4012), g1 = prmt(w0, w1, 0x3345);
    const uint32_t g2 = prmt(w1, w2, 0x2234), g3 = prmt(w2, 0u, 0x4123);
    raw3_pair(g0, g1, e);
    raw3_pair(g2, g3, e + 8);
  }
}

// Per-block channel constants of this thread's K chunk, in pair order.
template <int KB>
struct KConst {
  __half2 a[16];  // fast: s/M      safe: s
  __half2 c[16];  // fast: -1024s/M
  __half2 z[16];
  bool fast;
};

template <int KB, int I = 0>
AKV_DEV void k_consts_fill(const __half (&s)[32], const __half (&z)[32], KConst<KB>& kc) {
  if constexpr (I < 16) {
    constexpr PairIdx pi = kpair<KB>(I);
    constexpr int M = kmult<KB>(I);
    const __half2 s2 = __halves2half2(s[pi.a], s[pi.b]);
    kc.z[I] = __halves2half2(z[pi.a], z[pi.b]);
    kc.a[I] = kc.fast ? over_m<M>(s2) : s2;
    kc.c[I] = neg1024_over_m<M>(s2);
    k_consts_fill<KB, I + 1>(s, z, kc);
  }
}

template <int KB>
AKV_DEV void k_consts(const __half* ks, const __half* kz, KConst<KB>& kc) {
  __half s[32], z[32];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    *reinterpret_cast<uint4*>(s + 8 * k) = lds_v4(ks + 8 * k);
    *reinterpret_cast<uint4*>(z + 8 * k) = lds_v4(kz + 8 * k);
  }
  bool fast = true;
#pragma unroll
  for (int k = 0; k < 32; ++k) fast &= scale_is_fast(__half2float(s[k]));
  kc.fast = fast;
  k_consts_fill<KB>(s, z, kc);
}

template <int KB, int I = 0>
AKV_DEV void q_pairs(const __half (&qv)[32], uint32_t (&qp)[16]) {
  if constexpr (I < 16) {
    constexpr PairIdx pi = kpair<KB>(I);
    qp[I] = h2_as_u32(__halves2half2(qv[pi.a], qv[pi.b]));
    q_pairs<KB, I + 1>(qv, qp);
  }
}

template <int BITS, int I>
AKV_DEV uint32_t dq_pair(uint32_t x, __half2 a, __half2 c, __half2 z, bool fast) {
  constexpr int M = kmult<BITS>(I);
  return fast ? dq_fast<M>(x, a, c, z) : dq_safe<M>(x, a, z);
}

template <int KB, int I = 0>
AKV_DEV void k_dequant(uint32_t (&e)[16], const KConst<KB>& kc) {
  if constexpr (I < 16) {
    e[I] = dq_pair<KB, I>(e[I], kc.a[I], kc.c[I], kc.z[I], kc.fast);
    k_dequant<KB, I + 1>(e, kc);
  }
}

// ------------------------------------------------------------------ V codes -> A fragments
// Thread group g8 owns channels [16*g8, 16*g8+16).  For a token pair (ta, tb)
// produce e[ci] = (v_ta[ci], v_tb[ci]) dequantised, ci = 0..15.
template <int VB>
struct VRow {
  uint32_t w[VB == 2 ? 1 : 2];
};

template <int VB>
AKV_DEV VRow<VB> v_row_load(const uint8_t* row, int g8) {
  VRow<VB> r;
  if constexpr (VB == 4) {
    const uint2 w = lds_v2(row + 8 * g8);
    r.w[0] = w.x;
    r.w[1] = w.y;
  } else if constexpr (VB == 2) {
    r.w[0] = lds_u32(row + 4 * g8);
  } else {
    const int base = 6 * g8;
    const uint8_t* p = row + (base & ~3);
    const uint32_t lo = lds_u32(p), hi = lds_u32(p + 4);
    const int sh = (base & 3) * 8;
    const uint32_t v0 = __funnelshift_r(lo, hi, sh), v1 = __funnelshift_r(hi, 0u, sh);
    r.w[0] = prmt(v0, 0u, 0x4012);  // group 0, big-endian 24-bit
    r.w[1] = prmt(v0, v1, 0x3345);  // group 1
  }
  return r;
}

// raw magic pairs by channel index ci, plus each one's multiplier (compile time)
template <int VB>
constexpr int vmult(int ci) {
  if (VB == 4) return (ci & 1) ? 1 : 16;
  if (VB == 2) {
    constexpr int m[8] = {64, 16, 4, 1, 64, 16, 4, 256};
    return m[ci & 7];
  }
  constexpr int m3[8] = {64, 8, 1, 8, 1, 64, 8, 1};  // ci -> multiplier of code ci in raw3_pair order
  return m3[ci & 7];
}

template <int VB>
AKV_DEV void v_pair_raw(const VRow<VB>& a, const VRow<VB>& b, uint32_t (&e)[16]) {
  if constexpr (VB == 4) {
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const uint32_t x = prmt(a.w[k], b.w[k], 0x5410), y = prmt(a.w[k], b.w[k], 0x7632);
      const uint32_t x8 = x >> 8, y8 = y >> 8;
      e[8 * k + 1] = lop_magic<0x000F000Fu>(x);
      e[8 * k + 0] = lop_magic<0x00F000F0u>(x);
      e[8 * k + 3] = lop_magic<0x000F000Fu>(x8);
      e[8 * k + 2] = lop_magic<0x00F000F0u>(x8);
      e[8 * k + 5] = lop_magic<0x000F000Fu>(y);
      e[8 * k + 4] = lop_magic<0x00F000F0u>(y);
      e[8 * k + 7] = lop_magic<0x000F000Fu>(y8);
      e[8 * k + 6] = lop_magic<0x00F000F0u>(y8);
    }
  } else if constexpr (VB == 2) {
    const uint32_t xs[2] = {prmt(a.w[0], b.w[0], 0x5410), prmt(a.w[0], b.w[0], 0x7632)};
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const uint32_t x = xs[k], x8 = xs[k] >> 8;
      e[8 * k + 3] = lop_magic<0x00030003u>(x);
      e[8 * k + 2] = lop_magic<0x000C000Cu>(x);
      e[8 * k + 1] = lop_magic<0x00300030u>(x);
      e[8 * k + 0] = lop_magic<0x00C000C0u>(x);
      e[8 * k + 7] = lop_magic<0x03000300u>(x);
      e[8 * k + 6] = lop_magic<0x000C000Cu>(x8);
      e[8 * k + 5] = lop_magic<0x00300030u>(x8);
      e[8 * k + 4] = lop_magic<0x00C000C0u>(x8);
    }
  } else {
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      uint32_t t[8];
      raw3_pair(a.w[k], b.w[k], t);
#pragma unroll
      for (int j = 0; j < 8; ++j) e[8 * k + 7 - j] = t[j];
    }
  }
}

template <int VB, int CI = 0>
AKV_DEV void v_dequant(uint32_t (&e)[16], __half2 s2, __half2 z2, bool fast) {
  if constexpr (CI < 16) {
    constexpr int M = vmult<VB>(CI);
    e[CI] = fast ? dq_fast<M>(e[CI], over_m<M>(s2), neg1024_over_m<M>(s2), z2) : dq_safe<M>(e[CI], s2, z2);
    v_dequant<VB, CI + 1>(e, s2, z2, fast);
  }
}

// code of channel d in a packed row (akv/bitpack.py layout)
template <int BITS>
AKV_DEV uint32_t code_at(const uint8_t* row, int d) {
  if constexpr (BITS == 4) {
    const uint32_t byte = row[d >> 1];
    return (d & 1) ? (byte & 15u) : (byte >> 4);
  } else if constexpr (BITS == 2) {
    return (row[d >> 2] >> (6 - 2 * (d & 3))) & 3u;
  } else {
    const uint8_t* p = row + 3 * (d >> 3);
    const uint32_t word = (static_cast<uint32_t>(p[0]) << 16) | (p[1] << 8) | p[2];
    return (word >> (21 - 3 * (d & 7))) & 7u;
  }
}

// ------------------------------------------------------------------ shared softmax/PV state
struct WarpState {
  float acc[8][4];  // O^T: tile mt rows (g8 -> d=16*g8+2mt, g8+8 -> d+1), cols heads (2q4, 2q4+1)
  float m[2];       // running max (log2 units) for heads 2q4, 2q4+1
  float l[2];       // partial row sums (this thread's tokens only)
};

AKV_DEV void state_init(WarpState& s) {
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) s.acc[i][j] = 0.f;
  s.m[0] = s.m[1] = -INFINITY;
  s.l[0] = s.l[1] = 0.f;
}

// x[mt][4]: scaled logits (log2 units, -inf = masked) of this thread's 4
// tokens x 2 heads.  Rescales the state and turns x into probabilities.
AKV_DEV void online_softmax(WarpState& s, float (&x)[2][4]) {
  float mx[2];
  mx[0] = fmaxf(fmaxf(x[0][0], x[0][2]), fmaxf(x[1][0], x[1][2]));
  mx[1] = fmaxf(fmaxf(x[0][1], x[0][3]), fmaxf(x[1][1], x[1][3]));
#pragma unroll
  for (int o = 4; o < 32; o <<= 1) {
    mx[0] = fmaxf(mx[0], __shfl_xor_sync(0xffffffffu, mx[0], o));
    mx[1] = fmaxf(mx[1], __shfl_xor_sync(0xffffffffu, mx[1], o));
  }
  float alpha[2], base[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const float mn = fmaxf(s.m[h], mx[h]);
    base[h] = (mn == -INFINITY) ? 0.f : mn;
    alpha[h] = fast_exp2(s.m[h] - base[h]);
    s.m[h] = mn;
    s.l[h] *= alpha[h];
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    s.acc[i][0] *= alpha[0];
    s.acc[i][1] *= alpha[1];
    s.acc[i][2] *= alpha[0];
    s.acc[i][3] *= alpha[1];
  }
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      x[mt][j] = fast_exp2(x[mt][j] - base[j & 1]);
      s.l[j & 1] += x[mt][j];
    }
}

// P (fp32, S^T C-fragment layout) -> B fragments of the PV MMA as fp16 hi + lo.
AKV_DEV void p_fragments(const float (&x)[2][4], uint32_t (&ph)[2][2], uint32_t (&pl)[2][2]) {
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const __half2 hi = __floats2half2_rn(x[mt][2 * r], x[mt][2 * r + 1]);
      const float2 hf = __half22float2(hi);
      const __half2 lo = __floats2half2_rn(x[mt][2 * r] - hf.x, x[mt][2 * r + 1] - hf.y);
      ph[mt][r] = movmatrix_trans(h2_as_u32(hi));
      pl[mt][r] = movmatrix_trans(h2_as_u32(lo));
    }
}

// ------------------------------------------------------------------ epilogue
// Reduce the per-thread partials of one warp and park them in shared memory:
// red[h][d] (fp32, natural channel order), rm[h], rl[h].
AKV_DEV void warp_to_smem(WarpState& s, int lane, float* red, float* rm, float* rl) {
  const int g8 = lane >> 2, q4 = lane & 3;
#pragma unroll
  for (int h = 0; h < 2; ++h)
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) s.l[h] += __shfl_xor_sync(0xffffffffu, s.l[h], o);
#pragma unroll
  for (int mt = 0; mt < 8; ++mt) {
    const int d = 16 * g8 + 2 * mt;
    red[(2 * q4) * kHeadDim + d] = s.acc[mt][0];
    red[(2 * q4 + 1) * kHeadDim + d] = s.acc[mt][1];
    red[(2 * q4) * kHeadDim + d + 1] = s.acc[mt][2];
    red[(2 * q4 + 1) * kHeadDim + d + 1] = s.acc[mt][3];
  }
  if (g8 == 0) {
    rm[2 * q4] = s.m[0];
    rm[2 * q4 + 1] = s.m[1];
    rl[2 * q4] = s.l[0];
    rl[2 * q4 + 1] = s.l[1];
  }
}

// Merge the consumer warps' partials and write this CTA's split partial.
AKV_DEV void cta_write_partial(const DecodeParams& p, float* red, float* rm, float* rl, int b, int kvh, int hg,
                               int split) {
  const int nh = min(8, p.g - hg * 8);
  for (int i = threadIdx.x; i < nh * kHeadDim; i += blockDim.x) {
    const int h = i / kHeadDim, d = i % kHeadDim;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) M = fmaxf(M, rm[w * 8 + h]);
    const float base = (M == -INFINITY) ? 0.f : M;
    float acc = 0.f, L = 0.f;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) {
      const float f = fast_exp2(rm[w * 8 + h] - base);
      acc += f * red[(w * 8 + h) * kHeadDim + d];
      L += f * rl[w * 8 + h];
    }
    const int hq = kvh * p.g + hg * 8 + h;
    float* part = p.ws + ((static_cast<int64_t>(b) * p.Hq + hq) * p.splits + split) * (kHeadDim + 2);
    part[d] = acc;
    if (d == 0) {
      part[kHeadDim] = M;
      part[kHeadDim + 1] = L;
    }
  }
}

// ------------------------------------------------------------------ the kernel
template <int KB, int VB>
__global__ void __launch_bounds__(kDecodeThreads) mixed_decode_kernel(const DecodeParams p) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g8 = lane >> 2, q4 = lane & 3;
  const int split = blockIdx.x;
  const int kvh = blockIdx.y / p.n_hg, hg = blockIdx.y % p.n_hg;
  const int b = blockIdx.z;
  const bool warm_cta = split < p.warm_splits;

  // shared memory map
  const int rec = p.L.bytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + kStages;
  float* qs = reinterpret_cast<float*>(smem + 256);               // [8][128] query (fp32) for outliers
  unsigned char* stage0 = smem + 256 + 8 * kHeadDim * 4;          // [kStages][rec]
  // epilogue buffers alias the stages once the main loop is over
  float* red = reinterpret_cast<float*>(stage0);                  // [warps][8][128]
  float* rm = red + kConsumerWarps * 8 * kHeadDim;                // [warps][8]
  float* rl = rm + kConsumerWarps * 8;

  const int nh = min(8, p.g - hg * 8);
  const int qh_base = kvh * p.g + hg * 8;

  // this thread's query column (head g8 of the head group; zero padding beyond nh)
  __half qv[32];
  {
    const bool have = g8 < nh;
    const __half* qrow = p.q + b * p.q_sb + (qh_base + (have ? g8 : 0)) * p.q_sh + 32 * q4;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      uint4 v = have ? ldg_nc_v4(qrow + 8 * k) : make_uint4(0, 0, 0, 0);
      *reinterpret_cast<uint4*>(qv + 8 * k) = v;
    }
  }
  for (int i = threadIdx.x; i < 8 * kHeadDim; i += blockDim.x) {
    const int h = i / kHeadDim, d = i % kHeadDim;
    qs[i] = h < nh ? __half2float(p.q[b * p.q_sb + (qh_base + h) * p.q_sh + d]) : 0.f;
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    fence_mbar_init();
  }
  __syncthreads();

  WarpState st;
  state_init(st);

  if (warm_cta) {
    const int nblk_b = p.warm_len ? min(p.warm_len[b], p.n_warm_blocks) : p.n_warm_blocks;
    const int blo = split * p.wbps;
    const int bhi = min(nblk_b, blo + p.wbps);
    const int nb = max(0, bhi - blo);
    const uint8_t* wbase = p.warm + b * p.w_sb + kvh * p.w_sh + static_cast<int64_t>(blo) * rec;

    if (warp == kConsumerWarps) {
      // ---------------- producer: one lane streams records into the ring
      if (lane == 0) {
        int issued = 0;
        for (int i = 0; i < nb; ++i) {
          const int s = i % kStages;
          if (i >= kStages && !mbar_wait(&empty[s], ((i / kStages) - 1) & 1, p.status)) break;
          mbar_arrive_expect_tx(&full[s], rec);
          tma_load_1d(stage0 + s * rec, wbase + static_cast<int64_t>(i) * rec, rec, &full[s]);
          issued = i + 1;
        }
        // drain: every issued copy has landed before the ring memory is reused
        for (int i = max(0, issued - kStages); i < issued; ++i)
          mbar_wait(&full[i % kStages], (i / kStages) & 1, p.status);
      }
    } else {
      // ---------------- consumers
      uint32_t qp[16];
      q_pairs<KB>(qv, qp);
      const int n_out = p.L.n_outlier;
      const int kp = kHeadDim * KB / 8, vp = kHeadDim * VB / 8;

      for (int i = warp; i < nb; i += kConsumerWarps) {
        const int s = i % kStages;
        if (!mbar_wait(&full[s], (i / kStages) & 1, p.status)) break;
        const uint8_t* r = stage0 + s * rec;
        const uint8_t* kc = r + p.L.kc;
        const uint8_t* vc = r + p.L.vc;
        const __half* vsc = reinterpret_cast<const __half*>(r + p.L.vs);
        const __half* vzr = reinterpret_cast<const __half*>(r + p.L.vz);
        const uint32_t mask = lds_u32(r + p.L.mask);

        KConst<KB> kcst;
        k_consts<KB>(reinterpret_cast<const __half*>(r + p.L.ks) + 32 * q4,
                     reinterpret_cast<const __half*>(r + p.L.kz) + 32 * q4, kcst);

        // ---- S^T = K^ q  (tokens x heads), 2 m-tiles of 16 tokens
        float x[2][4];
#pragma unroll
        for (int mt = 0; mt < 2; ++mt) {
          uint32_t e0[16], e1[16];
          k_row_raw<KB>(kc + (16 * mt + g8) * kp, q4, e0);
          k_row_raw<KB>(kc + (16 * mt + g8 + 8) * kp, q4, e1);
          k_dequant<KB>(e0, kcst);
          k_dequant<KB>(e1, kcst);
          float c[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int ks = 0; ks < 8; ++ks)
            mma_16816(c, e0[2 * ks], e1[2 * ks], e0[2 * ks + 1], e1[2 * ks + 1], qp[2 * ks], qp[2 * ks + 1]);
#pragma unroll
          for (int j = 0; j < 4; ++j) x[mt][j] = c[j];
        }
        // K outlier channels: the dequantised value there is 0 (scale = zero = 0);
        // the reference overwrites it with the fp16 original.
        for (int j = 0; j < n_out; ++j) {
          const int d_o = reinterpret_cast<const int16_t*>(r + p.L.ki)[j];
          const float qa = qs[(2 * q4) * kHeadDim + d_o], qb = qs[(2 * q4 + 1) * kHeadDim + d_o];
          const __half* od = reinterpret_cast<const __half*>(r + p.L.ko);
#pragma unroll
          for (int mt = 0; mt < 2; ++mt)
#pragma unroll
            for (int rr = 0; rr < 2; ++rr) {
              const float o = __half2float(od[(16 * mt + 8 * rr + g8) * n_out + j]);
              x[mt][2 * rr] = fmaf(qa, o, x[mt][2 * rr]);
              x[mt][2 * rr + 1] = fmaf(qb, o, x[mt][2 * rr + 1]);
            }
        }
        bool valid[2][2];
#pragma unroll
        for (int mt = 0; mt < 2; ++mt)
#pragma unroll
          for (int rr = 0; rr < 2; ++rr) {
            valid[mt][rr] = (mask >> (16 * mt + 8 * rr + g8)) & 1u;
#pragma unroll
            for (int h = 0; h < 2; ++h)
              x[mt][2 * rr + h] = valid[mt][rr] ? x[mt][2 * rr + h] * p.scale_log2 : -INFINITY;
          }
        online_softmax(st, x);
        uint32_t ph[2][2], pl[2][2];
        p_fragments(x, ph, pl);

        // ---- O^T += V^ P  (head_dim x heads), k-steps of 16 tokens
#pragma unroll
        for (int ks = 0; ks < 2; ++ks) {
          const int ta = 16 * ks + 2 * q4;
          uint32_t e0[16], e1[16];
          {
            const VRow<VB> ra = v_row_load<VB>(vc + ta * vp, g8);
            const VRow<VB> rb = v_row_load<VB>(vc + (ta + 1) * vp, g8);
            v_pair_raw<VB>(ra, rb, e0);
            const __half2 s2 = __halves2half2(vsc[ta], vsc[ta + 1]);
            const __half2 z2 = __halves2half2(vzr[ta], vzr[ta + 1]);
            const bool fast = scale_is_fast(__low2float(s2)) && scale_is_fast(__high2float(s2));
            v_dequant<VB>(e0, s2, z2, fast);
          }
          {
            const VRow<VB> rc = v_row_load<VB>(vc + (ta + 8) * vp, g8);
            const VRow<VB> rd = v_row_load<VB>(vc + (ta + 9) * vp, g8);
            v_pair_raw<VB>(rc, rd, e1);
            const __half2 s2 = __halves2half2(vsc[ta + 8], vsc[ta + 9]);
            const __half2 z2 = __halves2half2(vzr[ta + 8], vzr[ta + 9]);
            const bool fast = scale_is_fast(__low2float(s2)) && scale_is_fast(__high2float(s2));
            v_dequant<VB>(e1, s2, z2, fast);
          }
#pragma unroll
          for (int mt = 0; mt < 8; ++mt) {
            mma_16816(st.acc[mt], e0[2 * mt], e0[2 * mt + 1], e1[2 * mt], e1[2 * mt + 1], ph[ks][0], ph[ks][1]);
            mma_16816(st.acc[mt], e0[2 * mt], e0[2 * mt + 1], e1[2 * mt], e1[2 * mt + 1], pl[ks][0], pl[ks][1]);
          }
        }

        // ---- V outlier channels: replace the dequantised code value by the fp16 original
        for (int j = 0; j < n_out; ++j) {
          const int d_o = reinterpret_cast<const int16_t*>(r + p.L.vi)[j];
          const __half* od = reinterpret_cast<const __half*>(r + p.L.vo);
          float corr[2] = {0.f, 0.f};
#pragma unroll
          for (int mt = 0; mt < 2; ++mt)
#pragma unroll
            for (int rr = 0; rr < 2; ++rr) {
              if (!valid[mt][rr]) continue;
              const int t = 16 * mt + 8 * rr + g8;
              const __half cv = __uint2half_rn(code_at<VB>(vc + t * vp, d_o));
              const float deq = __half2float(__hadd_rn(__hmul_rn(cv, vsc[t]), vzr[t]));
              const float diff = __half2float(od[t * n_out + j]) - deq;
#pragma unroll
              for (int h = 0; h < 2; ++h) corr[h] = fmaf(x[mt][2 * rr + h], diff, corr[h]);
            }
#pragma unroll
          for (int o = 4; o < 32; o <<= 1) {
            corr[0] += __shfl_xor_sync(0xffffffffu, corr[0], o);
            corr[1] += __shfl_xor_sync(0xffffffffu, corr[1], o);
          }
          if ((d_o >> 4) == g8) {
            const int ci = d_o & 15;
#pragma unroll
            for (int mt = 0; mt < 8; ++mt)
#pragma unroll
              for (int hf = 0; hf < 2; ++hf)
                if (ci == 2 * mt + hf) {
                  st.acc[mt][2 * hf] += corr[0];
                  st.acc[mt][2 * hf + 1] += corr[1];
                }
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
      }
    }
  } else {
    // ---------------- hot CTA: FP16 window, 128-bit loads, all warps consume (producer warp too)
    const int hs = split - p.warm_splits;
    const int nhot_b = p.hot_len ? min(p.hot_len[b], p.n_hot) : p.n_hot;
    const int nhb = (nhot_b + 31) / 32;
    const int blo = hs * p.hbps;
    const int bhi = min(nhb, blo + p.hbps);
    if (warp < kConsumerWarps) {
      uint32_t qn[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) qn[i] = h2_as_u32(__halves2half2(qv[2 * i], qv[2 * i + 1]));
      const __half* kb = p.hk + b * p.h_sb + kvh * p.h_sh;
      const __half* vb = p.hv + b * p.h_sb + kvh * p.h_sh;
      for (int blk = blo + warp; blk < bhi; blk += kConsumerWarps) {
        const int t0 = blk * 32;
        float x[2][4];
        bool valid[2][2];
#pragma unroll
        for (int mt = 0; mt < 2; ++mt) {
          uint32_t e0[16], e1[16];
#pragma unroll
          for (int rr = 0; rr < 2; ++rr) {
            const int t = t0 + 16 * mt + 8 * rr + g8;
            valid[mt][rr] = t < nhot_b;
            uint32_t* e = rr ? e1 : e0;
            const __half* row = kb + static_cast<int64_t>(valid[mt][rr] ? t : 0) * p.h_sn + 32 * q4;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const uint4 v = valid[mt][rr] ? ldg_nc_v4(row + 8 * k) : make_uint4(0, 0, 0, 0);
              e[4 * k + 0] = v.x;
              e[4 * k + 1] = v.y;
              e[4 * k + 2] = v.z;
              e[4 * k + 3] = v.w;
            }
          }
          float c[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int ks = 0; ks < 8; ++ks)
            mma_16816(c, e0[2 * ks], e1[2 * ks], e0[2 * ks + 1], e1[2 * ks + 1], qn[2 * ks], qn[2 * ks + 1]);
#pragma unroll
          for (int j = 0; j < 4; ++j) x[mt][j] = valid[mt][j >> 1] ? c[j] * p.scale_log2 : -INFINITY;
        }
        online_softmax(st, x);
        uint32_t ph[2][2], pl[2][2];
        p_fragments(x, ph, pl);
#pragma unroll
        for (int ks = 0; ks < 2; ++ks) {
          uint32_t va[4][8];
#pragma unroll
          for (int tt = 0; tt < 4; ++tt) {
            const int t = t0 + 16 * ks + 2 * q4 + (tt & 1) + 8 * (tt >> 1);
            const bool ok = t < nhot_b;
            const __half* row = vb + static_cast<int64_t>(ok ? t : 0) * p.h_sn + 16 * g8;
            const uint4 v0 = ok ? ldg_nc_v4(row) : make_uint4(0, 0, 0, 0);
            const uint4 v1 = ok ? ldg_nc_v4(row + 8) : make_uint4(0, 0, 0, 0);
            va[tt][0] = v0.x; va[tt][1] = v0.y; va[tt][2] = v0.z; va[tt][3] = v0.w;
            va[tt][4] = v1.x; va[tt][5] = v1.y; va[tt][6] = v1.z; va[tt][7] = v1.w;
          }
#pragma unroll
          for (int mt = 0; mt < 8; ++mt) {
            // channel pair (2mt, 2mt+1) of this thread group's chunk lives in word mt
            const uint32_t a0 = prmt(va[0][mt], va[1][mt], 0x5410);  // (ta, tb) at channel 2mt
            const uint32_t a1 = prmt(va[0][mt], va[1][mt], 0x7632);  // (ta, tb) at channel 2mt+1
            const uint32_t a2 = prmt(va[2][mt], va[3][mt], 0x5410);
            const uint32_t a3 = prmt(va[2][mt], va[3][mt], 0x7632);
            mma_16816(st.acc[mt], a0, a1, a2, a3, ph[ks][0], ph[ks][1]);
            mma_16816(st.acc[mt], a0, a1, a2, a3, pl[ks][0], pl[ks][1]);
          }
        }
      }
    }
  }

  // ---------------- epilogue: merge consumer warps, write the split partial
  __syncthreads();
  if (warp < kConsumerWarps)
    warp_to_smem(st, lane, red + warp * 8 * kHeadDim, rm + warp * 8, rl + warp * 8);
  __syncthreads();
  cta_write_partial(p, red, rm, rl, b, kvh, hg, split);
}

// ------------------------------------------------------------------ LSE combine
// Partial record of one (row, split): (acc[D], m, l) with acc unnormalised and
// relative to m (log2 units).  Row r, split s lives at part + s*ss + r*sr.
// Writes any of: fp16 out[r*o_sr + d], natural-log lse[r], and the merged
// partial record merged[r*(D+2) + ...] (for a further cross-GPU combine).
__global__ void lse_combine_kernel(const float* __restrict__ part, int64_t ss, int64_t sr, int rows, int splits,
                                   int D, __half* out, int64_t o_sr, float* lse, float* merged) {
  const int r = blockIdx.x;
  if (r >= rows) return;
  const float* base = part + static_cast<int64_t>(r) * sr;
  float M = -INFINITY;
  for (int s = 0; s < splits; ++s) M = fmaxf(M, base[s * ss + D]);
  const float mb = (M == -INFINITY) ? 0.f : M;
  float L = 0.f;
  for (int s = 0; s < splits; ++s) L += base[s * ss + D + 1] * exp2f(base[s * ss + D] - mb);
  const float inv = L > 0.f ? 1.f / L : 0.f;
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float o = 0.f;
    for (int s = 0; s < splits; ++s) o += base[s * ss + d] * exp2f(base[s * ss + D] - mb);
    if (out) out[static_cast<int64_t>(r) * o_sr + d] = __float2half_rn(o * inv);
    if (merged) merged[static_cast<int64_t>(r) * (D + 2) + d] = o;
  }
  if (threadIdx.x == 0) {
    if (lse) lse[r] = L > 0.f ? (M + log2f(L)) / kLog2e : -INFINITY;
    if (merged) {
      merged[static_cast<int64_t>(r) * (D + 2) + D] = M;
      merged[static_cast<int64_t>(r) * (D + 2) + D + 1] = L;
    }
  }
}

// ------------------------------------------------------------------ host side
struct DecodePlan {
  int n_hg, warm_splits, hot_splits, wbps, hbps, splits;
};

static DecodePlan plan_decode(int B, int Hq, int Hkv, int n_hot, int n_warm_blocks, int rec_bytes) {
  DecodePlan pl{};
  const int g = Hq / Hkv;
  pl.n_hg = (g + 7) / 8;
  const int units = B * Hkv * pl.n_hg;
  const int target = 148 * 6;  // ~2 waves of 3 resident CTAs per SM
  const int per_unit = max(1, (target + units - 1) / units);
  const int nhb = (n_hot + 31) / 32;
  const double wbytes = static_cast<double>(n_warm_blocks) * rec_bytes;
  const double hbytes = static_cast<double>(nhb) * 32 * kHeadDim * 4;
  const double tot = wbytes + hbytes;
  if (n_warm_blocks > 0) {
    int want = tot > 0 ? static_cast<int>(per_unit * wbytes / tot + 0.5) : 1;
    want = max(1, min(want, (n_warm_blocks + 3) / 4));
    pl.wbps = (n_warm_blocks + want - 1) / want;
    pl.warm_splits = (n_warm_blocks + pl.wbps - 1) / pl.wbps;
  }
  if (nhb > 0) {
    int want = tot > 0 ? static_cast<int>(per_unit * hbytes / tot + 0.5) : 1;
    want = max(1, min(want, nhb));
    pl.hbps = (nhb + want - 1) / want;
    pl.hot_splits = (nhb + pl.hbps - 1) / pl.hbps;
  }
  pl.splits = pl.warm_splits + pl.hot_splits;
  return pl;
}

static size_t decode_smem_bytes(int rec_bytes) {
  const size_t ring = static_cast<size_t>(kStages) * rec_bytes;
  const size_t epi = static_cast<size_t>(kConsumerWarps) * 8 * kHeadDim * 4 + kConsumerWarps * 8 * 8;
  return 256 + 8 * kHeadDim * 4 + (ring > epi ? ring : epi);
}

template <int KB, int VB>
static int launch_decode(const DecodeParams& p, cudaStream_t st) {
  const size_t smem = decode_smem_bytes(p.L.bytes);
  auto kern = mixed_decode_kernel<KB, VB>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) !=
      cudaSuccess)
    return AKV_ERR_LAUNCH;
  kern<<<dim3(p.splits, p.Hkv * p.n_hg, p.B), kDecodeThreads, smem, st>>>(p);
  return cudaGetLastError() == cudaSuccess ? AKV_OK : AKV_ERR_LAUNCH;
}

}  // namespace akv

using namespace akv;

// Upper bound on the split count of plan_decode for any record size: the warm
// and hot shares round to at most per_unit + 1 splits together.
static int max_splits(int B, int Hq, int Hkv, int n_hot, int n_warm_blocks) {
  const int g = Hq / Hkv;
  const int units = B * Hkv * ((g + 7) / 8);
  const int per_unit = max(1, (148 * 6 + units - 1) / units);
  const int cap = n_warm_blocks + (n_hot + 31) / 32;
  return max(1, min(per_unit + 2, cap));
}

extern "C" size_t akv_decode_workspace_bytes(int B, int Hq, int Hkv, int D, int n_hot, int n_warm_blocks) {
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv || D != kHeadDim || n_hot < 0 || n_warm_blocks < 0) return 0;
  return static_cast<size_t>(B) * Hq * max_splits(B, Hq, Hkv, n_hot, n_warm_blocks) * (D + 2) * sizeof(float);
}

extern "C" int akv_mixed_decode(const uint16_t* q, int64_t q_sb, int64_t q_sh, const uint16_t* hot_k,
                                const uint16_t* hot_v, int64_t h_sb, int64_t h_sh, int64_t h_sn, int n_hot,
                                const int32_t* hot_len, const uint8_t* warm, int64_t w_sb, int64_t w_sh,
                                const akv_warm_layout* layout, int n_warm_blocks, const int32_t* warm_len, int B,
                                int Hq, int Hkv, int D, float sm_scale, uint16_t* out, int64_t o_sb,
                                int64_t o_sh, float* lse, float* partial_out, void* workspace,
                                size_t workspace_bytes, int* status, void* stream) {
  if (!q || (!out && !partial_out)) return AKV_ERR_NULL;
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv || n_hot < 0 || n_warm_blocks < 0) return AKV_ERR_SHAPE;
  if (D != kHeadDim) return AKV_ERR_UNSUPPORTED;
  if (n_hot > 0 && (!hot_k || !hot_v)) return AKV_ERR_NULL;
  if (n_warm_blocks > 0 && (!warm || !layout)) return AKV_ERR_NULL;
  auto al = [](const void* ptr, int a) { return (reinterpret_cast<uintptr_t>(ptr) % a) == 0; };
  if (!al(q, 16) || q_sb % 8 || q_sh % 8) return AKV_ERR_ALIGN;
  if (out && (!al(out, 2) || o_sb != static_cast<int64_t>(Hq) * o_sh)) return AKV_ERR_UNSUPPORTED;
  if (n_hot > 0 && (!al(hot_k, 16) || !al(hot_v, 16) || h_sb % 8 || h_sh % 8 || h_sn % 8)) return AKV_ERR_ALIGN;
  akv_warm_layout L{};
  if (n_warm_blocks > 0) {
    L = *layout;
    if (L.head_dim != D) return AKV_ERR_SHAPE;
    if (L.key_bits < 2 || L.key_bits > 4 || L.value_bits < 2 || L.value_bits > 4) return AKV_ERR_BITS;
    if (L.n_outlier < 0 || L.n_outlier > kMaxDecodeOutliers) return AKV_ERR_UNSUPPORTED;
    if (L.bytes % 16 || !al(warm, 16) || w_sb % 16 || w_sh % 16) return AKV_ERR_ALIGN;
  }
  if (!workspace) return AKV_ERR_NULL;
  const DecodePlan pl = plan_decode(B, Hq, Hkv, n_hot, n_warm_blocks, n_warm_blocks > 0 ? L.bytes : 1);
  const int splits = max(pl.splits, 1);
  if (splits > max_splits(B, Hq, Hkv, n_hot, n_warm_blocks)) return AKV_ERR_UNSUPPORTED;  // planner invariant
  const size_t need = static_cast<size_t>(B) * Hq * splits * (D + 2) * sizeof(float);
  if (workspace_bytes < need || !al(workspace, 16)) return AKV_ERR_WORKSPACE;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  float* ws = static_cast<float*>(workspace);
  __half* outh = reinterpret_cast<__half*>(out);
  if (pl.splits == 0) {  // no tokens at all: a zeroed partial (m = 0, l = 0) combines to output 0, lse -inf
    if (cudaMemsetAsync(ws, 0, need, st) != cudaSuccess) return AKV_ERR_LAUNCH;
    lse_combine_kernel<<<B * Hq, 128, 0, st>>>(ws, D + 2, D + 2, B * Hq, 1, D, outh, o_sh, lse, partial_out);
    return cudaGetLastError() == cudaSuccess ? AKV_OK : AKV_ERR_LAUNCH;
  }
  DecodeParams p{};
  p.q = reinterpret_cast<const __half*>(q);
  p.q_sb = q_sb;
  p.q_sh = q_sh;
  p.hk = reinterpret_cast<const __half*>(hot_k);
  p.hv = reinterpret_cast<const __half*>(hot_v);
  p.h_sb = h_sb;
  p.h_sh = h_sh;
  p.h_sn = h_sn;
  p.n_hot = n_hot;
  p.hot_len = hot_len;
  p.warm = warm;
  p.w_sb = w_sb;
  p.w_sh = w_sh;
  p.L = L;
  p.n_warm_blocks = n_warm_blocks;
  p.warm_len = warm_len;
  p.B = B;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.g = Hq / Hkv;
  p.n_hg = pl.n_hg;
  p.scale_log2 = sm_scale * kLog2e;
  p.warm_splits = pl.warm_splits;
  p.hot_splits = pl.hot_splits;
  p.wbps = pl.wbps;
  p.hbps = pl.hbps;
  p.splits = pl.splits;
  p.ws = ws;
  p.status = status;
  int rc;
  const int kb = n_warm_blocks > 0 ? L.key_bits : 4, vb = n_warm_blocks > 0 ? L.value_bits : 4;
  switch (kb * 10 + vb) {
    case 22: rc = launch_decode<2, 2>(p, st); break;
    case 23: rc = launch_decode<2, 3>(p, st); break;
    case 24: rc = launch_decode<2, 4>(p, st); break;
    case 32: rc = launch_decode<3, 2>(p, st); break;
    case 33: rc = launch_decode<3, 3>(p, st); break;
    case 34: rc = launch_decode<3, 4>(p, st); break;
    case 42: rc = launch_decode<4, 2>(p, st); break;
    case 43: rc = launch_decode<4, 3>(p, st); break;
    default: rc = launch_decode<4, 4>(p, st); break;
  }
  if (rc != AKV_OK) return rc;
  lse_combine_kernel<<<B * Hq, 128, 0, st>>>(ws, D + 2, static_cast<int64_t>(pl.splits) * (D + 2), B * Hq,
                                             pl.splits, D, outh, o_sh, lse, partial_out);
  return cudaGetLastError() == cudaSuccess ? AKV_OK : AKV_ERR_LAUNCH;
}

extern "C" int akv_lse_combine(const float* part, int64_t part_ss, int64_t part_sr, int rows, int splits, int D,
                               uint16_t* out, int64_t o_sr, float* lse, float* merged, void* stream) {
  if (!part || (!out && !lse && !merged)) return AKV_ERR_NULL;
  if (rows <= 0 || splits <= 0 || D <= 0 || part_ss < 0 || part_sr < 0) return AKV_ERR_SHAPE;
  lse_combine_kernel<<<rows, 128, 0, static_cast<cudaStream_t>(stream)>>>(
      part, part_ss, part_sr, rows, splits, D, reinterpret_cast<__half*>(out), o_sr, lse, merged);
  return cudaGetLastError() == cudaSuccess ? AKV_OK : AKV_ERR_LAUNCH;
}

// ---------------------------------------------------------------------------
// Zero-allocation variant of akv_mixed_decode.
//
// Some callers cannot allocate device memory on the decode path: an attention
// backend hook inside another framework's serving loop is handed only the
// q / KV / output pointers and a stream, has no handle on that framework's
// memory pool, and must not call cudaMalloc there (it synchronises the device
// and is not allowed inside the engine's step).  For them the split-K partials
// live in this fixed device array instead of a caller workspace.  Every GPU
// that loads the library holds the array until the process exits.
// ---------------------------------------------------------------------------
namespace akv {
constexpr size_t kNoAllocScratchBytes = static_cast<size_t>(8) << 20;  // AKV_NOALLOC_SCRATCH_BYTES
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];
constexpr int kMaxDevices = 64;
static void* g_noalloc_ptr[kMaxDevices];  // device address of g_noalloc_scratch, per device
}  // namespace akv

extern "C" int akv_mixed_decode_noalloc(const uint16_t* q, int64_t q_sb, int64_t q_sh, const uint16_t* hot_k,
                                        const uint16_t* hot_v, int64_t h_sb, int64_t h_sh, int64_t h_sn, int n_hot,
                                        const int32_t* hot_len, const uint8_t* warm, int64_t w_sb, int64_t w_sh,
                                        const akv_warm_layout* layout, int n_warm_blocks, const int32_t* warm_len,
                                        int B, int Hq, int Hkv, int D, float sm_scale, uint16_t* out, int64_t o_sb,
                                        int64_t o_sh, float* lse, float* partial_out, int* status, void* stream) {
  const size_t need = akv_decode_workspace_bytes(B, Hq, Hkv, D, n_hot, n_warm_blocks);
  if (need == 0) return D != kHeadDim ? AKV_ERR_UNSUPPORTED : AKV_ERR_SHAPE;
  if (need > kNoAllocScratchBytes) return AKV_ERR_WORKSPACE;  // beyond the fixed scratch array
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return AKV_ERR_LAUNCH;
  if (!g_noalloc_ptr[dev]) {
    // one-time set-up per device, with that device current: the host-side name
    // g_noalloc_scratch is not a device address, so ask the runtime for it
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) return AKV_ERR_LAUNCH;
    g_noalloc_ptr[dev] = p;
  }
  return akv_mixed_decode(q, q_sb, q_sh, hot_k, hot_v, h_sb, h_sh, h_sn, n_hot, hot_len, warm, w_sb, w_sh, layout,
                          n_warm_blocks, warm_len, B, Hq, Hkv, D, sm_scale, out, o_sb, o_sh, lse, partial_out,
                          g_noalloc_ptr[dev], kNoAllocScratchBytes, status, stream);
}
