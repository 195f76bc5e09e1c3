// Mixed-tier decode attention: FP16 hot window + packed warm block records.
//
// softmax(q . [K_warm; K_hot]^T * sm_scale) . [V_warm; V_hot] for one query
// token per (batch row, query head), GQA-batched: one CTA owns one
// (batch row, KV head, <= 8 query heads) and a contiguous range of 32-token
// blocks (split-K over the sequence); an LSE combine merges the splits.
//
// Warm CTAs: every warp streams its own whole block records HBM -> SMEM with
// 1-D bulk TMA (cp.async.bulk + one mbarrier per stage) into three private
// stages, refilling a stage right after consuming it, and dequantises the
// blocks in registers exactly like the reference
// (akv/affine_quantizer.py:112-124, :178-189: fp16(fp16(code*scale) + zero),
// outlier channels replaced by their fp16 originals), so the contraction sees
// the same fp16 K/V values the reference attends over.  Packed codes become
// fp16 with the "1024 + code" magic (one LOP3 per pair), then three packed
// fp16 ops per pair: exact code, fp16(code*scale), + zero (no contraction).
// The contraction runs on mma.sync m16n8k16 (f16 in, f32 accumulate): tokens
// are M for q.K^T, head_dim is M for P.V, and the (<= 8) query heads of the KV
// head are N.  movmatrix transposes P (fp16) between the two.
//
// Hot CTAs read the FP16 window with 128-bit loads and use the same MMA
// layout with natural channel order.
#include <cuda_runtime.h>

#include <algorithm>
#include <cfloat>
#include <cmath>
#include <mutex>

#include "common.cuh"

namespace akv {

// head dims the decode kernel is built for (template parameter D): the K side
// gives each of a warp's four thread columns q4 the channels
// [q4*D/4, (q4+1)*D/4) (D/128 whole 32-channel record chunks, or half a chunk
// at D = 64), the V side gives each of its eight thread rows g8 the channels
// [g8*D/8, (g8+1)*D/8) (D/16 m-tiles of the P.V product)
constexpr bool decode_head_dim_ok(int D) { return D == 64 || D == 128 || D == 256; }
constexpr int kConsumerWarps = 4;
constexpr int kDecodeThreads = kConsumerWarps * 32;
constexpr int kStagesPerWarp = 2;                          // blocks each warp keeps in flight
constexpr int kStages = kConsumerWarps * kStagesPerWarp;
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
  // paged warm pool (nullptr: contiguous rows): record (b, kvh, blk) lives at
  // warm + btab[b * bt_sb + blk] * w_page + kvh * w_sh
  const int32_t* btab;
  int64_t bt_sb, w_page;
  int n_pages;  // pages in the pool: an entry outside [0, n_pages) records AKV_ERR_SHAPE and reads page 0
  akv_warm_layout L;
  int n_warm_blocks;
  const int32_t* warm_len;
  int B, Hq, Hkv, g, n_hg;
  float scale_log2;  // |sm_scale| * log2(e), at least FLT_MIN (scale 0: every logit weighs 2^0)
  float lazy_raw;    // kLazyMax / scale_log2: raw-logit headroom before the running max moves
  int q_neg;         // sm_scale < 0: the kernel negates q (exact) and uses |sm_scale|
  int warm_splits, hot_splits, wbps, hbps, splits;
  float* ws;  // split partials: row (b*Hq + hq)*splits + split holds (acc[D], m, l)
  int* status;
};

// ------------------------------------------------------------------ exact fp16 dequantisation
// x holds (1024 + M*c_a, 1024 + M*c_b) as fp16 (the LOP3 magic).
// c = fma(x, 1/M, -1024/M) is exact; fp16(c*s) and + zero round like the
// reference's `codes.half() * scale + zero` (two roundings, never fused).
template <int M>
AKV_DEV uint32_t dq(uint32_t x, __half2 s, __half2 z) {
  return h2_as_u32(__hadd2_rn(__hmul2_rn(u32_as_h2(fix_magic<M>(x)), s), z));
}

// The same value in two fused ops for records whose scales pass
// dq2_scale_ok: y = fma(x, s, b) = M*fp16(c*s) with b = -1024*s, then
// fma(y, 1/M, z) = fp16(fp16(c*s) + z).
template <int M>
AKV_DEV uint32_t dq2(uint32_t x, uint32_t s, uint32_t b, uint32_t z) {
  constexpr uint32_t inv = fp16_pow2_bits(-log2_pow2(M), false) * 0x10001u;  // (1/M, 1/M)
  uint32_t y, r;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(y) : "r"(x), "r"(s), "r"(b));
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(y), "r"(inv), "r"(z));
  return r;
}

// b = -1024 * s for a scale pair (exact for dq2_scale_ok scales)
AKV_DEV uint32_t neg1024(uint32_t s) {
  constexpr uint32_t k = fp16_pow2_bits(10, true) * 0x10001u;  // (-1024, -1024)
  uint32_t b;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(b) : "r"(s), "r"(k));
  return b;
}

// exact dequantisation of a magic pair: two-op form on flagged records
template <int M, bool FAST>
AKV_DEV uint32_t dqx(uint32_t x, uint32_t s, uint32_t b, uint32_t z) {
  if constexpr (FAST) return dq2<M>(x, s, b, z);
  else return dq<M>(x, u32_as_h2(s), u32_as_h2(z));
}

// ------------------------------------------------------------------ K codes -> A fragments
// Thread (g8, q4) holds, for one token row, the 32 codes of channel chunk q4
// as 16 half2 "pairs"; pair i feeds k-step i/2, low (i even) or high k slots.
// The channel order inside a chunk is permuted per bit width (kPairs*), with
// the magic multiplier of each pair in kMult*; the query fragment uses the
// same permutation.
__device__ constexpr int kMult4[16] = {1, 16, 1, 16, 1, 16, 1, 16, 1, 16, 1, 16, 1, 16, 1, 16};
__device__ constexpr int kMult2[16] = {1, 4, 16, 64, 256, 4, 16, 64, 1, 4, 16, 64, 256, 4, 16, 64};
__device__ constexpr int kMult3[16] = {1, 8, 64, 1, 8, 1, 8, 64, 1, 8, 64, 1, 8, 1, 8, 64};

// Lookups used only with compile-time indices (template recursion below), so
// every pair permutation and magic multiplier is a constant in the code.
template <int KB>
AKV_DEV constexpr PairIdx kpair(int i) {
  return key_pair(KB, i);
}
template <int BITS>
AKV_DEV constexpr int kmult(int i) {
  return BITS == 4 ? kMult4[i] : (BITS == 2 ? kMult2[i] : kMult3[i]);
}

// ---- K row chunk: the code words of thread q4's 32 channels of one token
// (3 bits: the four 24-bit groups, each turned big-endian into the low bits)
template <int KB>
struct KWords {
  uint32_t w[KB == 2 ? 2 : 4];
};

template <int KB>
AKV_DEV KWords<KB> k_words(const uint8_t* row, int q4) {
  KWords<KB> r;
  if constexpr (KB == 4) {
    const uint4 v = lds_v4(row + 16 * q4);
    r.w[0] = v.x;
    r.w[1] = v.y;
    r.w[2] = v.z;
    r.w[3] = v.w;
  } else if constexpr (KB == 2) {
    const uint2 v = lds_v2(row + 8 * q4);
    r.w[0] = v.x;
    r.w[1] = v.y;
  } else {
    const uint8_t* p = row + 12 * q4;
    const uint32_t w0 = lds_u32(p), w1 = lds_u32(p + 4), w2 = lds_u32(p + 8);
    r.w[0] = prmt(w0, 0u, 0x4012);
    r.w[1] = prmt(w0, w1, 0x3345);
    r.w[2] = prmt(w1, w2, 0x2234);
    r.w[3] = prmt(w2, 0u, 0x4123);
  }
  return r;
}

// D = 64: thread q4 owns half h = q4 & 1 of chunk q4 >> 1 (16 channels,
// pairs 8h .. 8h+7 of the chunk, which repeat the pattern of pairs 0..7 with
// channels + 16), moved into the words pairs 0..7 read.
template <int KB>
AKV_DEV KWords<KB> k_words_half(const uint8_t* row, int q4) {
  KWords<KB> r;
  if constexpr (KB == 4) {
    const uint2 v = lds_v2(row + 8 * q4);
    r.w[0] = v.x;
    r.w[1] = v.y;
    r.w[2] = r.w[3] = 0u;
  } else if constexpr (KB == 2) {
    r.w[0] = lds_u32(row + 4 * q4);
    r.w[1] = 0u;
  } else {
    const KWords<3> c = k_words<3>(row, q4 >> 1);
    const bool hi = q4 & 1;
    r.w[0] = hi ? c.w[2] : c.w[0];
    r.w[1] = hi ? c.w[3] : c.w[1];
    r.w[2] = r.w[3] = 0u;
  }
  return r;
}

// Magic pair I (codes kPairs*[I], multiplier kMult*[I]) of a K row chunk.
template <int KB, int I>
AKV_DEV uint32_t k_raw(const KWords<KB>& kw) {
  if constexpr (KB == 4) {
    constexpr int k = I / 4, sub = I % 4;
    const uint32_t x = sub < 2 ? kw.w[k] : (kw.w[k] >> 8);
    if constexpr (sub & 1) return lop_magic<0x00F000F0u>(x);
    else return lop_magic<0x000F000Fu>(x);
  } else if constexpr (KB == 2) {
    constexpr int k = I / 8, sub = I % 8;
    const uint32_t x = kw.w[k];
    if constexpr (sub == 0) return lop_magic<0x00030003u>(x);
    else if constexpr (sub == 1) return lop_magic<0x000C000Cu>(x);
    else if constexpr (sub == 2) return lop_magic<0x00300030u>(x);
    else if constexpr (sub == 3) return lop_magic<0x00C000C0u>(x);
    else if constexpr (sub == 4) return lop_magic<0x03000300u>(x);
    else if constexpr (sub == 5) return lop_magic<0x000C000Cu>(x >> 8);
    else if constexpr (sub == 6) return lop_magic<0x00300030u>(x >> 8);
    else return lop_magic<0x00C000C0u>(x >> 8);
  } else {
    constexpr int k = I / 8, sub = I % 8;  // group pair (2k, 2k+1): codes c7..c0 of each group
    const uint32_t wa = kw.w[2 * k], wb = kw.w[2 * k + 1];
    if constexpr (sub < 3) {
      const uint32_t y = prmt(wa, wb, 0x5410);
      if constexpr (sub == 0) return lop_magic<0x00070007u>(y);
      else if constexpr (sub == 1) return lop_magic<0x00380038u>(y);
      else return lop_magic<0x01C001C0u>(y);
    } else if constexpr (sub < 5) {
      const uint32_t y9 = prmt(wa, wb, 0x5410) >> 9;
      if constexpr (sub == 3) return lop_magic<0x00070007u>(y9);
      else return lop_magic<0x00380038u>(y9);
    } else {
      const uint32_t z = prmt(wa >> 15, wb >> 15, 0x5410);
      if constexpr (sub == 5) return lop_magic<0x00070007u>(z);
      else if constexpr (sub == 6) return lop_magic<0x00380038u>(z);
      else return lop_magic<0x01C001C0u>(z);
    }
  }
}

// query pairs of NP pairs (16 for a whole 32-channel chunk, 8 for a half)
// starting at channel BASE of the thread's query channels, in the K pair order
template <int KB, int NP, int BASE, int NQ, int I = 0>
AKV_DEV void q_pairs(const __half (&qv)[NQ], uint32_t (&qp)[NP]) {
  if constexpr (I < NP) {
    constexpr PairIdx pi = kpair<KB>(I);
    qp[I] = h2_as_u32(__halves2half2(qv[BASE + pi.a], qv[BASE + pi.b]));
    q_pairs<KB, NP, BASE, NQ, I + 1>(qv, qp);
  }
}

// q.K^T k-steps KS..KEND-1: per step, two channel pairs of the 4 token rows,
// dequantised exactly, into the two m-tile accumulators.  ks2 / kz2 point at
// this thread's chunk of the record's K scale / zero (decode pair order), so
// each step reads its two (scale, zero) pairs with two 8-byte loads.
template <int KB, bool FAST, int KS, int KEND, int QO, int NQP>
AKV_DEV void qk_steps(const KWords<KB> (&W)[2][2], const uint2* ks2, const uint2* kz2, const uint32_t (&qp)[NQP],
                      float (&c)[2][4]) {
  if constexpr (KS < KEND) {
    constexpr int I0 = 2 * KS, I1 = 2 * KS + 1;
    constexpr int M0 = kmult<KB>(I0), M1 = kmult<KB>(I1);
    const uint2 sp = ks2[KS], zp = kz2[KS];
    const uint32_t s0 = sp.x, s1 = sp.y, z0 = zp.x, z1 = zp.y;
    const uint32_t b0 = FAST ? neg1024(s0) : 0u, b1 = FAST ? neg1024(s1) : 0u;
#pragma unroll
    for (int mt = 0; mt < 2; ++mt) {
      const uint32_t a0 = dqx<M0, FAST>(k_raw<KB, I0>(W[mt][0]), s0, b0, z0);
      const uint32_t a1 = dqx<M0, FAST>(k_raw<KB, I0>(W[mt][1]), s0, b0, z0);
      const uint32_t a2 = dqx<M1, FAST>(k_raw<KB, I1>(W[mt][0]), s1, b1, z1);
      const uint32_t a3 = dqx<M1, FAST>(k_raw<KB, I1>(W[mt][1]), s1, b1, z1);
      mma_16816(c[mt], a0, a1, a2, a3, qp[QO + I0], qp[QO + I1]);
    }
    qk_steps<KB, FAST, KS + 1, KEND, QO, NQP>(W, ks2, kz2, qp, c);
  }
}

// ---- V token pair (ta, tb) of 16 channels ch0 .. ch0+15 (ch0 % 16 == 0) of
// thread group g8; EIGHT: only channels ch0 .. ch0+7 (head dim 64)
template <int VB>
struct VRow {
  uint32_t w[VB == 2 ? 1 : 2];
};

template <int VB, bool EIGHT = false>
AKV_DEV VRow<VB> v_row_load(const uint8_t* row, int ch0) {
  VRow<VB> r;
  if constexpr (EIGHT) {
    if constexpr (VB == 4) {
      r.w[0] = lds_u32(row + ch0 / 2);
      r.w[1] = 0u;
    } else if constexpr (VB == 2) {
      r.w[0] = *reinterpret_cast<const uint16_t*>(row + ch0 / 4);
    } else {
      const int base = ch0 * 3 / 8;  // 3 bytes: one 24-bit group
      const uint8_t* p = row + (base & ~3);
      const uint32_t v0 = __funnelshift_r(lds_u32(p), lds_u32(p + 4), (base & 3) * 8);
      r.w[0] = prmt(v0, 0u, 0x4012);
      r.w[1] = 0u;
    }
  } else if constexpr (VB == 4) {
    const uint2 w = lds_v2(row + ch0 / 2);
    r.w[0] = w.x;
    r.w[1] = w.y;
  } else if constexpr (VB == 2) {
    r.w[0] = lds_u32(row + ch0 / 4);
  } else {
    const int base = ch0 * 3 / 8;
    const uint8_t* p = row + (base & ~3);
    const uint32_t lo = lds_u32(p), hi = lds_u32(p + 4);
    const int sh = (base & 3) * 8;
    const uint32_t v0 = __funnelshift_r(lo, hi, sh), v1 = __funnelshift_r(hi, 0u, sh);
    r.w[0] = prmt(v0, 0u, 0x4012);  // group 0, big-endian 24-bit
    r.w[1] = prmt(v0, v1, 0x3345);  // group 1
  }
  return r;
}

// interleaved token pair: both tokens' codes side by side in each 16-bit half
template <int VB>
struct VPair {
  uint32_t x[VB == 2 ? 4 : (VB == 4 ? 8 : 6)];
};

template <int VB>
AKV_DEV VPair<VB> v_pair(const VRow<VB>& a, const VRow<VB>& b) {
  VPair<VB> v;
  if constexpr (VB == 2) {
    v.x[0] = prmt(a.w[0], b.w[0], 0x5410);  // codes 0..7
    v.x[1] = v.x[0] >> 8;
    v.x[2] = prmt(a.w[0], b.w[0], 0x7632);  // codes 8..15
    v.x[3] = v.x[2] >> 8;
  } else if constexpr (VB == 4) {
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      v.x[4 * k + 0] = prmt(a.w[k], b.w[k], 0x5410);
      v.x[4 * k + 1] = v.x[4 * k + 0] >> 8;
      v.x[4 * k + 2] = prmt(a.w[k], b.w[k], 0x7632);
      v.x[4 * k + 3] = v.x[4 * k + 2] >> 8;
    }
  } else {
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      v.x[3 * k + 0] = prmt(a.w[k], b.w[k], 0x5410);
      v.x[3 * k + 1] = v.x[3 * k + 0] >> 9;
      v.x[3 * k + 2] = prmt(a.w[k] >> 15, b.w[k] >> 15, 0x5410);
    }
  }
  return v;
}

// magic pair of channel CI (multiplier vmult<VB>(CI))
template <int VB, int CI>
AKV_DEV uint32_t v_raw(const VPair<VB>& v) {
  constexpr int k = CI / 8, sub = CI % 8;
  if constexpr (VB == 2) {
    const uint32_t x = v.x[2 * k], x8 = v.x[2 * k + 1];
    if constexpr (sub == 0) return lop_magic<0x00C000C0u>(x);
    else if constexpr (sub == 1) return lop_magic<0x00300030u>(x);
    else if constexpr (sub == 2) return lop_magic<0x000C000Cu>(x);
    else if constexpr (sub == 3) return lop_magic<0x00030003u>(x);
    else if constexpr (sub == 4) return lop_magic<0x00C000C0u>(x8);
    else if constexpr (sub == 5) return lop_magic<0x00300030u>(x8);
    else if constexpr (sub == 6) return lop_magic<0x000C000Cu>(x8);
    else return lop_magic<0x03000300u>(x);
  } else if constexpr (VB == 4) {
    const uint32_t* x = v.x + 4 * k;
    constexpr int src = sub / 2;  // 0: X, 1: X>>8, 2: Y, 3: Y>>8
    if constexpr (sub & 1) return lop_magic<0x000F000Fu>(x[src]);
    else return lop_magic<0x00F000F0u>(x[src]);
  } else {
    const uint32_t y = v.x[3 * k], y9 = v.x[3 * k + 1], z = v.x[3 * k + 2];
    if constexpr (sub == 0) return lop_magic<0x01C001C0u>(z);
    else if constexpr (sub == 1) return lop_magic<0x00380038u>(z);
    else if constexpr (sub == 2) return lop_magic<0x00070007u>(z);
    else if constexpr (sub == 3) return lop_magic<0x00380038u>(y9);
    else if constexpr (sub == 4) return lop_magic<0x00070007u>(y9);
    else if constexpr (sub == 5) return lop_magic<0x01C001C0u>(y);
    else if constexpr (sub == 6) return lop_magic<0x00380038u>(y);
    else return lop_magic<0x00070007u>(y);
  }
}

template <int VB>
__host__ __device__ constexpr int vmult(int ci) {
  if (VB == 4) return (ci & 1) ? 1 : 16;
  if (VB == 2) {
    constexpr int m[8] = {64, 16, 4, 1, 64, 16, 4, 256};
    return m[ci & 7];
  }
  constexpr int m3[8] = {64, 8, 1, 8, 1, 64, 8, 1};
  return m3[ci & 7];
}

// ------------------------------------------------------------------ shared softmax/PV state
template <int D>
struct WarpState {
  float acc[D / 16][4];  // O^T: tile mt rows (g8 -> d=(D/8)*g8+2mt, g8+8 -> d+1), cols heads (2q4, 2q4+1)
  float mr[2];      // running max of the raw logits q.k for heads 2q4, 2q4+1 (-inf: none yet)
  float nb[2];      // -mr * scale_log2: the exponent offset in use (0 while mr = -inf)
  float l[2];       // partial row sums (this thread's tokens only)
  // one-outlier records: sum_t p_t * original_t (side-tile row 0) and
  // sum_t p_t * -vd_t (row 8) for V outlier channel vch, held by lanes g8 = 0
  // until vch changes, then added to O^T row vch (flush_vout)
  float vo_acc[4];
  int vch;
};

template <int D>
AKV_DEV void state_init(WarpState<D>& s) {
#pragma unroll
  for (int i = 0; i < D / 16; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) s.acc[i][j] = 0.f;
  s.mr[0] = s.mr[1] = -INFINITY;
  s.nb[0] = s.nb[1] = 0.f;
  s.l[0] = s.l[1] = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) s.vo_acc[j] = 0.f;
  s.vch = -1;
}

// Add the side tile's correction sum_t p_t (original_t - vd_t) into O^T row
// vch and clear it.  Every lane takes part (shuffles); vch is warp-uniform.
template <int D>
AKV_DEV void flush_vout(WarpState<D>& s, int g8, int q4) {
  constexpr int kVpt = D / 8;  // V channels per thread row g8
  const float v0 = __shfl_sync(0xffffffffu, s.vo_acc[0] + s.vo_acc[2], q4);
  const float v1 = __shfl_sync(0xffffffffu, s.vo_acc[1] + s.vo_acc[3], q4);
  const int ch = s.vch;
  if (ch >= 0 && ch / kVpt == g8) {
    const int mt = (ch % kVpt) >> 1;
#pragma unroll
    for (int i = 0; i < D / 16; ++i) {
      if (i == mt) {
        if (ch & 1) {
          s.acc[i][2] += v0;
          s.acc[i][3] += v1;
        } else {
          s.acc[i][0] += v0;
          s.acc[i][1] += v1;
        }
      }
    }
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) s.vo_acc[j] = 0.f;
}

// x[mt][4]: raw logits q.k of this thread's 4 tokens x 2 heads (-inf =
// masked); p = 2^(x * scale_log2 + nb) overwrites x.  The running max moves
// (warp-wide max, rescale of acc and l) whenever some logit of the block
// exceeds it by more than lazy_raw = kLazyMax / scale_log2, otherwise the
// block costs no shuffles.  kLazyMax = 0: the offset is always the exact
// running max, so the largest weight so far is exactly 1 when P is rounded to
// fp16 for the P.V product.  A lazy offset (weights up to 2^8) saves ~3 % of
// the config-3 step but rounds the dominant weight too, and where one key
// carries a row that rounding (2^-11 relative) shows in the output: measured
// 2.2e-3 against fp32 attention on a random-init model's decode, twice the
// error of flash attention over the same fp16 view, which keeps the exact
// max.  acc / l and -nb + log2(l) do not depend on which offset was used.
// scale_log2 > 0, so a masked -inf logit gives p = 0.
constexpr float kLazyMax = 0.f;

template <int D>
AKV_DEV void online_softmax(WarpState<D>& s, float (&x)[2][4], float sl2, float lazy_raw) {
  float mx[2];
  mx[0] = fmaxf(fmaxf(x[0][0], x[0][2]), fmaxf(x[1][0], x[1][2]));
  mx[1] = fmaxf(fmaxf(x[0][1], x[0][3]), fmaxf(x[1][1], x[1][3]));
  if (__any_sync(0xffffffffu, mx[0] > s.mr[0] + lazy_raw || mx[1] > s.mr[1] + lazy_raw)) {
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
      mx[0] = fmaxf(mx[0], __shfl_xor_sync(0xffffffffu, mx[0], o));
      mx[1] = fmaxf(mx[1], __shfl_xor_sync(0xffffffffu, mx[1], o));
    }
    float alpha[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const float mn = fmaxf(s.mr[h], mx[h]);
      const float nbn = (mn == -INFINITY) ? 0.f : -mn * sl2;
      alpha[h] = (s.mr[h] == -INFINITY) ? 1.f : fast_exp2(fmaf(s.mr[h], sl2, nbn));
      s.mr[h] = mn;
      s.nb[h] = nbn;
      s.l[h] *= alpha[h];
    }
    s.vo_acc[0] *= alpha[0];
    s.vo_acc[1] *= alpha[1];
    s.vo_acc[2] *= alpha[0];
    s.vo_acc[3] *= alpha[1];
#pragma unroll
    for (int i = 0; i < D / 16; ++i) {
      s.acc[i][0] *= alpha[0];
      s.acc[i][1] *= alpha[1];
      s.acc[i][2] *= alpha[0];
      s.acc[i][3] *= alpha[1];
    }
  }
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      x[mt][j] = fast_exp2(fmaf(x[mt][j], sl2, s.nb[j & 1]));
      s.l[j & 1] += x[mt][j];
    }
}

// P (fp32, S^T C-fragment layout) -> B fragments of the PV MMA (fp16).
AKV_DEV void p_fragments(const float (&x)[2][4], uint32_t (&pb)[2][2]) {
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int r = 0; r < 2; ++r) pb[mt][r] = movmatrix_trans(pack_h2(x[mt][2 * r], x[mt][2 * r + 1]));
}

// P.V k-step over 16 tokens: m-tiles MT .. MEND-1 (channel pairs 2(mt%8),
// 2(mt%8)+1 of the 16-channel group the token-pair codes v0 / v1 hold), the
// two token pairs, dequantised exactly.
template <int VB, bool FAST, int MT, int MEND, int D>
AKV_DEV void pv_tiles(WarpState<D>& st, const VPair<VB>& v0, const VPair<VB>& v1, uint32_t s0, uint32_t b0,
                      uint32_t z0, uint32_t s1, uint32_t b1, uint32_t z1, const uint32_t (&pb)[2]) {
  if constexpr (MT < MEND) {
    constexpr int C0 = 2 * (MT % 8), C1 = 2 * (MT % 8) + 1;
    const uint32_t a0 = dqx<vmult<VB>(C0), FAST>(v_raw<VB, C0>(v0), s0, b0, z0);
    const uint32_t a1 = dqx<vmult<VB>(C1), FAST>(v_raw<VB, C1>(v0), s0, b0, z0);
    const uint32_t a2 = dqx<vmult<VB>(C0), FAST>(v_raw<VB, C0>(v1), s1, b1, z1);
    const uint32_t a3 = dqx<vmult<VB>(C1), FAST>(v_raw<VB, C1>(v1), s1, b1, z1);
    mma_16816(st.acc[MT], a0, a1, a2, a3, pb[0], pb[1]);
    pv_tiles<VB, FAST, MT + 1, MEND, D>(st, v0, v1, s0, b0, z0, s1, b1, z1, pb);
  }
}

// V outlier channel ch of a block: the reference attends over the fp16
// original there, the codes dequantise to vd.  O^T row ch gets
// sum_t (original_t - vd_t) p_t, as two MMAs (originals, then -vd, both exact
// fp16) whose A operand is zero except row ch.  ch is the same for the whole
// warp, so the target tile MT = (ch & 15) / 2 is a warp-uniform switch and
// every accumulator index stays a compile-time constant.
template <int MT, int D>
AKV_DEV void outlier_tile(WarpState<D>& st, const uint32_t (&ao)[4], const uint32_t (&an)[4],
                          const uint32_t (&pb)[2]) {
  mma_16816(st.acc[MT], ao[0], ao[1], ao[2], ao[3], pb[0], pb[1]);
  mma_16816(st.acc[MT], an[0], an[1], an[2], an[3], pb[0], pb[1]);
}

// tile mt (warp-uniform) as a chain of compile-time cases
template <int D, int MT = 0>
AKV_DEV void outlier_mma(WarpState<D>& st, int mt, const uint32_t (&ao)[4], const uint32_t (&an)[4],
                         const uint32_t (&pb)[2]) {
  if constexpr (MT + 1 < D / 16) {
    if (mt == MT) outlier_tile<MT, D>(st, ao, an, pb);
    else outlier_mma<D, MT + 1>(st, mt, ao, an, pb);
  } else {
    outlier_tile<MT, D>(st, ao, an, pb);
  }
}

// ------------------------------------------------------------------ epilogue
// Reduce the per-thread partials of one warp and park them in shared memory:
// red[h][d] (fp32, natural channel order), rm[h], rl[h].
template <int D>
AKV_DEV void warp_to_smem(WarpState<D>& s, int lane, float* red, float* rm, float* rl) {
  const int g8 = lane >> 2, q4 = lane & 3;
#pragma unroll
  for (int h = 0; h < 2; ++h)
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) s.l[h] += __shfl_xor_sync(0xffffffffu, s.l[h], o);
#pragma unroll
  for (int mt = 0; mt < D / 16; ++mt) {
    const int d = (D / 8) * g8 + 2 * mt;
    red[(2 * q4) * D + d] = s.acc[mt][0];
    red[(2 * q4 + 1) * D + d] = s.acc[mt][1];
    red[(2 * q4) * D + d + 1] = s.acc[mt][2];
    red[(2 * q4 + 1) * D + d + 1] = s.acc[mt][3];
  }
  if (g8 == 0) {  // partial (acc, m, l) with acc and l relative to 2^m, m = -nb (log2 units)
    rm[2 * q4] = s.l[0] == 0.f ? -INFINITY : -s.nb[0];
    rm[2 * q4 + 1] = s.l[1] == 0.f ? -INFINITY : -s.nb[1];
    rl[2 * q4] = s.l[0];
    rl[2 * q4 + 1] = s.l[1];
  }
}

// Merge the consumer warps' partials and write this CTA's split partial.
template <int D>
AKV_DEV void cta_write_partial(const DecodeParams& p, float* red, float* rm, float* rl, int b, int kvh, int hg,
                               int split) {
  const int nh = min(8, p.g - hg * 8);
  for (int i = threadIdx.x; i < nh * D; i += blockDim.x) {
    const int h = i / D, d = i % D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) M = fmaxf(M, rm[w * 8 + h]);
    const float base = (M == -INFINITY) ? 0.f : M;
    float acc = 0.f, L = 0.f;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) {
      const float f = fast_exp2(rm[w * 8 + h] - base);
      acc += f * red[(w * 8 + h) * D + d];
      L += f * rl[w * 8 + h];
    }
    const int hq = kvh * p.g + hg * 8 + h;
    float* part = p.ws + ((static_cast<int64_t>(b) * p.Hq + hq) * p.splits + split) * (D + 2);
    part[d] = acc;
    if (d == 0) {
      part[D] = M;
      part[D + 1] = L;
    }
  }
}

// ------------------------------------------------------------------ the kernel
// One warm block record (32 tokens of one (row, KV head)) staged at r:
// S^T = K^ q on the tensor cores, online softmax, O^T += V^ P.  FAST: every
// scale of the record passes dq2_scale_ok (record flags), so dequantisation
// takes two fused fp16 ops per code pair instead of four; the values are the
// same.  Offsets of the fixed fields are compile-time constants.
// NOUT: 0 = no outlier channels; 1 = one (K: q[ch] * original added to the
// logits with FFMAs, V: the side tile of WarpState); 2 = any n_out <= 8
// (extra MMAs per channel).
template <int D, int KB, int VB, int NOUT, bool FAST>
AKV_DEV void warm_block(WarpState<D>& st, const uint8_t* r, uint32_t mask, const uint32_t (&qp)[D / 8],
                        const float* qs, int n_out, float sl2, float lazy_raw, int g8, int q4) {
  constexpr RecLayout R = rec_layout(D, KB, VB, 0);
  constexpr RecLayout R1 = rec_layout(D, KB, VB, 1);
  constexpr int kp = D * KB / 8, vp = D * VB / 8;
  constexpr int kVpt = D / 8;  // V channels of thread row g8: [kVpt*g8, kVpt*(g8+1))

  // one outlier channel: fetch its ids, the query at the K channel and the K
  // originals of this thread's tokens before the main work
  float qk1[2] = {0.f, 0.f}, ko1[2][2] = {{0.f, 0.f}, {0.f, 0.f}};
  if constexpr (NOUT == 1) {
    const int kch = *reinterpret_cast<const int16_t*>(r + R1.ki);
    const int vch = *reinterpret_cast<const int16_t*>(r + R1.vi);
    qk1[0] = qs[(2 * q4) * D + kch];
    qk1[1] = qs[(2 * q4 + 1) * D + kch];
    const __half* ko = reinterpret_cast<const __half*>(r + R1.ko);
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int rr = 0; rr < 2; ++rr) ko1[mt][rr] = __half2float(ko[16 * mt + 8 * rr + g8]);
    if (vch != st.vch) {  // the V outlier channel moved: settle the side tile
      flush_vout(st, g8, q4);
      st.vch = vch;
    }
  }

  // ---- S^T = K^ q  (tokens x heads): rows 16mt + 8rr + g8, k-steps over channel pairs;
  // one pass of 8 k-steps per 32-channel chunk of the thread (4 k-steps over half a chunk at D = 64)
  float c[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
  const uint2* ks2 = reinterpret_cast<const uint2*>(r + R.ks);
  const uint2* kz2 = reinterpret_cast<const uint2*>(r + R.kz);
  if constexpr (D == 64) {
    KWords<KB> W[2][2];
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int rr = 0; rr < 2; ++rr) W[mt][rr] = k_words_half<KB>(r + R.kc + (16 * mt + 8 * rr + g8) * kp, q4);
    qk_steps<KB, FAST, 0, 4, 0, D / 8>(W, ks2 + 4 * q4, kz2 + 4 * q4, qp, c);
  } else {
    constexpr int kCh = D / 128;  // 32-channel chunks per thread
    {
      const int ch = kCh * q4;
      KWords<KB> W[2][2];
#pragma unroll
      for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int rr = 0; rr < 2; ++rr) W[mt][rr] = k_words<KB>(r + R.kc + (16 * mt + 8 * rr + g8) * kp, ch);
      qk_steps<KB, FAST, 0, 8, 0, D / 8>(W, ks2 + 8 * ch, kz2 + 8 * ch, qp, c);
    }
    if constexpr (kCh == 2) {
      const int ch = kCh * q4 + 1;
      KWords<KB> W[2][2];
#pragma unroll
      for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int rr = 0; rr < 2; ++rr) W[mt][rr] = k_words<KB>(r + R.kc + (16 * mt + 8 * rr + g8) * kp, ch);
      qk_steps<KB, FAST, 0, 8, 16, D / 8>(W, ks2 + 8 * ch, kz2 + 8 * ch, qp, c);
    }
  }
  // K outlier channels: their dequantised value is 0 (scale = zero = 0) and the
  // reference puts the fp16 original there.  One channel: + q[ch] * original
  // per logit.  General: one more MMA whose k slots 2q4, 2q4+1 are outliers
  // j = 2q4, 2q4+1 (n_outlier <= 8).
  if constexpr (NOUT == 1) {
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int rr = 0; rr < 2; ++rr)
#pragma unroll
        for (int h = 0; h < 2; ++h) c[mt][2 * rr + h] = fmaf(qk1[h], ko1[mt][rr], c[mt][2 * rr + h]);
  }
  if (NOUT == 2 && n_out > 0) {
    const __half* ko = reinterpret_cast<const __half*>(r + up16c(R.ki + 4 * n_out));
    const int16_t* kid = reinterpret_cast<const int16_t*>(r + R.ki);
    const int j0 = 2 * q4, j1 = 2 * q4 + 1;
    const __half hz = __float2half_rn(0.f);
    const __half qa = j0 < n_out ? __float2half_rn(qs[g8 * D + kid[j0]]) : hz;
    const __half qb = j1 < n_out ? __float2half_rn(qs[g8 * D + kid[j1]]) : hz;
    const uint32_t bq = h2_as_u32(__halves2half2(qa, qb));
#pragma unroll
    for (int mt = 0; mt < 2; ++mt) {
      uint32_t a[2];
#pragma unroll
      for (int rr = 0; rr < 2; ++rr) {
        const int t = 16 * mt + 8 * rr + g8;
        const __half oa = j0 < n_out ? ko[t * n_out + j0] : hz;
        const __half ob = j1 < n_out ? ko[t * n_out + j1] : hz;
        a[rr] = h2_as_u32(__halves2half2(oa, ob));
      }
      mma_16816(c[mt], a[0], a[1], 0u, 0u, bq, 0u);
    }
  }
  // raw logits; masked slots -inf (only partial blocks pay for the selects)
  if (mask != 0xffffffffu) {
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int rr = 0; rr < 2; ++rr) {
        const bool valid = (mask >> (16 * mt + 8 * rr + g8)) & 1u;
#pragma unroll
        for (int h = 0; h < 2; ++h) c[mt][2 * rr + h] = valid ? c[mt][2 * rr + h] : -INFINITY;
      }
  }
  online_softmax(st, c, sl2, lazy_raw);
  uint32_t pb[2][2];
  p_fragments(c, pb);

  // ---- O^T += V^ P  (head_dim x heads), k-steps of 16 tokens
  const __half* vsc = reinterpret_cast<const __half*>(r + R.vs);
  const __half* vzr = reinterpret_cast<const __half*>(r + R.vz);
#pragma unroll
  for (int ks = 0; ks < 2; ++ks) {
    const int ta = 16 * ks + 2 * q4;
    const uint8_t* vc = r + R.vc;
    const uint32_t s0 = lds_u32(vsc + ta), z0 = lds_u32(vzr + ta);
    const uint32_t s1 = lds_u32(vsc + ta + 8), z1 = lds_u32(vzr + ta + 8);
    const uint32_t b0 = FAST ? neg1024(s0) : 0u, b1 = FAST ? neg1024(s1) : 0u;
    constexpr bool kEight = D == 64;  // 8 V channels per thread row: half a 16-channel group
#pragma unroll
    for (int j = 0; j < (kEight ? 1 : kVpt / 16); ++j) {  // 16-channel groups of the thread row
      const int ch0 = kVpt * g8 + 16 * j;
      const VPair<VB> v0 = v_pair<VB>(v_row_load<VB, kEight>(vc + ta * vp, ch0),
                                      v_row_load<VB, kEight>(vc + (ta + 1) * vp, ch0));
      const VPair<VB> v1 = v_pair<VB>(v_row_load<VB, kEight>(vc + (ta + 8) * vp, ch0),
                                      v_row_load<VB, kEight>(vc + (ta + 9) * vp, ch0));
      if (j == 0) pv_tiles<VB, FAST, 0, (kEight ? 4 : 8), D>(st, v0, v1, s0, b0, z0, s1, b1, z1, pb[ks]);
      if constexpr (kVpt / 16 == 2)
        if (j == 1) pv_tiles<VB, FAST, 8, 16, D>(st, v0, v1, s0, b0, z0, s1, b1, z1, pb[ks]);
    }
  }

  // ---- V outlier channels: O^T row ch += sum_t p_t (original_t - vd_t).
  // One channel: rows 0 / 8 of the side tile take originals / -vd from lanes
  // g8 = 0 (one MMA per k-step, flushed when the channel moves).
  if constexpr (NOUT == 1) {
    const __half* vo = reinterpret_cast<const __half*>(r + R1.vo);
    const __half* vdq = reinterpret_cast<const __half*>(r + R1.vd);
    const bool lead = g8 == 0;
#pragma unroll
    for (int ks = 0; ks < 2; ++ks) {
      const int ta = 16 * ks + 2 * q4;
      const uint32_t o0 = lead ? lds_u32(vo + ta) : 0u, o1 = lead ? lds_u32(vo + ta + 8) : 0u;
      const uint32_t n0 = lead ? (lds_u32(vdq + ta) ^ 0x80008000u) : 0u;
      const uint32_t n1 = lead ? (lds_u32(vdq + ta + 8) ^ 0x80008000u) : 0u;
      mma_16816(st.vo_acc, o0, n0, o1, n1, pb[ks][0], pb[ks][1]);
    }
  }
  if (NOUT == 2 && n_out > 0) {
    const int o_vo = up16c(R.ki + 4 * n_out) + up16c(2 * kBlockTokens * n_out);
    const __half* vo = reinterpret_cast<const __half*>(r + o_vo);
    const __half* vdq = reinterpret_cast<const __half*>(r + o_vo + up16c(2 * kBlockTokens * n_out));
    const int16_t* vid = reinterpret_cast<const int16_t*>(r + R.ki + 2 * n_out);
    for (int j = 0; j < n_out; ++j) {
      const int ch = vid[j];
      const bool own = ch / kVpt == g8;
      const int hf = ch & 1;
#pragma unroll
      for (int ks = 0; ks < 2; ++ks) {
        const int ta = 16 * ks + 2 * q4;
        const uint32_t o0 = h2_as_u32(__halves2half2(vo[ta * n_out + j], vo[(ta + 1) * n_out + j]));
        const uint32_t o1 = h2_as_u32(__halves2half2(vo[(ta + 8) * n_out + j], vo[(ta + 9) * n_out + j]));
        const uint32_t d0 = h2_as_u32(__halves2half2(vdq[ta * n_out + j], vdq[(ta + 1) * n_out + j]));
        const uint32_t d1 = h2_as_u32(__halves2half2(vdq[(ta + 8) * n_out + j], vdq[(ta + 9) * n_out + j]));
        const uint32_t on = own ? 0xFFFFFFFFu : 0u;  // A is zero outside row ch
        const uint32_t m0 = hf ? 0u : on, m1 = hf ? on : 0u;
        const uint32_t ao[4] = {o0 & m0, o0 & m1, o1 & m0, o1 & m1};
        const uint32_t an[4] = {(d0 ^ 0x80008000u) & m0, (d0 ^ 0x80008000u) & m1, (d1 ^ 0x80008000u) & m0,
                                (d1 ^ 0x80008000u) & m1};
        outlier_mma<D>(st, (ch % kVpt) >> 1, ao, an, pb[ks]);
      }
    }
  }
}

// PAGED: warm records are found through the block table (p.btab), else row
// b's records are contiguous; a compile-time choice, so the contiguous kernel
// carries no table logic.
// resident CTAs per SM the kernel is built for: head dim 256 keeps twice the
// O^T accumulators and query pairs per thread, so it gets more registers
__host__ __device__ constexpr int decode_ctas_per_sm(int D) { return D == 256 ? 2 : 4; }

template <int D, int KB, int VB, int NOUT, bool PAGED>
__global__ void __launch_bounds__(kDecodeThreads, decode_ctas_per_sm(D)) mixed_decode_kernel(const DecodeParams p) {
  static_assert(decode_head_dim_ok(D), "head dim 64, 128 or 256");
  constexpr RecLayout R = rec_layout(D, KB, VB, 0);
  constexpr int kCpt = D / 4;  // K-side query channels of thread column q4: [kCpt*q4, kCpt*(q4+1))
  constexpr int kVpt = D / 8;  // V-side channels of thread row g8
  extern __shared__ __align__(128) unsigned char smem[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g8 = lane >> 2, q4 = lane & 3;
  const int split = blockIdx.x;
  const int kvh = blockIdx.y / p.n_hg, hg = blockIdx.y % p.n_hg;
  const int b = blockIdx.z;
  const bool warm_cta = split < p.warm_splits;

  // shared memory map
  const int rec = p.L.bytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);        // [kStages], 96 bytes
  float* qs = reinterpret_cast<float*>(smem + 256);               // [8][D] query (fp32) for outliers
  unsigned char* stage0 = smem + 256 + 8 * D * 4;                 // [kStages][rec]
  // epilogue buffers alias the stages once the main loop is over
  float* red = reinterpret_cast<float*>(stage0);                  // [warps][8][D]
  float* rm = red + kConsumerWarps * 8 * D;                       // [warps][8]
  float* rl = rm + kConsumerWarps * 8;

  const int nh = min(8, p.g - hg * 8);
  const int qh_base = kvh * p.g + hg * 8;
  const float sl2 = p.scale_log2, lazy_raw = p.lazy_raw;

  WarpState<D> st;
  state_init(st);

  // warm CTAs: every warp initialises its own stage barriers and puts its
  // first blocks in flight before anything else, so the query loads below
  // overlap the first copies instead of preceding them
  int nmine = 0;
  const uint8_t* wbase = nullptr;
  const int32_t* wtab = nullptr;  // paged pool: this row's block table, from this split's first block
  int32_t next_page = 0;          // lane 0: page of the warp's next refill, fetched one block ahead
  auto page_at = [&](int i) {
    int32_t pg = __ldg(wtab + i);
    if (static_cast<uint32_t>(pg) >= static_cast<uint32_t>(p.n_pages)) {
      set_status(p.status, AKV_ERR_SHAPE);
      pg = 0;
    }
    return pg;
  };
  uint64_t* wbar = full + warp * kStagesPerWarp;
  unsigned char* wstage = stage0 + warp * kStagesPerWarp * rec;
  if (warm_cta) {
    const int nblk_b = p.warm_len ? min(p.warm_len[b], p.n_warm_blocks) : p.n_warm_blocks;
    const int blo = split * p.wbps;
    const int bhi = min(nblk_b, blo + p.wbps);
    const int nb = max(0, bhi - blo);
    if constexpr (PAGED) {
      wtab = p.btab + b * p.bt_sb + blo;
      wbase = p.warm + kvh * p.w_sh;
    } else {
      wbase = p.warm + b * p.w_sb + kvh * p.w_sh + static_cast<int64_t>(blo) * rec;
    }
    // warp `warp` owns blocks i = warp + 4*li (li = 0, 1, ...) and stages
    // warp*kStagesPerWarp + li%kStagesPerWarp; lane 0 keeps them in flight
    nmine = nb > warp ? (nb - warp + kConsumerWarps - 1) / kConsumerWarps : 0;
    if (lane == 0) {
      for (int s = 0; s < kStagesPerWarp; ++s) mbar_init(&wbar[s], 1);
      fence_mbar_init();
      for (int li = 0; li < min(nmine, kStagesPerWarp); ++li) {
        const int i = warp + kConsumerWarps * li;
        const uint8_t* src = PAGED ? wbase + static_cast<int64_t>(page_at(i)) * p.w_page
                                   : wbase + static_cast<int64_t>(i) * rec;
        mbar_arrive_expect_tx(&wbar[li], rec);
        tma_load_1d(wstage + li * rec, src, rec, &wbar[li]);
      }
      if (PAGED && kStagesPerWarp < nmine) next_page = page_at(warp + kConsumerWarps * kStagesPerWarp);
    }
    __syncwarp();
  }

  // this thread's query column (head g8 of the head group; zero padding beyond nh);
  // a negative softmax scale is applied as -q (exact) with scale |sm_scale|
  const uint32_t qflip = p.q_neg ? 0x80008000u : 0u;
  __half qv[kCpt];
  {
    const bool have = g8 < nh;
    const __half* qrow = p.q + b * p.q_sb + (qh_base + (have ? g8 : 0)) * p.q_sh + kCpt * q4;
#pragma unroll
    for (int k = 0; k < kCpt / 8; ++k) {
      uint4 v = have ? ldg_nc_v4(qrow + 8 * k) : make_uint4(0, 0, 0, 0);
      v.x ^= qflip;
      v.y ^= qflip;
      v.z ^= qflip;
      v.w ^= qflip;
      *reinterpret_cast<uint4*>(qv + 8 * k) = v;
    }
  }
  if (warp == 0) {  // fp32 copy of the head group's queries for the outlier terms
#pragma unroll
    for (int k = 0; k < kCpt / 4; ++k) {
      const float4 f = make_float4(__half2float(qv[4 * k]), __half2float(qv[4 * k + 1]), __half2float(qv[4 * k + 2]),
                                   __half2float(qv[4 * k + 3]));
      *reinterpret_cast<float4*>(qs + g8 * D + kCpt * q4 + 4 * k) = f;
    }
  }
  __syncthreads();

  if (warm_cta) {
    // query pairs in the K pair order: 16 per 32-channel chunk (8 for the half chunk at D = 64)
    uint32_t qp[D / 8];
    if constexpr (D == 64) {
      q_pairs<KB, 8, 0, kCpt>(qv, qp);
    } else {
      uint32_t q0[16];
      q_pairs<KB, 16, 0, kCpt>(qv, q0);
#pragma unroll
      for (int i = 0; i < 16; ++i) qp[i] = q0[i];
      if constexpr (D == 256) {
        uint32_t q1[16];
        q_pairs<KB, 16, 32, kCpt>(qv, q1);
#pragma unroll
        for (int i = 0; i < 16; ++i) qp[16 + i] = q1[i];
      }
    }
    const int n_out = p.L.n_outlier;

    int waited = 0;  // blocks whose copy this warp has seen land
    for (int li = 0; li < nmine; ++li) {
      const int s = li % kStagesPerWarp;
      if (!mbar_wait(&wbar[s], (li / kStagesPerWarp) & 1, p.status)) break;
      waited = li + 1;
      const uint8_t* r = wstage + s * rec;
      const uint2 mf = lds_v2(r + R.mask);  // valid-slot mask, decode flags
      if ((mf.y & 0xFFFFu) == 0x0101u)
        warm_block<D, KB, VB, NOUT, true>(st, r, mf.x, qp, qs, n_out, sl2, lazy_raw, g8, q4);
      else
        warm_block<D, KB, VB, NOUT, false>(st, r, mf.x, qp, qs, n_out, sl2, lazy_raw, g8, q4);
      // refill this stage with the warp's block li+3 once every lane is done reading it
      __syncwarp();
      if (lane == 0 && li + kStagesPerWarp < nmine) {
        const int i = warp + kConsumerWarps * (li + kStagesPerWarp);
        const uint8_t* src = PAGED ? wbase + static_cast<int64_t>(next_page) * p.w_page
                                   : wbase + static_cast<int64_t>(i) * rec;
        if (PAGED && li + kStagesPerWarp + 1 < nmine) next_page = page_at(i + kConsumerWarps);
        fence_proxy_async_shared();
        mbar_arrive_expect_tx(&wbar[s], rec);
        tma_load_1d(wstage + s * rec, src, rec, &wbar[s]);
      }
    }
    // after a timed-out wait, let the copies still in flight land before the
    // stages are reused as epilogue scratch (bounded waits)
    if (lane == 0)
      for (int li = waited; li < min(nmine, waited + kStagesPerWarp); ++li)
        mbar_wait(&wbar[li % kStagesPerWarp], (li / kStagesPerWarp) & 1, p.status);
  } else {
    // ---------------- hot CTA: FP16 window, 128-bit loads
    const int hs = split - p.warm_splits;
    const int nhot_b = p.hot_len ? min(p.hot_len[b], p.n_hot) : p.n_hot;
    const int nhb = (nhot_b + 31) / 32;
    const int blo = hs * p.hbps;
    const int bhi = min(nhb, blo + p.hbps);
    // K rows in passes of up to 32 channels (16 words, 8 k-steps) of the thread's kCpt
    constexpr int kPassCh = kCpt < 32 ? kCpt : 32;
    constexpr int kPasses = kCpt / kPassCh;
    uint32_t qn[kCpt / 2];
#pragma unroll
    for (int i = 0; i < kCpt / 2; ++i) qn[i] = h2_as_u32(__halves2half2(qv[2 * i], qv[2 * i + 1]));
    const __half* kb = p.hk + b * p.h_sb + kvh * p.h_sh;
    const __half* vb = p.hv + b * p.h_sb + kvh * p.h_sh;
    for (int blk = blo + warp; blk < bhi; blk += kConsumerWarps) {
      const int t0 = blk * 32;
      float x[2][4];
      bool valid[2][2];
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
        float c[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int pass = 0; pass < kPasses; ++pass) {
          uint32_t e0[kPassCh / 2], e1[kPassCh / 2];
#pragma unroll
          for (int rr = 0; rr < 2; ++rr) {
            const int t = t0 + 16 * mt + 8 * rr + g8;
            valid[mt][rr] = t < nhot_b;
            uint32_t* e = rr ? e1 : e0;
            const __half* row =
                kb + static_cast<int64_t>(valid[mt][rr] ? t : 0) * p.h_sn + kCpt * q4 + kPassCh * pass;
#pragma unroll
            for (int k = 0; k < kPassCh / 8; ++k) {
              const uint4 v = valid[mt][rr] ? ldg_nc_v4(row + 8 * k) : make_uint4(0, 0, 0, 0);
              e[4 * k + 0] = v.x;
              e[4 * k + 1] = v.y;
              e[4 * k + 2] = v.z;
              e[4 * k + 3] = v.w;
            }
          }
#pragma unroll
          for (int ks = 0; ks < kPassCh / 4; ++ks)
            mma_16816(c, e0[2 * ks], e1[2 * ks], e0[2 * ks + 1], e1[2 * ks + 1], qn[kPassCh / 2 * pass + 2 * ks],
                      qn[kPassCh / 2 * pass + 2 * ks + 1]);
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) x[mt][j] = valid[mt][j >> 1] ? c[j] : -INFINITY;
      }
      online_softmax(st, x, sl2, lazy_raw);
      uint32_t pb[2][2];
      p_fragments(x, pb);
#pragma unroll
      for (int ks = 0; ks < 2; ++ks) {
        // the thread row's V channels in groups of 16 (8 at D = 64): m-tiles 8j .. 8j + kW - 1
        constexpr int kW = D == 64 ? 4 : 8;  // words (channel pairs) per group
#pragma unroll
        for (int j = 0; j < kVpt / (2 * kW); ++j) {
          uint32_t va[4][kW];
#pragma unroll
          for (int tt = 0; tt < 4; ++tt) {
            const int t = t0 + 16 * ks + 2 * q4 + (tt & 1) + 8 * (tt >> 1);
            const bool ok = t < nhot_b;
            const __half* row = vb + static_cast<int64_t>(ok ? t : 0) * p.h_sn + kVpt * g8 + 2 * kW * j;
#pragma unroll
            for (int k = 0; k < kW / 4; ++k) {
              const uint4 v = ok ? ldg_nc_v4(row + 8 * k) : make_uint4(0, 0, 0, 0);
              va[tt][4 * k + 0] = v.x;
              va[tt][4 * k + 1] = v.y;
              va[tt][4 * k + 2] = v.z;
              va[tt][4 * k + 3] = v.w;
            }
          }
#pragma unroll
          for (int m = 0; m < kW; ++m) {
            // channel pair (2mt, 2mt+1) of this thread row's channels lives in word m of group j
            const uint32_t a0 = prmt(va[0][m], va[1][m], 0x5410);  // (ta, tb) at channel 2mt
            const uint32_t a1 = prmt(va[0][m], va[1][m], 0x7632);  // (ta, tb) at channel 2mt+1
            const uint32_t a2 = prmt(va[2][m], va[3][m], 0x5410);
            const uint32_t a3 = prmt(va[2][m], va[3][m], 0x7632);
            mma_16816(st.acc[kW * j + m], a0, a1, a2, a3, pb[ks][0], pb[ks][1]);
          }
        }
      }
    }
  }

  // ---------------- epilogue: merge consumer warps, write the split partial
  if constexpr (NOUT == 1) flush_vout(st, g8, q4);
  __syncthreads();
  warp_to_smem(st, lane, red + warp * 8 * D, rm + warp * 8, rl + warp * 8);
  __syncthreads();
  cta_write_partial<D>(p, red, rm, rl, b, kvh, hg, split);
}

// ------------------------------------------------------------------ LSE combine
// Partial record of one (row, split): (acc[D], m, l) with acc unnormalised and
// relative to m (log2 units).  Row r, split s lives at part + s*ss + r*sr.
// Writes any of: fp16 out[r*o_sr + d], natural-log lse[r], and the merged
// partial record merged[r*(D+2) + ...] (for a further cross-GPU combine).
constexpr int kCombineMaxSplits = 256;  // splits whose weights are kept in shared memory
constexpr int kCombineThreads = 128;
constexpr int kCombineChunk = 32;                                 // channels per CTA
constexpr int kCombineGroups = kCombineThreads / kCombineChunk;  // split groups per CTA

// grid (rows, ceil(D / 32)): a CTA merges 32 channels of one row.  Warp 0
// turns the splits' (m, l) into weights w_s = 2^(m_s - M) in shared memory;
// thread (group, c) then sums channel c over the splits s = group (mod 4),
// eight loads in flight, and the four group sums meet in shared memory.
// Every warp's loads of one split are 128 contiguous bytes.
__global__ void __launch_bounds__(kCombineThreads) lse_combine_kernel(const float* __restrict__ part, int64_t ss,
                                                                      int64_t sr, int rows, int splits, int D,
                                                                      __half* out, int64_t o_sr, float* lse,
                                                                      float* merged) {
  __shared__ float w[kCombineMaxSplits];
  __shared__ float acc[kCombineGroups][kCombineChunk];
  __shared__ float sM, sL;
  // launched as a programmatic dependent of the decode kernel: wait until that
  // grid has completed and its partials are visible (a no-op otherwise)
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int r = blockIdx.x;
  if (r >= rows) return;
  const float* base = part + static_cast<int64_t>(r) * sr;
  const int lane = threadIdx.x & 31, grp = threadIdx.x >> 5;
  if (threadIdx.x < 32) {
    float M = -INFINITY;
    for (int s = lane; s < splits; s += 32) M = fmaxf(M, base[s * ss + D]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    const float mb = (M == -INFINITY) ? 0.f : M;
    float L = 0.f;
    for (int s = lane; s < splits; s += 32) {
      const float ws = exp2f(base[s * ss + D] - mb);
      if (s < kCombineMaxSplits) w[s] = ws;
      L += base[s * ss + D + 1] * ws;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
    if (lane == 0) {
      sM = M;
      sL = L;
    }
  }
  __syncthreads();
  const float M = sM, L = sL, mb = (M == -INFINITY) ? 0.f : M;
  const int d = blockIdx.y * kCombineChunk + lane;
  float o = 0.f;
  if (d < D) {
    const float* col = base + d;
    const int lim = min(splits, kCombineMaxSplits);
    int s = grp;
    for (; s + 7 * kCombineGroups < lim; s += 8 * kCombineGroups) {
      float v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = col[(s + j * kCombineGroups) * ss];
#pragma unroll
      for (int j = 0; j < 8; ++j) o = fmaf(v[j], w[s + j * kCombineGroups], o);
    }
    for (; s < splits; s += kCombineGroups)
      o = fmaf(col[s * ss], s < kCombineMaxSplits ? w[s] : exp2f(base[s * ss + D] - mb), o);
  }
  acc[grp][lane] = o;
  __syncthreads();
  if (grp == 0 && d < D) {
#pragma unroll
    for (int g = 1; g < kCombineGroups; ++g) o += acc[g][lane];
    const float inv = L > 0.f ? 1.f / L : 0.f;
    if (out) out[static_cast<int64_t>(r) * o_sr + d] = __float2half_rn(o * inv);
    if (merged) merged[static_cast<int64_t>(r) * (D + 2) + d] = o;
  }
  if (blockIdx.y == 0 && threadIdx.x == 0) {
    if (lse) lse[r] = L > 0.f ? (M + log2f(L)) / kLog2e : -INFINITY;
    if (merged) {
      merged[static_cast<int64_t>(r) * (D + 2) + D] = M;
      merged[static_cast<int64_t>(r) * (D + 2) + D + 1] = L;
    }
  }
}

static dim3 combine_grid(int rows, int D) { return dim3(rows, (D + kCombineChunk - 1) / kCombineChunk); }

// The split merge of a decode launch, as a programmatic dependent launch: the
// GPU processes its launch while the decode kernel is still running, and its
// griddepcontrol.wait holds it until the decode grid's partials are complete.
static int launch_combine_dependent(const float* part, int64_t ss, int64_t sr, int rows, int splits, int D,
                                    __half* out, int64_t o_sr, float* lse, float* merged, cudaStream_t st) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = combine_grid(rows, D);
  cfg.blockDim = dim3(kCombineThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, lse_combine_kernel, part, ss, sr, rows, splits, D, out, o_sr, lse, merged) ==
                 cudaSuccess
             ? AKV_OK
             : AKV_ERR_LAUNCH;
}

// ------------------------------------------------------------------ host side
struct DecodePlan {
  int n_hg, warm_splits, hot_splits, wbps, hbps, splits;
};

// Split-K plan.  A unit is one (batch row, KV head, <= 8 query heads); its
// tokens are split into warm and hot splits in proportion to their bytes.
// The split count per unit is chosen so that the grid fills its last wave of
// decode_slots(D) resident CTAs well, from at least ~3 waves (a half-empty last
// wave leaves SMs idle at the end of the launch); config 3 (128 units) gets
// 18 splits: 2,304 CTAs, 3.9 waves.
constexpr int kSms = 148;
// resident decode CTAs of the whole GPU at head dim D
static int decode_slots(int D) { return kSms * decode_ctas_per_sm(D); }
// Device time per byte of a hot CTA relative to a warm one: a hot warp streams
// plain fp16 rows (16 KB per 32-token block, two DRAM round trips, little
// arithmetic) while a warm warp dequantises ~3.9 KB records, so hot splits
// take proportionally more bytes.
constexpr double kHotCost = 0.75;

static void split_shares(int per_unit, int n_warm_blocks, int nhb, double wbytes, double hbytes, DecodePlan& pl) {
  const double tot = wbytes + hbytes;
  pl.warm_splits = pl.hot_splits = pl.wbps = pl.hbps = 0;
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
}

// Fewest 32-token blocks a split gets when the wave target would cut a unit
// finer (few units: batch 1, few KV heads): every warp then has several blocks
// to stream, and the split partials the combine reads stay few.
constexpr int kMinBlocksPerSplit = 16;

// Waves of resident CTAs the split count aims for: three when there are many
// units (config 3's 128: the smaller CTAs even out the tail), one when there
// are at most kFewUnits (a KV-head shard on 2-8 GPUs, batch 1 at 64 heads),
// where a three-wave target cuts every unit into short splits whose per-CTA
// set-up dominates (per layer, 1-wave vs 3-wave target: 8-GPU config-3 shard
// 29.4 vs 34.9 us, 4-GPU 52.1 vs 59.4, 2-GPU 91.4 vs 94.6, config-5b shard
// 30.9 vs 37.5; the full config-3 layer is 1.9 % slower with one wave).
constexpr int kFewUnits = 64;

// candidate split counts per unit: [lo, hi]; unit_blocks = warm + hot blocks of one unit
static void per_unit_range(int units, int unit_blocks, int slots, int& lo, int& hi) {
  const int waves = units <= kFewUnits ? 1 : 3;
  lo = max(1, (waves * slots + units - 1) / units);
  hi = lo + max(8, lo);
  const int cap = max(1, unit_blocks / kMinBlocksPerSplit);
  if (hi > cap) {
    hi = cap;
    lo = min(lo, cap);
  }
}

static DecodePlan plan_decode(int B, int Hq, int Hkv, int D, int n_hot, int n_warm_blocks, int rec_bytes) {
  DecodePlan pl{};
  const int g = Hq / Hkv;
  pl.n_hg = (g + 7) / 8;
  const int units = B * Hkv * pl.n_hg;
  const int nhb = (n_hot + 31) / 32;
  const double wbytes = static_cast<double>(n_warm_blocks) * rec_bytes;
  const double hbytes = static_cast<double>(nhb) * 32 * D * 4 * kHotCost;
  const int slots = decode_slots(D);
  int lo, hi;
  per_unit_range(units, n_warm_blocks + nhb, slots, lo, hi);
  double best = -1.0;
  DecodePlan cand = pl;
  for (int pu = lo; pu <= hi; ++pu) {
    split_shares(pu, n_warm_blocks, nhb, wbytes, hbytes, cand);
    const int64_t ctas = static_cast<int64_t>(units) * cand.splits;
    const int64_t waves = (ctas + slots - 1) / slots;
    const double fill = static_cast<double>(ctas) / static_cast<double>(waves * slots);
    if (fill > best + 0.03) {  // more splits only for a clearly fuller last wave
      best = fill;
      pl.warm_splits = cand.warm_splits;
      pl.hot_splits = cand.hot_splits;
      pl.wbps = cand.wbps;
      pl.hbps = cand.hbps;
      pl.splits = cand.splits;
    }
  }
  return pl;
}

static size_t decode_smem_bytes(int rec_bytes, int D) {
  const size_t ring = static_cast<size_t>(kStages) * rec_bytes;
  const size_t epi = static_cast<size_t>(kConsumerWarps) * 8 * D * 4 + kConsumerWarps * 8 * 8;
  return 256 + 8 * D * 4 + (ring > epi ? ring : epi);
}

template <int D, int KB, int VB, int NOUT>
static int launch_decode3(const DecodeParams& p, cudaStream_t st) {
  const size_t smem = decode_smem_bytes(p.L.bytes, D);
  auto kern = p.btab ? mixed_decode_kernel<D, KB, VB, NOUT, true> : mixed_decode_kernel<D, KB, VB, NOUT, false>;
  const bool ok = p.btab ? ensure_dynamic_smem<mixed_decode_kernel<D, KB, VB, NOUT, true>>(smem)
                         : ensure_dynamic_smem<mixed_decode_kernel<D, KB, VB, NOUT, false>>(smem);
  if (!ok) return AKV_ERR_LAUNCH;
  kern<<<dim3(p.splits, p.Hkv * p.n_hg, p.B), kDecodeThreads, smem, st>>>(p);
  return cudaGetLastError() == cudaSuccess ? AKV_OK : AKV_ERR_LAUNCH;
}

template <int D, int KB, int VB>
static int launch_decode(const DecodeParams& p, cudaStream_t st) {
  const int n = p.n_warm_blocks > 0 ? p.L.n_outlier : 0;
  if (n == 0) return launch_decode3<D, KB, VB, 0>(p, st);
  if (n == 1) return launch_decode3<D, KB, VB, 1>(p, st);
  return launch_decode3<D, KB, VB, 2>(p, st);
}

template <int D>
static int launch_decode_bits(const DecodeParams& p, int kb, int vb, cudaStream_t st) {
  switch (kb * 10 + vb) {
    case 22: return launch_decode<D, 2, 2>(p, st);
    case 23: return launch_decode<D, 2, 3>(p, st);
    case 24: return launch_decode<D, 2, 4>(p, st);
    case 32: return launch_decode<D, 3, 2>(p, st);
    case 33: return launch_decode<D, 3, 3>(p, st);
    case 34: return launch_decode<D, 3, 4>(p, st);
    case 42: return launch_decode<D, 4, 2>(p, st);
    case 43: return launch_decode<D, 4, 3>(p, st);
    default: return launch_decode<D, 4, 4>(p, st);
  }
}

}  // namespace akv

using namespace akv;

// Upper bound on the split count of plan_decode for any record size: the warm
// and hot shares of the largest candidate round to at most hi + 1 splits.
static int max_splits(int B, int Hq, int Hkv, int D, int n_hot, int n_warm_blocks) {
  const int g = Hq / Hkv;
  const int units = B * Hkv * ((g + 7) / 8);
  int lo, hi;
  per_unit_range(units, n_warm_blocks + (n_hot + 31) / 32, decode_slots(D), lo, hi);
  const int cap = n_warm_blocks + (n_hot + 31) / 32;
  return max(1, min(hi + 2, cap));
}

extern "C" size_t akv_decode_workspace_bytes(int B, int Hq, int Hkv, int D, int n_hot, int n_warm_blocks) {
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv || !decode_head_dim_ok(D) || n_hot < 0 || n_warm_blocks < 0)
    return 0;
  return static_cast<size_t>(B) * Hq * max_splits(B, Hq, Hkv, D, n_hot, n_warm_blocks) * (D + 2) * sizeof(float);
}

// Shared body of akv_mixed_decode (btab == nullptr: row b's records are
// contiguous at warm + b*w_sb + kvh*w_sh) and akv_mixed_decode_paged (row b's
// block blk is the record at warm + btab[b*bt_sb + blk]*w_page + kvh*w_sh).
static int decode_impl(const uint16_t* q, int64_t q_sb, int64_t q_sh, const uint16_t* hot_k, const uint16_t* hot_v,
                       int64_t h_sb, int64_t h_sh, int64_t h_sn, int n_hot, const int32_t* hot_len,
                       const uint8_t* warm, int64_t w_sb, int64_t w_sh, const int32_t* btab, int64_t bt_sb,
                       int64_t w_page, int n_pages, const akv_warm_layout* layout, int n_warm_blocks, const int32_t* warm_len,
                       int B, int Hq, int Hkv, int D, float sm_scale, uint16_t* out, int64_t o_sb, int64_t o_sh,
                       float* lse, float* partial_out, void* workspace, size_t workspace_bytes, int* status,
                       void* stream) {
  if (!q || (!out && !partial_out)) return AKV_ERR_NULL;
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv || n_hot < 0 || n_warm_blocks < 0) return AKV_ERR_SHAPE;
  if (!decode_head_dim_ok(D)) return AKV_ERR_UNSUPPORTED;
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
    if (L.bytes % 16 || !al(warm, 16) || w_sb % 16 || w_sh % 16 || w_page % 16) return AKV_ERR_ALIGN;
    if (btab && (bt_sb < n_warm_blocks || w_page <= 0 || n_pages <= 0)) return AKV_ERR_SHAPE;
    // the kernel addresses record fields at the offsets akv_warm_layout_init gives
    const RecLayout R = rec_layout(D, L.key_bits, L.value_bits, L.n_outlier);
    if (L.kc != R.kc || L.vc != R.vc || L.ks != R.ks || L.kz != R.kz || L.vs != R.vs || L.vz != R.vz ||
        L.mask != R.mask || L.flags != R.flags || L.ki != R.ki || L.vi != R.vi || L.ko != R.ko || L.vo != R.vo ||
        L.vd != R.vd || L.bytes != R.bytes)
      return AKV_ERR_UNSUPPORTED;
  }
  if (!workspace) return AKV_ERR_NULL;
  const DecodePlan pl = plan_decode(B, Hq, Hkv, D, n_hot, n_warm_blocks, n_warm_blocks > 0 ? L.bytes : 1);
  const int splits = max(pl.splits, 1);
  if (splits > max_splits(B, Hq, Hkv, D, n_hot, n_warm_blocks)) return AKV_ERR_UNSUPPORTED;  // planner invariant
  const size_t need = static_cast<size_t>(B) * Hq * splits * (D + 2) * sizeof(float);
  if (workspace_bytes < need || !al(workspace, 16)) return AKV_ERR_WORKSPACE;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  float* ws = static_cast<float*>(workspace);
  __half* outh = reinterpret_cast<__half*>(out);
  if (pl.splits == 0) {  // no tokens at all: a zeroed partial (m = 0, l = 0) combines to output 0, lse -inf
    if (cudaMemsetAsync(ws, 0, need, st) != cudaSuccess) return AKV_ERR_LAUNCH;
    lse_combine_kernel<<<combine_grid(B * Hq, D), kCombineThreads, 0, st>>>(ws, D + 2, D + 2, B * Hq, 1, D, outh, o_sh, lse, partial_out);
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
  p.btab = btab;
  p.bt_sb = bt_sb;
  p.w_page = w_page;
  p.n_pages = n_pages;
  p.L = L;
  p.n_warm_blocks = n_warm_blocks;
  p.warm_len = warm_len;
  p.B = B;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.g = Hq / Hkv;
  p.n_hg = pl.n_hg;
  p.q_neg = sm_scale < 0.f ? 1 : 0;
  p.scale_log2 = fmaxf(fabsf(sm_scale) * kLog2e, FLT_MIN);
  p.lazy_raw = kLazyMax / p.scale_log2;
  p.warm_splits = pl.warm_splits;
  p.hot_splits = pl.hot_splits;
  p.wbps = pl.wbps;
  p.hbps = pl.hbps;
  p.splits = pl.splits;
  p.ws = ws;
  p.status = status;
  int rc;
  const int kb = n_warm_blocks > 0 ? L.key_bits : 4, vb = n_warm_blocks > 0 ? L.value_bits : 4;
  if (D == 64) rc = launch_decode_bits<64>(p, kb, vb, st);
  else if (D == 256) rc = launch_decode_bits<256>(p, kb, vb, st);
  else rc = launch_decode_bits<128>(p, kb, vb, st);
  if (rc != AKV_OK) return rc;
  return launch_combine_dependent(ws, D + 2, static_cast<int64_t>(pl.splits) * (D + 2), B * Hq, pl.splits, D, outh,
                                  o_sh, lse, partial_out, st);
}

extern "C" int akv_mixed_decode(const uint16_t* q, int64_t q_sb, int64_t q_sh, const uint16_t* hot_k,
                                const uint16_t* hot_v, int64_t h_sb, int64_t h_sh, int64_t h_sn, int n_hot,
                                const int32_t* hot_len, const uint8_t* warm, int64_t w_sb, int64_t w_sh,
                                const akv_warm_layout* layout, int n_warm_blocks, const int32_t* warm_len, int B,
                                int Hq, int Hkv, int D, float sm_scale, uint16_t* out, int64_t o_sb,
                                int64_t o_sh, float* lse, float* partial_out, void* workspace,
                                size_t workspace_bytes, int* status, void* stream) {
  return decode_impl(q, q_sb, q_sh, hot_k, hot_v, h_sb, h_sh, h_sn, n_hot, hot_len, warm, w_sb, w_sh, nullptr, 0, 0, 0,
                     layout, n_warm_blocks, warm_len, B, Hq, Hkv, D, sm_scale, out, o_sb, o_sh, lse, partial_out,
                     workspace, workspace_bytes, status, stream);
}

extern "C" int akv_mixed_decode_args(const akv_decode_args* a, void* stream) {
  if (!a) return AKV_ERR_NULL;
  const size_t need = akv_decode_workspace_bytes(a->B, a->Hq, a->Hkv, a->D, a->n_hot, a->n_warm_blocks);
  if (need == 0) return decode_head_dim_ok(a->D) ? AKV_ERR_SHAPE : AKV_ERR_UNSUPPORTED;
  if (a->workspace_bytes < need) {
    if (a->workspace_need) *a->workspace_need = need;
    return AKV_ERR_WORKSPACE;
  }
  return akv_mixed_decode(a->q, a->q_sb, a->q_sh, a->hot_k, a->hot_v, a->h_sb, a->h_sh, a->h_sn, a->n_hot, a->hot_len,
                          a->warm, a->w_sb, a->w_sh, a->layout, a->n_warm_blocks, a->warm_len, a->B, a->Hq, a->Hkv,
                          a->D, a->sm_scale, a->out, a->o_sb, a->o_sh, a->lse, a->partial_out, a->workspace,
                          a->workspace_bytes, a->status, stream);
}

extern "C" int akv_mixed_decode_paged(const uint16_t* q, int64_t q_sb, int64_t q_sh, const uint16_t* hot_k,
                                      const uint16_t* hot_v, int64_t h_sb, int64_t h_sh, int64_t h_sn, int n_hot,
                                      const int32_t* hot_len, const uint8_t* pool, int n_pages,
                                      int64_t page_stride, int64_t head_stride, const int32_t* block_table,
                                      int64_t bt_stride,
                                      const akv_warm_layout* layout, int max_blocks, const int32_t* warm_len, int B,
                                      int Hq, int Hkv, int D, float sm_scale, uint16_t* out, int64_t o_sb,
                                      int64_t o_sh, float* lse, float* partial_out, void* workspace,
                                      size_t workspace_bytes, int* status, void* stream) {
  if (max_blocks > 0 && !block_table) return AKV_ERR_NULL;
  return decode_impl(q, q_sb, q_sh, hot_k, hot_v, h_sb, h_sh, h_sn, n_hot, hot_len, pool, 0, head_stride,
                     block_table, bt_stride, page_stride, n_pages, layout, max_blocks, warm_len, B, Hq, Hkv, D, sm_scale, out,
                     o_sb, o_sh, lse, partial_out, workspace, workspace_bytes, status, stream);
}

extern "C" int akv_lse_combine(const float* part, int64_t part_ss, int64_t part_sr, int rows, int splits, int D,
                               uint16_t* out, int64_t o_sr, float* lse, float* merged, void* stream) {
  if (!part || (!out && !lse && !merged)) return AKV_ERR_NULL;
  if (rows <= 0 || splits <= 0 || D <= 0 || part_ss < 0 || part_sr < 0) return AKV_ERR_SHAPE;
  lse_combine_kernel<<<combine_grid(rows, D), kCombineThreads, 0, static_cast<cudaStream_t>(stream)>>>(
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
// Device address of g_noalloc_scratch per device, looked up once per device
// under a std::once_flag, so first calls from several host threads are safe.
static void* g_noalloc_ptr[kMaxDevices];
static int g_noalloc_rc[kMaxDevices];
static std::once_flag g_noalloc_once[kMaxDevices];
}  // namespace akv

extern "C" int akv_mixed_decode_noalloc(const uint16_t* q, int64_t q_sb, int64_t q_sh, const uint16_t* hot_k,
                                        const uint16_t* hot_v, int64_t h_sb, int64_t h_sh, int64_t h_sn, int n_hot,
                                        const int32_t* hot_len, const uint8_t* warm, int64_t w_sb, int64_t w_sh,
                                        const akv_warm_layout* layout, int n_warm_blocks, const int32_t* warm_len,
                                        int B, int Hq, int Hkv, int D, float sm_scale, uint16_t* out, int64_t o_sb,
                                        int64_t o_sh, float* lse, float* partial_out, int* status, void* stream) {
  const size_t need = akv_decode_workspace_bytes(B, Hq, Hkv, D, n_hot, n_warm_blocks);
  if (need == 0) return !decode_head_dim_ok(D) ? AKV_ERR_UNSUPPORTED : AKV_ERR_SHAPE;
  if (need > kNoAllocScratchBytes) return AKV_ERR_WORKSPACE;  // beyond the fixed scratch array
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return AKV_ERR_LAUNCH;
  // one-time set-up per device, with that device current: the host-side name
  // g_noalloc_scratch is not a device address, so ask the runtime for it
  std::call_once(g_noalloc_once[dev], [dev] {
    void* p = nullptr;
    const bool ok = cudaGetSymbolAddress(&p, g_noalloc_scratch) == cudaSuccess && p;
    g_noalloc_ptr[dev] = ok ? p : nullptr;
    g_noalloc_rc[dev] = ok ? AKV_OK : AKV_ERR_LAUNCH;
  });
  if (g_noalloc_rc[dev] != AKV_OK) return g_noalloc_rc[dev];
  return akv_mixed_decode(q, q_sb, q_sh, hot_k, hot_v, h_sb, h_sh, h_sn, n_hot, hot_len, warm, w_sb, w_sh, layout,
                          n_warm_blocks, warm_len, B, Hq, Hkv, D, sm_scale, out, o_sb, o_sh, lse, partial_out,
                          g_noalloc_ptr[dev], kNoAllocScratchBytes, status, stream);
}
