// Block-affine quantise + bit-pack (warm-tier demotion) and its inverse.
//
// Numerics follow the reference quantiser op by op
// (akv/affine_quantizer.py:63-110 keys, :131-176 values):
//   scale = fp16(fp16(max - min) / maxval)      zero = min
//   code  = clamp(rint(fp16(fp16(x - zero) / scale)), 0, maxval), NaN -> 0
// Every fp16 op is an fp32 op rounded to fp16 (RNE); for + - * / that equals
// the correctly rounded fp16 op, which is what torch's CPU Half kernels do.
// The clamp(min=1e-8) of the reference is a no-op in fp16 (1e-8 underflows
// to 0), so a zero-range group keeps scale 0 and its 0/0 codes become 0.
//
// One CTA quantises one scale group (all heads of one batch row, up to three
// CTAs per SM): 1-D bulk TMA stages the group's fp16 rows in shared memory
// (one copy per head when the rows are contiguous, one per row for a gather),
// one pass over the columns yields the outlier norms and the key min/max, a
// pass over the rows yields the value min/max, and the encode pass turns 8
// channels of one token into BITS packed bytes per work item.  The division
// is exact without a divide, by Markstein's FMA remainder correction of a
// quotient estimate (P. Markstein, "Computation of elementary functions on
// the IBM RISC System/6000 processor", IBM J. Res. Dev. 34(1), 1990): with
// r = RN(1/s) precomputed per scale,
//   q0 = x*r,  e = fma(-s, q0, x),  q = fma(e, r, q0)   (packed fp32x2 ops)
// equals RN(x/s) for every pair of non-negative finite fp16 x and s (checked
// exhaustively against double division, all 2^30 pairs).  fp16(q) + 1024 in
// fp16 is 1024 + rint(fp16(q)) with ties to even, so one packed fp16 add
// rounds, and a max/min pair clamps (max(NaN, 1024) = 1024: NaN -> code 0).
#include <cuda_runtime.h>

#include <algorithm>

#include "common.cuh"

namespace akv {

struct QuantParams {
  const __half* src;
  int64_t sb, sh, sn;
  const int64_t* tok_idx;
  int64_t tok_sb;
  int64_t n_src;  // rows in the source: a tok_idx entry outside [0, n_src) records AKV_ERR_SHAPE, reads row 0
  int B, H, N, D, bits, is_key, group, n_out;
  akv_qdest dst;
  int* status;
  // chunked path (groups too large for one CTA): per-chunk partials and the
  // per-group results of the reduction, see QuantWs
  int n_chunks, n_groups, heads_per_cta;
  __half* ws_min;    // [B][n_chunks][H][D]
  __half* ws_max;    // [B][n_chunks][H][D]
  float* ws_sq;      // [B][n_chunks][H][D]   sum of squares
  __half* ws_zero;   // [B][n_groups][H][D]   keys: zero (min), outlier channels 0
  __half* ws_scale;  // [B][n_groups][H][D]   keys: scale
  int* ws_oidx;      // [B][n_groups][kMaxOutliersWs]
  // outlier scores from outside (heads sharded over GPUs): per (b, group) the
  // sum over ALL heads of the per-(head, channel) L2 norms, [B][n_groups][D];
  // score = score_sum / score_heads.  NULL: computed from this call's heads.
  const float* score_sum;
  int score_heads;
  float* norm_sums_out;  // akv_outlier_norm_sums: write [B][n_groups][D] sums over this call's heads
};

constexpr int kMaxOutliersWs = 32;
enum QuantMode { kQuantFull = 0, kQuantStats = 1, kQuantEncode = 2 };

constexpr int kQuantThreads = 256;
constexpr int kQuantCtasPerSm = 3;
constexpr int kMaxOutliers = 32;
constexpr int kEncChunk = 8;               // channels per encode work item (one 16-byte shared load)
constexpr float kZeroScale = 0x1p-100f;    // stands in for scale 0: x > 0 -> beyond fp16 -> maxval; 0 -> 0
constexpr uint32_t kMagic2 = 0x64006400u;  // (1024, 1024) as fp16x2

AKV_DEV char* vaddr(const akv_view& v, int b, int h, int blk, int slot) {
  return static_cast<char*>(v.ptr) + b * v.sb + h * v.sh + blk * v.sblk + slot * v.sslot;
}

// fp16 scale -> (s_eff, RN(1/s_eff)) for the exact division below.
AKV_DEV float scale_eff(__half s) {
  const float f = __half2float(s);
  return f == 0.f ? kZeroScale : f;
}

// RN(x / s) for x = fp16 value >= 0, s = scale_eff(), r = RN(1/s).
AKV_DEV float div_exact(float x, float s, float r) {
  const float q0 = __fmul_rn(x, r);
  const float e = __fmaf_rn(-s, q0, x);
  return __fmaf_rn(e, r, q0);
}

// Two lanes of div_exact: x2, r2 = (r0, r1), ns2 = (-s0, -s1).
AKV_DEV uint64_t div_exact2(uint64_t x2, uint64_t ns2, uint64_t r2) {
  const uint64_t q0 = f2_mul(x2, r2);
  return f2_fma(f2_fma(ns2, q0, x2), r2, q0);
}

// RN(1/s) for s an fp16 value or kZeroScale: one Newton-Raphson step
// y' = y + y*(1 - s*y) (residual by FMA, as in Markstein's method above) from
// the hardware approximation (within 1 ulp) lands on the correctly rounded
// reciprocal for every such s (checked exhaustively from starts up to 3 ulp off).
AKV_DEV float rcp_exact(float s) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(s));
  return __fmaf_rn(__fmaf_rn(-s, y, 1.0f), y, y);
}

// scale = fp16(fp16(hi - lo) / maxval) for two (lo, hi) pairs; the division
// by the constant maxval is div_exact with r = RN(1/maxval).  A range that
// overflowed fp16 stays inf (div_exact would turn inf into NaN).  With scale
// inf the encoder's quotients are NaN, which its clamp maps to code 0, the
// reference's code for x/inf = 0.
template <int BITS>
AKV_DEV __half2 affine_scale2(__half2 lo, __half2 hi) {
  constexpr float kMax = static_cast<float>((1 << BITS) - 1);
  constexpr float kInv = 1.0f / kMax;
  const float2 range = __half22float2(__hsub2_rn(hi, lo));
  const float q0 = range.x == INFINITY ? INFINITY : div_exact(range.x, kMax, kInv);
  const float q1 = range.y == INFINITY ? INFINITY : div_exact(range.y, kMax, kInv);
  return __floats2half2_rn(q0, q1);
}

// Two codes as (1024 + c0, 1024 + c1) fp16x2 ("magic" form: the low byte of
// each half is the code).
template <int BITS>
AKV_DEV uint32_t encode_pair(uint32_t x2, uint32_t z2, uint64_t ns2, uint64_t r2) {
  constexpr uint32_t top = kMagic2 + ((1u << BITS) - 1) * 0x00010001u;
  const float2 d = __half22float2(__hsub2_rn(u32_as_h2(x2), u32_as_h2(z2)));
  const float2 q = f2_split(div_exact2(f2_make(d.x, d.y), ns2, r2));
  __half2 h = __floats2half2_rn(q.x, q.y);
  h = __hadd2_rn(h, u32_as_h2(kMagic2));
  h = __hmin2(__hmax2(h, u32_as_h2(kMagic2)), u32_as_h2(top));
  return h2_as_u32(h);
}

template <int BITS>
AKV_DEV uint32_t encode_one(__half x, __half z, float s, float r) {
  const float d = __half2float(__hsub_rn(x, z));
  __half h = __hadd_rn(__float2half_rn(div_exact(d, s, r)), __ushort_as_half(0x6400));
  h = __hmin(__hmax(h, __ushort_as_half(0x6400)), __ushort_as_half(0x6400 + (1 << BITS) - 1));
  return __half_as_ushort(h) & 0xFFu;
}

// fp16 path.  For a scale s with 0 < s < 16384 and s * 2^15 >= 1/8, let
// m = 2^k scale s into s' = s*m in [1/8, 16384), ns = -s', r = RN16(1/s').
// Then  d = fp16(x - z) * m (exact),  q0 = fp16(d*r),  e = fma16(ns, q0, d),
// q = fma16(e, r, q0)  rounds (via + 1024) to the reference code for every fp16
// d and maxval 3, 7, 15 (checked exhaustively over all such s; the quotient q
// itself can be 1 ulp off, never across a rounding boundary of the code).  q
// is never negative or NaN there, so one min clamps.  Scale 0 also takes the
// fp16 path: it means max - min <= 7 * 2^-24, so every d is 0 or a few
// subnormal steps, and m = 2^15, ns = 0, r = 65504 send d > 0 past maxval and
// d = 0 to 0 (the reference's x/0 = inf and 0/0 = NaN -> 0).  Other scales
// (inf, >= 16384, < 2^-18) take the fp32 path.
AKV_DEV bool fast_coef(__half s, __half& m, __half& ns, __half& r) {
  const float f = __half2float(s);
  if (f == 0.f) {
    m = __ushort_as_half(0x7800);   // 2^15
    ns = __ushort_as_half(0);
    r = __ushort_as_half(0x7BFF);   // 65504
    return true;
  }
  if (!(f > 0.f && f < 16384.f)) return false;
  const int e = static_cast<int>((__float_as_uint(f) >> 23) & 0xFF) - 127;  // floor(log2 s)
  const int k = max(0, -3 - e);
  if (k > 15) return false;
  const float sp = f * __uint_as_float(static_cast<uint32_t>(k + 127) << 23);  // exact
  m = __ushort_as_half(static_cast<unsigned short>((k + 15) << 10));
  ns = __float2half_rn(-sp);
  r = __float2half_rn(rcp_exact(sp));  // RN16(RN32(1/s')) == RN16(1/s')
  return true;
}

// UNIT: every multiplier m of the group is 1 (all scales >= 1/8), so d needs no rescale.
template <int BITS, bool UNIT = false>
AKV_DEV uint32_t encode_pair16(uint32_t x2, uint32_t z2, uint32_t m2, uint32_t ns2, uint32_t r2) {
  constexpr uint32_t top = kMagic2 + ((1u << BITS) - 1) * 0x00010001u;
  const __half2 x_z = __hsub2_rn(u32_as_h2(x2), u32_as_h2(z2));
  const __half2 d = UNIT ? x_z : __hmul2_rn(x_z, u32_as_h2(m2));
  const __half2 q0 = __hmul2_rn(d, u32_as_h2(r2));
  const __half2 q = __hfma2(__hfma2(u32_as_h2(ns2), q0, d), u32_as_h2(r2), q0);
  return h2_as_u32(__hmin2(__hadd2_rn(q, u32_as_h2(kMagic2)), u32_as_h2(top)));
}

// 8 codes in magic form (m[i] = channels 2i, 2i+1) -> packed bytes (akv/bitpack.py):
//   4 bits: 4 bytes, even channel in the high nibble;
//   2 bits: 2 bytes (low half), first channel in the two high bits;
//   3 bits: one 24-bit big-endian group in bytes 0..2.
template <int BITS>
AKV_DEV uint32_t pack8(const uint32_t (&m)[4]) {
  if constexpr (BITS == 4) {
    const uint32_t va = prmt(m[0], m[1], 0x6420), vb = prmt(m[2], m[3], 0x6420);  // bytes = codes
    const uint32_t ta = ((va << 4) & 0x00F000F0u) | ((va >> 8) & 0x000F000Fu);
    const uint32_t tb = ((vb << 4) & 0x00F000F0u) | ((vb >> 8) & 0x000F000Fu);
    return prmt(ta, tb, 0x6420);
  } else if constexpr (BITS == 2) {
    // bytes (c0, c1, c2, c3) * (2^30 + 2^20 + 2^10 + 1): the top byte collects
    // c0<<6 | c1<<4 | c2<<2 | c3 and the cross terms stay below bit 24
    const uint32_t pa = prmt(m[0], m[1], 0x6420) * 0x40100401u;
    const uint32_t pb = prmt(m[2], m[3], 0x6420) * 0x40100401u;
    return prmt(pa, pb, 0x4473);
  } else {
    uint32_t w = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) w |= ((m[i] & 7u) << (21 - 6 * i)) | (((m[i] >> 16) & 7u) << (18 - 6 * i));
    return prmt(w, 0u, 0x4012);
  }
}

template <int BITS>
AKV_DEV void store_packed8(char* p, uint32_t w) {
  if constexpr (BITS == 4) {
    *reinterpret_cast<uint32_t*>(p) = w;
  } else if constexpr (BITS == 2) {
    *reinterpret_cast<uint16_t*>(p) = static_cast<uint16_t>(w);
  } else {
    p[0] = static_cast<char>(w);
    p[1] = static_cast<char>(w >> 8);
    p[2] = static_cast<char>(w >> 16);
  }
}

// Runs body(x, c, t) for the tokens t = sub, sub + step, ... < nt of one
// encode work item: x = the item's 8 staged channels of token t, c = where its
// packed codes go (nullptr: codes not written).  Both pointers advance by
// increments; a group longer than one block moves c to the next block record
// each time the slot passes 31.
template <typename Body>
AKV_DEV void walk_tokens(int sub, int nt, int step, const __half* xcol, int D, char* cbase, const akv_view& cv,
                         Body&& body) {
  const __half* x = xcol + sub * D;
  const int xstep = step * D;
  if (!cbase) {
#pragma unroll 4
    for (int t = sub; t < nt; t += step, x += xstep) body(x, static_cast<char*>(nullptr), t);
    return;
  }
  char* c = cbase + (sub >> 5) * cv.sblk + (sub & 31) * cv.sslot;
  const int64_t cstep = static_cast<int64_t>(step) * cv.sslot;
  if (nt <= kBlockTokens) {  // one block record
#pragma unroll 4
    for (int t = sub; t < nt; t += step, x += xstep, c += cstep) body(x, c, t);
    return;
  }
  const int64_t cwrap = cv.sblk - kBlockTokens * cv.sslot;
  int slot = sub & 31;
  for (int t = sub; t < nt; t += step, x += xstep, c += cstep) {
    body(x, c, t);
    for (slot += step; slot >= kBlockTokens; slot -= kBlockTokens) c += cwrap;
  }
}

template <int BITS>
AKV_DEV void unpack32(const uint32_t (&w)[BITS], uint32_t (&c)[32]) {
  if constexpr (BITS == 4) {
#pragma unroll
    for (int k = 0; k < 4; ++k)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint32_t byte = (w[k] >> (8 * i)) & 0xFF;
        c[8 * k + 2 * i] = byte >> 4;
        c[8 * k + 2 * i + 1] = byte & 0xF;
      }
  } else if constexpr (BITS == 2) {
#pragma unroll
    for (int k = 0; k < 2; ++k)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint32_t byte = (w[k] >> (8 * i)) & 0xFF;
#pragma unroll
        for (int j = 0; j < 4; ++j) c[16 * k + 4 * i + j] = (byte >> (6 - 2 * j)) & 3;
      }
  } else {
    uint32_t bytes[12];
#pragma unroll
    for (int k = 0; k < 3; ++k)
#pragma unroll
      for (int i = 0; i < 4; ++i) bytes[4 * k + i] = (w[k] >> (8 * i)) & 0xFF;
#pragma unroll
    for (int gq = 0; gq < 4; ++gq) {
      const uint32_t word = (bytes[3 * gq] << 16) | (bytes[3 * gq + 1] << 8) | bytes[3 * gq + 2];
#pragma unroll
      for (int j = 0; j < 8; ++j) c[8 * gq + j] = (word >> (21 - 3 * j)) & 7;
    }
  }
}

template <int BITS>
AKV_DEV void load_words(const char* p, uint32_t (&w)[BITS]) {
#pragma unroll
  for (int k = 0; k < BITS; ++k) w[k] = reinterpret_cast<const uint32_t*>(p)[k];
}

// Column statistics of one stats work item: 8 channels over n staged tokens
// `stride` halves apart: sums of squares (fp32, for the outlier norms) and,
// for keys, min / max.
template <bool IS_KEY, bool NORMS>
AKV_DEV void column_stats(const __half* x, int n, int stride, uint64_t (&s2)[4], __half2 (&mn)[4], __half2 (&mx)[4]) {
#pragma unroll 4
  for (int t = 0; t < n; ++t, x += stride) {
    const uint4 v = lds_v4(x);
    const uint32_t x4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const __half2 xh = u32_as_h2(x4[i]);
      if constexpr (NORMS) {
        const float2 f = __half22float2(xh);
        const uint64_t f2 = f2_make(f.x, f.y);
        s2[i] = f2_fma(f2, f2, s2[i]);
      }
      if constexpr (IS_KEY) {
        mn[i] = __hmin2(mn[i], xh);
        mx[i] = __hmax2(mx[i], xh);
      }
    }
  }
}

// Shared memory of one quantiser CTA (byte offsets; rows = H * nt):
//   xs    [rows][D]   fp16  the group's tokens (outlier channels zeroed later)
//   cz    [H][D]      fp16  keys: column min (= zero)
//   cs    [H][D]      fp16  keys: column max, then scale
//   co    keys:   km, kns, kr [H][D/2] fp16x2: fp16-path m, -s', 1/s' per channel pair
//         values: [rows] 16-byte records {z | m, -s' | 1/s' (fp16), -s_eff, 1/s_eff (fp32)}
//         -- shares its space with norms [H][D] fp32 and score [D] fp32, dead by then
//   oidx  [kMaxOutliers] int
//   flg   [H][nblk] u32  nonzero once a scale of that (head, block) is outside
//                        the decode's two-op dequantisation range
struct QuantSmem {
  size_t cz, cs, co, score, oidx, flg, total;
};

__host__ __device__ inline QuantSmem quant_smem_layout(int H, int nt, int D, int n_out, bool is_key) {
  QuantSmem m{};
  const size_t rows = static_cast<size_t>(H) * nt, hd = static_cast<size_t>(H) * D;
  const size_t kz = is_key ? hd : 0;
  m.cz = rows * D * 2;
  m.cs = m.cz + kz * 2;
  m.co = (m.cs + kz * 2 + 15) & ~static_cast<size_t>(15);
  const size_t cob = is_key ? hd * 6 : rows * 16;
  const size_t nsb = hd * 4 + static_cast<size_t>(D) * 4;
  m.score = m.co + hd * 4;
  m.oidx = m.co + (cob > nsb ? cob : nsb);
  m.flg = m.oidx + kMaxOutliers * 4;
  m.total = m.flg + static_cast<size_t>(H) * ((nt + kBlockTokens - 1) / kBlockTokens) * 4;
  return m;
}

// ---------------------------------------------------------------------------
// quantise.  MODE kQuantFull: grid (n_groups, B), one CTA per scale group
// (all heads).  Groups too large for one CTA take the chunked path: MODE
// kQuantStats (grid (n_chunks, B, head groups)) writes per-32-token-chunk
// column partials, quant_reduce_kernel turns them into the group's outlier
// channels and key scales, and MODE kQuantEncode (same grid) encodes each
// chunk with them.
// ---------------------------------------------------------------------------
// The CTA body, with its grid coordinates as arguments so that a fused
// kernel can run it for more than one tensor (demote_install_kernel).
// Returns false when the staging copy timed out (status set, nothing written).
template <int BITS, bool IS_KEY, int MODE>
__device__ __forceinline__ bool quantize_group_body(const QuantParams& p, int bx, int by, int bz,
                                                    unsigned char* smem_raw) {
  const int tid = threadIdx.x;
  const int b = by;
  const int t0 = MODE == kQuantFull ? bx * p.group : bx * kBlockTokens;  // multiple of 32, or 0
  const int chunk = bx;
  const int grp = t0 / p.group;
  const int h0 = MODE == kQuantFull ? 0 : bz * p.heads_per_cta;  // first head of this CTA
  const int blk0 = t0 / kBlockTokens;
  const int nt = MODE == kQuantFull ? min(p.group, p.N - t0) : min(kBlockTokens, p.N - t0);
  const int nblk = (nt + kBlockTokens - 1) / kBlockTokens;
  const int H = MODE == kQuantFull ? p.H : min(p.heads_per_cta, p.H - h0);  // heads in this CTA
  const int D = p.D, D2 = D / 2;
  const int rows = H * nt;
  const QuantSmem lay = quant_smem_layout(H, nt, D, p.n_out, IS_KEY);

  __half* xs = reinterpret_cast<__half*>(smem_raw);
  __half* cz = reinterpret_cast<__half*>(smem_raw + lay.cz);
  __half* cs = reinterpret_cast<__half*>(smem_raw + lay.cs);
  float* norms = reinterpret_cast<float*>(smem_raw + lay.co);
  float* score = reinterpret_cast<float*>(smem_raw + lay.score);
  uint32_t* km = reinterpret_cast<uint32_t*>(smem_raw + lay.co);  // keys
  uint32_t* kns = km + H * D2;
  uint32_t* kr = kns + H * D2;
  uint4* vco = reinterpret_cast<uint4*>(smem_raw + lay.co);       // values
  int* oidx = reinterpret_cast<int*>(smem_raw + lay.oidx);
  uint32_t* flg = reinterpret_cast<uint32_t*>(smem_raw + lay.flg);
  if (MODE != kQuantStats)
    for (int i = tid; i < H * nblk; i += kQuantThreads) flg[i] = 0;  // ordered by the staging barrier below

  // ---- stage the group's rows with 1-D bulk TMA (warp 0 issues, all wait)
  __shared__ __align__(8) uint64_t stage_bar;
  if (tid == 0) {
    mbar_init(&stage_bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (tid < 32) {
    if (tid == 0) mbar_arrive_expect_tx(&stage_bar, static_cast<uint32_t>(rows) * D * 2);
    __syncwarp();
    if (!p.tok_idx && p.sn == D) {  // each head's nt rows are one contiguous run
      for (int h = tid; h < H; h += 32)
        tma_load_1d(xs + h * nt * D, p.src + b * p.sb + (h0 + h) * p.sh + static_cast<int64_t>(t0) * D,
                    static_cast<uint32_t>(nt) * D * 2, &stage_bar);
    } else {
      for (int r = tid; r < rows; r += 32) {
        const int t = r % nt, h = r / nt;
        int64_t row = p.tok_idx ? p.tok_idx[b * p.tok_sb + t0 + t] : static_cast<int64_t>(t0 + t);
        if (p.tok_idx && static_cast<uint64_t>(row) >= static_cast<uint64_t>(p.n_src)) {
          set_status(p.status, AKV_ERR_SHAPE);
          row = 0;
        }
        tma_load_1d(xs + r * D, p.src + b * p.sb + (h0 + h) * p.sh + row * p.sn, D * 2, &stage_bar);
      }
    }
  }
  {
    const bool ok = mbar_wait(&stage_bar, 0, p.status);
    if (__syncthreads_or(!ok)) {  // timed out: let the copies land (bounded), then give up
      if (!ok) mbar_wait(&stage_bar, 0, p.status);
      return false;
    }
  }

  // ---- column statistics: outlier norms (affine_quantizer.py:75-85 / :143-151)
  //      and, for keys, the per-(head, channel) min/max.  A work item is 8
  //      channels of one head; two neighbouring lanes split its tokens.
  const int ncs = D / kEncChunk;
  const bool want_norms = p.n_out > 0 && !p.score_sum;  // this CTA computes outlier norms
  if (MODE == kQuantStats || (MODE == kQuantFull && (want_norms || IS_KEY))) {
    const int items = H * ncs * 2;
    for (int w0 = 0; w0 < items; w0 += kQuantThreads) {
      const int w = w0 + tid;
      const bool act = w < items;
      const unsigned mask = __ballot_sync(0xffffffffu, act);
      if (!act) continue;
      const int half = w & 1, col = w >> 1;
      const int h = col / ncs, c8 = col % ncs;
      const __half* base = xs + h * nt * D + c8 * kEncChunk;
      uint64_t s2[4];
      __half2 mn[4], mx[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        s2[i] = f2_make(0.f, 0.f);
        mn[i] = __float2half2_rn(INFINITY);
        mx[i] = __float2half2_rn(-INFINITY);
      }
      if (want_norms)
        column_stats<IS_KEY, true>(base + half * D, (nt - half + 1) >> 1, 2 * D, s2, mn, mx);
      else
        column_stats<IS_KEY, false>(base + half * D, (nt - half + 1) >> 1, 2 * D, s2, mn, mx);
      float s[8];
      if (want_norms) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 f = f2_split(s2[i]);
          s[2 * i] = f.x + __shfl_xor_sync(mask, f.x, 1);
          s[2 * i + 1] = f.y + __shfl_xor_sync(mask, f.y, 1);
        }
      }
      if constexpr (IS_KEY) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          mn[i] = __hmin2(mn[i], u32_as_h2(__shfl_xor_sync(mask, h2_as_u32(mn[i]), 1)));
          mx[i] = __hmax2(mx[i], u32_as_h2(__shfl_xor_sync(mask, h2_as_u32(mx[i]), 1)));
        }
      }
      if (MODE == kQuantStats && half == 0) {  // this chunk's partials
        const size_t o = ((static_cast<size_t>(b) * p.n_chunks + chunk) * p.H + h0 + h) * D + c8 * kEncChunk;
        if (want_norms) {
#pragma unroll
          for (int i = 0; i < 8; ++i) p.ws_sq[o + i] = s[i];
        }
        if constexpr (IS_KEY) {
          *reinterpret_cast<uint4*>(p.ws_min + o) =
              make_uint4(h2_as_u32(mn[0]), h2_as_u32(mn[1]), h2_as_u32(mn[2]), h2_as_u32(mn[3]));
          *reinterpret_cast<uint4*>(p.ws_max + o) =
              make_uint4(h2_as_u32(mx[0]), h2_as_u32(mx[1]), h2_as_u32(mx[2]), h2_as_u32(mx[3]));
        }
      }
      if (MODE == kQuantFull && half == 0) {
        const int c0 = h * D + c8 * kEncChunk;
        if (want_norms) {
#pragma unroll
          for (int i = 0; i < 8; ++i) norms[c0 + i] = sqrtf(s[i]);
        }
        if constexpr (IS_KEY) {
          *reinterpret_cast<uint4*>(cz + c0) =
              make_uint4(h2_as_u32(mn[0]), h2_as_u32(mn[1]), h2_as_u32(mn[2]), h2_as_u32(mn[3]));
          *reinterpret_cast<uint4*>(cs + c0) =
              make_uint4(h2_as_u32(mx[0]), h2_as_u32(mx[1]), h2_as_u32(mx[2]), h2_as_u32(mx[3]));
        }
      }
    }
    __syncthreads();
  }
  if constexpr (MODE == kQuantStats) return true;

  // ---- outlier channels: score = mean over heads of the norms, top-n
  //      (chunked path: the reduction kernel chose them for the whole group)
  if (MODE == kQuantEncode && p.n_out > 0) {
    for (int j = tid; j < p.n_out; j += kQuantThreads)
      oidx[j] = p.ws_oidx[(static_cast<size_t>(b) * p.n_groups + grp) * kMaxOutliersWs + j];
  }
  if (MODE == kQuantFull && p.n_out > 0) {
    for (int d = tid; d < D; d += kQuantThreads) {
      if (p.score_sum) {
        score[d] = p.score_sum[(static_cast<size_t>(b) * p.n_groups + grp) * D + d] / static_cast<float>(p.score_heads);
      } else {
        float s = 0.f;
        for (int h = 0; h < H; ++h) s += norms[h * D + d];
        score[d] = s / static_cast<float>(H);
      }
    }
    __syncthreads();
    if (tid < 32) {  // warp 0: top-n, largest first, lower index on ties
      for (int j = 0; j < p.n_out; ++j) {
        float best = -INFINITY;
        int bi = D;
        for (int d = tid; d < D; d += 32) {
          const float s = score[d];
          if (s > best || (s == best && d < bi)) { best = s; bi = d; }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          const float ob = __shfl_xor_sync(0xffffffffu, best, o);
          const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
          if (ob > best || (ob == best && oi < bi)) { best = ob; bi = oi; }
        }
        if (tid == 0) {
          oidx[j] = bi;
          score[bi] = -INFINITY;
        }
        __syncwarp();
      }
    }
  }
  if (p.n_out > 0) {
    __syncthreads();
    // side store: fp16 originals of the outlier channels (then zeroed in the
    // staged rows, affine_quantizer.py:84-85) and their ids
    const akv_view& od = p.dst.out_data;
    for (int r = tid; r < rows; r += kQuantThreads) {
      const int h = r / nt, t = r - (r / nt) * nt;
      __half* orow = od.ptr ? reinterpret_cast<__half*>(vaddr(od, b, h0 + h, blk0 + (t >> 5), t & 31)) : nullptr;
      for (int j = 0; j < p.n_out; ++j) {
        __half* x = xs + r * D + oidx[j];
        if (orow) orow[j] = *x;
        *x = __float2half_rn(0.0f);
      }
    }
    const akv_view& oi = p.dst.out_idx;
    if (oi.ptr) {
      for (int w = tid; w < H * nblk; w += kQuantThreads) {
        int16_t* ids = reinterpret_cast<int16_t*>(vaddr(oi, b, h0 + w / nblk, blk0 + w % nblk, 0));
        for (int j = 0; j < p.n_out; ++j) ids[j] = static_cast<int16_t>(oidx[j]);
      }
    }
    if (IS_KEY && MODE == kQuantFull) {  // a zeroed key column has min = max = 0
      for (int h = tid; h < H; h += kQuantThreads)
        for (int j = 0; j < p.n_out; ++j) cz[h * D + oidx[j]] = cs[h * D + oidx[j]] = __float2half_rn(0.0f);
    }
    __syncthreads();
  }

  bool all_fast = true;  // every scale of the group takes the fp16 path
  bool all_unit = true;  // ... and needs no power-of-two rescale (m = 1)
  if constexpr (IS_KEY) {
    // ---- keys: scale per (head, channel pair); 1/scale for the encoder; the
    //      scale / zero rows of every block record the group covers
    const akv_view& sv = p.dst.scale;
    const akv_view& zv = p.dst.zero;
    for (int w = tid; w < H * D2; w += kQuantThreads) {
      const int h = w / D2, dp = w - h * D2;
      __half2 lo, sc;
      // zero-range columns (max == min, the zeroed outlier channels among
      // them): x - zero is 0 for every token, so any multiplier encodes them
      bool flat0 = false, flat1 = false;
      if constexpr (MODE == kQuantEncode) {
        const size_t o = ((static_cast<size_t>(b) * p.n_groups + grp) * p.H + h0 + h) * D2 + dp;
        lo = reinterpret_cast<const __half2*>(p.ws_zero)[o];
        sc = reinterpret_cast<const __half2*>(p.ws_scale)[o];
        reinterpret_cast<__half2*>(cz)[w] = lo;
      } else {
        lo = reinterpret_cast<const __half2*>(cz)[w];
        const __half2 hi = reinterpret_cast<const __half2*>(cs)[w];
        sc = affine_scale2<BITS>(lo, hi);
        flat0 = __half2float(__low2half(hi)) == __half2float(__low2half(lo));
        flat1 = __half2float(__high2half(hi)) == __half2float(__high2half(lo));
      }
      reinterpret_cast<__half2*>(cs)[w] = sc;
      if (!dq2_scale_ok(__low2half(sc)) || !dq2_scale_ok(__high2half(sc))) flg[h * nblk] = 1u;
      __half m0, n0, r0, m1, n1, r1;
      if (!fast_coef(__low2half(sc), m0, n0, r0)) {
        m0 = n0 = r0 = __ushort_as_half(0);
        all_fast = false;
      }
      if (!fast_coef(__high2half(sc), m1, n1, r1)) {
        m1 = n1 = r1 = __ushort_as_half(0);
        all_fast = false;
      }
      km[w] = h2_as_u32(__halves2half2(m0, m1));
      all_unit = all_unit && ((km[w] & 0xFFFFu) == 0x3C00u || flat0) && ((km[w] >> 16) == 0x3C00u || flat1);
      kns[w] = h2_as_u32(__halves2half2(n0, n1));
      kr[w] = h2_as_u32(__halves2half2(r0, r1));
      if (p.dst.pair_order) {  // warm records: each 32-channel chunk in the decode pair order
        const int c0 = 2 * dp, base = c0 & ~31;
        const int s0 = base + key_pair_slot(BITS, c0 & 31), s1 = base + key_pair_slot(BITS, (c0 + 1) & 31);
        for (int bl = 0; bl < nblk; ++bl) {
          if (sv.ptr) {
            __half* o = reinterpret_cast<__half*>(vaddr(sv, b, h0 + h, blk0 + bl, 0));
            o[s0] = __low2half(sc);
            o[s1] = __high2half(sc);
          }
          if (zv.ptr) {
            __half* o = reinterpret_cast<__half*>(vaddr(zv, b, h0 + h, blk0 + bl, 0));
            o[s0] = __low2half(lo);
            o[s1] = __high2half(lo);
          }
        }
      } else {
        for (int bl = 0; bl < nblk; ++bl) {
          if (sv.ptr) reinterpret_cast<__half2*>(vaddr(sv, b, h0 + h, blk0 + bl, 0))[dp] = sc;
          if (zv.ptr) reinterpret_cast<__half2*>(vaddr(zv, b, h0 + h, blk0 + bl, 0))[dp] = lo;
        }
      }
    }
  } else {
    // ---- values: per-token min/max over D, one thread per row; the 16-byte
    //      chunks are visited from a row-dependent start so that neighbouring
    //      rows hit different banks
    for (int r = tid; r < rows; r += kQuantThreads) {
      const __half* xr = xs + r * D;
      __half2 mn = __float2half2_rn(INFINITY), mx = __float2half2_rn(-INFINITY);
      int c = r % ncs;
      for (int j = 0; j < ncs; ++j) {
        const uint4 v = lds_v4(xr + kEncChunk * c);
        const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          mn = __hmin2(mn, u32_as_h2(w4[i]));
          mx = __hmax2(mx, u32_as_h2(w4[i]));
        }
        c = (c + 1 == ncs) ? 0 : c + 1;
      }
      const __half lo = __hmin(__low2half(mn), __high2half(mn));
      const __half hi = __hmax(__low2half(mx), __high2half(mx));
      const __half sc = __low2half(affine_scale2<BITS>(__half2half2(lo), __half2half2(hi)));
      if (!dq2_scale_ok(sc)) flg[(r / nt) * nblk + ((r % nt) >> 5)] = 1u;
      const float se = scale_eff(sc), rc = rcp_exact(se);
      __half fm, fns, fr;
      if (!fast_coef(sc, fm, fns, fr)) {
        fm = fns = fr = __ushort_as_half(0);
        all_fast = false;
      }
      all_unit = all_unit && __half_as_ushort(fm) == 0x3C00u;
      vco[r] = make_uint4(__half_as_ushort(lo) | (static_cast<uint32_t>(__half_as_ushort(fm)) << 16),
                          __half_as_ushort(fns) | (static_cast<uint32_t>(__half_as_ushort(fr)) << 16),
                          __float_as_uint(-se), __float_as_uint(rc));
      const int h = r / nt, t = r - h * nt;
      const int blk = blk0 + (t >> 5), slot = t & 31;
      if (p.dst.scale.ptr) *reinterpret_cast<__half*>(vaddr(p.dst.scale, b, h0 + h, blk, slot)) = sc;
      if (p.dst.zero.ptr) *reinterpret_cast<__half*>(vaddr(p.dst.zero, b, h0 + h, blk, slot)) = lo;
      // what the zeroed outlier channel dequantises to (attention adds p . (original - this))
      if (p.n_out > 0 && p.dst.out_vdq.ptr) {
        __half* rp = reinterpret_cast<__half*>(vaddr(p.dst.out_vdq, b, h0 + h, blk, slot));
        const uint32_t c0 = encode_one<BITS>(__float2half_rn(0.0f), lo, se, rc);
        const __half deq = __hadd_rn(__hmul_rn(__uint2half_rn(c0), sc), lo);
        for (int j = 0; j < p.n_out; ++j) rp[j] = deq;
      }
    }
  }
  all_fast = __syncthreads_and(all_fast);
  all_unit = __syncthreads_and(all_unit) && all_fast;

  // ---- encode + pack: a work item is 8 channels of one head; its threads walk
  //      the tokens.  Keys keep the 8 channels' coefficients in registers and
  //      take the fp16 path unless one of the 8 scales needs the fp32 path;
  //      values read one 16-byte coefficient record per token.
  {
    const int cols = H * ncs;
    const int tpc = max(1, kQuantThreads / cols);
    const akv_view& cv = p.dst.codes;
    for (int w = tid; w < cols * tpc; w += kQuantThreads) {
      const int col = w % cols, sub = w / cols;
      const int h = col / ncs, c8 = col - h * ncs;
      char* cbase = cv.ptr ? vaddr(cv, b, h0 + h, blk0, 0) + c8 * BITS : nullptr;
      const __half* xcol = xs + h * nt * D + c8 * kEncChunk;
      uint32_t m[4];
      if constexpr (IS_KEY) {
        const int c0 = h * D + c8 * kEncChunk, p0 = c0 / 2;
        uint32_t z2[4], m2[4], ns2[4], r2[4];
        lds_u32x4(cz + c0, z2);
        lds_u32x4(km + p0, m2);
        lds_u32x4(kns + p0, ns2);
        lds_u32x4(kr + p0, r2);
        bool fast = all_fast;
        if (!fast) {
          fast = true;
#pragma unroll
          for (int i = 0; i < 4; ++i) fast = fast && (m2[i] & 0x7FFFu) && (m2[i] & 0x7FFF0000u);
        }
        if (all_unit) {
          walk_tokens(sub, nt, tpc, xcol, D, cbase, cv, [&](const __half* x, char* c, int) {
            uint32_t x2[4], mm[4];
            lds_u32x4(x, x2);
#pragma unroll
            for (int i = 0; i < 4; ++i) mm[i] = encode_pair16<BITS, true>(x2[i], z2[i], m2[i], ns2[i], r2[i]);
            if (c) store_packed8<BITS>(c, pack8<BITS>(mm));
          });
        } else if (fast) {
          walk_tokens(sub, nt, tpc, xcol, D, cbase, cv, [&](const __half* x, char* c, int) {
            uint32_t x2[4], mm[4];
            lds_u32x4(x, x2);
#pragma unroll
            for (int i = 0; i < 4; ++i) mm[i] = encode_pair16<BITS>(x2[i], z2[i], m2[i], ns2[i], r2[i]);
            if (c) store_packed8<BITS>(c, pack8<BITS>(mm));
          });
        } else {
          uint32_t s2[4];
          uint64_t nsf[4], rf[4];
          lds_u32x4(cs + c0, s2);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float s0 = scale_eff(__low2half(u32_as_h2(s2[i]))), s1 = scale_eff(__high2half(u32_as_h2(s2[i])));
            nsf[i] = f2_make(-s0, -s1);
            rf[i] = f2_make(rcp_exact(s0), rcp_exact(s1));
          }
          walk_tokens(sub, nt, tpc, xcol, D, cbase, cv, [&](const __half* x, char* c, int) {
            uint32_t x2[4], mm[4];
            lds_u32x4(x, x2);
#pragma unroll
            for (int i = 0; i < 4; ++i) mm[i] = encode_pair<BITS>(x2[i], z2[i], nsf[i], rf[i]);
            if (c) store_packed8<BITS>(c, pack8<BITS>(mm));
          });
        }
      } else if (all_unit) {
        const uint4* vrow = vco + h * nt;
        walk_tokens(sub, nt, tpc, xcol, D, cbase, cv, [&](const __half* x, char* c, int t) {
          const uint2 rec = *reinterpret_cast<const uint2*>(vrow + t);
          uint32_t x2[4], mm[4];
          lds_u32x4(x, x2);
          const uint32_t z2 = prmt(rec.x, rec.x, 0x1010);
          const uint32_t ns2 = prmt(rec.y, rec.y, 0x1010), r2 = prmt(rec.y, rec.y, 0x3232);
#pragma unroll
          for (int i = 0; i < 4; ++i) mm[i] = encode_pair16<BITS, true>(x2[i], z2, 0u, ns2, r2);
          if (c) store_packed8<BITS>(c, pack8<BITS>(mm));
        });
      } else if (all_fast) {
        const uint4* vrow = vco + h * nt;
        walk_tokens(sub, nt, tpc, xcol, D, cbase, cv, [&](const __half* x, char* c, int t) {
          const uint2 rec = *reinterpret_cast<const uint2*>(vrow + t);
          uint32_t x2[4], mm[4];
          lds_u32x4(x, x2);
          const uint32_t z2 = prmt(rec.x, rec.x, 0x1010), m2 = prmt(rec.x, rec.x, 0x3232);
          const uint32_t ns2 = prmt(rec.y, rec.y, 0x1010), r2 = prmt(rec.y, rec.y, 0x3232);
#pragma unroll
          for (int i = 0; i < 4; ++i) mm[i] = encode_pair16<BITS>(x2[i], z2, m2, ns2, r2);
          if (c) store_packed8<BITS>(c, pack8<BITS>(mm));
        });
      } else {
        for (int t = sub; t < nt; t += tpc) {
          const uint4 rec = vco[h * nt + t];
          uint32_t x2[4];
          lds_u32x4(xcol + t * D, x2);
          const uint32_t z2 = prmt(rec.x, rec.x, 0x1010);
          if (rec.x >> 16) {  // fp16 path
            const uint32_t m2 = prmt(rec.x, rec.x, 0x3232);
            const uint32_t ns2 = prmt(rec.y, rec.y, 0x1010), r2 = prmt(rec.y, rec.y, 0x3232);
#pragma unroll
            for (int i = 0; i < 4; ++i) m[i] = encode_pair16<BITS>(x2[i], z2, m2, ns2, r2);
          } else {
            const uint64_t nsf = f2_make(__uint_as_float(rec.z), __uint_as_float(rec.z));
            const uint64_t rf = f2_make(__uint_as_float(rec.w), __uint_as_float(rec.w));
#pragma unroll
            for (int i = 0; i < 4; ++i) m[i] = encode_pair<BITS>(x2[i], z2, nsf, rf);
          }
          if (cbase) store_packed8<BITS>(cbase + (t >> 5) * cv.sblk + (t & 31) * cv.sslot, pack8<BITS>(m));
        }
      }
    }
  }

  // ---- valid-slot masks and decode flags for the blocks this group wrote
  if (p.dst.mask.ptr || p.dst.flags.ptr) {
    for (int w = tid; w < H * nblk; w += kQuantThreads) {
      const int h = w / nblk, bl = blk0 + w % nblk;
      if (p.dst.mask.ptr) {
        const int lo = max(t0, bl * kBlockTokens) - bl * kBlockTokens;
        const int hi = min(t0 + nt, (bl + 1) * kBlockTokens) - bl * kBlockTokens;  // exclusive
        const uint32_t m = (hi - lo == 32) ? 0xffffffffu : (((1u << (hi - lo)) - 1u) << lo);
        *reinterpret_cast<uint32_t*>(vaddr(p.dst.mask, b, h0 + h, bl, 0)) = m;
      }
      if (p.dst.flags.ptr) {  // keys: one scale row per head for all its blocks
        const uint32_t bad = IS_KEY ? flg[h * nblk] : flg[w];
        *reinterpret_cast<uint8_t*>(vaddr(p.dst.flags, b, h0 + h, bl, 0)) = bad ? 0 : 1;
      }
    }
  }
  return true;
}

template <int BITS, bool IS_KEY, int MODE>
__global__ void __launch_bounds__(kQuantThreads, kQuantCtasPerSm) quantize_group_kernel(const QuantParams p) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  quantize_group_body<BITS, IS_KEY, MODE>(p, blockIdx.x, blockIdx.y, blockIdx.z, smem_raw);
}

// One demote event of a single token per batch row that also puts the new
// token in the freed slot: grid (1, B, 2), z = 0 quantises row b's K source
// row (all heads) into its record and z = 1 the V row, then the CTA writes
// the new token's K (or V) rows over the source row it has just staged (the
// staging wait orders the read before the overwrite; no other CTA reads that
// row).  One launch for what is otherwise two quantiser launches and two
// row copies per decode step.
struct InstallRows {
  const __half* nk;
  int64_t nk_sb, nk_sh;
  const __half* nv;
  int64_t nv_sb, nv_sh;
  int vec16;  // sources and destinations 16-byte aligned with strides in 8-half units
};

template <int KBITS, int VBITS>
__global__ void __launch_bounds__(kQuantThreads, kQuantCtasPerSm) demote_install_kernel(const QuantParams pk,
                                                                                         const QuantParams pv,
                                                                                         const InstallRows ins) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const bool key = blockIdx.z == 0;
  const bool ok = key ? quantize_group_body<KBITS, true, kQuantFull>(pk, 0, blockIdx.y, 0, smem_raw)
                      : quantize_group_body<VBITS, false, kQuantFull>(pv, 0, blockIdx.y, 0, smem_raw);
  if (!ok) return;
  const QuantParams& p = key ? pk : pv;
  const int b = blockIdx.y, D = p.D;
  const __half* src = key ? ins.nk + b * ins.nk_sb : ins.nv + b * ins.nv_sb;
  const int64_t s_sh = key ? ins.nk_sh : ins.nv_sh;
  __half* dst = const_cast<__half*>(p.src) + b * p.sb;
  if (ins.vec16) {
    const int per_row = D / 8;
    for (int i = threadIdx.x; i < p.H * per_row; i += blockDim.x) {
      const int h = i / per_row, c = (i % per_row) * 8;
      *reinterpret_cast<uint4*>(dst + h * p.sh + c) = *reinterpret_cast<const uint4*>(src + h * s_sh + c);
    }
  } else {
    for (int i = threadIdx.x; i < p.H * D; i += blockDim.x) {
      const int h = i / D, c = i % D;
      dst[h * p.sh + c] = src[h * s_sh + c];
    }
  }
}


// ---------------------------------------------------------------------------
// chunked path, step 2: one CTA per (group, b) folds the chunk partials in
// chunk order (a fixed summation order), picks the group's outlier channels
// (mean over all heads of the per-(head, channel) L2 norms, top-n, lower
// index on ties) and, for keys, computes zero / scale per (head, channel)
// with the outlier columns at 0 / 0.  Shared memory: [H][D] fp32 norms, or
// [H][D] fp16 min and max for keys without outliers, plus [D] fp32 scores.
// ---------------------------------------------------------------------------
template <int BITS, bool IS_KEY>
__global__ void __launch_bounds__(kQuantThreads) quant_reduce_kernel(const QuantParams p) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int tid = threadIdx.x;
  const int g = blockIdx.x, b = blockIdx.y;
  const int H = p.H, D = p.D, D2 = D / 2;
  const int c0 = g * p.group / kBlockTokens;
  const int c1 = min(p.n_chunks, ((g + 1) * p.group + kBlockTokens - 1) / kBlockTokens);
  float* norms = reinterpret_cast<float*>(smem_raw);              // [H][D]
  float* score = norms + static_cast<size_t>(H) * D;               // [D]
  __shared__ int oidx[kMaxOutliersWs];
  const size_t rowb = static_cast<size_t>(b) * p.n_chunks;

  if (p.n_out > 0 || p.norm_sums_out) {
    if (!p.score_sum) {
      for (int w = tid; w < H * D; w += kQuantThreads) {
        float sq = 0.f;
        for (int c = c0; c < c1; ++c) sq += p.ws_sq[((rowb + c) * H) * D + w];
        norms[w] = sqrtf(sq);
      }
      __syncthreads();
    }
    for (int d = tid; d < D; d += kQuantThreads) {
      const size_t o = (static_cast<size_t>(b) * p.n_groups + g) * D + d;
      if (p.score_sum) {
        score[d] = p.score_sum[o] / static_cast<float>(p.score_heads);
      } else {
        float s = 0.f;
        for (int h = 0; h < H; ++h) s += norms[h * D + d];
        if (p.norm_sums_out) p.norm_sums_out[o] = s;
        score[d] = s / static_cast<float>(H);
      }
    }
    if (p.norm_sums_out) return;
    __syncthreads();
    if (tid < 32) {
      for (int j = 0; j < p.n_out; ++j) {
        float best = -INFINITY;
        int bi = D;
        for (int d = tid; d < D; d += 32) {
          const float s = score[d];
          if (s > best || (s == best && d < bi)) { best = s; bi = d; }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          const float ob = __shfl_xor_sync(0xffffffffu, best, o);
          const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
          if (ob > best || (ob == best && oi < bi)) { best = ob; bi = oi; }
        }
        if (tid == 0) {
          oidx[j] = bi;
          score[bi] = -INFINITY;
          p.ws_oidx[(static_cast<size_t>(b) * p.n_groups + g) * kMaxOutliersWs + j] = bi;
        }
        __syncwarp();
      }
    }
    __syncthreads();
  }
  if constexpr (IS_KEY) {
    for (int w = tid; w < H * D2; w += kQuantThreads) {
      __half2 mn = __float2half2_rn(INFINITY), mx = __float2half2_rn(-INFINITY);
      for (int c = c0; c < c1; ++c) {
        const size_t o = (rowb + c) * H * D2 + w;
        mn = __hmin2(mn, reinterpret_cast<const __half2*>(p.ws_min)[o]);
        mx = __hmax2(mx, reinterpret_cast<const __half2*>(p.ws_max)[o]);
      }
      const int d0 = 2 * (w % D2);
      for (int j = 0; j < p.n_out; ++j) {  // zeroed outlier column: min = max = 0
        if (oidx[j] == d0) {
          mn = __halves2half2(__float2half_rn(0.f), __high2half(mn));
          mx = __halves2half2(__float2half_rn(0.f), __high2half(mx));
        }
        if (oidx[j] == d0 + 1) {
          mn = __halves2half2(__low2half(mn), __float2half_rn(0.f));
          mx = __halves2half2(__low2half(mx), __float2half_rn(0.f));
        }
      }
      const size_t o = (static_cast<size_t>(b) * p.n_groups + g) * H * D2 + w;
      reinterpret_cast<__half2*>(p.ws_zero)[o] = mn;
      reinterpret_cast<__half2*>(p.ws_scale)[o] = affine_scale2<BITS>(mn, mx);
    }
  }
}

// ---------------------------------------------------------------------------
// dequantise: one thread per (b, h, token, 32-code chunk)
// ---------------------------------------------------------------------------
struct DequantParams {
  akv_qdest src;
  const int64_t* tok_idx;
  int64_t tok_sb;
  int64_t n_src;  // tokens in the source: a tok_idx entry outside [0, n_src) records AKV_ERR_SHAPE, reads token 0
  int B, H, N, D, n_out;
  __half* out;
  int64_t osb, osh, osn;
  int* status;
};

template <int BITS, bool IS_KEY>
__global__ void dequantize_kernel(const DequantParams p) {
  const int nsu = p.D / 32;
  const int64_t total = static_cast<int64_t>(p.B) * p.H * p.N * nsu;
  for (int64_t w = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; w < total;
       w += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int su = static_cast<int>(w % nsu);
    int64_t r = w / nsu;
    const int n = static_cast<int>(r % p.N);
    r /= p.N;
    const int h = static_cast<int>(r % p.H);
    const int b = static_cast<int>(r / p.H);
    int64_t tok = p.tok_idx ? p.tok_idx[b * p.tok_sb + n] : n;
    if (p.tok_idx && static_cast<uint64_t>(tok) >= static_cast<uint64_t>(p.n_src)) {
      set_status(p.status, AKV_ERR_SHAPE);
      tok = 0;
    }
    const int blk = static_cast<int>(tok / kBlockTokens), slot = static_cast<int>(tok % kBlockTokens);
    uint32_t wds[BITS];
    load_words<BITS>(vaddr(p.src.codes, b, h, blk, slot) + su * 4 * BITS, wds);
    uint32_t c[32];
    unpack32<BITS>(wds, c);
    __half o[32];
    if constexpr (IS_KEY) {
      const __half* sc = reinterpret_cast<const __half*>(vaddr(p.src.scale, b, h, blk, 0)) + su * 32;
      const __half* zr = reinterpret_cast<const __half*>(vaddr(p.src.zero, b, h, blk, 0)) + su * 32;
      if (p.src.pair_order) {  // warm records: decode pair order within the chunk
#pragma unroll
        for (int k = 0; k < 32; ++k) {
          const int sl = key_pair_slot(BITS, k);
          o[k] = __hadd_rn(__hmul_rn(__uint2half_rn(c[k]), sc[sl]), zr[sl]);
        }
      } else {
#pragma unroll
        for (int k = 0; k < 32; ++k) o[k] = __hadd_rn(__hmul_rn(__uint2half_rn(c[k]), sc[k]), zr[k]);
      }
    } else {
      const __half sc = *reinterpret_cast<const __half*>(vaddr(p.src.scale, b, h, blk, slot));
      const __half zr = *reinterpret_cast<const __half*>(vaddr(p.src.zero, b, h, blk, slot));
#pragma unroll
      for (int k = 0; k < 32; ++k) o[k] = __hadd_rn(__hmul_rn(__uint2half_rn(c[k]), sc), zr);
    }
    if (p.n_out > 0) {
      const int16_t* ids = reinterpret_cast<const int16_t*>(vaddr(p.src.out_idx, b, h, blk, 0));
      const __half* dat = reinterpret_cast<const __half*>(vaddr(p.src.out_data, b, h, blk, slot));
      for (int j = 0; j < p.n_out; ++j) {
        const int d = ids[j] - su * 32;
#pragma unroll
        for (int k = 0; k < 32; ++k)
          if (d == k) o[k] = dat[j];
      }
    }
    __half* dst = p.out + b * p.osb + h * p.osh + n * p.osn + su * 32;
#pragma unroll
    for (int k = 0; k < 4; ++k) reinterpret_cast<uint4*>(dst)[k] = reinterpret_cast<const uint4*>(o)[k];
  }
}

// ---------------------------------------------------------------------------
// standalone bit packing (akv/bitpack.py), any row width, zero right-padding
// ---------------------------------------------------------------------------
__global__ void pack_codes_kernel(const uint8_t* codes, int64_t rows, int dim, int bits, uint8_t* out) {
  const int per = bits == 4 ? 2 : (bits == 3 ? 8 : 4);   // codes per pack group
  const int gbytes = bits == 3 ? 3 : 1;                  // bytes per pack group
  const int ngr = (dim + per - 1) / per;
  const int64_t total = rows * ngr;
  for (int64_t w = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; w < total;
       w += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int gi = static_cast<int>(w % ngr);
    const int64_t r = w / ngr;
    const uint8_t* src = codes + r * dim;
    uint32_t c[8];
    for (int j = 0; j < per; ++j) {
      const int d = gi * per + j;
      c[j] = d < dim ? src[d] : 0u;
    }
    uint8_t* dst = out + r * static_cast<int64_t>(ngr) * gbytes + gi * gbytes;
    if (bits == 4) {
      dst[0] = static_cast<uint8_t>(((c[0] & 15) << 4) | (c[1] & 15));
    } else if (bits == 2) {
      dst[0] = static_cast<uint8_t>(((c[0] & 3) << 6) | ((c[1] & 3) << 4) | ((c[2] & 3) << 2) | (c[3] & 3));
    } else {
      uint32_t word = 0;
      for (int j = 0; j < 8; ++j) word |= (c[j] & 7) << (21 - 3 * j);
      dst[0] = static_cast<uint8_t>(word >> 16);
      dst[1] = static_cast<uint8_t>(word >> 8);
      dst[2] = static_cast<uint8_t>(word);
    }
  }
}

__global__ void unpack_codes_kernel(const uint8_t* packed, int64_t rows, int dim, int bits, uint8_t* out) {
  const int per = bits == 4 ? 2 : (bits == 3 ? 8 : 4);
  const int gbytes = bits == 3 ? 3 : 1;
  const int ngr = (dim + per - 1) / per;
  const int64_t total = rows * ngr;
  for (int64_t w = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; w < total;
       w += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int gi = static_cast<int>(w % ngr);
    const int64_t r = w / ngr;
    const uint8_t* src = packed + r * static_cast<int64_t>(ngr) * gbytes + gi * gbytes;
    uint32_t c[8];
    if (bits == 4) {
      c[0] = src[0] >> 4;
      c[1] = src[0] & 15;
    } else if (bits == 2) {
      for (int j = 0; j < 4; ++j) c[j] = (src[0] >> (6 - 2 * j)) & 3;
    } else {
      const uint32_t word = (static_cast<uint32_t>(src[0]) << 16) | (src[1] << 8) | src[2];
      for (int j = 0; j < 8; ++j) c[j] = (word >> (21 - 3 * j)) & 7;
    }
    uint8_t* dst = out + r * dim;
    for (int j = 0; j < per; ++j) {
      const int d = gi * per + j;
      if (d < dim) dst[d] = static_cast<uint8_t>(c[j]);
    }
  }
}

// ---------------------------------------------------------------------------
// host launchers
// ---------------------------------------------------------------------------
static inline bool aligned(const void* p, int a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

size_t quant_smem_bytes(int H, int nt, int D, int n_out, bool is_key) {
  return quant_smem_layout(H, nt, D, n_out, is_key).total;
}

constexpr size_t kQuantSmemLimit = 220 * 1024;

// How one akv_quantize call runs: one CTA per scale group when the group's
// rows fit in shared memory, else the chunked path (32-token chunks, heads
// split into groups of heads_per_cta) with a caller workspace.
struct QuantPlan {
  bool chunked;
  int n_groups, n_chunks, heads_per_cta;
  size_t smem, reduce_smem;
  size_t off_min, off_max, off_sq, off_zero, off_scale, off_oidx, ws_bytes;
};

static size_t up256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

static QuantPlan plan_quant(int B, int H, int N, int D, int group, int n_out, bool is_key,
                            bool force_chunked = false) {
  QuantPlan pl{};
  pl.n_groups = (N + group - 1) / group;
  pl.smem = quant_smem_bytes(H, std::min(group, N), D, n_out, is_key);
  if (pl.smem <= kQuantSmemLimit && !force_chunked) return pl;
  pl.chunked = true;
  pl.n_chunks = (N + kBlockTokens - 1) / kBlockTokens;
  int hs = H;
  while (hs > 1 && quant_smem_bytes(hs, kBlockTokens, D, n_out, is_key) > kQuantSmemLimit) --hs;
  pl.heads_per_cta = hs;
  pl.smem = quant_smem_bytes(hs, kBlockTokens, D, n_out, is_key);
  pl.reduce_smem = (static_cast<size_t>(H) * D + D) * sizeof(float);
  const size_t part = static_cast<size_t>(B) * pl.n_chunks * H * D;
  const size_t grp = static_cast<size_t>(B) * pl.n_groups * H * D;
  pl.off_min = 0;
  pl.off_max = pl.off_min + up256(part * 2);
  pl.off_sq = pl.off_max + up256(part * 2);
  pl.off_zero = pl.off_sq + up256(part * 4);
  pl.off_scale = pl.off_zero + up256(grp * 2);
  pl.off_oidx = pl.off_scale + up256(grp * 2);
  pl.ws_bytes = pl.off_oidx + up256(static_cast<size_t>(B) * pl.n_groups * kMaxOutliersWs * 4);
  return pl;
}

template <typename K>
static bool set_smem(K kern, size_t smem) {
  return smem <= 48 * 1024 ||
         cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) ==
             cudaSuccess;
}

template <int BITS, bool IS_KEY>
static int launch_quant(QuantParams p, const QuantPlan& pl, void* ws, cudaStream_t st) {
  p.n_groups = pl.n_groups;
  if (!pl.chunked) {
    auto kern = quantize_group_kernel<BITS, IS_KEY, kQuantFull>;
    if (!set_smem(kern, pl.smem)) return AKV_ERR_LAUNCH;
    kern<<<dim3(pl.n_groups, p.B), kQuantThreads, pl.smem, st>>>(p);
    return cudaGetLastError() == cudaSuccess ? AKV_OK : AKV_ERR_LAUNCH;
  }
  char* w = static_cast<char*>(ws);
  p.n_chunks = pl.n_chunks;
  p.n_groups = pl.n_groups;
  p.heads_per_cta = pl.heads_per_cta;
  p.ws_min = reinterpret_cast<__half*>(w + pl.off_min);
  p.ws_max = reinterpret_cast<__half*>(w + pl.off_max);
  p.ws_sq = reinterpret_cast<float*>(w + pl.off_sq);
  p.ws_zero = reinterpret_cast<__half*>(w + pl.off_zero);
  p.ws_scale = reinterpret_cast<__half*>(w + pl.off_scale);
  p.ws_oidx = reinterpret_cast<int*>(w + pl.off_oidx);
  const dim3 grid(pl.n_chunks, p.B, (p.H + pl.heads_per_cta - 1) / pl.heads_per_cta);
  if (IS_KEY || (p.n_out > 0 && !p.score_sum)) {
    auto stats = quantize_group_kernel<BITS, IS_KEY, kQuantStats>;
    auto reduce = quant_reduce_kernel<BITS, IS_KEY>;
    if (!set_smem(stats, pl.smem) || !set_smem(reduce, pl.reduce_smem)) return AKV_ERR_LAUNCH;
    stats<<<grid, kQuantThreads, pl.smem, st>>>(p);
    reduce<<<dim3(pl.n_groups, p.B), kQuantThreads, pl.reduce_smem, st>>>(p);
  } else if (p.n_out > 0) {  // external scores: the reduction only picks the outlier channels
    auto reduce = quant_reduce_kernel<BITS, IS_KEY>;
    if (!set_smem(reduce, pl.reduce_smem)) return AKV_ERR_LAUNCH;
    reduce<<<dim3(pl.n_groups, p.B), kQuantThreads, pl.reduce_smem, st>>>(p);
  }
  auto enc = quantize_group_kernel<BITS, IS_KEY, kQuantEncode>;
  if (!set_smem(enc, pl.smem)) return AKV_ERR_LAUNCH;
  enc<<<grid, kQuantThreads, pl.smem, st>>>(p);
  return cudaGetLastError() == cudaSuccess ? AKV_OK : AKV_ERR_LAUNCH;
}

template <int BITS, bool IS_KEY>
static int launch_dequant(const DequantParams& p, cudaStream_t st) {
  const int64_t total = static_cast<int64_t>(p.B) * p.H * p.N * (p.D / 32);
  const int threads = 256;
  const int64_t blocks = std::min<int64_t>((total + threads - 1) / threads, 148 * 32);
  dequantize_kernel<BITS, IS_KEY><<<static_cast<unsigned>(blocks), threads, 0, st>>>(p);
  return cudaGetLastError() == cudaSuccess ? AKV_OK : AKV_ERR_LAUNCH;
}

}  // namespace akv

using namespace akv;

extern "C" size_t akv_quantize_workspace_bytes(int B, int H, int N, int D, int group, int n_outlier, int is_key) {
  if (B <= 0 || H <= 0 || N <= 0 || D <= 0 || D % 32 != 0 || D > 256) return 0;
  if (n_outlier < 0 || n_outlier > kMaxOutliers || n_outlier > D) return 0;
  if (group <= 0 || group > N) group = N;
  const QuantPlan pl = plan_quant(B, H, N, D, group, n_outlier, is_key != 0);
  return pl.chunked ? pl.ws_bytes : 0;
}

extern "C" int akv_quantize(const uint16_t* src, int64_t src_sb, int64_t src_sh, int64_t src_sn,
                            const int64_t* tok_idx, int64_t tok_sb, int64_t n_src, int B, int H, int N, int D,
                            int bits, int is_key, int group, int n_outlier, const akv_qdest* dst, int* status,
                            void* stream) {
  return akv_quantize_ws(src, src_sb, src_sh, src_sn, tok_idx, tok_sb, n_src, B, H, N, D, bits, is_key, group,
                         n_outlier, dst, nullptr, 0, status, stream);
}

extern "C" int akv_quantize_ws(const uint16_t* src, int64_t src_sb, int64_t src_sh, int64_t src_sn,
                               const int64_t* tok_idx, int64_t tok_sb, int64_t n_src, int B, int H, int N, int D,
                               int bits, int is_key, int group, int n_outlier, const akv_qdest* dst,
                               void* workspace, size_t workspace_bytes, int* status, void* stream) {
  return akv_quantize_ext(src, src_sb, src_sh, src_sn, tok_idx, tok_sb, n_src, B, H, N, D, bits, is_key, group,
                          n_outlier, dst, nullptr, 0, workspace, workspace_bytes, status, stream);
}

// Checks of one quantiser call and its parameter block (akv_quantize_ext and
// the fused single-token demotion share them).
static int prepare_quant(const uint16_t* src, int64_t src_sb, int64_t src_sh, int64_t src_sn, const int64_t* tok_idx,
                         int64_t tok_sb, int64_t n_src, int B, int H, int N, int D, int bits, int is_key, int group,
                         int n_outlier, const akv_qdest* dst, const float* score_sum, int score_heads, int* status,
                         QuantParams& p, QuantPlan& pl) {
  if (!src || !dst) return AKV_ERR_NULL;
  if (tok_idx && n_src <= 0) return AKV_ERR_SHAPE;
  if (score_sum && score_heads <= 0) return AKV_ERR_SHAPE;
  if (bits < 2 || bits > 4) return AKV_ERR_BITS;
  if (B <= 0 || H <= 0 || N <= 0 || D <= 0 || D % 32 != 0 || D > 256) return AKV_ERR_SHAPE;
  if (group <= 0) group = N;
  if (group > N) group = N;
  if (N > group && group % kBlockTokens != 0) return AKV_ERR_SHAPE;
  if (n_outlier < 0 || n_outlier > kMaxOutliers || n_outlier > D) return AKV_ERR_SHAPE;
  if (!aligned(src, 16) || src_sb % 8 || src_sh % 8 || src_sn % 8) return AKV_ERR_ALIGN;
  if (dst->codes.ptr && (!aligned(dst->codes.ptr, 4) || dst->codes.sb % 4 || dst->codes.sh % 4 ||
                         dst->codes.sblk % 4 || dst->codes.sslot % 4))
    return AKV_ERR_ALIGN;
  if (is_key && dst->scale.ptr && (!aligned(dst->scale.ptr, 4) || dst->scale.sb % 4 || dst->scale.sh % 4 ||
                                   dst->scale.sblk % 4))
    return AKV_ERR_ALIGN;
  if (is_key && dst->zero.ptr && (!aligned(dst->zero.ptr, 4) || dst->zero.sb % 4 || dst->zero.sh % 4 ||
                                  dst->zero.sblk % 4))
    return AKV_ERR_ALIGN;
  if (dst->mask.ptr && !aligned(dst->mask.ptr, 4)) return AKV_ERR_ALIGN;
  if (dst->out_vdq.ptr && (!aligned(dst->out_vdq.ptr, 2) || dst->out_vdq.sslot % 2)) return AKV_ERR_ALIGN;
  pl = plan_quant(B, H, N, D, group, n_outlier, is_key != 0);
  if (pl.smem > kQuantSmemLimit) return AKV_ERR_UNSUPPORTED;
  p = QuantParams{};
  p.src = reinterpret_cast<const __half*>(src);
  p.sb = src_sb;
  p.sh = src_sh;
  p.sn = src_sn;
  p.tok_idx = tok_idx;
  p.tok_sb = tok_sb;
  p.n_src = n_src;
  p.B = B;
  p.H = H;
  p.N = N;
  p.D = D;
  p.bits = bits;
  p.is_key = is_key;
  p.group = group;
  p.n_out = n_outlier;
  p.dst = *dst;
  p.status = status;
  p.score_sum = score_sum;
  p.score_heads = score_heads;
  p.n_groups = pl.n_groups;
  return AKV_OK;
}

extern "C" int akv_quantize_ext(const uint16_t* src, int64_t src_sb, int64_t src_sh, int64_t src_sn,
                                const int64_t* tok_idx, int64_t tok_sb, int64_t n_src, int B, int H, int N, int D,
                                int bits, int is_key, int group, int n_outlier, const akv_qdest* dst,
                                const float* score_sum, int score_heads, void* workspace, size_t workspace_bytes,
                                int* status, void* stream) {
  QuantParams p;
  QuantPlan pl;
  const int rc = prepare_quant(src, src_sb, src_sh, src_sn, tok_idx, tok_sb, n_src, B, H, N, D, bits, is_key, group,
                               n_outlier, dst, score_sum, score_heads, status, p, pl);
  if (rc != AKV_OK) return rc;
  if (pl.chunked && (!workspace || workspace_bytes < pl.ws_bytes || !aligned(workspace, 256))) return AKV_ERR_WORKSPACE;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (bits * 2 + (is_key ? 1 : 0)) {
    case 5: return launch_quant<2, true>(p, pl, workspace, st);
    case 4: return launch_quant<2, false>(p, pl, workspace, st);
    case 7: return launch_quant<3, true>(p, pl, workspace, st);
    case 6: return launch_quant<3, false>(p, pl, workspace, st);
    case 9: return launch_quant<4, true>(p, pl, workspace, st);
    default: return launch_quant<4, false>(p, pl, workspace, st);
  }
}

extern "C" int akv_dequantize(const akv_qdest* src, const int64_t* tok_idx, int64_t tok_sb, int64_t n_src, int B,
                              int H, int N, int D, int bits, int is_key, int n_outlier, uint16_t* out,
                              int64_t out_sb, int64_t out_sh, int64_t out_sn, int* status, void* stream) {
  if (!src || !out || !src->codes.ptr || !src->scale.ptr || !src->zero.ptr) return AKV_ERR_NULL;
  if (tok_idx && n_src <= 0) return AKV_ERR_SHAPE;
  if (n_outlier > 0 && (!src->out_idx.ptr || !src->out_data.ptr)) return AKV_ERR_NULL;
  if (bits < 2 || bits > 4) return AKV_ERR_BITS;
  if (B <= 0 || H <= 0 || N < 0 || D <= 0 || D % 32 != 0 || D > 256) return AKV_ERR_SHAPE;
  if (N == 0) return AKV_OK;
  if (!aligned(out, 16) || out_sb % 8 || out_sh % 8 || out_sn % 8) return AKV_ERR_ALIGN;
  if (!aligned(src->codes.ptr, 4) || src->codes.sb % 4 || src->codes.sh % 4 || src->codes.sblk % 4 ||
      src->codes.sslot % 4)
    return AKV_ERR_ALIGN;
  DequantParams p{*src, tok_idx, tok_sb, n_src, B, H, N, D, n_outlier, reinterpret_cast<__half*>(out),
                  out_sb, out_sh, out_sn, status};
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (bits * 2 + (is_key ? 1 : 0)) {
    case 5: return launch_dequant<2, true>(p, st);
    case 4: return launch_dequant<2, false>(p, st);
    case 7: return launch_dequant<3, true>(p, st);
    case 6: return launch_dequant<3, false>(p, st);
    case 9: return launch_dequant<4, true>(p, st);
    default: return launch_dequant<4, false>(p, st);
  }
}

extern "C" int akv_pack_codes(const uint8_t* codes, int64_t rows, int dim, int bits, uint8_t* packed,
                              void* stream) {
  if (!codes || !packed) return AKV_ERR_NULL;
  if (bits < 2 || bits > 4) return AKV_ERR_BITS;
  if (rows < 0 || dim <= 0) return AKV_ERR_SHAPE;
  if (rows == 0) return AKV_OK;
  const int per = bits == 4 ? 2 : (bits == 3 ? 8 : 4);
  const int64_t total = rows * ((dim + per - 1) / per);
  const int64_t blocks = std::min<int64_t>((total + 255) / 256, 148 * 16);
  pack_codes_kernel<<<static_cast<unsigned>(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      codes, rows, dim, bits, packed);
  return cudaGetLastError() == cudaSuccess ? AKV_OK : AKV_ERR_LAUNCH;
}

extern "C" int akv_unpack_codes(const uint8_t* packed, int64_t rows, int dim, int bits, uint8_t* codes,
                                void* stream) {
  if (!codes || !packed) return AKV_ERR_NULL;
  if (bits < 2 || bits > 4) return AKV_ERR_BITS;
  if (rows < 0 || dim <= 0) return AKV_ERR_SHAPE;
  if (rows == 0) return AKV_OK;
  const int per = bits == 4 ? 2 : (bits == 3 ? 8 : 4);
  const int64_t total = rows * ((dim + per - 1) / per);
  const int64_t blocks = std::min<int64_t>((total + 255) / 256, 148 * 16);
  unpack_codes_kernel<<<static_cast<unsigned>(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      packed, rows, dim, bits, codes);
  return cudaGetLastError() == cudaSuccess ? AKV_OK : AKV_ERR_LAUNCH;
}

// Sum over this call's heads of the per-(head, channel) L2 norms over each
// scale group's tokens: the partial outlier score of heads held by one GPU,
// all-reduced over the GPUs before akv_quantize_ext (the reference scores
// channels by the mean over all heads, affine_quantizer.py:79 / :146).
// Always the chunked statistics path; workspace from
// akv_outlier_norm_sums_workspace_bytes.
static QuantPlan plan_norms(int B, int H, int N, int D, int group) {
  return plan_quant(B, H, N, D, group, 1, false, true);
}

extern "C" size_t akv_outlier_norm_sums_workspace_bytes(int B, int H, int N, int D, int group) {
  if (B <= 0 || H <= 0 || N <= 0 || D <= 0 || D % 32 != 0 || D > 256) return 0;
  if (group <= 0 || group > N) group = N;
  return plan_norms(B, H, N, D, group).ws_bytes;
}

extern "C" int akv_outlier_norm_sums(const uint16_t* src, int64_t src_sb, int64_t src_sh, int64_t src_sn,
                                     const int64_t* tok_idx, int64_t tok_sb, int64_t n_src, int B, int H, int N,
                                     int D, int group, float* out, void* workspace, size_t workspace_bytes,
                                     int* status, void* stream) {
  if (!src || !out) return AKV_ERR_NULL;
  if (tok_idx && n_src <= 0) return AKV_ERR_SHAPE;
  if (B <= 0 || H <= 0 || N <= 0 || D <= 0 || D % 32 != 0 || D > 256) return AKV_ERR_SHAPE;
  if (group <= 0 || group > N) group = N;
  if (N > group && group % kBlockTokens != 0) return AKV_ERR_SHAPE;
  if (!aligned(src, 16) || src_sb % 8 || src_sh % 8 || src_sn % 8) return AKV_ERR_ALIGN;
  const QuantPlan pl = plan_norms(B, H, N, D, group);
  if (pl.smem > kQuantSmemLimit) return AKV_ERR_UNSUPPORTED;
  if (!workspace || workspace_bytes < pl.ws_bytes || !aligned(workspace, 256)) return AKV_ERR_WORKSPACE;
  QuantParams p{};
  p.src = reinterpret_cast<const __half*>(src);
  p.sb = src_sb;
  p.sh = src_sh;
  p.sn = src_sn;
  p.tok_idx = tok_idx;
  p.tok_sb = tok_sb;
  p.n_src = n_src;
  p.status = status;
  p.B = B;
  p.H = H;
  p.N = N;
  p.D = D;
  p.bits = 4;
  p.group = group;
  p.n_out = 1;
  p.n_chunks = pl.n_chunks;
  p.n_groups = pl.n_groups;
  p.heads_per_cta = pl.heads_per_cta;
  char* w = static_cast<char*>(workspace);
  p.ws_sq = reinterpret_cast<float*>(w + pl.off_sq);
  p.norm_sums_out = out;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  auto stats = quantize_group_kernel<4, false, kQuantStats>;
  auto reduce = quant_reduce_kernel<4, false>;
  if (!set_smem(stats, pl.smem) || !set_smem(reduce, pl.reduce_smem)) return AKV_ERR_LAUNCH;
  stats<<<dim3(pl.n_chunks, B, (H + pl.heads_per_cta - 1) / pl.heads_per_cta), kQuantThreads, pl.smem, st>>>(p);
  reduce<<<dim3(pl.n_groups, B), kQuantThreads, pl.reduce_smem, st>>>(p);
  return cudaGetLastError() == cudaSuccess ? AKV_OK : AKV_ERR_LAUNCH;
}

// ---------------------------------------------------------------------------
// One demotion event into new warm block records: the K and V destinations
// (the record fields akv_warm_layout describes) are built here, and the two
// quantiser launches issued back to back, so a caller appending to an arena
// makes one call per event.
// ---------------------------------------------------------------------------
static akv_qdest record_qdest(uint8_t* base, int64_t sb, int64_t sh, const akv_warm_layout& L, bool is_key) {
  akv_qdest d{};
  const int64_t sblk = L.bytes;
  const int n = L.n_outlier;
  auto view = [&](int off, int64_t sslot) { return akv_view{base + off, sb, sh, sblk, sslot}; };
  if (is_key) {
    d.pair_order = 1;  // records keep K scale / zero in the decode pair order
    d.codes = view(L.kc, L.head_dim * L.key_bits / 8);
    d.scale = view(L.ks, 0);
    d.zero = view(L.kz, 0);
    if (n) {
      d.out_data = view(L.ko, 2 * n);
      d.out_idx = view(L.ki, 0);
    }
  } else {
    d.codes = view(L.vc, L.head_dim * L.value_bits / 8);
    d.scale = view(L.vs, 2);
    d.zero = view(L.vz, 2);
    if (n) {
      d.out_data = view(L.vo, 2 * n);
      d.out_idx = view(L.vi, 0);
      d.out_vdq = view(L.vd, 2 * n);
    }
  }
  d.mask = view(L.mask, 0);
  d.flags = view(L.flags + (is_key ? 0 : 1), 0);
  return d;
}

extern "C" size_t akv_warm_append_workspace_bytes(int B, int H, int N, int D, int group, int n_outlier) {
  const size_t k = akv_quantize_workspace_bytes(B, H, N, D, group, n_outlier, 1);
  const size_t v = akv_quantize_workspace_bytes(B, H, N, D, group, n_outlier, 0);
  return k > v ? k : v;
}

extern "C" int akv_warm_append(uint8_t* arena, int64_t a_sb, int64_t a_sh, const akv_warm_layout* layout, int blk0,
                               const uint16_t* k, int64_t k_sb, int64_t k_sh, int64_t k_sn, const uint16_t* v,
                               int64_t v_sb, int64_t v_sh, int64_t v_sn, const int64_t* tok_idx, int64_t tok_sb,
                               int64_t n_src, int B, int H, int N, int group, void* workspace,
                               size_t workspace_bytes, int* status, void* stream) {
  if (!arena || !layout || !k || !v) return AKV_ERR_NULL;
  if (blk0 < 0) return AKV_ERR_SHAPE;
  const akv_warm_layout L = *layout;
  uint8_t* base = arena + static_cast<int64_t>(blk0) * L.bytes;
  const akv_qdest dk = record_qdest(base, a_sb, a_sh, L, true);
  const akv_qdest dv = record_qdest(base, a_sb, a_sh, L, false);
  int rc = akv_quantize_ext(k, k_sb, k_sh, k_sn, tok_idx, tok_sb, n_src, B, H, N, L.head_dim, L.key_bits, 1, group,
                            L.n_outlier, &dk, nullptr, 0, workspace, workspace_bytes, status, stream);
  if (rc != AKV_OK) return rc;
  return akv_quantize_ext(v, v_sb, v_sh, v_sn, tok_idx, tok_sb, n_src, B, H, N, L.head_dim, L.value_bits, 0, group,
                          L.n_outlier, &dv, nullptr, 0, workspace, workspace_bytes, status, stream);
}

template <int KBITS, int VBITS>
static int launch_demote_install(const QuantParams& pk, const QuantParams& pv, const InstallRows& ins, size_t smem,
                                 int B, cudaStream_t st) {
  auto kern = demote_install_kernel<KBITS, VBITS>;
  if (!set_smem(kern, smem)) return AKV_ERR_LAUNCH;
  kern<<<dim3(1, B, 2), kQuantThreads, smem, st>>>(pk, pv, ins);
  return cudaGetLastError() == cudaSuccess ? AKV_OK : AKV_ERR_LAUNCH;
}

extern "C" int akv_warm_demote_install(uint8_t* arena, int64_t a_sb, int64_t a_sh, const akv_warm_layout* layout,
                                       int blk0, uint16_t* k, int64_t k_sb, int64_t k_sh, uint16_t* v, int64_t v_sb,
                                       int64_t v_sh, const uint16_t* nk, int64_t nk_sb, int64_t nk_sh,
                                       const uint16_t* nv, int64_t nv_sb, int64_t nv_sh, int B, int H, int* status,
                                       void* stream) {
  if (!arena || !layout || !k || !v || !nk || !nv) return AKV_ERR_NULL;
  if (blk0 < 0) return AKV_ERR_SHAPE;
  const akv_warm_layout L = *layout;
  const int D = L.head_dim;
  uint8_t* base = arena + static_cast<int64_t>(blk0) * L.bytes;
  const akv_qdest dk = record_qdest(base, a_sb, a_sh, L, true);
  const akv_qdest dv = record_qdest(base, a_sb, a_sh, L, false);
  QuantParams pk, pv;
  QuantPlan lk, lv;
  int rc = prepare_quant(k, k_sb, k_sh, D, nullptr, 0, 0, B, H, 1, D, L.key_bits, 1, 1, L.n_outlier, &dk, nullptr, 0,
                         status, pk, lk);
  if (rc != AKV_OK) return rc;
  rc = prepare_quant(v, v_sb, v_sh, D, nullptr, 0, 0, B, H, 1, D, L.value_bits, 0, 1, L.n_outlier, &dv, nullptr, 0,
                     status, pv, lv);
  if (rc != AKV_OK) return rc;
  if (lk.chunked || lv.chunked) return AKV_ERR_UNSUPPORTED;  // one token never is
  InstallRows ins{reinterpret_cast<const __half*>(nk), nk_sb, nk_sh, reinterpret_cast<const __half*>(nv), nv_sb,
                  nv_sh, 0};
  ins.vec16 = aligned(nk, 16) && aligned(nv, 16) && nk_sb % 8 == 0 && nk_sh % 8 == 0 && nv_sb % 8 == 0 &&
              nv_sh % 8 == 0;  // the destinations passed the quantiser's 16-byte checks
  const size_t smem = std::max(lk.smem, lv.smem);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (L.key_bits * 8 + L.value_bits) {
    case 18: return launch_demote_install<2, 2>(pk, pv, ins, smem, B, st);
    case 19: return launch_demote_install<2, 3>(pk, pv, ins, smem, B, st);
    case 20: return launch_demote_install<2, 4>(pk, pv, ins, smem, B, st);
    case 26: return launch_demote_install<3, 2>(pk, pv, ins, smem, B, st);
    case 27: return launch_demote_install<3, 3>(pk, pv, ins, smem, B, st);
    case 28: return launch_demote_install<3, 4>(pk, pv, ins, smem, B, st);
    case 34: return launch_demote_install<4, 2>(pk, pv, ins, smem, B, st);
    case 35: return launch_demote_install<4, 3>(pk, pv, ins, smem, B, st);
    case 36: return launch_demote_install<4, 4>(pk, pv, ins, smem, B, st);
    default: return AKV_ERR_BITS;
  }
}
