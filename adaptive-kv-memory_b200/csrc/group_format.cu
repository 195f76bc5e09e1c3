// Per-token, per-D-group ("group format") quantised tiers of the reference's
// older kernel API: akv/triton_ops.py (fused_quantized_attention,
// fused_mixed_precision_attention, _dequantize_packed :657-715) and
// akv/triton_kernels.py (fused_decode_attention :281-423,
// fused_quantize_evict :426-500).
//
// A row of D channels is padded with zeros to a multiple of group_size and
// stored as one packed byte row: bits 8 one code per byte; bits 4 channel 2j
// in the high nibble of byte j; bits 2 channel 4j in bits 7..6 of byte j,
// then 5..4, 3..2, 1..0.  Each group g of a row has an fp16 scale and zero.
//
// Kernels:
//   group_dequant_kernel    codes -> fp16, fp32 arithmetic like
//                           _dequantize_packed (asymmetric c*s + z as a
//                           product then a sum; symmetric (c - max/2)*s)
//   group_quantize_kernel   fp16 rows (optionally gathered by index) ->
//                           packed codes + fp16 scale / zero per group, in the
//                           fp16 arithmetic of fused_quantize_evict (every
//                           torch half op is a float op rounded to fp16)
//   attention_probs_kernel  softmax weights exp(sm_scale*q.k - lse) of a
//                           key tier, given the natural-log LSE over all
//                           tiers (the attention-weight output of
//                           fused_mixed_precision_attention :466-515)
#include <cuda_runtime.h>

#include <algorithm>

#include "common.cuh"

namespace akv {

static inline bool gf_aligned(const void* p, int a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// code of channel d in a packed row
template <int BITS>
AKV_DEV uint32_t gf_code(const uint8_t* row, int d) {
  if constexpr (BITS == 8) {
    return row[d];
  } else if constexpr (BITS == 4) {
    const uint32_t b = row[d >> 1];
    return (d & 1) ? (b & 15u) : (b >> 4);
  } else {
    const uint32_t b = row[d >> 2];
    return (b >> (6 - 2 * (d & 3))) & 3u;
  }
}

// One thread per 8 channels of one (h, n) row.
template <int BITS>
__global__ void group_dequant_kernel(const uint8_t* packed, int64_t p_sh, int64_t p_sn, const __half* sc,
                                     const __half* zr, int64_t s_sh, int64_t s_sn, int H, int N, int D, int gsize,
                                     const int32_t* symmetric, __half* out, int64_t o_sh, int64_t o_sn) {
  const int nc = D / 8;
  const int64_t total = static_cast<int64_t>(H) * N * nc;
  const bool sym = symmetric != nullptr && *symmetric != 0;
  constexpr float kHalfRange = static_cast<float>(((1 << BITS) - 1) / 2);  // max_val // 2
  for (int64_t w = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; w < total;
       w += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int c8 = static_cast<int>(w % nc);
    const int64_t r = w / nc;
    const int n = static_cast<int>(r % N), h = static_cast<int>(r / N);
    const uint8_t* row = packed + h * p_sh + n * p_sn;
    const __half* srow = sc + h * s_sh + n * s_sn;
    const __half* zrow = zr + h * s_sh + n * s_sn;
    __align__(16) __half o[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int d = 8 * c8 + i;
      const float c = static_cast<float>(gf_code<BITS>(row, d));
      const int g = d / gsize;
      const float s = __half2float(srow[g]);
      const float v = sym ? __fmul_rn(__fsub_rn(c, kHalfRange), s) : __fadd_rn(__fmul_rn(c, s), __half2float(zrow[g]));
      o[i] = __float2half_rn(v);
    }
    *reinterpret_cast<uint4*>(out + h * o_sh + n * o_sn + 8 * c8) = *reinterpret_cast<const uint4*>(o);
  }
}

// fp16 op of torch: float op, rounded to fp16
AKV_DEV __half h_sub(__half a, __half b) { return __float2half_rn(__fsub_rn(__half2float(a), __half2float(b))); }
AKV_DEV __half h_div(__half a, __half b) { return __float2half_rn(__fdiv_rn(__half2float(a), __half2float(b))); }

// One warp per (row, group); lanes stride over the group's channels.
template <int BITS>
__global__ void group_quantize_kernel(const __half* src, int64_t s_sn, const int64_t* row_idx, int64_t n_src, int n,
                                      int D, int gsize, int n_groups, uint8_t* packed, int64_t row_bytes,
                                      __half* scales, __half* zeros, int* status) {
  constexpr int kMax = (1 << BITS) - 1;
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x / 32);
  const int64_t total = static_cast<int64_t>(n) * n_groups;
  for (int64_t w = blockIdx.x * static_cast<int64_t>(blockDim.x / 32) + threadIdx.x / 32; w < total; w += warps) {
    const int g = static_cast<int>(w % n_groups);
    const int64_t r = w / n_groups;
    int64_t sr = row_idx ? row_idx[r] : r;
    if (row_idx && static_cast<uint64_t>(sr) >= static_cast<uint64_t>(n_src)) {
      if (lane == 0) set_status(status, AKV_ERR_SHAPE);
      sr = 0;
    }
    const __half* x = src + sr * s_sn;
    const int d0 = g * gsize;
    // min / max over the group, zero padding beyond D included (F.pad)
    float mn = INFINITY, mx = -INFINITY;
    for (int i = lane; i < gsize; i += 32) {
      const int d = d0 + i;
      const float v = d < D ? __half2float(x[d]) : 0.f;
      mn = fminf(mn, v);
      mx = fmaxf(mx, v);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    }
    const __half hmn = __float2half_rn(mn), hmx = __float2half_rn(mx);  // exact: fp16 values
    // scales = (max - min) / max_int, clamp(min=1e-8): every positive fp16
    // exceeds 1e-8 and fp16(1e-8) is 0, so the clamp changes nothing
    const __half scale = h_div(h_sub(hmx, hmn), __float2half_rn(static_cast<float>(kMax)));
    if (lane == 0) {
      scales[r * n_groups + g] = scale;
      zeros[r * n_groups + g] = hmn;
    }
    // codes: round-half-even of fp16((x - zero) / scale), clamped; NaN (0/0
    // of a constant group) writes code 0
    uint8_t* prow = packed + r * row_bytes;
    constexpr int kPer = 8 / BITS;  // codes per byte
    for (int j = lane; j < gsize / kPer; j += 32) {
      uint32_t byte = 0;
#pragma unroll
      for (int t = 0; t < kPer; ++t) {
        const int d = d0 + j * kPer + t;
        const __half v = d < D ? x[d] : __float2half_rn(0.f);
        const float qf = __half2float(h_div(h_sub(v, hmn), scale));
        const float rq = rintf(qf);  // fp16 integers and halves are exact in fp32
        const uint32_t c = (rq >= 0.f) ? static_cast<uint32_t>(fminf(rq, static_cast<float>(kMax))) : 0u;
        byte |= c << (8 - BITS * (t + 1));
      }
      prow[(d0 / kPer) + j] = static_cast<uint8_t>(byte);
    }
  }
}

// One warp per (b, h, key n); lanes stride over D; loops over the M queries.
__global__ void attention_probs_kernel(const __half* q, int64_t q_sb, int64_t q_sh, int64_t q_sm, const __half* k,
                                       int64_t k_sb, int64_t k_sh, int64_t k_sn, const float* lse, int B, int H, int M,
                                       int N, int D, float sm_scale, float* out, int64_t o_sb, int64_t o_sh,
                                       int64_t o_sm, int col0) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x / 32);
  const int64_t total = static_cast<int64_t>(B) * H * N;
  for (int64_t w = blockIdx.x * static_cast<int64_t>(blockDim.x / 32) + threadIdx.x / 32; w < total; w += warps) {
    const int n = static_cast<int>(w % N);
    const int64_t bh = w / N;
    const int h = static_cast<int>(bh % H), b = static_cast<int>(bh / H);
    const __half* kr = k + b * k_sb + h * k_sh + n * k_sn;
    float kv[8];  // D <= 256
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int d = lane + 32 * i;
      kv[i] = d < D ? __half2float(kr[d]) : 0.f;
    }
    for (int m = 0; m < M; ++m) {
      const __half* qr = q + b * q_sb + h * q_sh + m * q_sm;
      float acc = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int d = lane + 32 * i;
        if (d < D) acc = fmaf(__half2float(qr[d]), kv[i], acc);
      }
#pragma unroll
      for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
      if (lane == 0) {
        const float l = lse[bh * M + m];
        out[b * o_sb + h * o_sh + m * o_sm + col0 + n] = isinf(l) ? 0.f : expf(sm_scale * acc - l);
      }
    }
  }
}

static unsigned gf_blocks(int64_t work, int per_block) {
  return static_cast<unsigned>(std::max<int64_t>(1, std::min<int64_t>((work + per_block - 1) / per_block, 148 * 16)));
}

}  // namespace akv

using namespace akv;

extern "C" int akv_group_dequant(const uint8_t* packed, int64_t p_sh, int64_t p_sn, const uint16_t* scales,
                                 const uint16_t* zeros, int64_t s_sh, int64_t s_sn, int H, int N, int D, int group_size,
                                 int bits, const int32_t* symmetric, uint16_t* out, int64_t o_sh, int64_t o_sn,
                                 void* stream) {
  if (!packed || !scales || !zeros || !out) return AKV_ERR_NULL;
  if (bits != 2 && bits != 4 && bits != 8) return AKV_ERR_BITS;
  if (H <= 0 || N < 0 || D <= 0 || D % 8 != 0 || group_size <= 0) return AKV_ERR_SHAPE;
  if (N == 0) return AKV_OK;
  if (!gf_aligned(out, 16) || o_sh % 8 || o_sn % 8) return AKV_ERR_ALIGN;
  const int64_t total = static_cast<int64_t>(H) * N * (D / 8);
  auto st = static_cast<cudaStream_t>(stream);
  auto s = reinterpret_cast<const __half*>(scales);
  auto z = reinterpret_cast<const __half*>(zeros);
  auto o = reinterpret_cast<__half*>(out);
  const unsigned nb = gf_blocks(total, 256);
  if (bits == 2)
    group_dequant_kernel<2><<<nb, 256, 0, st>>>(packed, p_sh, p_sn, s, z, s_sh, s_sn, H, N, D, group_size, symmetric,
                                                o, o_sh, o_sn);
  else if (bits == 4)
    group_dequant_kernel<4><<<nb, 256, 0, st>>>(packed, p_sh, p_sn, s, z, s_sh, s_sn, H, N, D, group_size, symmetric,
                                                o, o_sh, o_sn);
  else
    group_dequant_kernel<8><<<nb, 256, 0, st>>>(packed, p_sh, p_sn, s, z, s_sh, s_sn, H, N, D, group_size, symmetric,
                                                o, o_sh, o_sn);
  return cudaGetLastError() == cudaSuccess ? AKV_OK : AKV_ERR_LAUNCH;
}

extern "C" int akv_int4_group_dequant(const uint8_t* packed, int64_t p_sh, int64_t p_sn, const uint16_t* scales,
                                      const uint16_t* zeros, int64_t s_sh, int64_t s_sn, int H, int N, int D,
                                      int group_size, uint16_t* out, int64_t o_sh, int64_t o_sn, void* stream) {
  return akv_group_dequant(packed, p_sh, p_sn, scales, zeros, s_sh, s_sn, H, N, D, group_size, 4, nullptr, out, o_sh,
                           o_sn, stream);
}

extern "C" int akv_group_quantize(const uint16_t* src, int64_t s_sn, const int64_t* row_idx, int64_t n_src, int n,
                                  int D, int group_size, int bits, uint8_t* packed, int64_t row_bytes,
                                  uint16_t* scales, uint16_t* zeros, int* status, void* stream) {
  if (!src || !packed || !scales || !zeros) return AKV_ERR_NULL;
  if (bits != 2 && bits != 4 && bits != 8) return AKV_ERR_BITS;
  if (n < 0 || D <= 0 || group_size <= 0 || group_size % (8 / bits) != 0) return AKV_ERR_SHAPE;
  const int n_groups = (D + group_size - 1) / group_size;
  if (row_bytes < static_cast<int64_t>(n_groups) * group_size * bits / 8) return AKV_ERR_SHAPE;
  if (row_idx && n_src <= 0) return AKV_ERR_SHAPE;
  if (n == 0) return AKV_OK;
  const int64_t total = static_cast<int64_t>(n) * n_groups;
  auto st = static_cast<cudaStream_t>(stream);
  auto x = reinterpret_cast<const __half*>(src);
  auto s = reinterpret_cast<__half*>(scales);
  auto z = reinterpret_cast<__half*>(zeros);
  const unsigned nb = gf_blocks(total, 8);
  if (bits == 2)
    group_quantize_kernel<2><<<nb, 256, 0, st>>>(x, s_sn, row_idx, n_src, n, D, group_size, n_groups, packed,
                                                 row_bytes, s, z, status);
  else if (bits == 4)
    group_quantize_kernel<4><<<nb, 256, 0, st>>>(x, s_sn, row_idx, n_src, n, D, group_size, n_groups, packed,
                                                 row_bytes, s, z, status);
  else
    group_quantize_kernel<8><<<nb, 256, 0, st>>>(x, s_sn, row_idx, n_src, n, D, group_size, n_groups, packed,
                                                 row_bytes, s, z, status);
  return cudaGetLastError() == cudaSuccess ? AKV_OK : AKV_ERR_LAUNCH;
}

extern "C" int akv_attention_probs(const uint16_t* q, int64_t q_sb, int64_t q_sh, int64_t q_sm, const uint16_t* k,
                                   int64_t k_sb, int64_t k_sh, int64_t k_sn, const float* lse, int B, int H, int M,
                                   int N, int D, float sm_scale, float* out, int64_t o_sb, int64_t o_sh, int64_t o_sm,
                                   int col0, void* stream) {
  if (!q || !k || !lse || !out) return AKV_ERR_NULL;
  if (B <= 0 || H <= 0 || M <= 0 || N < 0 || D <= 0 || D > 256 || col0 < 0) return AKV_ERR_SHAPE;
  if (N == 0) return AKV_OK;
  const int64_t total = static_cast<int64_t>(B) * H * N;
  attention_probs_kernel<<<gf_blocks(total, 8), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const __half*>(q), q_sb, q_sh, q_sm, reinterpret_cast<const __half*>(k), k_sb, k_sh, k_sn, lse,
      B, H, M, N, D, sm_scale, out, o_sb, o_sh, o_sm, col0);
  return cudaGetLastError() == cudaSuccess ? AKV_OK : AKV_ERR_LAUNCH;
}
