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
// One CTA quantises one scale group (all heads of one batch row): it stages
// the group's fp16 rows in shared memory with 128-bit loads, runs the
// outlier-channel selection and the min/max reductions there, then encodes
// and packs 32 codes per thread.
#include <cuda_runtime.h>

#include <algorithm>

#include "common.cuh"

namespace akv {

struct QuantParams {
  const __half* src;
  int64_t sb, sh, sn;
  const int64_t* tok_idx;
  int64_t tok_sb;
  int B, H, N, D, bits, is_key, group, n_out;
  akv_qdest dst;
  int* status;
};

constexpr int kQuantThreads = 256;
constexpr int kMaxOutliers = 32;

__host__ __device__ inline int pad_pitch(int D) { return D + 8; }  // halves; +16 B per row

AKV_DEV char* vaddr(const akv_view& v, int b, int h, int blk, int slot) {
  return static_cast<char*>(v.ptr) + b * v.sb + h * v.sh + blk * v.sblk + slot * v.sslot;
}

AKV_DEV uint32_t quant_code(float x, float zero, float scale, float maxval) {
  const float diff = __half2float(__float2half_rn(__fsub_rn(x, zero)));
  float r = __half2float(__float2half_rn(__fdiv_rn(diff, scale)));
  r = rintf(r);
  r = fminf(fmaxf(r, 0.0f), maxval);  // fmaxf(NaN, 0) == 0: the reference's NaN -> 0 cast
  return static_cast<uint32_t>(r);
}

// Pack 32 codes (c[0..31]) into 4*BITS bytes following akv/bitpack.py, as
// little-endian u32 words w[0..BITS-1].
template <int BITS>
AKV_DEV void pack32(const uint32_t (&c)[32], uint32_t (&w)[BITS]) {
  if constexpr (BITS == 4) {
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      uint32_t x = 0;
#pragma unroll
      for (int i = 0; i < 4; ++i) x |= ((c[8 * k + 2 * i] << 4) | c[8 * k + 2 * i + 1]) << (8 * i);
      w[k] = x;
    }
  } else if constexpr (BITS == 2) {
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      uint32_t x = 0;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int j = 16 * k + 4 * i;
        x |= ((c[j] << 6) | (c[j + 1] << 4) | (c[j + 2] << 2) | c[j + 3]) << (8 * i);
      }
      w[k] = x;
    }
  } else {  // 3 bits: 8 codes -> 24-bit big-endian group -> 3 bytes
    uint32_t bytes[12];
#pragma unroll
    for (int gq = 0; gq < 4; ++gq) {
      uint32_t word = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) word |= c[8 * gq + j] << (21 - 3 * j);
      bytes[3 * gq + 0] = (word >> 16) & 0xFF;
      bytes[3 * gq + 1] = (word >> 8) & 0xFF;
      bytes[3 * gq + 2] = word & 0xFF;
    }
#pragma unroll
    for (int k = 0; k < 3; ++k)
      w[k] = bytes[4 * k] | (bytes[4 * k + 1] << 8) | (bytes[4 * k + 2] << 16) | (bytes[4 * k + 3] << 24);
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
AKV_DEV void store_words(char* p, const uint32_t (&w)[BITS]) {
  if constexpr (BITS == 4) {
    if ((reinterpret_cast<uintptr_t>(p) & 15) == 0) {
      *reinterpret_cast<uint4*>(p) = make_uint4(w[0], w[1], w[2], w[3]);
      return;
    }
  } else if constexpr (BITS == 2) {
    if ((reinterpret_cast<uintptr_t>(p) & 7) == 0) {
      *reinterpret_cast<uint2*>(p) = make_uint2(w[0], w[1]);
      return;
    }
  }
#pragma unroll
  for (int k = 0; k < BITS; ++k) reinterpret_cast<uint32_t*>(p)[k] = w[k];
}

template <int BITS>
AKV_DEV void load_words(const char* p, uint32_t (&w)[BITS]) {
#pragma unroll
  for (int k = 0; k < BITS; ++k) w[k] = reinterpret_cast<const uint32_t*>(p)[k];
}

// ---------------------------------------------------------------------------
// quantise: grid (n_groups, B), block kQuantThreads
// ---------------------------------------------------------------------------
template <int BITS, bool IS_KEY>
__global__ void __launch_bounds__(kQuantThreads) quantize_group_kernel(const QuantParams p) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int tid = threadIdx.x;
  const int b = blockIdx.y;
  const int t0 = blockIdx.x * p.group;
  const int nt = min(p.group, p.N - t0);
  const int H = p.H, D = p.D;
  const int pitch = pad_pitch(D);
  const float maxval = static_cast<float>((1 << BITS) - 1);

  __half* xs = reinterpret_cast<__half*>(smem_raw);                      // [H][nt][pitch]
  __half* kmin = xs + static_cast<size_t>(H) * nt * pitch;               // [H][D] (keys)
  __half* kmax = kmin + H * D;                                           // [H][D] -> scale
  float* norms = reinterpret_cast<float*>(kmax + H * D);                 // [H][D]
  float* score = norms + H * D;                                          // [D]
  int* oidx = reinterpret_cast<int*>(score + D);                         // [kMaxOutliers]
  __half* od_s = reinterpret_cast<__half*>(oidx + kMaxOutliers);         // [H][nt][n_out] originals

  // ---- stage the group's rows (128-bit loads, 16 B per thread-iteration)
  const int vpr = D / 8;
  for (int v = tid; v < H * nt * vpr; v += kQuantThreads) {
    const int c = v % vpr;
    const int r = v / vpr;
    const int t = r % nt;
    const int h = r / nt;
    const int64_t row = p.tok_idx ? p.tok_idx[b * p.tok_sb + t0 + t] : static_cast<int64_t>(t0 + t);
    const __half* g = p.src + b * p.sb + h * p.sh + row * p.sn + c * 8;
    *reinterpret_cast<uint4*>(xs + (static_cast<size_t>(h) * nt + t) * pitch + c * 8) = ldg_nc_v4(g);
  }
  __syncthreads();

  const __half2* xs2 = reinterpret_cast<const __half2*>(xs);
  const int p2 = pitch / 2;

  // ---- outlier channels (affine_quantizer.py:75-85 / :143-151)
  if (p.n_out > 0) {
    for (int w = tid; w < H * (D / 2); w += kQuantThreads) {
      const int h = w / (D / 2), dp = w % (D / 2);
      float s0 = 0.f, s1 = 0.f;
      for (int t = 0; t < nt; ++t) {
        const float2 x = __half22float2(xs2[(h * nt + t) * p2 + dp]);
        s0 = fmaf(x.x, x.x, s0);
        s1 = fmaf(x.y, x.y, s1);
      }
      norms[h * D + 2 * dp] = sqrtf(s0);
      norms[h * D + 2 * dp + 1] = sqrtf(s1);
    }
    __syncthreads();
    for (int d = tid; d < D; d += kQuantThreads) {
      float s = 0.f;
      for (int h = 0; h < H; ++h) s += norms[h * D + d];
      score[d] = s / static_cast<float>(H);
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
    __syncthreads();
    // side store: fp16 originals of the outlier channels, then their ids
    const akv_view& od = p.dst.out_data;
    for (int w = tid; w < H * nt * p.n_out; w += kQuantThreads) {
      const int j = w % p.n_out;
      const int t = (w / p.n_out) % nt;
      const int h = w / (p.n_out * nt);
      const int tt = t0 + t;
      const __half o = xs[(static_cast<size_t>(h) * nt + t) * pitch + oidx[j]];
      od_s[w] = o;  // w == (h*nt + t)*n_out + j
      if (od.ptr) reinterpret_cast<__half*>(vaddr(od, b, h, tt / kBlockTokens, tt % kBlockTokens))[j] = o;
    }
    const akv_view& oi = p.dst.out_idx;
    if (oi.ptr) {
      const int blk0 = t0 / kBlockTokens, nblk = (t0 + nt - 1) / kBlockTokens - blk0 + 1;
      for (int w = tid; w < H * nblk * p.n_out; w += kQuantThreads) {
        const int j = w % p.n_out;
        const int bl = (w / p.n_out) % nblk;
        const int h = w / (p.n_out * nblk);
        reinterpret_cast<int16_t*>(vaddr(oi, b, h, blk0 + bl, 0))[j] = static_cast<int16_t>(oidx[j]);
      }
    }
    __syncthreads();
    // zero the outlier channels before min/max (affine_quantizer.py:84-85)
    for (int w = tid; w < H * nt * p.n_out; w += kQuantThreads) {
      const int j = w % p.n_out;
      const int r = w / p.n_out;
      xs[static_cast<size_t>(r) * pitch + oidx[j]] = __float2half_rn(0.0f);
    }
    __syncthreads();
  }

  // ---- keys: per-(head, channel) min/max over the group's tokens -> scale/zero
  if constexpr (IS_KEY) {
    for (int w = tid; w < H * (D / 2); w += kQuantThreads) {
      const int h = w / (D / 2), dp = w % (D / 2);
      __half2 mn = __float2half2_rn(INFINITY), mx = __float2half2_rn(-INFINITY);
      for (int t = 0; t < nt; ++t) {
        const __half2 x = xs2[(h * nt + t) * p2 + dp];
        mn = __hmin2(mn, x);
        mx = __hmax2(mx, x);
      }
      const float2 lo = __half22float2(mn), hi = __half22float2(mx);
      const float sc0 = __half2float(__float2half_rn(__fsub_rn(hi.x, lo.x)));
      const float sc1 = __half2float(__float2half_rn(__fsub_rn(hi.y, lo.y)));
      reinterpret_cast<__half2*>(kmin)[w] = mn;
      reinterpret_cast<__half2*>(kmax)[w] =
          __halves2half2(__float2half_rn(__fdiv_rn(sc0, maxval)), __float2half_rn(__fdiv_rn(sc1, maxval)));
    }
    __syncthreads();
    const int blk0 = t0 / kBlockTokens, nblk = (t0 + nt - 1) / kBlockTokens - blk0 + 1;
    for (int w = tid; w < H * nblk * (D / 2); w += kQuantThreads) {
      const int dp = w % (D / 2);
      const int bl = (w / (D / 2)) % nblk;
      const int h = w / ((D / 2) * nblk);
      if (p.dst.scale.ptr)
        reinterpret_cast<__half2*>(vaddr(p.dst.scale, b, h, blk0 + bl, 0))[dp] =
            reinterpret_cast<const __half2*>(kmax)[h * (D / 2) + dp];
      if (p.dst.zero.ptr)
        reinterpret_cast<__half2*>(vaddr(p.dst.zero, b, h, blk0 + bl, 0))[dp] =
            reinterpret_cast<const __half2*>(kmin)[h * (D / 2) + dp];
    }
  }

  // ---- encode + pack: one thread per (head, token, 32-code chunk)
  const int nsu = D / 32;  // 1..8, divides 32
  const int total = H * nt * nsu;
  const int rounds = (total + kQuantThreads - 1) / kQuantThreads;
  for (int rd = 0; rd < rounds; ++rd) {
    const int w = rd * kQuantThreads + tid;
    const bool valid = w < total;
    const int su = w % nsu;
    const int r = valid ? w / nsu : 0;
    const int t = r % nt;
    const int h = r / nt;
    const __half* row = xs + static_cast<size_t>(r) * pitch + su * 32;
    __half x[32];
#pragma unroll
    for (int k = 0; k < 4; ++k) *reinterpret_cast<uint4*>(x + 8 * k) = lds_v4(row + 8 * k);
    float zf[32], sf[32];
    if constexpr (IS_KEY) {
#pragma unroll
      for (int k = 0; k < 32; ++k) {
        zf[k] = __half2float(kmin[h * D + su * 32 + k]);
        sf[k] = __half2float(kmax[h * D + su * 32 + k]);
      }
    } else {
      // per-token min/max over D: reduce this chunk, then across the nsu lanes of the row
      __half mn = x[0], mx = x[0];
#pragma unroll
      for (int k = 1; k < 32; ++k) {
        mn = __hmin(mn, x[k]);
        mx = __hmax(mx, x[k]);
      }
      for (int o = 1; o < nsu; o <<= 1) {
        const __half omn = __shfl_xor_sync(0xffffffffu, mn, o);
        const __half omx = __shfl_xor_sync(0xffffffffu, mx, o);
        mn = __hmin(mn, omn);
        mx = __hmax(mx, omx);
      }
      const float lo = __half2float(mn), hi = __half2float(mx);
      const float range = __half2float(__float2half_rn(__fsub_rn(hi, lo)));
      const __half sc = __float2half_rn(__fdiv_rn(range, maxval));
      if (valid && su == 0) {
        const int tt = t0 + t;
        if (p.dst.scale.ptr)
          *reinterpret_cast<__half*>(vaddr(p.dst.scale, b, h, tt / kBlockTokens, tt % kBlockTokens)) = sc;
        if (p.dst.zero.ptr)
          *reinterpret_cast<__half*>(vaddr(p.dst.zero, b, h, tt / kBlockTokens, tt % kBlockTokens)) = mn;
      }
#pragma unroll
      for (int k = 0; k < 32; ++k) {
        zf[k] = lo;
        sf[k] = __half2float(sc);
      }
    }
    if (!valid) continue;
    uint32_t c[32];
#pragma unroll
    for (int k = 0; k < 32; ++k) c[k] = quant_code(__half2float(x[k]), zf[k], sf[k], maxval);
    if constexpr (!IS_KEY) {
      // outlier residual: fp16 original minus what the zeroed channel dequantises to
      if (p.n_out > 0 && p.dst.out_resid.ptr) {
        const int tt = t0 + t;
        float* rp = reinterpret_cast<float*>(vaddr(p.dst.out_resid, b, h, tt / kBlockTokens, tt % kBlockTokens));
        for (int j = 0; j < p.n_out; ++j) {
          const int d = oidx[j] - su * 32;
          if (d < 0 || d >= 32) continue;
          uint32_t cv = 0;
#pragma unroll
          for (int k = 0; k < 32; ++k)
            if (k == d) cv = c[k];
          const __half deq = __hadd_rn(__hmul_rn(__uint2half_rn(cv), __float2half_rn(sf[0])), __float2half_rn(zf[0]));
          rp[j] = __half2float(od_s[(h * nt + t) * p.n_out + j]) - __half2float(deq);
        }
      }
    }
    uint32_t wds[BITS];
    pack32<BITS>(c, wds);
    const int tt = t0 + t;
    if (p.dst.codes.ptr)
      store_words<BITS>(vaddr(p.dst.codes, b, h, tt / kBlockTokens, tt % kBlockTokens) + su * 4 * BITS, wds);
  }

  // ---- valid-slot masks for the blocks this group wrote
  if (p.dst.mask.ptr) {
    const int blk0 = t0 / kBlockTokens, blk1 = (t0 + nt - 1) / kBlockTokens;
    for (int w = tid; w < H * (blk1 - blk0 + 1); w += kQuantThreads) {
      const int bl = blk0 + w % (blk1 - blk0 + 1);
      const int h = w / (blk1 - blk0 + 1);
      const int lo = max(t0, bl * kBlockTokens) - bl * kBlockTokens;
      const int hi = min(t0 + nt, (bl + 1) * kBlockTokens) - bl * kBlockTokens;  // exclusive
      const uint32_t m = (hi - lo == 32) ? 0xffffffffu : (((1u << (hi - lo)) - 1u) << lo);
      *reinterpret_cast<uint32_t*>(vaddr(p.dst.mask, b, h, bl, 0)) = m;
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
  int B, H, N, D, n_out;
  __half* out;
  int64_t osb, osh, osn;
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
    const int64_t tok = p.tok_idx ? p.tok_idx[b * p.tok_sb + n] : n;
    const int blk = static_cast<int>(tok / kBlockTokens), slot = static_cast<int>(tok % kBlockTokens);
    uint32_t wds[BITS];
    load_words<BITS>(vaddr(p.src.codes, b, h, blk, slot) + su * 4 * BITS, wds);
    uint32_t c[32];
    unpack32<BITS>(wds, c);
    __half o[32];
    if constexpr (IS_KEY) {
      const __half* sc = reinterpret_cast<const __half*>(vaddr(p.src.scale, b, h, blk, 0)) + su * 32;
      const __half* zr = reinterpret_cast<const __half*>(vaddr(p.src.zero, b, h, blk, 0)) + su * 32;
#pragma unroll
      for (int k = 0; k < 32; ++k) o[k] = __hadd_rn(__hmul_rn(__uint2half_rn(c[k]), sc[k]), zr[k]);
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

size_t quant_smem_bytes(int H, int nt, int D, int n_out) {
  return static_cast<size_t>(H) * nt * pad_pitch(D) * 2 + static_cast<size_t>(H) * D * 4 +
         static_cast<size_t>(H) * D * 4 + D * 4 + kMaxOutliers * 4 + static_cast<size_t>(H) * nt * n_out * 2;
}

template <int BITS, bool IS_KEY>
static int launch_quant(const QuantParams& p, cudaStream_t st) {
  const int ngroups = (p.N + p.group - 1) / p.group;
  const int nt = min(p.group, p.N);
  const size_t smem = quant_smem_bytes(p.H, nt, p.D, p.n_out);
  auto kern = quantize_group_kernel<BITS, IS_KEY>;
  if (smem > 48 * 1024) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) !=
        cudaSuccess)
      return AKV_ERR_LAUNCH;
  }
  kern<<<dim3(ngroups, p.B), kQuantThreads, smem, st>>>(p);
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

extern "C" int akv_quantize(const uint16_t* src, int64_t src_sb, int64_t src_sh, int64_t src_sn,
                            const int64_t* tok_idx, int64_t tok_sb, int B, int H, int N, int D, int bits,
                            int is_key, int group, int n_outlier, const akv_qdest* dst, int* status,
                            void* stream) {
  if (!src || !dst) return AKV_ERR_NULL;
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
  if (dst->out_resid.ptr && (!aligned(dst->out_resid.ptr, 4) || dst->out_resid.sslot % 4)) return AKV_ERR_ALIGN;
  if (quant_smem_bytes(H, group, D, n_outlier) > 220 * 1024) return AKV_ERR_UNSUPPORTED;
  QuantParams p{reinterpret_cast<const __half*>(src), src_sb, src_sh, src_sn, tok_idx, tok_sb, B, H, N, D,
                bits, is_key, group, n_outlier, *dst, status};
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (bits * 2 + (is_key ? 1 : 0)) {
    case 5: return launch_quant<2, true>(p, st);
    case 4: return launch_quant<2, false>(p, st);
    case 7: return launch_quant<3, true>(p, st);
    case 6: return launch_quant<3, false>(p, st);
    case 9: return launch_quant<4, true>(p, st);
    default: return launch_quant<4, false>(p, st);
  }
}

extern "C" int akv_dequantize(const akv_qdest* src, const int64_t* tok_idx, int64_t tok_sb, int B, int H, int N,
                              int D, int bits, int is_key, int n_outlier, uint16_t* out, int64_t out_sb,
                              int64_t out_sh, int64_t out_sn, void* stream) {
  if (!src || !out || !src->codes.ptr || !src->scale.ptr || !src->zero.ptr) return AKV_ERR_NULL;
  if (n_outlier > 0 && (!src->out_idx.ptr || !src->out_data.ptr)) return AKV_ERR_NULL;
  if (bits < 2 || bits > 4) return AKV_ERR_BITS;
  if (B <= 0 || H <= 0 || N < 0 || D <= 0 || D % 32 != 0 || D > 256) return AKV_ERR_SHAPE;
  if (N == 0) return AKV_OK;
  if (!aligned(out, 16) || out_sb % 8 || out_sh % 8 || out_sn % 8) return AKV_ERR_ALIGN;
  if (!aligned(src->codes.ptr, 4) || src->codes.sb % 4 || src->codes.sh % 4 || src->codes.sblk % 4 ||
      src->codes.sslot % 4)
    return AKV_ERR_ALIGN;
  DequantParams p{*src, tok_idx, tok_sb, B, H, N, D, n_outlier, reinterpret_cast<__half*>(out),
                  out_sb, out_sh, out_sn};
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
