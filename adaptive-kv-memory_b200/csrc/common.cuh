// Device helpers shared by the warm-tier kernels (sm_100a).
//
// Everything here is hand-written inline PTX / CUDA intrinsics:
//   * mbarrier + cp.async.bulk (1-D TMA) for streaming warm records into SMEM,
//   * mma.sync m16n8k16 (f16 x f16 -> f32) and movmatrix for the decode
//     contraction,
//   * the "1024 + code" fp16 bit trick that turns packed integer codes into
//     exact fp16 values with one LOP3 and one HFMA2 per pair.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

#include <atomic>

#include "akv_b200.h"

#define AKV_DEV __device__ __forceinline__

namespace akv {

constexpr int kBlockTokens = 32;   // tokens per warm block record

// Byte offsets inside one warm block record (the akv_warm_layout fields);
// akv_warm_layout_init and the decode kernel's compile-time offsets both
// come from here.  Everything up to ki depends only on (D, kb, vb).
struct RecLayout {
  int kc, vc, ks, kz, vs, vz, mask, flags, ki, vi, ko, vo, vd, bytes;
};

__host__ __device__ constexpr int up16c(int x) { return (x + 15) & ~15; }

// Decode pair order of a key chunk.  The decode kernel turns the packed K
// codes of 32 channels (one 16/12/8-byte chunk of a token row) into 16 fp16
// pairs with one LOP3 "magic" each; pair i holds channels (a, b) =
// key_pair(bits, i) of the chunk, chosen so that both codes sit in the low 10
// bits of their 16-bit half (4 bits: nibbles n and n+4 of a byte pair; 2/3
// bits: codes 8 apart).  Warm records store the K scale and zero of each
// chunk in this order (word i = (channel a, channel b)), so the decoder reads
// each pair's scale and zero with one load.
struct PairIdx {
  int a, b;
};

__host__ __device__ constexpr PairIdx key_pair(int bits, int i) {
  const int j = i % 8;
  if (bits == 4) {
    const int a = 8 * (i / 4) + ((i % 4) ^ 1);
    return PairIdx{a, a + 4};
  }
  const int a = 16 * (i / 8) + (bits == 2 ? (j < 4 ? 3 - j : 11 - j) : 7 - j);
  return PairIdx{a, a + 8};
}

// slot (0..31) of channel c (0..31) of a chunk in the decode pair order (the
// inverse of key_pair in closed form: channel c is the a (b) member of pair i
// and sits in slot 2i (2i + 1))
__host__ __device__ constexpr int key_pair_slot(int bits, int c) {
  if (bits == 4) return 2 * (4 * (c >> 3) + ((c & 3) ^ 1)) + ((c & 7) >> 2);
  return 2 * (8 * (c >> 4) + ((c & 7) ^ (bits == 2 ? 3 : 7))) + ((c & 15) >> 3);
}

__host__ __device__ constexpr RecLayout rec_layout(int D, int kb, int vb, int n) {
  RecLayout r{};
  r.kc = 0;
  r.vc = up16c(kBlockTokens * D * kb / 8);
  r.ks = r.vc + up16c(kBlockTokens * D * vb / 8);
  r.kz = r.ks + up16c(2 * D);
  r.vs = r.kz + up16c(2 * D);
  r.vz = r.vs + up16c(2 * kBlockTokens);
  r.mask = r.vz + up16c(2 * kBlockTokens);  // u32 valid-slot mask
  r.flags = r.mask + 4;                      // u8[4]: K / V decode flags
  r.ki = r.mask + 8;                         // n int16 K outlier ids
  r.vi = r.ki + 2 * n;                       // n int16 V outlier ids
  r.ko = up16c(r.ki + 4 * n);
  r.vo = r.ko + up16c(2 * kBlockTokens * n);
  r.vd = r.vo + up16c(2 * kBlockTokens * n);
  r.bytes = r.vd + up16c(2 * kBlockTokens * n);
  return r;
}

// Every mbarrier wait is bounded in time: after kWaitLimitNs of global-timer
// time without the phase completing it records AKV_ERR_TIMEOUT in the status
// word and the kernel stops issuing work.  Each try_wait asks the hardware to
// suspend the waiting thread for up to kSuspendHintNs (it resumes as soon as
// the phase completes), so waiting warps leave the issue slots to the warps
// that have work instead of spinning.
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s
constexpr uint32_t kSuspendHintNs = 1000000u;     // 1 ms

// ---------------------------------------------------------------- launch set-up
// Dynamic shared memory above 48 KB needs a per-function attribute; setting
// it costs a driver call, so each kernel instance (template argument) keeps
// the largest size it has been given per device and sets it only when a
// larger one is asked for.
template <auto Kern>
inline bool ensure_dynamic_smem(size_t smem) {
  if (smem <= 48 * 1024) return true;
  constexpr int kDevices = 64;
  static std::atomic<int> have[kDevices];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  if (dev < 0 || dev >= kDevices)
    return cudaFuncSetAttribute(Kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) ==
           cudaSuccess;
  int cur = have[dev].load(std::memory_order_acquire);
  if (cur >= static_cast<int>(smem)) return true;
  if (cudaFuncSetAttribute(Kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) != cudaSuccess)
    return false;
  while (cur < static_cast<int>(smem) && !have[dev].compare_exchange_weak(cur, static_cast<int>(smem))) {
  }
  return true;
}

// ---------------------------------------------------------------- status// ---------------------------------------------------------------- status
AKV_DEV void set_status(int* status, int code) {
  if (status) atomicCAS(status, 0, code);
}

// ---------------------------------------------------------------- smem
AKV_DEV uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- mbarrier
AKV_DEV void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

AKV_DEV void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

AKV_DEV void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
               : "memory");
}

AKV_DEV void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
                   smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

AKV_DEV bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(kSuspendHintNs)
      : "memory");
  return ok != 0;
}

AKV_DEV uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait: returns false (and records a timeout) if the phase does not
// complete within limit_ns (kWaitLimitNs in every kernel; the self-test entry
// akv_selftest_wait passes a short one).
AKV_DEV bool mbar_wait(uint64_t* bar, uint32_t parity, int* status, uint64_t limit_ns = kWaitLimitNs) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (global_timer_ns() - t0 > limit_ns) {
      set_status(status, AKV_ERR_TIMEOUT);
      return false;
    }
  }
  return true;
}

// Order this thread's earlier generic-proxy shared-memory accesses before
// later async-proxy (TMA) writes to the same buffer.
AKV_DEV void fence_proxy_async_shared() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// 1-D bulk TMA copy global -> shared, completion counted on an mbarrier.
// dst/src 16-byte aligned, bytes a multiple of 16.  One CTA only.
AKV_DEV void tma_load_1d(void* dst_smem, const void* src_gmem, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst_smem)),
      "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// ---------------------------------------------------------------- loads
// 16-byte global -> shared copy that bypasses registers and L1 (cp.async.cg);
// both addresses 16-byte aligned.
AKV_DEV void cp_async16(void* dst_smem, const void* src_gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst_smem)), "l"(src_gmem) : "memory");
}

// Wait until every cp.async this thread issued has landed in shared memory.
AKV_DEV void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

AKV_DEV uint4 ldg_nc_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

AKV_DEV uint4 lds_v4(const void* p) { return *reinterpret_cast<const uint4*>(p); }
AKV_DEV void lds_u32x4(const void* p, uint32_t (&w)[4]) {
  const uint4 v = *reinterpret_cast<const uint4*>(p);
  w[0] = v.x;
  w[1] = v.y;
  w[2] = v.z;
  w[3] = v.w;
}
AKV_DEV uint2 lds_v2(const void* p) { return *reinterpret_cast<const uint2*>(p); }
AKV_DEV uint32_t lds_u32(const void* p) { return *reinterpret_cast<const uint32_t*>(p); }

// ---------------------------------------------------------------- bit tricks
AKV_DEV uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) { return __byte_perm(a, b, sel); }

// (x & mask) | 0x64006400 in one LOP3: each 16-bit half becomes the fp16
// value 1024 + (x & mask_half) as long as the mask lies in bits 0..9.
template <uint32_t MASK>
AKV_DEV uint32_t lop_magic(uint32_t x) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(x), "n"(MASK), "n"(0x64006400u));
  return r;
}

// fp16 bits of +-2^e (|e| <= 14), as a compile-time constant
constexpr uint32_t fp16_pow2_bits(int e, bool negative) {
  return (negative ? 0x8000u : 0u) | (static_cast<uint32_t>(15 + e) << 10);
}

constexpr int log2_pow2(int m) { return m <= 1 ? 0 : 1 + log2_pow2(m / 2); }

// Undo the magic offset exactly: (1024 + m*c)/m - 1024/m == c for power-of-two m.
// Both constants are exact fp16 powers of two, written as compile-time bit
// patterns (no runtime conversion).
template <int MULT>
AKV_DEV uint32_t fix_magic(uint32_t x) {
  constexpr int k = log2_pow2(MULT);
  constexpr uint32_t inv = fp16_pow2_bits(-k, false) * 0x10001u;     // (1/m, 1/m)
  constexpr uint32_t off = fp16_pow2_bits(10 - k, true) * 0x10001u;  // (-1024/m, -1024/m)
  uint32_t r;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(x), "r"(inv), "r"(off));
  return r;
}

// Scales for which the decode's two-op dequantisation is exact: +0 or
// [2^-14, 65504/1024].  With x = 1024 + M*c (the magic form, M = 2^k),
//   y = fma(x, s, -1024*s) = fp16(M*c*s) = M*fp16(c*s)   (-1024*s exact, no overflow,
//                                                          c*s normal or 0)
//   fma(y, 1/M, z) = fp16(fp16(c*s) + z)                  (y/M exact)
// which is the reference's codes.half() * scale + zero with both roundings
// (checked exhaustively over every such scale, code, multiplier and a
// stride-7 sample of all fp16 zeros).  The quantiser flags each warm record
// whose scales all qualify.
AKV_DEV bool dq2_scale_ok(__half s) {
  const unsigned short u = __half_as_ushort(s);
  return u == 0 || (u >= 0x0400 && u <= 0x53FF);
}

template <uint32_t MASK, int MULT>
AKV_DEV uint32_t code_pair(uint32_t x) {
  return fix_magic<MULT>(lop_magic<MASK>(x));
}

AKV_DEV uint32_t h2_as_u32(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
AKV_DEV __half2 u32_as_h2(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }

AKV_DEV uint32_t pack_h2(float lo, float hi) { return h2_as_u32(__floats2half2_rn(lo, hi)); }

// ---------------------------------------------------------------- MMA
// D = A(16x16, row) * B(16x8, col) + D, f16 inputs, f32 accumulate.
AKV_DEV void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                       uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Transpose an 8x8 b16 matrix held in the m8n8 fragment layout.
AKV_DEV uint32_t movmatrix_trans(uint32_t a) {
  uint32_t d;
  asm("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(d) : "r"(a));
  return d;
}

// ---------------------------------------------------------------- packed fp32 (sm_100)
// Two IEEE fp32 lanes per 64-bit register; each lane rounds like the scalar op.
AKV_DEV uint64_t f2_make(float lo, float hi) {
  uint64_t d;
  asm("mov.b64 %0, {%1, %2};" : "=l"(d) : "f"(lo), "f"(hi));
  return d;
}

AKV_DEV float2 f2_split(uint64_t v) {
  float2 r;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
  return r;
}

AKV_DEV uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

AKV_DEV uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}

// c + a*b for fp16 a, b and fp32 c with one rounding; the fp16 product is
// exact in fp32, so this equals fmaf(float(a), float(b), c).
AKV_DEV float fma_f16_f32(__half a, __half b, float c) {
  float d;
  asm("fma.rn.f32.f16 %0, %1, %2, %3;" : "=f"(d) : "h"(__half_as_ushort(a)), "h"(__half_as_ushort(b)), "f"(c));
  return d;
}

AKV_DEV float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

}  // namespace akv
