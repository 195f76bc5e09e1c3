// Mixed-tier prefill attention on the 5th-generation tensor cores (tcgen05).
//
// Many query tokens at once (a prompt, or a chunk of one) attend over the
// FP16 hot tier and the packed warm block records, causally by token
// position: query token i sees key token j iff pos(j) <= pos(i).  This is the
// attention the reference runs with SDPA over AKVLayer's chronological FP16
// view (akv/drop_in.py:753-787) during prefill; here the warm tier is read
// from its packed records and dequantised exactly like the reference
// (fp16(fp16(code*scale) + zero), outlier channels replaced by their fp16
// originals, akv/affine_quantizer.py:112-124, :178-189) into shared memory,
// one 128-token tile at a time, and never written back to HBM.
//
// One CTA (4 warps) owns 128 query rows of one (batch row, query head) and
// loops over 128-token key tiles (4 warm records, or 128 hot rows):
//   S = Q K^T     tcgen05.mma kind::f16, M=128 N=128, K=128 (8 k-steps),
//                 operands in shared memory, accumulator in tensor memory
//   softmax       thread t owns query row t = TMEM lane t (tcgen05.ld),
//                 online max with lazy rescaling; P is written back over S
//                 in tensor memory as two fp16 terms hi + lo (exact to ~2^-22)
//   O += P V      two tcgen05.mma per k-step (hi, lo) with A read from tensor
//                 memory, V read MN-major from shared memory, O accumulated in
//                 tensor memory
// Q and hot K/V tiles arrive by tensor TMA (cp.async.bulk.tensor, this GPU's
// memory only, one CTA per copy); warm tiles are dequantised by the CTA's threads.
// Two CTAs fit on an SM (96 KB of tiles, 256 TMEM columns each), so one CTA's
// MMAs overlap the other's softmax and dequantisation.
//
// Shared-memory operand layout (no swizzle, the UMMA "interleaved" canonical
// form): element (row r, col c) of a 128 x 128 fp16 tile sits at byte
//   (r % 8) * 16 + (r / 8) * 128 + (c / 8) * 2048 + (c % 8) * 2
// i.e. 8-row x 16-byte core matrices, 16 of them down the rows (128 B apart),
// one 2 KB column block per 8 columns.  As a K-major operand (rows = M or N,
// cols = K) the stride between 8-row groups is 128 B and between 8-column
// groups 2048 B; read MN-major (V: rows = keys = K, cols = channels = N) the
// roles swap.  A tensor TMA box of {8 channels, 128 rows} lands exactly one
// 2 KB column block.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cfloat>
#include <climits>
#include <cmath>
#include <mutex>

#include "common.cuh"

namespace akv {
namespace prefill {

constexpr int kD = 128;         // head dim
constexpr int kTile = 128;      // query rows per CTA, key tokens per tile
constexpr int kThreads = 128;   // 4 warps: thread t <-> query row t <-> TMEM lane t
constexpr int kTileBytes = kTile * kD * 2;  // 32 KB
constexpr int kTmemCols = 256;  // S at columns [0, 128), O at [128, 256)
constexpr float kLazy = 8.f;    // log2 headroom before the running max moves
constexpr float kLog2e = 1.4426950408889634f;

struct Params {
  const __half* q;
  int64_t q_sb, q_sh, q_sm;
  const int32_t* q_pos;
  int64_t qp_sb;
  int M;
  const __half* hk;
  const __half* hv;
  int64_t h_sb, h_sh, h_sn;
  int n_hot;
  const int32_t* hot_pos;
  int64_t hp_sb;
  const uint8_t* warm;
  int64_t w_sb, w_sh;
  akv_warm_layout L;
  int n_warm_blocks;
  const int32_t* warm_pos;  // [b * wp_sb + slot], slot = block * 32 + s
  int64_t wp_sb;
  int B, Hq, Hkv, g;
  float scale_log2;
  __half* out;
  int64_t o_sb, o_sh, o_sm;
  float* lse;  // [(b * Hq + h) * M + m]
  int* status;
};

// ------------------------------------------------------------------ tcgen05 helpers
// Shared-memory matrix descriptor, no swizzle: start address, leading-dimension
// byte offset (between core matrices along K), stride-dimension byte offset
// (between 8-row groups along M/N), all >> 4; bits 46-47 = 1 (sm_100 format).
AKV_DEV uint64_t smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) | (static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16) |
         (static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}

// Instruction descriptor of kind::f16: fp16 A and B, fp32 accumulator,
// A K-major, B K-major (b_mn = 0) or MN-major (b_mn = 1), shape M x N.
constexpr uint32_t instr_desc(int M, int N, int b_mn) {
  return (1u << 4) | (static_cast<uint32_t>(b_mn) << 16) | (static_cast<uint32_t>(N >> 3) << 17) |
         (static_cast<uint32_t>(M >> 4) << 24);
}

AKV_DEV void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
      : "memory");
}

// The same with A (M x K fp16, two K elements per 32-bit column) read from tensor memory.
AKV_DEV void umma_f16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
      : "memory");
}

// Arrive on `bar` once every tcgen05 operation this thread issued has completed.
AKV_DEV void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

AKV_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
AKV_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 32 consecutive fp32 columns of this thread's TMEM lane (warp w reads lanes 32w..32w+31).
AKV_DEV void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

AKV_DEV void tmem_st32(uint32_t taddr, const float (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
      "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
      "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
      "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
      "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
      "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
}

AKV_DEV void tmem_st32u(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
      "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]),
      "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]),
      "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}

AKV_DEV void tmem_st16u(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}

AKV_DEV void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
AKV_DEV void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Tensor TMA: box {8 channels, 128 rows, 1, 1} at (c0, c1, c2, c3) -> one 2 KB column block.
AKV_DEV void tma_load_4d(void* dst, const CUtensorMap* map, int c0, int c1, int c2, int c3, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
      "[%6];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar))
      : "memory");
}

// byte offset of element (r, c) in a tile (see the layout note above)
AKV_DEV uint32_t tile_off(int r, int c) {
  return static_cast<uint32_t>((r & 7) * 16 + (r >> 3) * 128 + (c >> 3) * 2048 + (c & 7) * 2);
}

// ------------------------------------------------------------------ warm tile rows
// Thread t handles token t of a warm tile (record t / 32, slot t % 32).  Its
// packed K and V code rows, its V scale / zero and its outlier originals are
// fetched into registers one visible tile ahead (16-byte loads, all in flight
// together); lane l of the record's warp also fetches bytes 8l..8l+7 of the
// record's K scales and zeros (stored in the decode pair order).  So the
// global-memory latency of the next tile hides behind the tensor-core work and
// the softmax of the current one.
constexpr int kPrefetchOut = 2;  // outlier channels kept in registers (more: read at dequantisation)

template <int KB, int VB>
struct WarmRow {
  uint4 k[KB];          // K codes: 128 * KB / 8 bytes
  uint4 v[VB];          // V codes
  uint2 ks2, kz2;       // this lane's K scale / zero pair words 2l, 2l+1 of its record
  uint2 ids;            // outlier ids: K at bytes 2j, V at bytes 2n + 2j (n <= 2)
  uint32_t vsz;         // V scale (low half) and zero (high half) of this token
  __half ko[kPrefetchOut], vo[kPrefetchOut];
  const uint8_t* rec;   // nullptr: beyond the written blocks
  int kp;               // the token's position (INT_MAX: empty slot)
  bool valid;           // slot holds a token (mask bit set)
};

template <int KB, int VB>
AKV_DEV void load_warm_row(const Params& p, int b, int kvh, int tile, int t, WarmRow<KB, VB>& w) {
  const int blk = tile * 4 + (t >> 5), slot = t & 31;
  w.valid = false;
  w.rec = nullptr;
  w.kp = INT_MAX;
  if (blk >= p.n_warm_blocks) return;
  const uint8_t* rec = p.warm + b * p.w_sb + kvh * p.w_sh + static_cast<int64_t>(blk) * p.L.bytes;
  w.rec = rec;
  const int n = p.L.n_outlier;
  w.ks2 = __ldg(reinterpret_cast<const uint2*>(rec + p.L.ks) + slot);
  w.kz2 = __ldg(reinterpret_cast<const uint2*>(rec + p.L.kz) + slot);
  w.ids = n > 0 ? __ldg(reinterpret_cast<const uint2*>(rec + p.L.ki)) : make_uint2(0u, 0u);
  const uint32_t mask = __ldg(reinterpret_cast<const uint32_t*>(rec + p.L.mask));
  w.valid = (mask >> slot) & 1u;
  const int kp = __ldg(p.warm_pos + b * p.wp_sb + blk * 32 + slot);
  w.kp = w.valid ? kp : INT_MAX;
  const uint4* kr = reinterpret_cast<const uint4*>(rec + p.L.kc + slot * (kD * KB / 8));
  const uint4* vr = reinterpret_cast<const uint4*>(rec + p.L.vc + slot * (kD * VB / 8));
#pragma unroll
  for (int i = 0; i < KB; ++i) w.k[i] = __ldg(kr + i);
#pragma unroll
  for (int i = 0; i < VB; ++i) w.v[i] = __ldg(vr + i);
  w.vsz = static_cast<uint32_t>(__half_as_ushort(__ldg(reinterpret_cast<const __half*>(rec + p.L.vs) + slot))) |
          (static_cast<uint32_t>(__half_as_ushort(__ldg(reinterpret_cast<const __half*>(rec + p.L.vz) + slot))) << 16);
#pragma unroll
  for (int j = 0; j < kPrefetchOut; ++j) {
    w.ko[j] = j < n ? __ldg(reinterpret_cast<const __half*>(rec + p.L.ko) + slot * n + j) : __float2half_rn(0.f);
    w.vo[j] = j < n ? __ldg(reinterpret_cast<const __half*>(rec + p.L.vo) + slot * n + j) : __float2half_rn(0.f);
  }
}

// K scales / zeros of this warp's record in natural channel order: pair word
// wi holds channels key_pair(KB, wi % 16) of 32-channel chunk wi / 16.
template <int KB, int VB>
AKV_DEV void stage_kscale(const WarmRow<KB, VB>& w, int lane, __half* ks, __half* kz) {
  const uint32_t sw[2] = {w.ks2.x, w.ks2.y}, zw[2] = {w.kz2.x, w.kz2.y};
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int wi = 2 * lane + j;
    const PairIdx pi = key_pair(KB, wi & 15);
    const int c0 = 32 * (wi >> 4);
    const bool have = w.rec != nullptr;
    ks[c0 + pi.a] = __ushort_as_half(have ? static_cast<unsigned short>(sw[j] & 0xFFFFu) : 0);
    ks[c0 + pi.b] = __ushort_as_half(have ? static_cast<unsigned short>(sw[j] >> 16) : 0);
    kz[c0 + pi.a] = __ushort_as_half(have ? static_cast<unsigned short>(zw[j] & 0xFFFFu) : 0);
    kz[c0 + pi.b] = __ushort_as_half(have ? static_cast<unsigned short>(zw[j] >> 16) : 0);
  }
}

// code of channel C in a packed row held as 32-bit words (akv/bitpack.py
// layouts: 4 bits even channel in the high nibble, 2 bits MSB first, 3 bits
// 24-bit big-endian groups); C is a template argument, so every shift and
// word index is a constant
template <int BITS, int C, int NW>
AKV_DEV uint32_t code_of(const uint32_t (&w)[NW]) {
  if constexpr (BITS == 4) {
    constexpr int by = C >> 1;
    return (w[by >> 2] >> (8 * (by & 3) + ((C & 1) ? 0 : 4))) & 15u;
  } else if constexpr (BITS == 2) {
    constexpr int by = C >> 2;
    return (w[by >> 2] >> (8 * (by & 3) + 6 - 2 * (C & 3))) & 3u;
  } else {
    constexpr int b0 = 3 * (C >> 3);       // bytes b0..b0+2 form a big-endian 24-bit word
    constexpr int bit = 21 - 3 * (C & 7);  // code j of the group at bits 21-3j .. 23-3j
    const uint32_t w24 = (((w[b0 >> 2] >> (8 * (b0 & 3))) & 0xFFu) << 16) |
                         (((w[(b0 + 1) >> 2] >> (8 * ((b0 + 1) & 3))) & 0xFFu) << 8) |
                         ((w[(b0 + 2) >> 2] >> (8 * ((b0 + 2) & 3))) & 0xFFu);
    return (w24 >> bit) & 7u;
  }
}

// channels (C, C+1) (C even) as exact fp16 codes.  4 and 2 bits: the byte
// holding both codes is copied into both 16-bit halves (PRMT), one LOP3 keeps
// each half's code bits in place and ORs in the exponent of 1024, giving
// (1024 + M0*c0, 1024 + M1*c1) with power-of-two M, and one HFMA2
// x * (1/M0, 1/M1) - (1024/M0, 1024/M1) gives (c0, c1) exactly.  3 bits:
// the codes are extracted and (1024 + code) - 1024 is formed directly.
template <int BITS, int C, int NW>
AKV_DEV __half2 code_pair_h2(const uint32_t (&w)[NW]) {
  if constexpr (BITS == 4 || BITS == 2) {
    constexpr int by = BITS == 4 ? C >> 1 : C >> 2;  // byte of the row holding channels C and C+1
    constexpr uint32_t k = by & 3;
    const uint32_t y = prmt(w[by >> 2], 0u, k | (4u << 4) | (k << 8) | (4u << 12));  // (byte, byte)
    // code masks in the byte (even channel first) and their multipliers
    constexpr uint32_t m0 = BITS == 4 ? 0xF0u : ((C & 2) ? 0x0Cu : 0xC0u);
    constexpr uint32_t m1 = BITS == 4 ? 0x0Fu : ((C & 2) ? 0x03u : 0x30u);
    constexpr int e0 = BITS == 4 ? 4 : ((C & 2) ? 2 : 6), e1 = BITS == 4 ? 0 : ((C & 2) ? 0 : 4);
    uint32_t x;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(x) : "r"(y), "n"(m0 | (m1 << 16)), "n"(0x64006400u));
    constexpr uint32_t inv = fp16_pow2_bits(-e0, false) | (fp16_pow2_bits(-e1, false) << 16);
    constexpr uint32_t off = fp16_pow2_bits(10 - e0, true) | (fp16_pow2_bits(10 - e1, true) << 16);
    uint32_t r;
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(x), "r"(inv), "r"(off));
    return u32_as_h2(r);
  } else {
    const uint32_t u = code_of<BITS, C>(w) | (code_of<BITS, C + 1>(w) << 16) | 0x64006400u;
    return __hsub2(u32_as_h2(u), u32_as_h2(0x64006400u));
  }
}

// one 8-channel column block CB of the K row (per-channel scale / zero) or
// of the V row (per-token scale / zero), exactly dequantised
template <int BITS, bool IS_KEY, int CB, int NW>
AKV_DEV void dq_block(const uint32_t (&w)[NW], const __half* ks, const __half* kz, __half2 vs2, __half2 vz2,
                      bool valid, unsigned char* tile, int t) {
  if constexpr (CB < kD / 8) {
    uint4 o = make_uint4(0u, 0u, 0u, 0u);
    if (valid) {
      __half2 s[4], z[4];
      if constexpr (IS_KEY) {
        const uint4 s4 = *reinterpret_cast<const uint4*>(ks + CB * 8);
        const uint4 z4 = *reinterpret_cast<const uint4*>(kz + CB * 8);
        s[0] = u32_as_h2(s4.x), s[1] = u32_as_h2(s4.y), s[2] = u32_as_h2(s4.z), s[3] = u32_as_h2(s4.w);
        z[0] = u32_as_h2(z4.x), z[1] = u32_as_h2(z4.y), z[2] = u32_as_h2(z4.z), z[3] = u32_as_h2(z4.w);
      } else {
        s[0] = s[1] = s[2] = s[3] = vs2;
        z[0] = z[1] = z[2] = z[3] = vz2;
      }
      o.x = h2_as_u32(__hadd2_rn(__hmul2_rn(code_pair_h2<BITS, 8 * CB>(w), s[0]), z[0]));
      o.y = h2_as_u32(__hadd2_rn(__hmul2_rn(code_pair_h2<BITS, 8 * CB + 2>(w), s[1]), z[1]));
      o.z = h2_as_u32(__hadd2_rn(__hmul2_rn(code_pair_h2<BITS, 8 * CB + 4>(w), s[2]), z[2]));
      o.w = h2_as_u32(__hadd2_rn(__hmul2_rn(code_pair_h2<BITS, 8 * CB + 6>(w), s[3]), z[3]));
    }
    *reinterpret_cast<uint4*>(tile + tile_off(t, CB * 8)) = o;
    dq_block<BITS, IS_KEY, CB + 1>(w, ks, kz, vs2, vz2, valid, tile, t);
  }
}

// Row t of the K (IS_KEY) or V tile from the prefetched registers, exactly
// like the reference: fp16(fp16(code * scale) + zero) per element
// (__hmul2_rn then __hadd2_rn), outlier channels then overwritten with their
// fp16 originals.  Invalid slots get zero rows (their softmax weight is 0
// and must not meet a non-finite value).
template <int KB, int VB, bool IS_KEY>
AKV_DEV void dequant_row(const WarmRow<KB, VB>& w, const Params& p, const __half* ks, const __half* kz,
                         unsigned char* tile, int t) {
  constexpr int BITS = IS_KEY ? KB : VB;
  uint32_t cw[4 * BITS];
#pragma unroll
  for (int i = 0; i < BITS; ++i) {
    const uint4 q = IS_KEY ? w.k[i] : w.v[i < VB ? i : 0];
    cw[4 * i] = q.x;
    cw[4 * i + 1] = q.y;
    cw[4 * i + 2] = q.z;
    cw[4 * i + 3] = q.w;
  }
  const __half2 vs2 = u32_as_h2((w.vsz & 0xFFFFu) * 0x10001u), vz2 = u32_as_h2((w.vsz >> 16) * 0x10001u);
  dq_block<BITS, IS_KEY, 0>(cw, ks, kz, vs2, vz2, w.valid, tile, t);
  const int n = p.L.n_outlier;
  if (w.valid && n > 0) {  // outlier channels: the fp16 originals replace the dequantised values
    const int slot = t & 31;
    for (int j = 0; j < n; ++j) {
      int ch;
      __half val;
      if (n <= kPrefetchOut) {  // ids: K at 16-bit word j, V at word n + j of the 8 prefetched bytes
        const int q = IS_KEY ? j : n + j;
        const uint32_t wd = q < 2 ? w.ids.x : w.ids.y;
        ch = static_cast<int16_t>((wd >> (16 * (q & 1))) & 0xFFFFu);
        val = IS_KEY ? (j == 0 ? w.ko[0] : w.ko[1]) : (j == 0 ? w.vo[0] : w.vo[1]);
      } else {
        ch = reinterpret_cast<const int16_t*>(w.rec + (IS_KEY ? p.L.ki : p.L.vi))[j];
        val = reinterpret_cast<const __half*>(w.rec + (IS_KEY ? p.L.ko : p.L.vo))[slot * n + j];
      }
      *reinterpret_cast<__half*>(tile + tile_off(t, ch)) = val;
    }
  }
}

// ------------------------------------------------------------------ tile visibility
// Key position of thread t's key in tile `tile` (INT_MAX: no key there, or
// an empty warm slot).
AKV_DEV int key_pos(const Params& p, int b, int kvh, int n_wtiles, int tile, int t) {
  if (tile < n_wtiles) {
    const int blk = tile * 4 + (t >> 5), slot = t & 31;
    if (blk >= p.n_warm_blocks) return INT_MAX;
    const uint8_t* rec = p.warm + b * p.w_sb + kvh * p.w_sh + static_cast<int64_t>(blk) * p.L.bytes;
    const uint32_t mask = __ldg(reinterpret_cast<const uint32_t*>(rec + p.L.mask));
    return ((mask >> slot) & 1u) ? __ldg(p.warm_pos + b * p.wp_sb + blk * 32 + slot) : INT_MAX;
  }
  const int j = (tile - n_wtiles) * kTile + t;
  return j < p.n_hot ? __ldg(p.hot_pos + b * p.hp_sb + j) : INT_MAX;
}

constexpr int kScanTiles = 32;  // tiles whose visibility one scan step decides

// ------------------------------------------------------------------ the kernel
struct Maps {
  CUtensorMap q, hk, hv;
};

template <int KB, int VB>
__global__ void __launch_bounds__(kThreads, 2) prefill_kernel(const Params p, const __grid_constant__ Maps maps) {
  extern __shared__ __align__(1024) unsigned char smem[];
  unsigned char* qtile = smem;                    // Q, 32 KB
  unsigned char* ktile = smem + kTileBytes;       // K
  unsigned char* vtile = smem + 2 * kTileBytes;   // V
  unsigned char* aux = smem + 3 * kTileBytes;
  __half* kscale = reinterpret_cast<__half*>(aux);             // [4][128] natural channel order
  __half* kzero = kscale + 4 * kD;                              // [4][128]
  int32_t* kpos = reinterpret_cast<int32_t*>(kzero + 4 * kD);  // [128] key positions (INT_MAX: invisible)
  uint64_t* bars = reinterpret_cast<uint64_t*>(kpos + kTile);  // load, s, o
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 4);
  __shared__ uint32_t s_vis, s_notfull;  // the current scan window: bit j = tile c0 + j visible / not fully visible
  __shared__ int s_qmax[4], s_qmin[4];

  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int m0 = blockIdx.x * kTile;
  const int h = blockIdx.y, b = blockIdx.z;
  const int kvh = h / p.g;
  uint64_t* bar_load = bars;
  uint64_t* bar_s = bars + 1;
  uint64_t* bar_o = bars + 2;

  // ---- set-up: barriers, tensor memory, this thread's query position
  if (t == 0) {
    mbar_init(bar_load, 1);
    mbar_init(bar_s, 1);
    mbar_init(bar_o, 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  const int mrow = m0 + t;
  const bool row_ok = mrow < p.M;
  const int qpos = row_ok ? __ldg(p.q_pos + b * p.qp_sb + mrow) : INT_MIN;
  {
    const int qmx = __reduce_max_sync(0xffffffffu, qpos);
    const int qmn = __reduce_min_sync(0xffffffffu, row_ok ? qpos : INT_MAX);
    if (lane == 0) {
      s_qmax[warp] = qmx;
      s_qmin[warp] = qmn;
    }
  }
  // ---- Q tile: 16 column blocks by tensor TMA (rows beyond M read as zeros)
  if (t == 0) {
    mbar_arrive_expect_tx(bar_load, kTileBytes);
    for (int cb = 0; cb < kD / 8; ++cb) tma_load_4d(qtile + cb * 2048, &maps.q, cb * 8, m0, h, b, bar_load);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS = tmem, tO = tmem + kTile;
  const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;  // this warp's TMEM lanes
  const int cta_qmax = max(max(s_qmax[0], s_qmax[1]), max(s_qmax[2], s_qmax[3]));
  const int cta_qmin = min(min(s_qmin[0], s_qmin[1]), min(s_qmin[2], s_qmin[3]));

  uint32_t ph_load = 0, ph_s = 0, ph_o = 0;
  bool ok = true;  // no bounded wait has run out
  if (!mbar_wait(bar_load, ph_load, p.status)) {
    mbar_wait(bar_load, ph_load, p.status);
    ok = false;
  }
  ok = !__syncthreads_or(!ok);
  ph_load ^= 1;

  const uint32_t idesc_s = instr_desc(kTile, kTile, 0);  // S = Q K^T: B (= K) K-major
  const uint32_t idesc_o = instr_desc(kTile, kD, 1);     // O = P V:   B (= V) MN-major
  const uint32_t q_addr = smem_u32(qtile), k_addr = smem_u32(ktile), v_addr = smem_u32(vtile);

  const int n_wtiles = (p.n_warm_blocks + 3) / 4;
  const int n_tiles = n_wtiles + (p.n_hot + kTile - 1) / kTile;

  // visibility of tiles [c0, c0 + 32): one scan step reads every key position
  // of the window (32 loads per thread in flight) and ORs the per-tile flags
  int win = -1;
  auto scan = [&](int c0) {
    __syncthreads();  // every thread has read the previous window's flags before they are cleared
    if (t == 0) s_vis = s_notfull = 0u;
    __syncthreads();
    int kp[kScanTiles];
#pragma unroll
    for (int j = 0; j < kScanTiles; ++j) kp[j] = c0 + j < n_tiles ? key_pos(p, b, kvh, n_wtiles, c0 + j, t) : INT_MAX;
    uint32_t vis = 0u, nf = 0u;
#pragma unroll
    for (int j = 0; j < kScanTiles; ++j) {
      vis |= static_cast<uint32_t>(kp[j] <= cta_qmax) << j;
      nf |= static_cast<uint32_t>(kp[j] > cta_qmin) << j;
    }
    vis = __reduce_or_sync(0xffffffffu, vis);
    nf = __reduce_or_sync(0xffffffffu, nf);
    if (lane == 0) {
      atomicOr(&s_vis, vis);
      atomicOr(&s_notfull, nf);
    }
    __syncthreads();
    win = c0;
  };
  // first visible tile at or after `from` (n_tiles: none); uniform over the CTA
  auto next_visible = [&](int from) {
    while (from < n_tiles) {
      const int c0 = from - from % kScanTiles;
      if (win != c0) scan(c0);
      const uint32_t bits = s_vis >> (from - c0);
      if (bits) return from + __ffs(bits) - 1;
      from = c0 + kScanTiles;
    }
    return n_tiles;
  };

  float m_run = -INFINITY;  // running max of this row's scaled logits (log2 units)
  float l_run = 0.f;        // running sum of 2^(s - m_run)
  bool o_live = false;      // O holds accumulated values (a P.V has been issued)
  bool pv_pending = false;  // a P.V MMA may still read the V tile and the P columns

  WarmRow<KB, VB> wr;
  int cur = next_visible(0);
  if (cur < n_wtiles) load_warm_row<KB, VB>(p, b, kvh, cur, t, wr);
  while (cur < n_tiles && ok) {
    const bool warm_tile = cur < n_wtiles;
    const bool full = !((s_notfull >> (cur - win)) & 1u);  // every key valid and visible to every row
    const int nxt = next_visible(cur + 1);                  // (may rescan: uniform)

    // -- the previous tile's P.V reads V and the P columns; S of the previous
    // tile is complete, so a warm tile's K rows are dequantised first, while
    // that P.V may still run
    if (warm_tile) {
      kpos[t] = wr.kp;
      stage_kscale<KB, VB>(wr, lane, kscale + warp * kD, kzero + warp * kD);
      __syncwarp();
      dequant_row<KB, VB, true>(wr, p, kscale + warp * kD, kzero + warp * kD, ktile, t);
    }
    if (pv_pending) {
      if (!mbar_wait(bar_o, ph_o, p.status)) {
        mbar_wait(bar_o, ph_o, p.status);
        ok = false;
      }
      ph_o ^= 1;
      pv_pending = false;
      tc_fence_after();
    }
    if (__syncthreads_or(!ok)) break;

    if (warm_tile) {
      dequant_row<KB, VB, false>(wr, p, nullptr, nullptr, vtile, t);
      fence_proxy_async_shared();  // generic-proxy tile writes -> visible to the tensor cores
      if (nxt < n_wtiles) load_warm_row<KB, VB>(p, b, kvh, nxt, t, wr);  // next tile's rows in flight
    } else {
      kpos[t] = key_pos(p, b, kvh, n_wtiles, cur, t);
      if (t == 0) {
        const int j0 = (cur - n_wtiles) * kTile;
        mbar_arrive_expect_tx(bar_load, 2 * kTileBytes);
        for (int cb = 0; cb < kD / 8; ++cb) {
          tma_load_4d(ktile + cb * 2048, &maps.hk, cb * 8, j0, kvh, b, bar_load);
          tma_load_4d(vtile + cb * 2048, &maps.hv, cb * 8, j0, kvh, b, bar_load);
        }
      }
      if (!mbar_wait(bar_load, ph_load, p.status)) {  // let the copies land (bounded) before giving up
        mbar_wait(bar_load, ph_load, p.status);
        ok = false;
      }
      ph_load ^= 1;
    }
    tc_fence_before();
    if (__syncthreads_or(!ok)) break;

    // -- S = Q K^T  (8 k-steps of 16 channels; operands advance 2 column blocks per step)
    if (t == 0) {
      tc_fence_after();
#pragma unroll
      for (int ks = 0; ks < kD / 16; ++ks) {
        const uint64_t a = smem_desc(q_addr + ks * 4096, 2048, 128);
        const uint64_t bd = smem_desc(k_addr + ks * 4096, 2048, 128);
        umma_f16(tS, a, bd, idesc_s, ks > 0 ? 1u : 0u);
      }
      umma_commit(bar_s);
    }
    if (!mbar_wait(bar_s, ph_s, p.status)) {  // the MMA still owns the tiles: wait once more (bounded)
      mbar_wait(bar_s, ph_s, p.status);
      ok = false;
    }
    ph_s ^= 1;
    tc_fence_after();
    if (__syncthreads_or(!ok)) break;

    // -- softmax, pass 1: this row's max over the tile (S read 32 columns at a time)
    const float sl2 = p.scale_log2;
    float mx = -INFINITY;
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
      float sv[32];
      tmem_ld32(tS + lane_base + c * 32, sv);
      tmem_wait_ld();
      if (full) {
#pragma unroll
        for (int i = 0; i < 32; ++i) mx = fmaxf(mx, sv[i]);
      } else {
        const int4* kp4 = reinterpret_cast<const int4*>(kpos + c * 32);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int4 k4 = kp4[i];
          mx = fmaxf(mx, k4.x <= qpos ? sv[4 * i] : -INFINITY);
          mx = fmaxf(mx, k4.y <= qpos ? sv[4 * i + 1] : -INFINITY);
          mx = fmaxf(mx, k4.z <= qpos ? sv[4 * i + 2] : -INFINITY);
          mx = fmaxf(mx, k4.w <= qpos ? sv[4 * i + 3] : -INFINITY);
        }
      }
    }
    mx = mx * sl2;  // scale_log2 > 0: the max of the scaled logits
    const bool move = mx > m_run + kLazy;
    float alpha = 1.f;
    if (move) {
      alpha = (m_run == -INFINITY) ? 0.f : exp2f(m_run - mx);
      m_run = mx;
      l_run *= alpha;
    }
    if (__any_sync(0xffffffffu, move) && o_live) {  // rescale this warp's O rows in tensor memory
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        float o[32];
        tmem_ld32(tO + lane_base + c * 32, o);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) o[i] *= alpha;
        tmem_st32(tO + lane_base + c * 32, o);
      }
      tmem_wait_st();
    }
    // -- pass 2: P = 2^(s - m) as an exact-to-2^-22 pair of fp16 terms, hi =
    // fp16(P) and lo = fp16(P - hi), written over the S columns just read:
    // keys 32c .. 32c+31 -> hi in columns 32c .. 32c+15, lo in 32c+16 .. 32c+31
    // (two keys per column), so P.V runs as two MMAs with A in tensor memory
    const float mb = (m_run == -INFINITY) ? 0.f : m_run;
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
      float sv[32];
      tmem_ld32(tS + lane_base + c * 32, sv);
      tmem_wait_ld();
      const int4* kp4 = reinterpret_cast<const int4*>(kpos + c * 32);
      uint32_t hi[16], lo[16];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int4 k4 = full ? make_int4(INT_MIN, INT_MIN, INT_MIN, INT_MIN) : kp4[i];
        const int kk[4] = {k4.x, k4.y, k4.z, k4.w};
        float pr[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) pr[e] = kk[e] <= qpos ? fast_exp2(fmaf(sv[4 * i + e], sl2, -mb)) : 0.f;
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const __half2 hh = __floats2half2_rn(pr[2 * e], pr[2 * e + 1]);
          const float2 hf = __half22float2(hh);
          hi[2 * i + e] = h2_as_u32(hh);
          lo[2 * i + e] = h2_as_u32(__floats2half2_rn(pr[2 * e] - hf.x, pr[2 * e + 1] - hf.y));
          l_run += pr[2 * e] + pr[2 * e + 1];
        }
      }
      tmem_st16u(tS + lane_base + 32 * c, hi);
      tmem_st16u(tS + lane_base + 32 * c + 16, lo);
    }
    tmem_wait_st();
    tc_fence_before();
    __syncthreads();

    // -- O += P V  (8 k-steps of 16 keys, hi then lo term; A from tensor memory)
    if (t == 0) {
      tc_fence_after();
#pragma unroll
      for (int ks = 0; ks < kTile / 16; ++ks) {
        const uint64_t bd = smem_desc(v_addr + ks * 256, 128, 2048);  // V: MN-major (keys = K, channels = N)
        const uint32_t col = 32 * (ks >> 1) + 8 * (ks & 1);
        umma_f16_ts(tO, tS + col, bd, idesc_o, (o_live || ks > 0) ? 1u : 0u);
        umma_f16_ts(tO, tS + col + 16, bd, idesc_o, 1u);
      }
      umma_commit(bar_o);
    }
    o_live = true;
    pv_pending = true;
    cur = nxt;
  }

  // ---- epilogue: O / l -> fp16 rows
  if (pv_pending) {
    if (!mbar_wait(bar_o, ph_o, p.status)) mbar_wait(bar_o, ph_o, p.status);
    tc_fence_after();
  }
  __syncthreads();
  const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
#pragma unroll 1
  for (int c = 0; c < 4; ++c) {
    float o[32];
    if (o_live) {
      tmem_ld32(tO + lane_base + c * 32, o);
      tmem_wait_ld();
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i) o[i] = 0.f;
    }
    if (row_ok) {
      __align__(16) __half2 oh[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) oh[i] = __floats2half2_rn(o[2 * i] * inv, o[2 * i + 1] * inv);
      __half* dst = p.out + b * p.o_sb + h * p.o_sh + static_cast<int64_t>(mrow) * p.o_sm + c * 32;
#pragma unroll
      for (int q = 0; q < 4; ++q) reinterpret_cast<uint4*>(dst)[q] = reinterpret_cast<const uint4*>(oh)[q];
    }
  }
  if (row_ok && p.lse)
    p.lse[(static_cast<int64_t>(b) * p.Hq + h) * p.M + mrow] = l_run > 0.f ? (m_run + log2f(l_run)) / kLog2e : -INFINITY;
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

constexpr size_t kSmemBytes = 3 * kTileBytes + 2 * 4 * kD * 2 + kTile * 4 + 64 + 1024;

// ------------------------------------------------------------------ host: tensor maps
using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiled encoder() {
  static EncodeTiled fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiled>(f);
  });
  return fn;
}

// 4-D fp16 map over (channel, row, head, batch), box {8, 128, 1, 1}, zero fill
// outside [0, rows): element strides in elements (row, head, batch).
static bool make_map(CUtensorMap* m, const void* base, int rows, int heads, int batch, int64_t s_row, int64_t s_head,
                     int64_t s_batch) {
  EncodeTiled enc = encoder();
  if (!enc) return false;
  const cuuint64_t dims[4] = {static_cast<cuuint64_t>(kD), static_cast<cuuint64_t>(rows),
                              static_cast<cuuint64_t>(heads), static_cast<cuuint64_t>(batch)};
  // a stride is never used for a dimension of extent 1, but must still be a multiple of 16 bytes
  auto st = [](int64_t s, int n) { return static_cast<cuuint64_t>(n > 1 ? s * 2 : 16); };
  const cuuint64_t strides[3] = {st(s_row, rows), st(s_head, heads), st(s_batch, batch)};
  const cuuint32_t box[4] = {8, static_cast<cuuint32_t>(kTile), 1, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int KB, int VB>
static int launch(const Params& p, const Maps& maps, cudaStream_t st) {
  auto kern = prefill_kernel<KB, VB>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kSmemBytes)) !=
      cudaSuccess)
    return AKV_ERR_LAUNCH;
  kern<<<dim3((p.M + kTile - 1) / kTile, p.Hq, p.B), kThreads, kSmemBytes, st>>>(p, maps);
  return cudaGetLastError() == cudaSuccess ? AKV_OK : AKV_ERR_LAUNCH;
}

}  // namespace prefill
}  // namespace akv

using namespace akv;

extern "C" int akv_prefill_attention(const uint16_t* q, int64_t q_sb, int64_t q_sh, int64_t q_sm,
                                     const int32_t* q_pos, int64_t qp_sb, int M, const uint16_t* hot_k,
                                     const uint16_t* hot_v, int64_t h_sb, int64_t h_sh, int64_t h_sn, int n_hot,
                                     const int32_t* hot_pos, int64_t hp_sb, const uint8_t* warm, int64_t w_sb,
                                     int64_t w_sh, const akv_warm_layout* layout, int n_warm_blocks,
                                     const int32_t* warm_pos, int64_t wp_sb, int B, int Hq, int Hkv, int D,
                                     float sm_scale, uint16_t* out, int64_t o_sb, int64_t o_sh, int64_t o_sm,
                                     float* lse, int* status, void* stream) {
  using namespace akv::prefill;
  if (!q || !q_pos || !out) return AKV_ERR_NULL;
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv || M <= 0 || n_hot < 0 || n_warm_blocks < 0) return AKV_ERR_SHAPE;
  if (D != kD) return AKV_ERR_UNSUPPORTED;
  if (Hq > 65535 || B > 65535) return AKV_ERR_SHAPE;
  if (n_hot > 0 && (!hot_k || !hot_v || !hot_pos)) return AKV_ERR_NULL;
  if (n_warm_blocks > 0 && (!warm || !layout || !warm_pos)) return AKV_ERR_NULL;
  auto al = [](const void* ptr, int a) { return (reinterpret_cast<uintptr_t>(ptr) % a) == 0; };
  // tensor TMA: 16-byte aligned bases and strides
  if (!al(q, 16) || q_sb % 8 || q_sh % 8 || q_sm % 8) return AKV_ERR_ALIGN;
  if (n_hot > 0 && (!al(hot_k, 16) || !al(hot_v, 16) || h_sb % 8 || h_sh % 8 || h_sn % 8)) return AKV_ERR_ALIGN;
  if (!al(out, 16) || o_sb % 8 || o_sh % 8 || o_sm % 8) return AKV_ERR_ALIGN;
  akv_warm_layout L{};
  if (n_warm_blocks > 0) {
    L = *layout;
    if (L.head_dim != D) return AKV_ERR_SHAPE;
    if (L.key_bits < 2 || L.key_bits > 4 || L.value_bits < 2 || L.value_bits > 4) return AKV_ERR_BITS;
    const RecLayout R = rec_layout(D, L.key_bits, L.value_bits, L.n_outlier);
    if (L.kc != R.kc || L.vc != R.vc || L.ks != R.ks || L.kz != R.kz || L.vs != R.vs || L.vz != R.vz ||
        L.mask != R.mask || L.ki != R.ki || L.vi != R.vi || L.ko != R.ko || L.vo != R.vo || L.bytes != R.bytes)
      return AKV_ERR_UNSUPPORTED;
    if (!al(warm, 16) || w_sb % 16 || w_sh % 16) return AKV_ERR_ALIGN;
  }
  Maps maps{};
  if (!make_map(&maps.q, q, M, Hq, B, q_sm, q_sh, q_sb)) return AKV_ERR_UNSUPPORTED;
  if (n_hot > 0) {
    if (!make_map(&maps.hk, hot_k, n_hot, Hkv, B, h_sn, h_sh, h_sb)) return AKV_ERR_UNSUPPORTED;
    if (!make_map(&maps.hv, hot_v, n_hot, Hkv, B, h_sn, h_sh, h_sb)) return AKV_ERR_UNSUPPORTED;
  }
  Params p{};
  p.q = reinterpret_cast<const __half*>(q);
  p.q_sb = q_sb;
  p.q_sh = q_sh;
  p.q_sm = q_sm;
  p.q_pos = q_pos;
  p.qp_sb = qp_sb;
  p.M = M;
  p.hk = reinterpret_cast<const __half*>(hot_k);
  p.hv = reinterpret_cast<const __half*>(hot_v);
  p.h_sb = h_sb;
  p.h_sh = h_sh;
  p.h_sn = h_sn;
  p.n_hot = n_hot;
  p.hot_pos = hot_pos;
  p.hp_sb = hp_sb;
  p.warm = warm;
  p.w_sb = w_sb;
  p.w_sh = w_sh;
  p.L = L;
  p.n_warm_blocks = n_warm_blocks;
  p.warm_pos = warm_pos;
  p.wp_sb = wp_sb;
  p.B = B;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.g = Hq / Hkv;
  p.scale_log2 = sm_scale * kLog2e;
  p.out = reinterpret_cast<__half*>(out);
  p.o_sb = o_sb;
  p.o_sh = o_sh;
  p.o_sm = o_sm;
  p.lse = lse;
  p.status = status;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int kb = n_warm_blocks > 0 ? L.key_bits : 4, vb = n_warm_blocks > 0 ? L.value_bits : 4;
  switch (kb * 10 + vb) {
    case 22: return launch<2, 2>(p, maps, st);
    case 23: return launch<2, 3>(p, maps, st);
    case 24: return launch<2, 4>(p, maps, st);
    case 32: return launch<3, 2>(p, maps, st);
    case 33: return launch<3, 3>(p, maps, st);
    case 34: return launch<3, 4>(p, maps, st);
    case 42: return launch<4, 2>(p, maps, st);
    case 43: return launch<4, 3>(p, maps, st);
    default: return launch<4, 4>(p, maps, st);
  }
}
