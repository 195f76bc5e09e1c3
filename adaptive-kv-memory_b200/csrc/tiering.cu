// Tier-management kernels: importance update, demote selection (bottom-k),
// row gather for demote/promote, and cold-tier copies; plus the ABI helpers.
#include <cuda_runtime.h>

#include <algorithm>

#include "common.cuh"

namespace akv {

// ---------------------------------------------------------------------------
// importance update (akv/triton_ops.py:604-650, CPU branch semantics)
//   imp[n]    = sum_m ( sum_{b,h} attn[b,h,m,n] / (B*H) )
//   scores[n] = fl(fl(scores[n] * decay) + imp[n])
//
// Both sums add in the order of torch's CPU reduction of a contiguous tensor
// over its outer dimension (the reference's attention_weights.float()
// .mean(dim=(0, 1)).sum(dim=0); the restated ordering is PyTorch's
// cascade_sum / multi_row_sum / row_sum in aten/src/ATen/native/cpu/
// SumKernel.cpp, BSD licence):
//  * a column whose index lies below the last multiple of twice the CPU
//    vector width `vw` (floats per SIMD register of the machine running the
//    reference: 16 with AVX-512, 8 with AVX2; torch sums those columns in
//    blocks of four and two registers) sums its R rows in "cascade"
//    order: with lp = max(4, ceil(log2(R)) / 4), the rows are added one by
//    one to level 0; after every 2^lp rows level 0 is added to level 1 (and
//    cleared), level 1 to level 2 when the row count is a multiple of 2^(2lp),
//    level 2 to level 3 at multiples of 2^(3lp); at the end the levels are
//    added in order 0 + 1 + 2 + 3;
//  * the remaining columns (one register's worth and the scalar tail) sum
//    four interleaved cascades (rows
//    4i + k, i < R/4) with the last R % 4 rows added to cascade 0, then
//    cascades 1, 2, 3 added to it in order.
// The mean divides the (b, h) sum by B*H (sum, then a true division, as
// torch's CPU mean does).  The flattened (m, n) column index decides the
// order of the (b, h) sum, n alone that of the sum over m.
// ---------------------------------------------------------------------------
struct TorchCascade {
  float acc[4];
  int i, lp, mask;
  AKV_DEV void init(int size) {
    int cl = 0;
    while ((1 << cl) < size) ++cl;  // ceil(log2(size)), 0 for size <= 1
    lp = cl / 4 > 4 ? cl / 4 : 4;
    mask = (1 << lp) - 1;
    i = 0;
    acc[0] = acc[1] = acc[2] = acc[3] = 0.f;
  }
  AKV_DEV void push(float v) {
    acc[0] = __fadd_rn(acc[0], v);
    if ((++i & mask) == 0) {  // a full step of 2^lp rows
      acc[1] = __fadd_rn(acc[1], acc[0]);
      acc[0] = 0.f;
      if ((i & (mask << lp)) == 0) {
        acc[2] = __fadd_rn(acc[2], acc[1]);
        acc[1] = 0.f;
        if ((i & (mask << (2 * lp))) == 0) {
          acc[3] = __fadd_rn(acc[3], acc[2]);
          acc[2] = 0.f;
        }
      }
    }
  }
  AKV_DEV float result() const {
    return __fadd_rn(__fadd_rn(__fadd_rn(acc[0], acc[1]), acc[2]), acc[3]);
  }
};

// torch-order sum of the BH rows of one column (row stride rs).  Rows are
// loaded kRowsInFlight at a time so a thread keeps several loads in flight
// while the additions keep their order; ILP selects the four-interleaved-
// cascade form.
constexpr int kRowsInFlight = 16;
template <bool ILP>
AKV_DEV float bh_column_sum(const float* __restrict__ col, int64_t rs, int BH) {
  if constexpr (!ILP) {
    TorchCascade c;
    c.init(BH);
    int bh = 0;
    for (; bh + kRowsInFlight <= BH; bh += kRowsInFlight) {
      float v[kRowsInFlight];
#pragma unroll
      for (int j = 0; j < kRowsInFlight; ++j) v[j] = __ldg(col + (bh + j) * rs);
#pragma unroll
      for (int j = 0; j < kRowsInFlight; ++j) c.push(v[j]);
    }
    for (; bh < BH; ++bh) c.push(__ldg(col + bh * rs));
    return c.result();
  } else {
    TorchCascade c0, c1, c2, c3;
    c0.init(BH / 4);
    c1.init(BH / 4);
    c2.init(BH / 4);
    c3.init(BH / 4);
    const int full = BH / 4 * 4;
    int bh = 0;
    for (; bh + kRowsInFlight <= full; bh += kRowsInFlight) {
      float v[kRowsInFlight];
#pragma unroll
      for (int j = 0; j < kRowsInFlight; ++j) v[j] = __ldg(col + (bh + j) * rs);
#pragma unroll
      for (int j = 0; j < kRowsInFlight; j += 4) {
        c0.push(v[j]);
        c1.push(v[j + 1]);
        c2.push(v[j + 2]);
        c3.push(v[j + 3]);
      }
    }
    for (; bh + 4 <= full; bh += 4) {  // groups of four left
      c0.push(__ldg(col + bh * rs));
      c1.push(__ldg(col + (bh + 1) * rs));
      c2.push(__ldg(col + (bh + 2) * rs));
      c3.push(__ldg(col + (bh + 3) * rs));
    }
    float s = c0.result();
    for (; bh < BH; ++bh) s = __fadd_rn(s, __ldg(col + bh * rs));  // the last BH % 4 rows go into cascade 0
    s = __fadd_rn(s, c1.result());
    s = __fadd_rn(s, c2.result());
    return __fadd_rn(s, c3.result());
  }
}

// attention received by position n: imp = torch-order sum over m of
// fl(torch-order sum over (b, h) of attn[bh, m, n] / (B*H)).
AKV_DEV float attn_received_col(const float* __restrict__ attn, int BH, int M, int Na, int n, int vw) {
  const float cnt = static_cast<float>(BH);
  const int64_t rs = static_cast<int64_t>(M) * Na;  // stride between (b,h) rows = columns of the (b,h) sum
  const int64_t jv1 = rs / (2 * vw) * (2 * vw);
  const int jv2 = Na / (2 * vw) * (2 * vw);
  auto avg_of = [&](int m) {
    const float* col = attn + static_cast<int64_t>(m) * Na + n;
    const float s = static_cast<int64_t>(m) * Na + n >= jv1 ? bh_column_sum<true>(col, rs, BH)
                                                              : bh_column_sum<false>(col, rs, BH);
    return __fdiv_rn(s, cnt);
  };
  if (M == 1) return avg_of(0);
  if (n < jv2) {
    TorchCascade c;
    c.init(M);
    for (int m = 0; m < M; ++m) c.push(avg_of(m));
    return c.result();
  }
  TorchCascade c0, c1, c2, c3;
  c0.init(M / 4);
  c1.init(M / 4);
  c2.init(M / 4);
  c3.init(M / 4);
  const int full = M / 4 * 4;
  int m = 0;
  for (; m < full; m += 4) {
    c0.push(avg_of(m));
    c1.push(avg_of(m + 1));
    c2.push(avg_of(m + 2));
    c3.push(avg_of(m + 3));
  }
  float imp = c0.result();
  for (; m < M; ++m) imp = __fadd_rn(imp, avg_of(m));
  imp = __fadd_rn(imp, c1.result());
  imp = __fadd_rn(imp, c2.result());
  return __fadd_rn(imp, c3.result());
}

__global__ void importance_update_kernel(const float* __restrict__ attn, int B, int H, int M, int Na,
                                         float* __restrict__ scores, int N, float decay, int vw) {
  const int n = blockIdx.x * blockDim.x + threadIdx.x;
  if (n >= N) return;
  const float imp = n < Na ? attn_received_col(attn, B * H, M, Na, n, vw) : 0.f;
  scores[n] = __fadd_rn(__fmul_rn(scores[n], decay), imp);
}

// ---------------------------------------------------------------------------
// ImportanceBasedMigrator (akv/vmm.py:113-245) on the GPU.
//
// update (:121-164): attention received per position = sum over queries of the
// mean over batch and heads (the same reduction order as above); positions in
// [n_prev, Na) are new and start at score 0, last access = step, retrieval 0;
// scores = fl(fl(scores*decay) + received); last access = step where
// received > 0.01.
// ---------------------------------------------------------------------------
__global__ void migrator_update_kernel(const float* __restrict__ attn, int B, int H, int M, int Na,
                                       float* __restrict__ scores, int64_t* __restrict__ access,
                                       float* __restrict__ retrieval, int n_prev, int64_t step, float decay, int vw) {
  const int n = blockIdx.x * blockDim.x + threadIdx.x;
  if (n >= Na) return;
  const float imp = attn_received_col(attn, B * H, M, Na, n, vw);
  float sc = scores[n];
  if (n >= n_prev) {
    sc = 0.f;
    access[n] = step;
    retrieval[n] = 0.f;
  }
  scores[n] = __fadd_rn(__fmul_rn(sc, decay), imp);
  if (imp > 0.01f) access[n] = step;
}

// Order-preserving u32 key of a float and back (for max / min by integer
// atomics); a min is kept as the max of the complemented key, so zeroed words
// are the identity of all three reductions.
AKV_DEV uint32_t mig_key(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
AKV_DEV float mig_unkey(uint32_t k) { return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k); }

// compute_importance (:175-219), step 1: max of scores, min of last access,
// max of retrieval over [0, N) -> red[0..2] as keys (zeroed before the
// launch); every CTA reduces a grid-stride share, then folds it in with one
// atomic per quantity (max and min do not depend on the order)
__global__ void migrator_reduce_kernel(const float* __restrict__ scores, const int64_t* __restrict__ access,
                                       const float* __restrict__ retrieval, int N, uint32_t* red) {
  __shared__ float smax[32], rmax[32];
  __shared__ float amin[32];
  float a = -INFINITY, r = -INFINITY, t = INFINITY;
  // four positions per thread and trip with 16-byte loads when all three
  // arrays are 16-byte aligned (several loads in flight per thread), the
  // rest one by one
  const bool vec = ((reinterpret_cast<uintptr_t>(scores) | reinterpret_cast<uintptr_t>(retrieval) |
                     reinterpret_cast<uintptr_t>(access)) & 15u) == 0;
  int done = 0;
  if (vec) {
    const int ng = N / 4;
    for (int g = blockIdx.x * blockDim.x + threadIdx.x; g < ng; g += gridDim.x * blockDim.x) {
      const float4 sv = __ldg(reinterpret_cast<const float4*>(scores) + g);
      const float4 rv = __ldg(reinterpret_cast<const float4*>(retrieval) + g);
      const longlong2 a0 = __ldg(reinterpret_cast<const longlong2*>(access) + 2 * g);
      const longlong2 a1 = __ldg(reinterpret_cast<const longlong2*>(access) + 2 * g + 1);
      a = fmaxf(fmaxf(a, fmaxf(sv.x, sv.y)), fmaxf(sv.z, sv.w));
      r = fmaxf(fmaxf(r, fmaxf(rv.x, rv.y)), fmaxf(rv.z, rv.w));
      t = fminf(fminf(t, fminf(static_cast<float>(a0.x), static_cast<float>(a0.y))),
                fminf(static_cast<float>(a1.x), static_cast<float>(a1.y)));
    }
    done = 4 * ng;
  }
  for (int i = done + blockIdx.x * blockDim.x + threadIdx.x; i < N; i += gridDim.x * blockDim.x) {
    a = fmaxf(a, scores[i]);
    r = fmaxf(r, retrieval[i]);
    t = fminf(t, static_cast<float>(access[i]));  // access.float().min()
  }
  for (int o = 16; o > 0; o >>= 1) {
    a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
    r = fmaxf(r, __shfl_xor_sync(0xffffffffu, r, o));
    t = fminf(t, __shfl_xor_sync(0xffffffffu, t, o));
  }
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    smax[w] = a;
    rmax[w] = r;
    amin[w] = t;
  }
  __syncthreads();
  if (w == 0) {
    const int nw = blockDim.x >> 5;
    a = lane < nw ? smax[lane] : -INFINITY;
    r = lane < nw ? rmax[lane] : -INFINITY;
    t = lane < nw ? amin[lane] : INFINITY;
    for (int o = 16; o > 0; o >>= 1) {
      a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
      r = fmaxf(r, __shfl_xor_sync(0xffffffffu, r, o));
      t = fminf(t, __shfl_xor_sync(0xffffffffu, t, o));
    }
    if (lane == 0) {
      atomicMax(red, mig_key(a));
      atomicMax(red + 1, ~mig_key(t));
      atomicMax(red + 2, mig_key(r));
    }
  }
}

// step 2: importance = w_a*attn_norm + w_r*recency + w_t*retr_norm, each op
// rounded like torch's, protected ends at +inf
__global__ void migrator_importance_kernel(const float* __restrict__ scores, const int64_t* __restrict__ access,
                                           const float* __restrict__ retrieval, int N, int64_t step,
                                           const uint32_t* __restrict__ red, float w_a, float w_r, float w_t,
                                           int n_first, int n_last, float* __restrict__ out) {
  const int n = blockIdx.x * blockDim.x + threadIdx.x;
  if (n >= N) return;
  const float smax = mig_unkey(red[0]), amin = mig_unkey(~red[1]), rmax = mig_unkey(red[2]);
  const float attn_norm = __fdiv_rn(scores[n], fmaxf(smax, 1e-10f));
  // max(1.0, step - access.min()) is Python double arithmetic, then a float32 divisor
  const double den = fmax(1.0, static_cast<double>(step) - static_cast<double>(amin));
  const float recency = __fdiv_rn(__fsub_rn(static_cast<float>(access[n]), amin), static_cast<float>(den));
  const float retr = __fdiv_rn(retrieval[n], __fadd_rn(fmaxf(rmax, 1e-10f), 1e-10f));
  float imp = __fadd_rn(__fadd_rn(__fmul_rn(w_a, attn_norm), __fmul_rn(w_r, recency)), __fmul_rn(w_t, retr));
  if (n < n_first || n >= N - n_last) imp = INFINITY;
  out[n] = imp;
}

// ---------------------------------------------------------------------------
// bottom-k selection with protected ends (akv/drop_in.py:392-413)
//
// Scores map to order-preserving u32 keys; protected positions get the key
// of +inf.  The k-th smallest key is found by an 8-bit radix select (four
// passes, most significant byte first), then a stable compaction emits, in
// ascending index order, every position below that key plus the first
// (k - count_below) positions equal to it.  Every step is a short launch
// over the whole GPU (no CTA waits on another):
//   per pass: sel_hist_kernel (per-CTA shared histograms of the keys that
//   match the prefix so far, lanes of a warp that hit one bin adding with a
//   single atomic, then added into the pass's global histogram; the last CTA
//   to arrive scans that histogram and extends the prefix by the byte of the
//   k-th key); then sel_count_kernel (per-CTA counts of keys below / equal to
//   the threshold) and sel_compact_kernel (each CTA places its contiguous
//   slice after the lower CTAs' counts and writes it in index order).
// Workspace (u32): hist[4][256] and the per-pass arrival counters done[4]
// (zeroed first), state {prefix, mask, remaining}, counts[grid][2].
// ---------------------------------------------------------------------------
constexpr int kSelThreads = 256;
constexpr int kSelWarps = kSelThreads / 32;
constexpr int kSelMaxCtas = 2 * 148;
constexpr size_t kSelWsWords = 4 * 256 + 4 + 4 + 2 * kSelMaxCtas;
constexpr size_t kSelZeroWords = 4 * 256 + 4;  // histograms and per-pass arrival counters, zeroed per call

AKV_DEV uint32_t order_key(float f) {
  uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// keys of positions 4g .. 4g+3 (beyond n: key 0, valid false); one 16-byte
// load when the scores are 16-byte aligned
AKV_DEV void sel_keys4(const float* s, bool vec, int g, int n, int pf, int pl, uint32_t (&key)[4], bool (&valid)[4]) {
  const int i0 = 4 * g;
  float v[4];
  if (vec && i0 + 3 < n) {
    const float4 f = __ldg(reinterpret_cast<const float4*>(s) + g);
    v[0] = f.x;
    v[1] = f.y;
    v[2] = f.z;
    v[3] = f.w;
  } else {
#pragma unroll
    for (int e = 0; e < 4; ++e) v[e] = i0 + e < n ? __ldg(s + i0 + e) : 0.f;
  }
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const int i = i0 + e;
    valid[e] = i < n;
    key[e] = !valid[e] ? 0u : ((i < pf || i >= n - pl) ? order_key(INFINITY) : order_key(v[e]));
  }
}

struct SelArgs {
  const float* scores;
  int n, k, pf, pl, vec;
  int ng, per_cta;  // 4-position groups in total / per CTA slice (multiple of 32)
  uint32_t* ws;
  int64_t* out;
};

AKV_DEV uint32_t* sel_hist(const SelArgs& a, int pass) { return a.ws + pass * 256; }
AKV_DEV uint32_t* sel_done(const SelArgs& a) { return a.ws + 4 * 256; }
AKV_DEV uint32_t* sel_state(const SelArgs& a) { return a.ws + 4 * 256 + 4; }
AKV_DEV uint32_t* sel_counts(const SelArgs& a) { return a.ws + 4 * 256 + 8; }

// The whole CTA (256 threads, one bin each): the bin holding the rem-th
// smallest key of this pass is the first whose inclusive count reaches rem
// (bin 255 if none of the first 255 does), found with a block-wide scan of
// the histogram; the threshold state moves on by one byte.
AKV_DEV void sel_pick(const SelArgs& a, int pass) {
  static_assert(kSelThreads == 256, "one thread per histogram bin");
  __shared__ uint32_t wsum[8];
  __shared__ uint32_t s_bin, s_below;
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  uint32_t* st = sel_state(a);
  const uint32_t prefix = pass ? __ldcg(st) : 0u, mask = pass ? __ldcg(st + 1) : 0u;
  const uint32_t rem = pass ? __ldcg(st + 2) : static_cast<uint32_t>(a.k);
  const uint32_t v = __ldcg(sel_hist(a, pass) + tid);
  uint32_t x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) wsum[w] = x;
  __syncthreads();
  uint32_t off = 0;
  for (int i = 0; i < w; ++i) off += wsum[i];
  const uint32_t incl = x + off, excl = incl - v;
  if (tid == 255) {  // the fallback: bin 255 after everything below it
    s_bin = 255u;
    s_below = excl;
  }
  __syncthreads();
  if (tid < 255 && excl < rem && incl >= rem) {  // exactly one bin, the first reaching rem
    s_bin = static_cast<uint32_t>(tid);
    s_below = excl;
  }
  __syncthreads();
  if (tid == 0) {
    const int shift = 24 - 8 * pass;
    st[0] = prefix | (s_bin << shift);
    st[1] = mask | (255u << shift);
    st[2] = rem - s_below;
  }
}

__global__ void __launch_bounds__(kSelThreads) sel_hist_kernel(const SelArgs a, int pass) {
  __shared__ uint32_t hist[256];
  const int tid = threadIdx.x, lane = tid & 31;
  hist[tid] = 0;
  const uint32_t prefix = pass ? sel_state(a)[0] : 0u, mask = pass ? sel_state(a)[1] : 0u;
  const int shift = 24 - 8 * pass;
  __syncthreads();
  const int g0 = blockIdx.x * a.per_cta, g1 = g0 + a.per_cta;
  for (int g = g0 + tid; g < g1; g += kSelThreads) {  // per_cta is a multiple of 32: whole warps every trip
    uint32_t key[4];
    bool valid[4];
    sel_keys4(a.scores, a.vec, g, a.n, a.pf, a.pl, key, valid);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const bool hit = valid[e] && (key[e] & mask) == prefix;
      const uint32_t bin = (key[e] >> shift) & 255u;
      const uint32_t voters = __ballot_sync(0xffffffffu, hit);
      if (hit) {
        const uint32_t peers = __match_any_sync(voters, bin);
        if ((peers & ((1u << lane) - 1u)) == 0) atomicAdd(&hist[bin], __popc(peers));
      }
    }
  }
  __syncthreads();
  const uint32_t c = hist[tid];
  if (c) atomicAdd(&sel_hist(a, pass)[tid], c);
  // the last CTA to finish the pass picks the next threshold byte
  __threadfence();
  __syncthreads();
  __shared__ bool last;
  if (tid == 0) last = atomicAdd(sel_done(a) + pass, 1u) == gridDim.x - 1;
  __syncthreads();
  if (last) {
    __threadfence();
    sel_pick(a, pass);
  }
}

// keys below / equal to the threshold in this CTA's slice
__global__ void __launch_bounds__(kSelThreads) sel_count_kernel(const SelArgs a) {
  __shared__ uint32_t wl[kSelWarps], we[kSelWarps];
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const uint32_t thr = sel_state(a)[0];
  uint32_t c_lt = 0, c_eq = 0;
  const int g0 = blockIdx.x * a.per_cta, g1 = g0 + a.per_cta;
  for (int g = g0 + tid; g < g1; g += kSelThreads) {
    uint32_t key[4];
    bool valid[4];
    sel_keys4(a.scores, a.vec, g, a.n, a.pf, a.pl, key, valid);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      c_lt += valid[e] && key[e] < thr;
      c_eq += valid[e] && key[e] == thr;
    }
  }
  c_lt = __reduce_add_sync(0xffffffffu, c_lt);
  c_eq = __reduce_add_sync(0xffffffffu, c_eq);
  if (lane == 0) {
    wl[wid] = c_lt;
    we[wid] = c_eq;
  }
  __syncthreads();
  if (tid == 0) {
    uint32_t tl = 0, te = 0;
    for (int w = 0; w < kSelWarps; ++w) {
      tl += wl[w];
      te += we[w];
    }
    sel_counts(a)[2 * blockIdx.x] = tl;
    sel_counts(a)[2 * blockIdx.x + 1] = te;
  }
}

// stable compaction of this CTA's slice: warp w of the CTA owns the
// contiguous groups [g0 + w*wt, g0 + (w+1)*wt); lane l holds positions
// 4l .. 4l+3 of each 128-position trip
__global__ void __launch_bounds__(kSelThreads) sel_compact_kernel(const SelArgs a) {
  __shared__ uint32_t wl[kSelWarps], we[kSelWarps];
  __shared__ uint32_t s_base_lt, s_base_eq;
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const uint32_t thr = sel_state(a)[0], take_eq = sel_state(a)[2];
  if (tid < 32) {  // entries of the lower CTAs
    uint32_t bl = 0, be = 0;
    for (int c = lane; c < static_cast<int>(blockIdx.x); c += 32) {
      bl += sel_counts(a)[2 * c];
      be += sel_counts(a)[2 * c + 1];
    }
    bl = __reduce_add_sync(0xffffffffu, bl);
    be = __reduce_add_sync(0xffffffffu, be);
    if (lane == 0) {
      s_base_lt = bl;
      s_base_eq = be;
    }
  }
  const int wt = a.per_cta / kSelWarps;  // multiple of 32 (per_cta is a multiple of 32 * kSelWarps)
  const int g_begin = blockIdx.x * a.per_cta + wid * wt, g_end = g_begin + wt;
  uint32_t c_lt = 0, c_eq = 0;
  for (int g = g_begin + lane; g < g_end; g += 32) {
    uint32_t key[4];
    bool valid[4];
    sel_keys4(a.scores, a.vec, g, a.n, a.pf, a.pl, key, valid);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      c_lt += valid[e] && key[e] < thr;
      c_eq += valid[e] && key[e] == thr;
    }
  }
  c_lt = __reduce_add_sync(0xffffffffu, c_lt);
  c_eq = __reduce_add_sync(0xffffffffu, c_eq);
  if (lane == 0) {
    wl[wid] = c_lt;
    we[wid] = c_eq;
  }
  __syncthreads();
  uint32_t base_lt = s_base_lt, base_eq = s_base_eq;
  for (int w = 0; w < wid; ++w) {
    base_lt += wl[w];
    base_eq += we[w];
  }
  if (base_lt + min(base_eq, take_eq) >= static_cast<uint32_t>(a.k)) return;  // everything selected lies before
  const uint32_t below = (1u << lane) - 1u;
  for (int g = g_begin + lane; g < g_end; g += 32) {
    uint32_t key[4];
    bool valid[4];
    sel_keys4(a.scores, a.vec, g, a.n, a.pf, a.pl, key, valid);
    uint32_t blt[4], beq[4], lanes_lt = 0, lanes_eq = 0;  // entries of lower lanes
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      blt[e] = __ballot_sync(0xffffffffu, valid[e] && key[e] < thr);
      beq[e] = __ballot_sync(0xffffffffu, valid[e] && key[e] == thr);
      lanes_lt += __popc(blt[e] & below);
      lanes_eq += __popc(beq[e] & below);
    }
    uint32_t my_lt = base_lt + lanes_lt, my_eq = base_eq + lanes_eq;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const bool lt = valid[e] && key[e] < thr;
      const bool eq = valid[e] && key[e] == thr;
      // output position = number of selected entries with a smaller index;
      // selected = lt, or eq with rank < take_eq
      if (lt || (eq && my_eq < take_eq)) a.out[my_lt + min(my_eq, take_eq)] = 4 * g + e;
      my_lt += lt;
      my_eq += eq;
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      base_lt += __popc(blt[e]);
      base_eq += __popc(beq[e]);
    }
  }
}

// ---------------------------------------------------------------------------
// row gather: 16-byte vectors, one (b, h, row) per warp-stride
// ---------------------------------------------------------------------------
__global__ void gather_rows_kernel(const char* __restrict__ src, int64_t s_sb, int64_t s_sh, int64_t s_sn,
                                   int64_t n_src, const int64_t* __restrict__ idx, int n, int B, int H,
                                   int64_t row_bytes, char* __restrict__ dst, int64_t d_sb, int64_t d_sh,
                                   int64_t d_sn, int* status) {
  const int64_t vpr = row_bytes / 16;
  const int64_t total = static_cast<int64_t>(B) * H * n * vpr;
  for (int64_t w = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; w < total;
       w += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t v = w % vpr;
    int64_t r = w / vpr;
    const int i = static_cast<int>(r % n);
    r /= n;
    const int h = static_cast<int>(r % H);
    const int b = static_cast<int>(r / H);
    int64_t row = idx[i];
    if (static_cast<uint64_t>(row) >= static_cast<uint64_t>(n_src)) {  // out of range: flag it, read row 0
      set_status(status, AKV_ERR_SHAPE);
      row = 0;
    }
    const uint4 x = ldg_nc_v4(src + b * s_sb + h * s_sh + row * s_sn + v * 16);
    *reinterpret_cast<uint4*>(dst + b * d_sb + h * d_sh + i * d_sn + v * 16) = x;
  }
}

// dst[b, h, dst_idx[i]] <- src[b, h, src_idx ? src_idx[i] : i]; indices
// outside their tier record AKV_ERR_SHAPE and read / write row 0.
__global__ void scatter_rows_kernel(const char* __restrict__ src, int64_t s_sb, int64_t s_sh, int64_t s_sn,
                                    int64_t n_src, const int64_t* __restrict__ src_idx,
                                    const int64_t* __restrict__ dst_idx, int n, int B, int H, int64_t row_bytes,
                                    char* __restrict__ dst, int64_t d_sb, int64_t d_sh, int64_t d_sn, int64_t n_dst,
                                    int* status) {
  const int64_t vpr = row_bytes / 16;
  const int64_t total = static_cast<int64_t>(B) * H * n * vpr;
  for (int64_t w = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; w < total;
       w += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t v = w % vpr;
    int64_t r = w / vpr;
    const int i = static_cast<int>(r % n);
    r /= n;
    const int h = static_cast<int>(r % H);
    const int b = static_cast<int>(r / H);
    int64_t sr = src_idx ? src_idx[i] : i;
    int64_t dr = dst_idx[i];
    if (static_cast<uint64_t>(sr) >= static_cast<uint64_t>(n_src)) {
      set_status(status, AKV_ERR_SHAPE);
      sr = 0;
    }
    if (static_cast<uint64_t>(dr) >= static_cast<uint64_t>(n_dst)) {
      set_status(status, AKV_ERR_SHAPE);
      dr = 0;
    }
    const uint4 x = *reinterpret_cast<const uint4*>(src + b * s_sb + h * s_sh + sr * s_sn + v * 16);
    *reinterpret_cast<uint4*>(dst + b * d_sb + h * d_sh + dr * d_sn + v * 16) = x;
  }
}

// Self-test of the bounded mbarrier wait every kernel uses: one CTA waits on
// phase 0 of a barrier with arrival count 1.  arrive = 1: thread 0 arrives
// first and the wait completes; arrive = 0: nothing arrives, the wait runs out
// after limit_ns, records AKV_ERR_TIMEOUT in *status and the kernel returns.
// result[0] = 1 when every thread's wait completed, 2 when it ran out.
__global__ void selftest_wait_kernel(int arrive, uint64_t limit_ns, int* status, int* result) {
  __shared__ uint64_t bar;
  __shared__ int ran_out;
  if (threadIdx.x == 0) {
    ran_out = 0;
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (arrive && threadIdx.x == 0) mbar_arrive(&bar);
  if (!mbar_wait(&bar, 0, status, limit_ns)) atomicExch(&ran_out, 1);
  __syncthreads();
  if (threadIdx.x == 0) result[0] = ran_out ? 2 : 1;
}

}  // namespace akv

using namespace akv;

extern "C" const char* akv_strerror(int status) {
  switch (status) {
    case AKV_OK: return "ok";
    case AKV_ERR_SHAPE: return "bad or unsupported shape";
    case AKV_ERR_BITS: return "bit width must be 2, 3 or 4";
    case AKV_ERR_ALIGN: return "pointer or stride misaligned";
    case AKV_ERR_UNSUPPORTED: return "request not supported by this build";
    case AKV_ERR_LAUNCH: return "CUDA launch or runtime error";
    case AKV_ERR_TIMEOUT: return "device-side wait timed out";
    case AKV_ERR_NULL: return "required pointer is NULL";
    case AKV_ERR_WORKSPACE: return "workspace too small";
    default: return "unknown status";
  }
}

extern "C" int akv_abi_version(void) { return AKV_ABI_VERSION; }

extern "C" int akv_warm_layout_init(int D, int kb, int vb, int n, akv_warm_layout* L) {
  if (!L) return AKV_ERR_NULL;
  if (kb < 2 || kb > 4 || vb < 2 || vb > 4) return AKV_ERR_BITS;
  if (D <= 0 || D % 32 || D > 256 || n < 0 || n > D) return AKV_ERR_SHAPE;
  const RecLayout r = rec_layout(D, kb, vb, n);
  L->head_dim = D;
  L->key_bits = kb;
  L->value_bits = vb;
  L->n_outlier = n;
  L->kc = r.kc;
  L->vc = r.vc;
  L->ks = r.ks;
  L->kz = r.kz;
  L->vs = r.vs;
  L->vz = r.vz;
  L->mask = r.mask;
  L->flags = r.flags;
  L->ki = r.ki;
  L->vi = r.vi;
  L->ko = r.ko;
  L->vo = r.vo;
  L->vd = r.vd;
  L->bytes = r.bytes;
  return AKV_OK;
}

// Floats per SIMD register of the CPU whose torch reduction order the
// importance sums follow (16: AVX-512, 8: AVX2 / default builds).
static int g_reduction_width = 16;

extern "C" int akv_set_reduction_width(int floats) {
  if (floats != 4 && floats != 8 && floats != 16) return AKV_ERR_SHAPE;
  g_reduction_width = floats;
  return AKV_OK;
}

extern "C" int akv_importance_update(const float* attn, int B, int H, int M, int Na, float* scores, int N,
                                     float decay, void* stream) {
  if (!scores || (!attn && Na > 0)) return AKV_ERR_NULL;
  if (B <= 0 || H <= 0 || M <= 0 || Na < 0 || N < 0) return AKV_ERR_SHAPE;
  if (N == 0) return AKV_OK;
  importance_update_kernel<<<(N + 255) / 256, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      attn, B, H, M, Na, scores, N, decay, g_reduction_width);
  return cudaGetLastError() == cudaSuccess ? AKV_OK : AKV_ERR_LAUNCH;
}

extern "C" size_t akv_select_workspace_bytes(int n) { return n >= 0 ? kSelWsWords * sizeof(uint32_t) : 0; }

extern "C" int akv_select_bottomk(const float* scores, int n, int k, int protect_first, int protect_last,
                                  int64_t* idx_out, void* workspace, size_t workspace_bytes, void* stream) {
  if (!scores || !idx_out) return AKV_ERR_NULL;
  if (n < 0 || k < 0 || k > n || protect_first < 0 || protect_last < 0) return AKV_ERR_SHAPE;
  if (k == 0) return AKV_OK;
  if (!workspace || workspace_bytes < kSelWsWords * sizeof(uint32_t)) return AKV_ERR_WORKSPACE;
  if (reinterpret_cast<uintptr_t>(workspace) % 16) return AKV_ERR_ALIGN;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  SelArgs a{};
  a.scores = scores;
  a.n = n;
  a.k = k;
  a.pf = std::min(protect_first, n);
  a.pl = std::min(protect_last, n);
  a.vec = (reinterpret_cast<uintptr_t>(scores) % 16) == 0;
  a.ng = (n + 3) / 4;
  // slices of whole warp tiles (32 groups per warp per trip, kSelWarps warps)
  constexpr int unit = 32 * kSelWarps;
  const int ctas = std::max(1, std::min(kSelMaxCtas, (a.ng + unit - 1) / unit));
  a.per_cta = (a.ng + ctas * unit - 1) / (ctas * unit) * unit;
  const int grid = (a.ng + a.per_cta - 1) / a.per_cta;
  a.ws = static_cast<uint32_t*>(workspace);
  a.out = idx_out;
  if (cudaMemsetAsync(workspace, 0, kSelZeroWords * sizeof(uint32_t), st) != cudaSuccess) return AKV_ERR_LAUNCH;
  for (int pass = 0; pass < 4; ++pass) sel_hist_kernel<<<grid, kSelThreads, 0, st>>>(a, pass);
  sel_count_kernel<<<grid, kSelThreads, 0, st>>>(a);
  sel_compact_kernel<<<grid, kSelThreads, 0, st>>>(a);
  return cudaGetLastError() == cudaSuccess ? AKV_OK : AKV_ERR_LAUNCH;
}

extern "C" int akv_gather_rows(const void* src, int64_t s_sb, int64_t s_sh, int64_t s_sn, int64_t n_src,
                               const int64_t* idx, int n, int B, int H, int64_t row_bytes, void* dst, int64_t d_sb,
                               int64_t d_sh, int64_t d_sn, int* status, void* stream) {
  if (!src || !dst || (!idx && n > 0)) return AKV_ERR_NULL;
  if (n < 0 || B <= 0 || H <= 0 || row_bytes <= 0 || n_src <= 0) return AKV_ERR_SHAPE;
  if (n == 0) return AKV_OK;
  auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) % 16) == 0; };
  if (row_bytes % 16 || !al(src) || !al(dst) || s_sb % 16 || s_sh % 16 || s_sn % 16 || d_sb % 16 || d_sh % 16 ||
      d_sn % 16)
    return AKV_ERR_ALIGN;
  const int64_t total = static_cast<int64_t>(B) * H * n * (row_bytes / 16);
  const int64_t blocks = std::min<int64_t>((total + 255) / 256, 148 * 16);
  gather_rows_kernel<<<static_cast<unsigned>(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const char*>(src), s_sb, s_sh, s_sn, n_src, idx, n, B, H, row_bytes, static_cast<char*>(dst),
      d_sb, d_sh, d_sn, status);
  return cudaGetLastError() == cudaSuccess ? AKV_OK : AKV_ERR_LAUNCH;
}

extern "C" int akv_scatter_rows(const void* src, int64_t s_sb, int64_t s_sh, int64_t s_sn, int64_t n_src,
                                const int64_t* src_idx, const int64_t* dst_idx, int n, int B, int H,
                                int64_t row_bytes, void* dst, int64_t d_sb, int64_t d_sh, int64_t d_sn, int64_t n_dst,
                                int* status, void* stream) {
  if (!src || !dst || !dst_idx) return AKV_ERR_NULL;
  if (n < 0 || B <= 0 || H <= 0 || row_bytes <= 0 || row_bytes % 16 || n_src <= 0 || n_dst <= 0)
    return AKV_ERR_SHAPE;
  if (n == 0) return AKV_OK;
  if (reinterpret_cast<uintptr_t>(src) % 16 || reinterpret_cast<uintptr_t>(dst) % 16 || s_sb % 16 || s_sh % 16 ||
      s_sn % 16 || d_sb % 16 || d_sh % 16 || d_sn % 16)
    return AKV_ERR_ALIGN;
  const int64_t total = static_cast<int64_t>(B) * H * n * (row_bytes / 16);
  const int64_t blocks = std::min<int64_t>((total + 255) / 256, 148 * 16);
  scatter_rows_kernel<<<static_cast<unsigned>(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const char*>(src), s_sb, s_sh, s_sn, n_src, src_idx, dst_idx, n, B, H, row_bytes,
      static_cast<char*>(dst), d_sb, d_sh, d_sn, n_dst, status);
  return cudaGetLastError() == cudaSuccess ? AKV_OK : AKV_ERR_LAUNCH;
}

extern "C" int akv_selftest_wait(int arrive, int64_t limit_ns, int* status, int* result, void* stream) {
  if (!status || !result) return AKV_ERR_NULL;
  if (limit_ns <= 0 || limit_ns > static_cast<int64_t>(kWaitLimitNs)) return AKV_ERR_SHAPE;
  selftest_wait_kernel<<<1, 64, 0, static_cast<cudaStream_t>(stream)>>>(arrive, static_cast<uint64_t>(limit_ns),
                                                                         status, result);
  return cudaGetLastError() == cudaSuccess ? AKV_OK : AKV_ERR_LAUNCH;
}

extern "C" int akv_cold_copy(void* dst, int64_t dst_stride, const void* src, int64_t src_stride, int64_t chunk_bytes,
                             int64_t count, int dir, void* stream, void* event) {
  if (!dst || !src) return AKV_ERR_NULL;
  if (chunk_bytes <= 0 || count < 0 || dst_stride < chunk_bytes || src_stride < chunk_bytes) return AKV_ERR_SHAPE;
  if (dir != 0 && dir != 1) return AKV_ERR_SHAPE;
  if (count == 0) return AKV_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const cudaMemcpyKind kind = dir == 0 ? cudaMemcpyDeviceToHost : cudaMemcpyHostToDevice;
  if (cudaMemcpy2DAsync(dst, static_cast<size_t>(dst_stride), src, static_cast<size_t>(src_stride),
                        static_cast<size_t>(chunk_bytes), static_cast<size_t>(count), kind, st) != cudaSuccess)
    return AKV_ERR_LAUNCH;
  if (event && cudaEventRecord(static_cast<cudaEvent_t>(event), st) != cudaSuccess) return AKV_ERR_LAUNCH;
  return AKV_OK;
}

extern "C" int akv_migrator_update(const float* attn, int B, int H, int M, int Na, float* scores, int64_t* last_access,
                                   float* retrieval, int n_prev, int64_t step, float decay, void* stream) {
  if (!attn || !scores || !last_access || !retrieval) return AKV_ERR_NULL;
  if (B <= 0 || H <= 0 || M <= 0 || Na < 0 || n_prev < 0) return AKV_ERR_SHAPE;
  if (Na == 0) return AKV_OK;
  migrator_update_kernel<<<(Na + 255) / 256, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      attn, B, H, M, Na, scores, last_access, retrieval, n_prev, step, decay, g_reduction_width);
  return cudaGetLastError() == cudaSuccess ? AKV_OK : AKV_ERR_LAUNCH;
}

extern "C" int akv_migrator_importance(const float* scores, const int64_t* last_access, const float* retrieval, int N,
                                       int64_t step, float w_attn, float w_recency, float w_retrieval,
                                       int protect_first, int protect_last, float* out, void* workspace,
                                       size_t workspace_bytes, void* stream) {
  if (!scores || !last_access || !retrieval || !out) return AKV_ERR_NULL;
  if (N < 0 || protect_first < 0 || protect_last < 0) return AKV_ERR_SHAPE;
  if (N == 0) return AKV_OK;
  if (!workspace || workspace_bytes < 16) return AKV_ERR_WORKSPACE;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint32_t* red = static_cast<uint32_t*>(workspace);
  if (cudaMemsetAsync(red, 0, 3 * sizeof(uint32_t), st) != cudaSuccess) return AKV_ERR_LAUNCH;
  const int ctas = std::max(1, std::min(2 * 148, (N + 4 * 1024 - 1) / (4 * 1024)));
  migrator_reduce_kernel<<<ctas, 1024, 0, st>>>(scores, last_access, retrieval, N, red);
  migrator_importance_kernel<<<(N + 255) / 256, 256, 0, st>>>(scores, last_access, retrieval, N, step, red, w_attn,
                                                               w_recency, w_retrieval, std::min(protect_first, N),
                                                               std::min(protect_last, N), out);
  return cudaGetLastError() == cudaSuccess ? AKV_OK : AKV_ERR_LAUNCH;
}
