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
// One thread per column n; the (b,h) sum runs in order, like a sequential
// reduction of the reference's mean over dims (0, 1).
// ---------------------------------------------------------------------------
__global__ void importance_update_kernel(const float* __restrict__ attn, int B, int H, int M, int Na,
                                         float* __restrict__ scores, int N, float decay) {
  const int n = blockIdx.x * blockDim.x + threadIdx.x;
  if (n >= N) return;
  float imp = 0.f;
  if (n < Na) {
    const float inv = static_cast<float>(B * H);
    for (int m = 0; m < M; ++m) {
      float s = 0.f;
      for (int bh = 0; bh < B * H; ++bh) s = __fadd_rn(s, attn[(static_cast<int64_t>(bh) * M + m) * Na + n]);
      imp = __fadd_rn(imp, __fdiv_rn(s, inv));
    }
  }
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
                                       float* __restrict__ retrieval, int n_prev, int64_t step, float decay) {
  const int n = blockIdx.x * blockDim.x + threadIdx.x;
  if (n >= Na) return;
  const float cnt = static_cast<float>(B * H);
  float imp = 0.f;
  for (int m = 0; m < M; ++m) {
    float s = 0.f;
    for (int bh = 0; bh < B * H; ++bh) s = __fadd_rn(s, attn[(static_cast<int64_t>(bh) * M + m) * Na + n]);
    imp = __fadd_rn(imp, __fdiv_rn(s, cnt));
  }
  float sc = scores[n];
  if (n >= n_prev) {
    sc = 0.f;
    access[n] = step;
    retrieval[n] = 0.f;
  }
  scores[n] = __fadd_rn(__fmul_rn(sc, decay), imp);
  if (imp > 0.01f) access[n] = step;
}

// compute_importance (:175-219), step 1: max of scores, min of last access,
// max of retrieval over [0, N) -> red[0..2] (one CTA)
__global__ void migrator_reduce_kernel(const float* __restrict__ scores, const int64_t* __restrict__ access,
                                       const float* __restrict__ retrieval, int N, float* red) {
  __shared__ float smax[32], rmax[32];
  __shared__ float amin[32];
  float a = -INFINITY, r = -INFINITY, t = INFINITY;
  for (int i = threadIdx.x; i < N; i += blockDim.x) {
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
      red[0] = a;
      red[1] = t;
      red[2] = r;
    }
  }
}

// step 2: importance = w_a*attn_norm + w_r*recency + w_t*retr_norm, each op
// rounded like torch's, protected ends at +inf
__global__ void migrator_importance_kernel(const float* __restrict__ scores, const int64_t* __restrict__ access,
                                           const float* __restrict__ retrieval, int N, int64_t step,
                                           const float* __restrict__ red, float w_a, float w_r, float w_t,
                                           int n_first, int n_last, float* __restrict__ out) {
  const int n = blockIdx.x * blockDim.x + threadIdx.x;
  if (n >= N) return;
  const float smax = red[0], amin = red[1], rmax = red[2];
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
// of +inf.  A single CTA finds the k-th smallest key by an 8-bit radix select
// (4 passes of a 256-bin histogram), then a stable compaction emits, in
// ascending index order, every position below the threshold key plus the
// first (k - count_below) positions equal to it.
// ---------------------------------------------------------------------------
constexpr int kSelThreads = 1024;

AKV_DEV uint32_t order_key(float f) {
  uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

AKV_DEV uint32_t sel_key(const float* s, int i, int n, int pf, int pl) {
  if (i < pf || i >= n - pl) return order_key(INFINITY);
  return order_key(s[i]);
}

__global__ void __launch_bounds__(kSelThreads) select_bottomk_kernel(const float* __restrict__ scores, int n, int k,
                                                                     int pf, int pl, int64_t* __restrict__ out) {
  __shared__ uint32_t hist[256];
  __shared__ uint32_t s_prefix, s_mask, s_remaining;
  __shared__ uint32_t warp_cnt[kSelThreads / 32];
  __shared__ uint32_t s_base_lt, s_base_eq;
  const int tid = threadIdx.x;
  if (tid == 0) {
    s_prefix = 0;
    s_mask = 0;
    s_remaining = static_cast<uint32_t>(k);
  }
  __syncthreads();
  // radix select of the k-th smallest key, most significant byte first
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = tid; i < 256; i += kSelThreads) hist[i] = 0;
    __syncthreads();
    const uint32_t prefix = s_prefix, mask = s_mask;
    for (int i = tid; i < n; i += kSelThreads) {
      const uint32_t key = sel_key(scores, i, n, pf, pl);
      if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 255u], 1u);
    }
    __syncthreads();
    if (tid == 0) {
      uint32_t rem = s_remaining, acc = 0;
      int bin = 0;
      for (; bin < 256; ++bin) {
        if (acc + hist[bin] >= rem) break;
        acc += hist[bin];
      }
      s_remaining = rem - acc;
      s_prefix = prefix | (static_cast<uint32_t>(bin) << shift);
      s_mask = mask | (255u << shift);
    }
    __syncthreads();
  }
  const uint32_t thr = s_prefix;       // key of the k-th smallest
  const uint32_t take_eq = s_remaining;  // how many keys == thr to take (lowest indices first)
  // stable compaction in index order, chunk by chunk
  if (tid == 0) {
    s_base_lt = 0;
    s_base_eq = 0;
  }
  __syncthreads();
  const int lane = tid & 31, wid = tid >> 5;
  for (int base = 0; base < n; base += kSelThreads) {
    const int i = base + tid;
    uint32_t key = i < n ? sel_key(scores, i, n, pf, pl) : 0xffffffffu;
    const bool lt = i < n && key < thr;
    const bool eq = i < n && key == thr;
    // ranks of `eq` entries in index order
    const uint32_t beq = __ballot_sync(0xffffffffu, eq);
    const uint32_t blt = __ballot_sync(0xffffffffu, lt);
    if (lane == 0) warp_cnt[wid] = (__popc(blt) << 16) | __popc(beq);
    __syncthreads();
    uint32_t pre_lt = 0, pre_eq = 0, tot_lt = 0, tot_eq = 0;
    for (int w = 0; w < kSelThreads / 32; ++w) {
      const uint32_t c = warp_cnt[w];
      if (w < wid) {
        pre_lt += c >> 16;
        pre_eq += c & 0xffffu;
      }
      tot_lt += c >> 16;
      tot_eq += c & 0xffffu;
    }
    const uint32_t my_lt = s_base_lt + pre_lt + __popc(blt & ((1u << lane) - 1u));
    const uint32_t my_eq = s_base_eq + pre_eq + __popc(beq & ((1u << lane) - 1u));
    // output position = number of selected entries with smaller index
    // selected = lt, or eq with rank < take_eq
    if (lt || (eq && my_eq < take_eq)) {
      const uint32_t eq_before = min(my_eq, take_eq);
      out[my_lt + eq_before] = i;
    }
    __syncthreads();
    if (tid == 0) {
      s_base_lt += tot_lt;
      s_base_eq += tot_eq;
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// row gather: 16-byte vectors, one (b, h, row) per warp-stride
// ---------------------------------------------------------------------------
__global__ void gather_rows_kernel(const char* __restrict__ src, int64_t s_sb, int64_t s_sh, int64_t s_sn,
                                   const int64_t* __restrict__ idx, int n, int B, int H, int64_t row_bytes,
                                   char* __restrict__ dst, int64_t d_sb, int64_t d_sh, int64_t d_sn) {
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
    const uint4 x = ldg_nc_v4(src + b * s_sb + h * s_sh + idx[i] * s_sn + v * 16);
    *reinterpret_cast<uint4*>(dst + b * d_sb + h * d_sh + i * d_sn + v * 16) = x;
  }
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

extern "C" int akv_importance_update(const float* attn, int B, int H, int M, int Na, float* scores, int N,
                                     float decay, void* stream) {
  if (!scores || (!attn && Na > 0)) return AKV_ERR_NULL;
  if (B <= 0 || H <= 0 || M <= 0 || Na < 0 || N < 0) return AKV_ERR_SHAPE;
  if (N == 0) return AKV_OK;
  importance_update_kernel<<<(N + 255) / 256, 256, 0, static_cast<cudaStream_t>(stream)>>>(attn, B, H, M, Na,
                                                                                          scores, N, decay);
  return cudaGetLastError() == cudaSuccess ? AKV_OK : AKV_ERR_LAUNCH;
}

extern "C" size_t akv_select_workspace_bytes(int n) { return n >= 0 ? 16 : 0; }

extern "C" int akv_select_bottomk(const float* scores, int n, int k, int protect_first, int protect_last,
                                  int64_t* idx_out, void* workspace, size_t workspace_bytes, void* stream) {
  (void)workspace;
  (void)workspace_bytes;
  if (!scores || !idx_out) return AKV_ERR_NULL;
  if (n < 0 || k < 0 || k > n || protect_first < 0 || protect_last < 0) return AKV_ERR_SHAPE;
  if (k == 0) return AKV_OK;
  if (protect_first > n) protect_first = n;
  if (protect_last > n) protect_last = n;
  select_bottomk_kernel<<<1, kSelThreads, 0, static_cast<cudaStream_t>(stream)>>>(scores, n, k, protect_first,
                                                                                 protect_last, idx_out);
  return cudaGetLastError() == cudaSuccess ? AKV_OK : AKV_ERR_LAUNCH;
}

extern "C" int akv_gather_rows(const void* src, int64_t s_sb, int64_t s_sh, int64_t s_sn, const int64_t* idx, int n,
                               int B, int H, int64_t row_bytes, void* dst, int64_t d_sb, int64_t d_sh, int64_t d_sn,
                               void* stream) {
  if (!src || !dst || (!idx && n > 0)) return AKV_ERR_NULL;
  if (n < 0 || B <= 0 || H <= 0 || row_bytes <= 0) return AKV_ERR_SHAPE;
  if (n == 0) return AKV_OK;
  auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) % 16) == 0; };
  if (row_bytes % 16 || !al(src) || !al(dst) || s_sb % 16 || s_sh % 16 || s_sn % 16 || d_sb % 16 || d_sh % 16 ||
      d_sn % 16)
    return AKV_ERR_ALIGN;
  const int64_t total = static_cast<int64_t>(B) * H * n * (row_bytes / 16);
  const int64_t blocks = std::min<int64_t>((total + 255) / 256, 148 * 16);
  gather_rows_kernel<<<static_cast<unsigned>(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const char*>(src), s_sb, s_sh, s_sn, idx, n, B, H, row_bytes, static_cast<char*>(dst), d_sb,
      d_sh, d_sn);
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
      attn, B, H, M, Na, scores, last_access, retrieval, n_prev, step, decay);
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
  float* red = static_cast<float*>(workspace);
  migrator_reduce_kernel<<<1, 1024, 0, st>>>(scores, last_access, retrieval, N, red);
  migrator_importance_kernel<<<(N + 255) / 256, 256, 0, st>>>(scores, last_access, retrieval, N, step, red, w_attn,
                                                               w_recency, w_retrieval, std::min(protect_first, N),
                                                               std::min(protect_last, N), out);
  return cudaGetLastError() == cudaSuccess ? AKV_OK : AKV_ERR_LAUNCH;
}
