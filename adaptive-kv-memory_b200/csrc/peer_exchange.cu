// The cross-GPU step of a sequence-split decode (batch 1, very long context:
// every GPU holds a contiguous share of the warm blocks) over NVLink peer
// memory instead of a collective library call.
//
// Each GPU ends its decode with one merged partial record (acc[D], m, l) per
// (batch row, query head) for the tokens it holds.  akv_peer_publish writes
// that record into slot `rank` of every GPU's gather buffer with plain P2P
// stores and, once all of them are written (system-scope fences), sets flag
// `rank` in every GPU's flag array to the step's epoch; akv_peer_combine waits
// (bounded) for all flags of the epoch in its own memory and merges the world
// records with the same log-sum-exp arithmetic as the split combine.  Gather
// slots alternate between two halves by epoch parity: a GPU cannot publish
// epoch e + 2 before every GPU has finished combining epoch e (its combine of
// e + 1 waits for their publishes of e + 1, which follow their combines of e).
//
// Peer addresses come from CUDA IPC handles opened with lazy peer access
// (akv_ipc_open); only plain loads and stores touch peer memory, issued by
// these kernels (no TMA copy, no library kernel).
#include <cuda_runtime.h>

#include <cfloat>
#include <cmath>
#include <cstring>

#include "common.cuh"

namespace akv {

constexpr int kPeerThreads = 128;
constexpr uint64_t kPeerWaitNs = 2000000000ull;  // 2 s

// grid (rows): block r copies record r to every rank's slot, then the last
// block to finish raises this rank's flag at every rank
__global__ void __launch_bounds__(kPeerThreads) peer_publish_kernel(const float* __restrict__ part, int64_t part_sr,
                                                                    int rows, int D, float* const* peer_gather,
                                                                    int* const* peer_flags, int world, int rank,
                                                                    int epoch, int* counter) {
  const int r = blockIdx.x;
  const int rec = D + 2;
  const int64_t slot = (static_cast<int64_t>(epoch & 1) * world + rank) * rows * rec + static_cast<int64_t>(r) * rec;
  const float* src = part + static_cast<int64_t>(r) * part_sr;
  for (int p = 0; p < world; ++p) {
    float* dst = peer_gather[p] + slot;
    for (int i = threadIdx.x; i < rec; i += blockDim.x) dst[i] = src[i];
  }
  __threadfence_system();  // this thread's stores, to every GPU, before the arrival below
  __syncthreads();
  __shared__ bool last;
  if (threadIdx.x == 0) last = atomicAdd(counter + (epoch & 1), 1) == static_cast<int>(gridDim.x) - 1;
  __syncthreads();
  if (last && threadIdx.x == 0) {
    __threadfence_system();
    for (int p = 0; p < world; ++p) atomicExch_system(peer_flags[p] + rank, epoch);
    counter[epoch & 1] = 0;  // ready for epoch + 2 (stream order: the next publish follows this kernel)
  }
}

AKV_DEV int load_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// grid (rows, ceil(D / 32)): wait for every rank's flag of this epoch, then
// merge the world records of row r (channels 32 * blockIdx.y ..)
__global__ void __launch_bounds__(32) peer_combine_kernel(const float* __restrict__ gather,
                                                                    const int* flags, int rows, int D, int world,
                                                                    int epoch, __half* out, int64_t o_sr, float* lse,
                                                                    int* status) {
  __shared__ int ok;
  if (threadIdx.x == 0) {
    ok = 1;
    const uint64_t t0 = global_timer_ns();
    for (int p = 0; p < world; ++p) {
      while (load_acquire_sys(flags + p) < epoch) {
        if (global_timer_ns() - t0 > kPeerWaitNs) {
          set_status(status, AKV_ERR_TIMEOUT);
          ok = 0;
          break;
        }
        __nanosleep(256);
      }
      if (!ok) break;
    }
  }
  __syncthreads();
  const int r = blockIdx.x;
  const int d = blockIdx.y * 32 + threadIdx.x;
  if (!ok) {  // a rank never published: output zeros, lse -inf (status says why)
    if (d < D && out) out[static_cast<int64_t>(r) * o_sr + d] = __float2half_rn(0.f);
    if (blockIdx.y == 0 && threadIdx.x == 0 && lse) lse[r] = -INFINITY;
    return;
  }
  const int rec = D + 2;
  const float* base = gather + static_cast<int64_t>(epoch & 1) * world * rows * rec + static_cast<int64_t>(r) * rec;
  const int64_t ss = static_cast<int64_t>(rows) * rec;
  float M = -INFINITY;
  for (int p = 0; p < world; ++p) M = fmaxf(M, base[p * ss + D]);
  const float mb = (M == -INFINITY) ? 0.f : M;
  float L = 0.f, o = 0.f;
  for (int p = 0; p < world; ++p) {
    const float w = exp2f(base[p * ss + D] - mb);
    L += base[p * ss + D + 1] * w;
    if (d < D) o = fmaf(base[p * ss + d], w, o);
  }
  if (d < D && out) {
    const float inv = L > 0.f ? 1.f / L : 0.f;
    out[static_cast<int64_t>(r) * o_sr + d] = __float2half_rn(o * inv);
  }
  if (blockIdx.y == 0 && threadIdx.x == 0 && lse) lse[r] = L > 0.f ? (M + log2f(L)) / 1.4426950408889634f : -INFINITY;
}

}  // namespace akv

using namespace akv;

extern "C" int akv_peer_publish(const float* part, int64_t part_sr, int rows, int D, float* const* peer_gather,
                                int* const* peer_flags, int world, int rank, int epoch, int* counter, void* stream) {
  if (!part || !peer_gather || !peer_flags || !counter) return AKV_ERR_NULL;
  if (rows <= 0 || D <= 0 || world <= 0 || rank < 0 || rank >= world || epoch <= 0 || part_sr < D + 2)
    return AKV_ERR_SHAPE;
  peer_publish_kernel<<<rows, kPeerThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      part, part_sr, rows, D, peer_gather, peer_flags, world, rank, epoch, counter);
  return cudaGetLastError() == cudaSuccess ? AKV_OK : AKV_ERR_LAUNCH;
}

extern "C" int akv_peer_combine(const float* gather, const int* flags, int rows, int D, int world, int epoch,
                                uint16_t* out, int64_t o_sr, float* lse, int* status, void* stream) {
  if (!gather || !flags || (!out && !lse)) return AKV_ERR_NULL;
  if (rows <= 0 || D <= 0 || world <= 0 || epoch <= 0) return AKV_ERR_SHAPE;
  peer_combine_kernel<<<dim3(rows, (D + 31) / 32), 32, 0, static_cast<cudaStream_t>(stream)>>>(
      gather, flags, rows, D, world, epoch, reinterpret_cast<__half*>(out), o_sr, lse, status);
  return cudaGetLastError() == cudaSuccess ? AKV_OK : AKV_ERR_LAUNCH;
}

extern "C" int akv_peer_alloc(size_t bytes, void** dev_ptr_out) {
  if (!dev_ptr_out) return AKV_ERR_NULL;
  if (bytes == 0) return AKV_ERR_SHAPE;
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) return AKV_ERR_LAUNCH;
  if (cudaMemset(p, 0, bytes) != cudaSuccess) {
    cudaFree(p);
    return AKV_ERR_LAUNCH;
  }
  *dev_ptr_out = p;
  return AKV_OK;
}

extern "C" int akv_peer_free(void* dev_ptr) {
  if (!dev_ptr) return AKV_ERR_NULL;
  return cudaFree(dev_ptr) == cudaSuccess ? AKV_OK : AKV_ERR_LAUNCH;
}

extern "C" int akv_ipc_export(const void* dev_ptr, void* handle_out) {
  if (!dev_ptr || !handle_out) return AKV_ERR_NULL;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, const_cast<void*>(dev_ptr)) != cudaSuccess) return AKV_ERR_LAUNCH;
  memcpy(handle_out, &h, sizeof(h));
  return AKV_OK;
}

extern "C" int akv_ipc_open(const void* handle, void** dev_ptr_out) {
  if (!handle || !dev_ptr_out) return AKV_ERR_NULL;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  if (cudaIpcOpenMemHandle(dev_ptr_out, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return AKV_ERR_LAUNCH;
  return AKV_OK;
}

extern "C" int akv_ipc_close(void* dev_ptr) {
  if (!dev_ptr) return AKV_ERR_NULL;
  return cudaIpcCloseMemHandle(dev_ptr) == cudaSuccess ? AKV_OK : AKV_ERR_LAUNCH;
}
