// Cross-GPU exchange of split-KV decode partials over peer memory (NVLink), without NCCL.
//
// Long-context decode splits one sequence's KV cache by position over the ranks; every
// rank ends a step with a normalised partial (o, m, l) per q-head (a few KB). Here each
// rank pushes its partial straight into every rank's mailbox with plain stores through
// CUDA IPC mappings, raises a flag in each mailbox, waits (bounded) for the flags of all
// ranks in its own mailbox, and merges the partials (log-sum-exp). One small kernel per
// step, no host involvement, so the whole decode step can be replayed from a CUDA graph.
//
// Mailbox of a rank: see peer.cuh (this kernel uses the call flags and the partials). A
// call's epoch e = (*epoch) + 1 selects parity e & 1: a rank can be at most one call ahead
// of another (it waits for all flags of its own call), so the other parity is never
// overwritten while it is read.
// No TMA, no multicast, no multimem: plain ld/st to peer memory.
#include <cuda_runtime.h>

#include <cstring>

#include "peer.cuh"

namespace tasft {
namespace {

constexpr int kPeerThreads = 512;


constexpr int kRowChunk = 128;  // rows whose merge weights sit in shared memory at once
constexpr int kMaxWorld = 8;

template <typename T>
__global__ void __launch_bounds__(kPeerThreads) peer_combine_kernel(tasft_peer_combine_args a) {
  const int world = a.world, rank = a.rank, D = a.D;
  const int64_t rows = a.rows;
  const int64_t slab = rows * (D + 2);  // floats of one rank's partial
  const uint32_t e = *a.epoch + 1u;
  const int par = (int)(e & 1u);
  const int64_t foff = peer_part_off(world, rows, D);  // float offset of the partials
  // 1. push this rank's (o | m, l) rows into slot [par][rank] of every mailbox, 8 bytes per
  //    store (a row is D + 2 floats, D even: rows stay 8-byte aligned)
  const int64_t rp = (D + 2) / 2;  // float2 per mailbox row
  for (int p = 0; p < world; ++p) {
    float2* dst = reinterpret_cast<float2*>(reinterpret_cast<float*>(a.mailboxes[p]) + foff +
                                            ((int64_t)par * world + rank) * slab);
    for (int64_t x = threadIdx.x; x < rows * rp; x += blockDim.x) {
      const int64_t r = x / rp, c = x % rp;
      dst[x] = c < D / 2 ? reinterpret_cast<const float2*>(a.part_o + r * D)[c]
                         : reinterpret_cast<const float2*>(a.part_ml)[r];
    }
  }
  __syncthreads();
  // 2. publish: the data stores above happen-before the flag
  if (threadIdx.x == 0) {
    __threadfence_system();
    for (int p = 0; p < world; ++p) st_release_sys(reinterpret_cast<uint32_t*>(a.mailboxes[p]) + rank, e);
  }
  // 3. wait for every rank's flag in this rank's own mailbox (bounded)
  __shared__ int s_timeout;
  if (threadIdx.x == 0) s_timeout = 0;
  __syncthreads();
  if (threadIdx.x < world) {
    const uint32_t* flag = reinterpret_cast<const uint32_t*>(a.mailboxes[rank]) + threadIdx.x;
    const uint64_t t0 = globaltimer_ns();
    while ((int32_t)(ld_acquire_sys(flag) - e) < 0) {
      if (globaltimer_ns() - t0 > a.timeout_ns) {
        atomicOr(&s_timeout, 1);
        break;
      }
    }
  }
  __syncthreads();
  if (s_timeout && threadIdx.x == 0) set_err(a.err, TASFT_DEVERR_TIMEOUT);
  // 4. merge the world partials of this parity: per chunk of rows, the weights
  //    w_g = l_g e^(m_g - max) and their sum first (all (rank, row) pairs loaded at once), then every
  //    output element as one pass of independent loads
  const float* box = reinterpret_cast<const float*>(a.mailboxes[rank]) + foff + (int64_t)par * world * slab;
  __shared__ float s_w[kMaxWorld][kRowChunk];
  __shared__ float s_m[kMaxWorld][kRowChunk];
  __shared__ float s_den[kRowChunk];
  for (int64_t r0 = 0; r0 < rows; r0 += kRowChunk) {
    const int nr = rows - r0 < kRowChunk ? (int)(rows - r0) : kRowChunk;
    for (int x = threadIdx.x; x < world * nr; x += blockDim.x) {
      const int g = x / nr, r = x % nr;
      const float* pr = box + g * slab + (r0 + r) * (D + 2);
      const float l = pr[D + 1];
      s_w[g][r] = l;
      s_m[g][r] = l > 0.f ? pr[D] : -INFINITY;
    }
    __syncthreads();
    for (int r = threadIdx.x; r < nr; r += blockDim.x) {
      float mt = -INFINITY;
      for (int g = 0; g < world; ++g) mt = fmaxf(mt, s_m[g][r]);
      float den = 0.f;
      for (int g = 0; g < world; ++g) {
        const float w = s_m[g][r] == -INFINITY ? 0.f : s_w[g][r] * __expf(s_m[g][r] - mt);
        s_w[g][r] = w;
        den += w;
      }
      s_den[r] = den;
    }
    __syncthreads();
#pragma unroll 4
    for (int x = threadIdx.x; x < nr * D; x += blockDim.x) {
      const int r = x / D, c = x % D;
      float num = 0.f;
      for (int g = 0; g < world; ++g) num = fmaf(s_w[g][r], box[g * slab + (r0 + r) * (D + 2) + c], num);
      const float den = s_den[r];
      reinterpret_cast<T*>(a.out)[(r0 + r) * D + c] = from_f<T>(den > 0.f ? num / den : 0.f);
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) *a.epoch = e;
}

}  // namespace
}  // namespace tasft

using namespace tasft;

extern "C" int64_t tasft_peer_mailbox_bytes(int32_t world, int64_t rows, int32_t D) {
  if (world <= 0 || rows <= 0 || D <= 0) return -1;
  return peer_mailbox_bytes(world, rows, D);
}

extern "C" int tasft_peer_alloc(int64_t bytes, void** ptr) {
  if (!ptr || bytes <= 0) return TASFT_ERR_INVALID_ARG;
  *ptr = nullptr;
  if (cudaMalloc(ptr, (size_t)bytes) != cudaSuccess) return TASFT_ERR_CUDA;
  if (cudaMemset(*ptr, 0, (size_t)bytes) != cudaSuccess) return TASFT_ERR_CUDA;
  return TASFT_OK;
}

extern "C" int tasft_peer_free(void* ptr) {
  return ptr && cudaFree(ptr) != cudaSuccess ? TASFT_ERR_CUDA : TASFT_OK;
}

extern "C" int tasft_ipc_handle(void* ptr, uint8_t* handle64) {
  if (!ptr || !handle64) return TASFT_ERR_INVALID_ARG;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, ptr) != cudaSuccess) return TASFT_ERR_CUDA;
  static_assert(sizeof(h) == 64, "IPC handle size");
  memcpy(handle64, &h, 64);
  return TASFT_OK;
}

extern "C" int tasft_ipc_open(const uint8_t* handle64, void** ptr) {
  if (!handle64 || !ptr) return TASFT_ERR_INVALID_ARG;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle64, 64);
  *ptr = nullptr;
  return cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess ? TASFT_OK : TASFT_ERR_CUDA;
}

extern "C" int tasft_ipc_close(void* ptr) {
  return ptr && cudaIpcCloseMemHandle(ptr) != cudaSuccess ? TASFT_ERR_CUDA : TASFT_OK;
}

extern "C" int tasft_peer_combine(const tasft_peer_combine_args* ap, tasft_stream_t stream) {
  if (!ap) return TASFT_ERR_INVALID_ARG;
  const tasft_peer_combine_args& a = *ap;
  if (!a.part_o || !a.part_ml || !a.mailboxes || !a.epoch || !a.out) return TASFT_ERR_INVALID_ARG;
  if (a.world <= 0 || a.world > kMaxWorld || a.rank < 0 || a.rank >= a.world || a.rows <= 0 || a.D <= 0)
    return TASFT_ERR_INVALID_ARG;
  // 8-byte pushes: D even, partial rows 8-byte aligned
  if ((a.D & 1) || (reinterpret_cast<uintptr_t>(a.part_o) & 7u) || (reinterpret_cast<uintptr_t>(a.part_ml) & 7u))
    return TASFT_ERR_INVALID_ARG;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  switch (a.dtype) {
    case TASFT_F32: peer_combine_kernel<float><<<1, kPeerThreads, 0, st>>>(a); break;
    case TASFT_BF16: peer_combine_kernel<__nv_bfloat16><<<1, kPeerThreads, 0, st>>>(a); break;
    case TASFT_F16: peer_combine_kernel<__half><<<1, kPeerThreads, 0, st>>>(a); break;
    default: return TASFT_ERR_UNSUPPORTED;
  }
  count_launch();
  return launch_status();
}
