// Decode entry point that allocates nothing.
//
// Some callers cannot hand this library a workspace: a plugin whose host process owns
// every device allocation and passes the plugin only its input and output buffers, or a
// serving loop that must never call cudaMalloc (it can synchronise the device and can
// fail under memory pressure at the worst moment). For them the split-KV scratch of the
// decode kernels (per-split partial results and the per-(sequence, kv-head) tickets)
// lives in one file-scope device array of fixed size, kNoAllocScratchBytes.
//
// Rules for users of tasft_bsa_decode_fwd_noalloc:
//   * The array exists once per GPU that loads the library and stays allocated until
//     the process exits.
//   * The first call on each device looks up the array's device address
//     (cudaGetSymbolAddress) with that device current; make that first call before any
//     stream capture begins.
//   * Every call on a device shares the array and leaves its last contents behind. The
//     ticket counters are cleared (cudaMemsetAsync on the caller's stream) at the start
//     of every call. Calls whose executions overlap on the GPU -- on different streams,
//     or without ordering between them -- race on the array and give wrong results.
//     Order them on one stream.
//   * A call that needs more scratch than kNoAllocScratchBytes returns TASFT_ERR_TOO_LARGE
//     before anything is launched. With num_splits == 1 no scratch is used at all.
#include <mutex>

#include "decode.cuh"

namespace tasft {

int decode_check_args(const tasft_decode_args& a);
int decode_pick_splits(const tasft_decode_args& a);
int decode_run(const tasft_decode_args& a, const DecodeWs& ws, int nsplit, cudaStream_t st);

namespace {

constexpr int64_t kNoAllocScratchBytes = 4ll << 20;  // 4 MiB per device
constexpr int kMaxDevices = 64;

// The scratch itself. In host code this name only stands in for the symbol; the device
// address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) uint8_t g_decode_scratch[kNoAllocScratchBytes];

std::mutex g_mu;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of the scratch on the current device (looked up once per device).
int scratch_for_current_device(void** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return TASFT_ERR_CUDA;
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_decode_scratch);
    if (e != cudaSuccess || p == nullptr) {
      if (debug_enabled()) debug_log("cudaGetSymbolAddress(g_decode_scratch) failed: %s", cudaGetErrorString(e));
      return TASFT_ERR_CUDA;
    }
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return TASFT_OK;
}

}  // namespace
}  // namespace tasft

using namespace tasft;

extern "C" int64_t tasft_decode_noalloc_capacity(void) { return kNoAllocScratchBytes; }

extern "C" int tasft_bsa_decode_fwd_noalloc(const tasft_decode_args* ap, tasft_stream_t stream) {
  if (!ap) return TASFT_ERR_INVALID_ARG;
  const tasft_decode_args& a = *ap;
  int rc = decode_check_args(a);
  if (rc != TASFT_OK) return rc;
  const int nsplit = decode_pick_splits(a);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  DecodeWs ws{nullptr, nullptr, 0};
  if (nsplit > 1) {
    // same layout as tasft_decode_workspace_size: tickets (padded to 256 B), then partials
    const int64_t tick = ((int64_t)(a.B * a.Hk + 2) * 4 + 255) / 256 * 256;
    const int64_t need = tick + (int64_t)a.B * a.Hq * nsplit * (a.D + 2) * 4;
    if (need > kNoAllocScratchBytes) {
      if (debug_enabled())
        debug_log("decode_noalloc: needs %lld bytes of scratch, capacity is %lld", (long long)need,
                  (long long)kNoAllocScratchBytes);
      return TASFT_ERR_TOO_LARGE;
    }
    void* base = nullptr;
    rc = scratch_for_current_device(&base);
    if (rc != TASFT_OK) return rc;
    if (cudaMemsetAsync(base, 0, (size_t)tick, st) != cudaSuccess) return TASFT_ERR_CUDA;
    ws.max_splits = nsplit;
    ws.ticket = reinterpret_cast<int32_t*>(base);
    ws.part = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(base) + tick);
  }
  return decode_run(a, ws, nsplit, st);
}
