// Gate threshold calibration: tau such that a target fraction of the gate's block scores
// is kept, measured on calibration scores instead of the reference's weight-norm heuristic
// (tasft/bundle/export.py:327-360 sets "estimated_sparsity = 0.5 + 0.1 * |w_out|").
//
// tau = the keep-th largest score, found exactly by a radix select over the 32-bit
// pattern of the scores (mapped so that unsigned order is float order), one 8-bit digit
// per pass, histograms in shared memory; then one pass counts the scores >= tau (the
// reference keeps soft >= tau, tasft/modules/attn_gate.py:475, so ties at tau are kept).
// A single CTA: calibration runs once per layer offline, and the scores of a layer are a
// few MB at most. Deterministic.
#include "common.cuh"

namespace tasft {
namespace {

constexpr int kCalibThreads = 1024;

__device__ __forceinline__ uint32_t order_bits(float f) {
  const uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float from_order_bits(uint32_t u) {
  return __uint_as_float((u & 0x80000000u) ? (u & 0x7fffffffu) : ~u);
}

__global__ void __launch_bounds__(kCalibThreads) calib_tau_kernel(tasft_calib_args a) {
  __shared__ unsigned long long hist[256];
  __shared__ uint32_t s_prefix, s_mask;
  __shared__ long long s_remaining;
  if (threadIdx.x == 0) {
    s_prefix = 0;
    s_mask = 0;
    s_remaining = a.keep;
  }
  __syncthreads();
  if (a.keep <= 0 || a.keep > a.n) {
    if (threadIdx.x == 0) {
      *a.tau = a.keep <= 0 ? INFINITY : -INFINITY;  // keep nothing / everything
      if (a.kept) *a.kept = a.keep <= 0 ? 0 : a.n;
    }
    return;
  }
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    const uint32_t prefix = s_prefix, mask = s_mask;
    for (int64_t i = threadIdx.x; i < a.n; i += blockDim.x) {
      const uint32_t u = order_bits(a.scores[i]);
      if ((u & mask) == prefix) atomicAdd(&hist[(u >> shift) & 255u], 1ull);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      long long rem = s_remaining;
      int d = 255;
      for (; d > 0; --d) {
        if ((long long)hist[d] >= rem) break;
        rem -= (long long)hist[d];
      }
      s_remaining = rem;
      s_prefix = prefix | ((uint32_t)d << shift);
      s_mask = mask | (255u << shift);
    }
    __syncthreads();
  }
  const float tau = from_order_bits(s_prefix);
  if (a.kept) {
    __shared__ unsigned long long s_cnt;
    if (threadIdx.x == 0) s_cnt = 0;
    __syncthreads();
    unsigned long long c = 0;
    for (int64_t i = threadIdx.x; i < a.n; i += blockDim.x) c += a.scores[i] >= tau ? 1ull : 0ull;
    atomicAdd(&s_cnt, c);
    __syncthreads();
    if (threadIdx.x == 0) *a.kept = (int64_t)s_cnt;
  }
  if (threadIdx.x == 0) *a.tau = tau;
}

}  // namespace
}  // namespace tasft

using namespace tasft;

extern "C" int tasft_calibrate_tau(const tasft_calib_args* ap, tasft_stream_t stream) {
  if (!ap || !ap->scores || !ap->tau || ap->n <= 0) return TASFT_ERR_INVALID_ARG;
  calib_tau_kernel<<<1, kCalibThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(*ap);
  count_launch();
  return launch_status();
}
