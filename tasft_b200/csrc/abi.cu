// C-ABI entry points that dispatch between kernel variants, plus status strings,
// version and launch accounting.
#include "common.cuh"

#include <cstdarg>
#include <cstdio>
#include <cstdlib>

namespace tasft {
std::atomic<int64_t> g_launches{0};

bool debug_enabled() {
  static const bool on = std::getenv("TASFT_DEBUG") != nullptr;
  return on;
}
void debug_log(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  std::fprintf(stderr, "[tasft_b200] ");
  std::vfprintf(stderr, fmt, ap);
  std::fprintf(stderr, "\n");
  va_end(ap);
}
int prefill_simt(const tasft_prefill_args& a, cudaStream_t st, const int32_t* cu = nullptr);
// Returns TASFT_ERR_UNSUPPORTED when the tcgen05 kernel does not cover the shape.
// `cu` (cu_seqlens, B + 1 entries) and `total` describe packed sequences; nullptr / 0 otherwise.
int prefill_tc(const tasft_prefill_args& a, cudaStream_t st, const int32_t* cu = nullptr, int total = 0,
               float* bmax = nullptr, int emulate_bf16 = 0);
}  // namespace tasft

using namespace tasft;

extern "C" int tasft_bsa_prefill_fwd(const tasft_prefill_args* ap, tasft_stream_t stream) {
  if (!ap) return TASFT_ERR_INVALID_ARG;
  const tasft_prefill_args& a = *ap;
  if (!a.q || !a.k || !a.v || !a.out || !a.kept_idx || !a.kept_cnt) return TASFT_ERR_INVALID_ARG;
  if (a.B <= 0 || a.Hq <= 0 || a.Hk <= 0 || a.S <= 0 || a.D <= 0 || a.Hm <= 0) return TASFT_ERR_INVALID_ARG;
  if (a.Hq % a.Hk != 0 || a.Hq % a.Hm != 0) return TASFT_ERR_INVALID_ARG;
  if (a.q_stride[3] != 1 || a.k_stride[3] != 1 || a.v_stride[3] != 1 || a.o_stride[3] != 1)
    return TASFT_ERR_INVALID_ARG;
  if (a.block != 32 && a.block != 64 && a.block != 128) return TASFT_ERR_UNSUPPORTED;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (!a.force_simt) {
    const int rc = prefill_tc(a, st);
    if (rc != TASFT_ERR_UNSUPPORTED) return rc;
  }
  return prefill_simt(a, st);
}

extern "C" int tasft_bsa_prefill_varlen_fwd(const tasft_prefill_varlen_args* vp, tasft_stream_t stream) {
  if (!vp || !vp->cu_seqlens) return TASFT_ERR_INVALID_ARG;
  const tasft_prefill_args& a = vp->base;
  if (!a.q || !a.k || !a.v || !a.out || !a.kept_idx || !a.kept_cnt) return TASFT_ERR_INVALID_ARG;
  if (a.B <= 0 || a.Hq <= 0 || a.Hk <= 0 || a.S <= 0 || a.D <= 0 || a.Hm <= 0 || vp->total <= 0)
    return TASFT_ERR_INVALID_ARG;
  if (a.Hq % a.Hk != 0 || a.Hq % a.Hm != 0) return TASFT_ERR_INVALID_ARG;
  if (a.q_stride[3] != 1 || a.k_stride[3] != 1 || a.v_stride[3] != 1 || a.o_stride[3] != 1)
    return TASFT_ERR_INVALID_ARG;
  if (a.block != 32 && a.block != 64 && a.block != 128) return TASFT_ERR_UNSUPPORTED;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (!a.force_simt) {
    const int rc = prefill_tc(a, st, vp->cu_seqlens, vp->total);
    if (rc != TASFT_ERR_UNSUPPORTED) return rc;
  }
  return prefill_simt(a, st, vp->cu_seqlens);
}

extern "C" const char* tasft_status_string(int status) {
  switch (status) {
    case TASFT_OK: return "ok";
    case TASFT_ERR_INVALID_ARG: return "invalid argument";
    case TASFT_ERR_UNSUPPORTED: return "unsupported dtype, head_dim or block size";
    case TASFT_ERR_CUDA: return "CUDA runtime error";
    case TASFT_ERR_WORKSPACE: return "workspace missing or too small";
    case TASFT_ERR_TOO_LARGE: return "size exceeds a fixed capacity";
    default: return "unknown status";
  }
}

extern "C" int tasft_abi_version(void) { return TASFT_ABI_VERSION; }

extern "C" int64_t tasft_launch_count(void) { return g_launches.load(); }
