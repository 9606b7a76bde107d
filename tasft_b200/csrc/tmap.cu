// Host-side TMA tensor-map construction (driver entry point fetched through the runtime,
// so the library needs no link-time dependency on libcuda).
#include <cudaTypedefs.h>
#include <mutex>

#include "tc.cuh"

namespace tasft {

static PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

bool make_tmap_bhsd(CUtensorMap* map, const void* base, int B, int H, int S, int D, const int64_t* st, int elem_bytes,
                    int box_rows) {
  auto fn = get_encode();
  if (!fn) return false;
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0) return false;
  if (st[3] != 1) return false;
  for (int i = 0; i < 3; ++i)
    if ((st[i] * elem_bytes) % 16 != 0 || st[i] <= 0) return false;
  if (D % 64 != 0) return false;
  cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)S, (cuuint64_t)H, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)(st[2] * elem_bytes), (cuuint64_t)(st[1] * elem_bytes),
                           (cuuint64_t)(st[0] * elem_bytes)};
  cuuint32_t box[4] = {64, (cuuint32_t)box_rows, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUtensorMapDataType dt = elem_bytes == 2 ? CU_TENSOR_MAP_DATA_TYPE_UINT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  const CUresult r = fn(map, dt, 4, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS && debug_enabled()) debug_log("cuTensorMapEncodeTiled failed: %d", (int)r);
  return r == CUDA_SUCCESS;
}

bool make_tmap_paged(CUtensorMap* map, const void* base, int pages, int page_size, int H, int D, const int64_t* st,
                     int box_rows) {
  auto fn = get_encode();
  if (!fn) return false;
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0) return false;
  if (st[3] != 1 || D % 64 != 0) return false;
  for (int i = 0; i < 3; ++i)
    if ((st[i] * 2) % 16 != 0 || st[i] <= 0) return false;
  cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)H, (cuuint64_t)page_size, (cuuint64_t)pages};
  cuuint64_t strides[3] = {(cuuint64_t)(st[2] * 2), (cuuint64_t)(st[1] * 2), (cuuint64_t)(st[0] * 2)};
  cuuint32_t box[4] = {64, 1, (cuuint32_t)box_rows, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 4, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS && debug_enabled()) debug_log("cuTensorMapEncodeTiled (paged) failed: %d", (int)r);
  return r == CUDA_SUCCESS;
}

}  // namespace tasft
