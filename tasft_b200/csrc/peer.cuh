// Layout of a rank's peer mailbox and the flag operations shared by the peer-memory merge
// (peer.cu) and the split decode whose merge kernel exchanges directly (decode_mma.cu).
//
//   [call flags: world uint32, then the per-call CTA counter at index world; 256-B padded]
//   [row flags: world x rows uint32, 256-B padded]
//   [partials: 2 parity x world x rows x (D + 2) fp32: normalised o, then m (base e), l]
// A call's epoch e = (*epoch) + 1 selects parity e & 1 and is the value written to the flags.
#pragma once

#include "common.cuh"

namespace tasft {

__host__ __device__ inline int64_t peer_flags_bytes(int world) { return ((int64_t)(world + 1) * 4 + 255) / 256 * 256; }
__host__ __device__ inline int64_t peer_rowflags_bytes(int world, int64_t rows) {
  return ((int64_t)world * rows * 4 + 255) / 256 * 256;
}
// float offset of the partials
__host__ __device__ inline int64_t peer_part_off(int world, int64_t rows) {
  return (peer_flags_bytes(world) + peer_rowflags_bytes(world, rows)) / 4;
}
__host__ __device__ inline int64_t peer_mailbox_bytes(int world, int64_t rows, int D) {
  return peer_part_off(world, rows) * 4 + (int64_t)2 * world * rows * (D + 2) * 4;
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

}  // namespace tasft
