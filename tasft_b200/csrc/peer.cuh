// Layout of a rank's peer mailbox and the flag operations shared by the peer-memory merge
// (peer.cu) and the split decode whose merge kernel exchanges directly (decode_mma.cu).
//
//   [call flags: world uint32, then the per-call CTA counter at index world; 256-B padded]
//   [row words: 2 parity x world x rows x (D + 2) uint64, each (fp32 value bits | epoch << 32):
//    normalised o, then m (base e), l; written by tasft_bsa_decode_peer_fwd]
//   [partials: 2 parity x world x rows x (D + 2) fp32, written by tasft_peer_combine]
// A call's epoch e = (*epoch) + 1 selects parity e & 1 and is the value of the flags. A row
// word carries its own epoch, so one 8-byte store publishes a value: the reader spins on the
// word itself and needs no fence or separate flag.
#pragma once

#include "common.cuh"

namespace tasft {

__host__ __device__ inline int64_t peer_flags_bytes(int world) { return ((int64_t)(world + 1) * 4 + 255) / 256 * 256; }
// uint64 offset of the row words
__host__ __device__ inline int64_t peer_word_off(int world) { return peer_flags_bytes(world) / 8; }
__host__ __device__ inline int64_t peer_words_bytes(int world, int64_t rows, int D) {
  return (int64_t)2 * world * rows * (D + 2) * 8;
}
// float offset of the partials
__host__ __device__ inline int64_t peer_part_off(int world, int64_t rows, int D) {
  return (peer_flags_bytes(world) + peer_words_bytes(world, rows, D)) / 4;
}
__host__ __device__ inline int64_t peer_mailbox_bytes(int world, int64_t rows, int D) {
  return peer_part_off(world, rows, D) * 4 + (int64_t)2 * world * rows * (D + 2) * 4;
}

__device__ __forceinline__ void st_relaxed_sys_u64(uint64_t* p, uint64_t v) {
  asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_relaxed_sys_u64(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
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
