// Shared pieces of the two decode kernels: split-KV workspace and the per-unit finish
// (direct output for one split; otherwise partial + atomic ticket, and the last split to
// finish merges all partials -- no CTA ever waits on another).
#pragma once

#include "common.cuh"

namespace tasft {

struct DecodeWs {
  float* part;      // [B*Hq, nsplit, D + 2]  (normalised o, m (base e), l)
  int32_t* ticket;  // [B*Hk] + 2 work counters, cleared by the host before each split call
  int max_splits;
};

__device__ __forceinline__ void named_bar(int id, int n) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

// res: shared [grp][D + 2] = (o / l, m, l) of this CTA for each q-head of the group.
// Executed by `nthr` threads (tid in [0, nthr)) that share named barrier `bar_id`.
template <typename T>
__device__ void decode_finish(const tasft_decode_args& a, const DecodeWs& ws, int nsplit, int split, int unit, int b,
                              int hk, int grp, const float* res, int tid, int nthr, int bar_id, int* s_last) {
  const int D = a.D;
  if (nsplit == 1) {
    for (int x = tid; x < grp * D; x += nthr) {
      const int g = x / D, d = x % D;
      const int hq = hk * grp + g;
      const float o = res[g * (D + 2) + d];
      if (a.out) reinterpret_cast<T*>(a.out)[b * a.o_stride[0] + hq * a.o_stride[1] + d] = from_f<T>(o);
      const int64_t row = (int64_t)b * a.Hq + hq;
      if (a.part_o) a.part_o[row * D + d] = o;
      if (a.part_ml && d == 0) {
        a.part_ml[row * 2] = res[g * (D + 2) + D];
        a.part_ml[row * 2 + 1] = res[g * (D + 2) + D + 1];
      }
    }
    return;
  }
  for (int x = tid; x < grp * (D + 2); x += nthr) {
    const int g = x / (D + 2), d = x % (D + 2);
    const int64_t row = (int64_t)b * a.Hq + hk * grp + g;
    ws.part[(row * ws.max_splits + split) * (D + 2) + d] = res[g * (D + 2) + d];
  }
  __threadfence();
  named_bar(bar_id, nthr);
  if (tid == 0) {
    const int prev = atomicAdd(&ws.ticket[unit], 1);
    const int last = prev == nsplit - 1;
    if (last) ws.ticket[unit] = 0;  // ready for the next call
    *s_last = last;
  }
  named_bar(bar_id, nthr);
  if (!*s_last) return;
  __threadfence();
  for (int x = tid; x < grp * D; x += nthr) {
    const int g = x / D, d = x % D;
    const int64_t row = (int64_t)b * a.Hq + hk * grp + g;
    const float* pr = ws.part + row * ws.max_splits * (D + 2);
    float mt = -INFINITY;
    for (int sp = 0; sp < nsplit; ++sp) {
      if (__ldcg(pr + sp * (D + 2) + D + 1) > 0.f) mt = fmaxf(mt, __ldcg(pr + sp * (D + 2) + D));
    }
    float num = 0.f, den = 0.f;
    for (int sp = 0; sp < nsplit; ++sp) {
      const float l = __ldcg(pr + sp * (D + 2) + D + 1);
      if (l > 0.f) {
        const float w = l * __expf(__ldcg(pr + sp * (D + 2) + D) - mt);
        num = fmaf(w, __ldcg(pr + sp * (D + 2) + d), num);
        den += w;
      }
    }
    const float o = den > 0.f ? num / den : 0.f;
    const int hq = hk * grp + g;
    if (a.out) reinterpret_cast<T*>(a.out)[b * a.o_stride[0] + hq * a.o_stride[1] + d] = from_f<T>(o);
    if (a.part_o) a.part_o[row * D + d] = o;
    if (a.part_ml && d == 0) {
      a.part_ml[row * 2] = mt;
      a.part_ml[row * 2 + 1] = den;
    }
  }
}

// whether the tensor-core decode takes these arguments (bf16/f16, block 64, D 64/128, group <= 8)
bool decode_mma_ok(const tasft_decode_args& a);
// Cross-GPU exchange done by the wide-split merge kernel (world == 0: off)
struct PeerMode {
  void* const* mailboxes;
  uint32_t* epoch;
  int world, rank;
  uint64_t timeout_ns;
};
int decode_mma(const tasft_decode_args& a, const DecodeWs& ws, int nsplit, cudaStream_t st,
               const PeerMode& pm = PeerMode{nullptr, nullptr, 0, 0, 0});
// Paged-cache variant (k_cache / v_cache are page pools, see tasft_bsa_decode_paged_fwd).
int decode_mma_paged(const tasft_decode_args& a, const DecodeWs& ws, int nsplit, const int32_t* table, int max_pages,
                     int page_size, int num_pages, cudaStream_t st);

}  // namespace tasft
