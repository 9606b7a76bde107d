// Block-sparse causal GQA prefill on the 5th-generation tensor cores (sm_100a).
//
// Same contract as the reference kernel (tasft/kernels/block_sparse_fa.py:108-269,
// launched at :454-552): per q-block, visit the kept k-blocks in ascending order with
// an fp32 online softmax, p cast to the value dtype before P.V, rows with nothing kept
// give 0. Only the data movement and the arithmetic engine differ.
//
// CTA = one 128-row M tile made of two 64-row "slots" that share one kv-head:
//   GQA (Hq/Hk >= 2): two q-heads of the group at the same q-block;
//   MHA (Hq/Hk == 1): one head at two consecutive q-blocks.
// The CTA walks the union of the two slots' kept lists; a per-entry 2-bit mask says
// which slot keeps the block (the other slot's rows get p = 0). With lists at kv-head
// granularity both slots keep the same blocks and nothing is wasted.
//
// Warp roles (192 threads, 2 CTAs per SM):
//   warp 0     TMA producer: Q once, then K and V tiles of each kept block (2-stage ring)
//   warp 1     MMA issuer:   S = Q K^T (SS, M128 N64) into a double-buffered TMEM tile,
//                            O += P V (TS: P read from TMEM where it overwrote S)
//   warps 2-5  softmax:      one thread per row; tcgen05.ld S, mask, online max with a
//                            lazy O rescale (only when the max grows by > 2^8), p = 2^x,
//                            tcgen05.st P (bf16) back into TMEM, epilogue O / l.
// Every mbarrier wait is bounded (TASFT_DEVERR_TIMEOUT) so a broken pipeline returns.
#include "tc.cuh"

namespace tasft {

namespace {

constexpr int kThreads = 192;
constexpr int kBlk = 64;           // block size (tokens) handled by this kernel
constexpr int kMaxNB = 1024;       // max blocks per sequence (S <= 65536)
constexpr uint32_t kTmemCols = 256;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescaleThreshold = 8.0f;  // log2 units

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <int D>
struct Smem {
  static constexpr int kChunks = D / 64;                  // 64-element (128 B) swizzle atoms along D
  static constexpr int kQBytes = kChunks * 128 * 128;     // 128 rows x 128 B per chunk
  static constexpr int kKVTileBytes = kChunks * 64 * 128; // 64 rows x 128 B per chunk
  static constexpr int kStageBytes = 2 * kKVTileBytes;    // K + V
  static constexpr int kQOff = 0;
  static constexpr int kStageOff = kQOff + kQBytes;
  static constexpr int kListOff = kStageOff + 2 * kStageBytes;
  static constexpr int kBitmapOff = kListOff + kMaxNB * 4;
  static constexpr int kBarOff = kBitmapOff + 2 * (kMaxNB / 32) * 4;
  static constexpr int kNumBars = 11;
  static constexpr int kMiscOff = kBarOff + kNumBars * 8;
  static constexpr int kBytes = kMiscOff + 16;
  static constexpr int kAlloc = kBytes + 1024;  // slack for 1024-byte alignment
};

struct Work {
  int b, hk, head[2], qbs[2];
  bool valid[2];
};

__device__ __forceinline__ Work decode_work(const tasft_prefill_args& a, int NB) {
  const int grp = a.Hq / a.Hk;
  const int pairs = grp >= 2 ? (grp + 1) / 2 : 1;
  const int nbp = grp >= 2 ? NB : (NB + 1) / 2;
  const int inner = a.B * a.Hk * pairs;
  const int id = blockIdx.x;
  const int qbo = id / inner;
  const int rem = id % inner;
  const int p = rem % pairs;
  Work w;
  w.hk = (rem / pairs) % a.Hk;
  w.b = rem / (pairs * a.Hk);
  const int qslot = nbp - 1 - qbo;  // heavy (late) q-blocks first
  for (int s = 0; s < 2; ++s) {
    if (grp >= 2) {
      w.head[s] = w.hk * grp + 2 * p + s;
      w.qbs[s] = qslot;
      w.valid[s] = (2 * p + s) < grp;
    } else {
      w.head[s] = w.hk;
      w.qbs[s] = 2 * qslot + s;
      w.valid[s] = w.qbs[s] < NB;
    }
  }
  return w;
}

template <int D, bool kF16>
__global__ void __launch_bounds__(kThreads, 2)
    bsa_prefill_tc_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
                          const __grid_constant__ CUtensorMap tmv, const tasft_prefill_args a, const int NB) {
  using L = Smem<D>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint8_t* sQ = smem + L::kQOff;
  int32_t* list = reinterpret_cast<int32_t*>(smem + L::kListOff);
  uint32_t* bitmap = reinterpret_cast<uint32_t*>(smem + L::kBitmapOff);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* bar_q = bars + 0;
  uint64_t* kv_full = bars + 1;   // [2]
  uint64_t* kv_empty = bars + 3;  // [2]
  uint64_t* s_full = bars + 5;    // [2]
  uint64_t* p_ready = bars + 7;   // [2]
  uint64_t* pv_done = bars + 9;
  // Single-use barrier for the epilogue. pv_done cannot serve: when the softmax warps
  // finish the last block, P.V of block n-2 may still run, and a parity wait cannot tell
  // "phase n-2 pending" from "phase n-1 done".
  uint64_t* o_final = bars + 10;
  uint32_t* misc = reinterpret_cast<uint32_t*>(smem + L::kMiscOff);  // [0] tmem base, [1] list length, [2] abort

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const Work w = decode_work(a, NB);
  const int words = (NB + 31) / 32;

  // ---------------- setup ----------------
  if (warp == 0 && lane == 0) {
    mbar_init(bar_q, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_ready[i], 128);
    }
    mbar_init(pv_done, 1);
    mbar_init(o_final, 1);
    fence_barrier_init();
    misc[2] = 0;
  }
  if (warp == 1) {
    tc::tmem_alloc(&misc[0], kTmemCols);
    tc::tmem_relinquish();
  }
  for (int i = threadIdx.x; i < 2 * words; i += kThreads) bitmap[i] = 0;
  __syncthreads();
  // union of the two slots' kept lists as bitmaps
  const int grp_m = a.Hq / a.Hm;
  for (int s = 0; s < 2; ++s) {
    if (!w.valid[s]) continue;
    const int hm = w.head[s] / grp_m;
    const int64_t lrow = ((int64_t)w.b * a.Hm + hm) * NB + w.qbs[s];
    const int cnt = min(a.kept_cnt[lrow], NB);
    const int32_t* idx = a.kept_idx + lrow * NB;
    for (int t = threadIdx.x; t < cnt; t += kThreads) {
      const int kb = idx[t];
      if (kb < 0 || kb >= NB) {
        set_err(a.err, TASFT_DEVERR_INDEX);
        continue;
      }
      if (a.causal && kb > w.qbs[s]) continue;
      atomicOr(&bitmap[s * words + (kb >> 5)], 1u << (kb & 31));
    }
  }
  __syncthreads();
  if (warp == 0) {
    int n = 0;
    for (int wd = 0; wd < words; ++wd) {
      const uint32_t m0 = bitmap[wd], m1 = bitmap[words + wd];
      const uint32_t bit = 1u << lane;
      const bool any = ((m0 | m1) & bit) != 0;
      const unsigned bal = __ballot_sync(0xffffffffu, any);
      if (any) {
        const int pos = n + __popc(bal & (bit - 1u));
        const int slots = ((m0 & bit) ? 1 : 0) | ((m1 & bit) ? 2 : 0);
        list[pos] = (wd * 32 + lane) | (slots << 16);
      }
      n += __popc(bal);
    }
    if (lane == 0) misc[1] = n;
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = misc[0];
  const int n = misc[1];
  const uint32_t tS0 = tmem;            // S buffers: columns [0,64) and [64,128)
  const uint32_t tO = tmem + 128;       // O: columns [128, 128 + D)

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      tc::prefetch_tmap(&tmq);
      tc::prefetch_tmap(&tmk);
      tc::prefetch_tmap(&tmv);
      const int nvalid = (w.valid[0] ? 1 : 0) + (w.valid[1] ? 1 : 0);
      mbar_arrive_expect_tx(bar_q, nvalid * L::kChunks * 64 * 128);
      for (int s = 0; s < 2; ++s) {
        if (!w.valid[s]) continue;
        for (int c = 0; c < L::kChunks; ++c)
          tc::tma_load_4d(sQ + c * 128 * 128 + s * 64 * 128, &tmq, c * 64, w.qbs[s] * kBlk, w.head[s], w.b, bar_q);
      }
      int issued = 0;
      for (int j = 0; j < n; ++j) {
        const int st = j & 1;
        if (j >= 2 && !mbar_wait(&kv_empty[st], ((j >> 1) - 1) & 1)) {
          set_err(a.err, TASFT_DEVERR_TIMEOUT);
          break;
        }
        const int kb = list[j] & 0xffff;
        uint8_t* sK = smem + L::kStageOff + st * L::kStageBytes;
        uint8_t* sV = sK + L::kKVTileBytes;
        mbar_arrive_expect_tx(&kv_full[st], L::kStageBytes);
        for (int c = 0; c < L::kChunks; ++c) {
          tc::tma_load_4d(sK + c * 64 * 128, &tmk, c * 64, kb * kBlk, w.hk, w.b, &kv_full[st]);
          tc::tma_load_4d(sV + c * 64 * 128, &tmv, c * 64, kb * kBlk, w.hk, w.b, &kv_full[st]);
        }
        ++issued;
      }
      // do not leave the CTA while copies into its shared memory are in flight
      mbar_wait(bar_q, 0);
      for (int j = max(0, issued - 2); j < issued; ++j) mbar_wait(&kv_full[j & 1], (j >> 1) & 1);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t fmt = kF16 ? 0u : 1u;
      constexpr uint32_t idesc_s = tc::make_idesc(128, 64, fmt, false);
      constexpr uint32_t idesc_o = tc::make_idesc(128, D, fmt, true);
      const uint32_t q_addr = smem_u32(sQ);
      bool ok = mbar_wait(bar_q, 0);
      auto issue_s = [&](int j) {
        const int st = j & 1;
        const uint32_t k_addr = smem_u32(smem + L::kStageOff + st * L::kStageBytes);
        const uint32_t dst = tS0 + st * 64;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint64_t ad = tc::make_sdesc(q_addr + (kk >> 2) * 128 * 128 + (kk & 3) * 32, 16, 1024);
          const uint64_t bd = tc::make_sdesc(k_addr + (kk >> 2) * 64 * 128 + (kk & 3) * 32, 16, 1024);
          tc::mma_ss(dst, ad, bd, idesc_s, kk > 0 ? 1u : 0u);
        }
        tc::mma_commit(&s_full[st]);
      };
      if (ok && n > 0) {
        ok = mbar_wait(&kv_full[0], 0);
        if (ok) {
          tc::tc_fence_after();
          issue_s(0);
        }
      }
      for (int j = 0; ok && j < n; ++j) {
        if (j + 1 < n) {
          ok = mbar_wait(&kv_full[(j + 1) & 1], ((j + 1) >> 1) & 1);
          if (ok && j >= 1) ok = mbar_wait(pv_done, (j - 1) & 1);
          if (!ok) break;
          tc::tc_fence_after();
          issue_s(j + 1);
        }
        ok = mbar_wait(&p_ready[j & 1], (j >> 1) & 1);
        if (!ok) break;
        tc::tc_fence_after();
        const uint32_t v_addr = smem_u32(smem + L::kStageOff + (j & 1) * L::kStageBytes + L::kKVTileBytes);
        const uint32_t p_tmem = tS0 + (j & 1) * 64;
#pragma unroll
        for (int kk = 0; kk < kBlk / 16; ++kk) {
          const uint64_t bd = tc::make_sdesc(v_addr + kk * 16 * 128, 64 * 128, 1024);
          tc::mma_ts(tO, p_tmem + kk * 8, bd, idesc_o, (j > 0 || kk > 0) ? 1u : 0u);
        }
        tc::mma_commit(&kv_empty[j & 1]);
        tc::mma_commit(pv_done);
        if (j == n - 1) tc::mma_commit(o_final);
      }
      if (!ok) {
        set_err(a.err, TASFT_DEVERR_TIMEOUT);
        atomicExch(&misc[2], 1u);
      }
    }
  } else {
    // ---------------- softmax + epilogue (warps 2..5) ----------------
    const int quarter = warp & 3;            // TMEM lanes [32*quarter, 32*quarter + 32)
    const int r = quarter * 32 + lane;       // tile row
    const int slot = r >> 6;
    const int qpos = w.qbs[slot] * kBlk + (r & 63);
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const float sl2 = a.scale * kLog2e;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < n; ++j) {
      if (!__all_sync(0xffffffffu, mbar_wait(&s_full[j & 1], (j >> 1) & 1))) { ok = false; break; }
      tc::tc_fence_after();
      const int entry = list[j];
      const int kb = entry & 0xffff;
      const bool active = w.valid[slot] && ((entry >> (16 + slot)) & 1);
      uint32_t sraw[64];
      tc::tmem_ld64_sync(tS0 + (j & 1) * 64 + lane_off, sraw);
      const int kbase = kb * kBlk;
      // keys valid for this row: < S, and <= qpos when causal
      int lim = a.S - kbase;
      if (a.causal) lim = min(lim, qpos - kbase + 1);
      if (!active) lim = 0;
      lim = max(0, min(lim, kBlk));
      float x[64];
      float mb = -INFINITY;
#pragma unroll
      for (int c = 0; c < 64; ++c) {
        x[c] = __uint_as_float(sraw[c]) * sl2;
        if (c < lim) mb = fmaxf(mb, x[c]);
      }
      const float m_new = fmaxf(m, mb);
      bool need = (m != -INFINITY) && (m_new > m + kRescaleThreshold);
      if (m == -INFINITY) m = m_new;  // O row is still exactly zero: no rescale
      const bool warp_need = __any_sync(0xffffffffu, need);
      if (warp_need) {
        // O must hold every earlier P.V before it is rescaled
        if (!__all_sync(0xffffffffu, mbar_wait(pv_done, (j - 1) & 1))) { ok = false; break; }
        tc::tc_fence_after();
        const float alpha = need ? ex2(m - m_new) : 1.0f;
        for (int c0 = 0; c0 < D; c0 += 32) {
          uint32_t o[32];
          tc::tmem_ld32_sync(tO + c0 + lane_off, o);
#pragma unroll
          for (int c = 0; c < 32; ++c) o[c] = __float_as_uint(__uint_as_float(o[c]) * alpha);
          tc::tmem_st32(tO + c0 + lane_off, o);
        }
        tc::tmem_wait_st();
        if (need) {
          l *= alpha;
          m = m_new;
        }
      }
      uint32_t pk[32];
      float rs = 0.f;
#pragma unroll
      for (int c = 0; c < 32; ++c) {
        const float p0 = (2 * c < lim) ? ex2(x[2 * c] - m) : 0.f;
        const float p1 = (2 * c + 1 < lim) ? ex2(x[2 * c + 1] - m) : 0.f;
        rs += p0 + p1;
        pk[c] = kF16 ? tc::pack_f16x2(p0, p1) : tc::pack_bf16x2(p0, p1);
      }
      l += rs;
      tc::tmem_st32(tS0 + (j & 1) * 64 + lane_off, pk);
      tc::tmem_wait_st();
      tc::tc_fence_before();
      mbar_arrive(&p_ready[j & 1]);
    }
    if (ok && n > 0) {
      ok = __all_sync(0xffffffffu, mbar_wait(o_final, 0));
      tc::tc_fence_after();
    }
    if (!ok) set_err(a.err, TASFT_DEVERR_TIMEOUT);
    // epilogue: O / l -> global (rows >= S and invalid slots are not stored)
    const bool store = w.valid[slot] && qpos < a.S;
    using T = typename std::conditional<kF16, __half, __nv_bfloat16>::type;
    T* orow = reinterpret_cast<T*>(a.out) + w.b * a.o_stride[0] + (int64_t)w.head[slot] * a.o_stride[1] +
              (int64_t)qpos * a.o_stride[2];
    const float inv = (l > 0.f) ? 1.0f / l : 0.f;
    for (int c0 = 0; c0 < D; c0 += 32) {
      uint32_t o[32];
      if (n > 0) {
        tc::tmem_ld32_sync(tO + c0 + lane_off, o);
      } else {
#pragma unroll
        for (int c = 0; c < 32; ++c) o[c] = 0u;
      }
      if (store) {
        uint32_t pk[16];
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          const float v0 = ok ? __uint_as_float(o[2 * c]) * inv : 0.f;
          const float v1 = ok ? __uint_as_float(o[2 * c + 1]) * inv : 0.f;
          pk[c] = kF16 ? tc::pack_f16x2(v0, v1) : tc::pack_bf16x2(v0, v1);
        }
        uint4* dst = reinterpret_cast<uint4*>(orow + c0);
#pragma unroll
        for (int v = 0; v < 4; ++v) dst[v] = make_uint4(pk[4 * v], pk[4 * v + 1], pk[4 * v + 2], pk[4 * v + 3]);
      }
    }
  }
  // ---------------- teardown ----------------
  __syncwarp();
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, kTmemCols);
  }
}

template <int D, bool kF16>
int launch_tc(const tasft_prefill_args& a, cudaStream_t st) {
  const int es = 2;
  const int NB = (a.S + kBlk - 1) / kBlk;
  CUtensorMap mq, mk, mv;
  if (!make_tmap_bhsd(&mq, a.q, a.B, a.Hq, a.S, D, a.q_stride, es, 64)) return TASFT_ERR_UNSUPPORTED;
  if (!make_tmap_bhsd(&mk, a.k, a.B, a.Hk, a.S, D, a.k_stride, es, 64)) return TASFT_ERR_UNSUPPORTED;
  if (!make_tmap_bhsd(&mv, a.v, a.B, a.Hk, a.S, D, a.v_stride, es, 64)) return TASFT_ERR_UNSUPPORTED;
  const int grp = a.Hq / a.Hk;
  const int pairs = grp >= 2 ? (grp + 1) / 2 : 1;
  const int nbp = grp >= 2 ? NB : (NB + 1) / 2;
  const int64_t grid = (int64_t)a.B * a.Hk * pairs * nbp;
  auto kern = bsa_prefill_tc_kernel<D, kF16>;
  const int smem = Smem<D>::kAlloc;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return TASFT_ERR_CUDA;
  kern<<<(unsigned)grid, kThreads, smem, st>>>(mq, mk, mv, a, NB);
  count_launch();
  return launch_status();
}

}  // namespace

int prefill_tc(const tasft_prefill_args& a, cudaStream_t st) {
  if (a.block != kBlk) return TASFT_ERR_UNSUPPORTED;
  if (a.dtype != TASFT_BF16 && a.dtype != TASFT_F16) return TASFT_ERR_UNSUPPORTED;
  if (a.D != 64 && a.D != 128) return TASFT_ERR_UNSUPPORTED;
  const int NB = (a.S + kBlk - 1) / kBlk;
  if (NB > kMaxNB) return TASFT_ERR_UNSUPPORTED;
  // vectorised epilogue stores: 16-byte aligned rows
  if (!aligned16(a.out) || (a.o_stride[0] % 8) || (a.o_stride[1] % 8) || (a.o_stride[2] % 8))
    return TASFT_ERR_UNSUPPORTED;
  const bool f16 = a.dtype == TASFT_F16;
  if (a.D == 128) return f16 ? launch_tc<128, true>(a, st) : launch_tc<128, false>(a, st);
  return f16 ? launch_tc<64, true>(a, st) : launch_tc<64, false>(a, st);
}

}  // namespace tasft
