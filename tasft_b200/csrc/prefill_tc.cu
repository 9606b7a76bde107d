// Block-sparse causal GQA prefill on the 5th-generation tensor cores (sm_100a).
//
// Same contract as the reference kernel (tasft/kernels/block_sparse_fa.py:108-269,
// launched at :454-552): per q-block, visit the kept k-blocks in ascending order with
// an fp32 online softmax, p cast to the value dtype before P.V, rows with nothing kept
// give 0. Only the data movement and the arithmetic engine differ.
//
// Tile = one 128-row M tile made of two 64-row "slots" that share one kv-head:
//   GQA (Hq/Hk >= 2): two q-heads of the group at the same q-block;
//   MHA (Hq/Hk == 1): one head at two consecutive q-blocks.
// A tile walks the union of its two slots' kept lists; a per-entry 2-bit mask says
// which slot keeps the block (the other slot's rows get p = 0). With lists at kv-head
// granularity both slots keep the same blocks and nothing is wasted.
//
// Persistent CTAs (2 per SM, 192 threads) take tiles in a static stride over a
// heavy-first order. Warp roles:
//   warp 0     producer: builds the next tile's union list (double-buffered), loads Q
//              once the previous tile's last S = Q K^T has run, and streams K and V tiles
//              of every kept block through separate 2-stage rings (TMA, 128B swizzle)
//   warp 1     MMA issuer: S = Q K^T (SS, M128 N64) into a double-buffered TMEM tile,
//              O += P V (TS: P read from TMEM where it overwrote S)
//   warps 2-5  softmax: one thread per row; tcgen05.ld S, mask, online max with a lazy
//              O rescale (only when the max grows by > 2^8), p = 2^x, tcgen05.st P (bf16)
//              back into TMEM, epilogue O / l, which overlaps the next tile's loads.
// Packed sequences (cu_seqlens, the vLLM prefill layout) use the same kernel: the tensors
// are one [1, H, total, D] map, every row coordinate is offset by its sequence's start,
// and keys and stores are bounded by the sequence's own length.
// Every mbarrier phase is indexed by a global block counter or by the CTA's tile counter,
// and every wait is arranged so the waiter is at most one phase behind (a parity wait
// cannot tell phase k from phase k + 2). Every wait is bounded (TASFT_DEVERR_TIMEOUT).
#include <cstdlib>

#include "tc.cuh"

namespace tasft {

namespace {

constexpr int kThreads = 192;
constexpr int kBlk = 64;           // block size (tokens) handled by this kernel
constexpr int kMaxNB = 1024;       // max blocks per sequence (S <= 65536)
constexpr int kWords = kMaxNB / 32;
constexpr uint32_t kTmemCols = 256;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescaleThreshold = 8.0f;  // log2 units

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// ---- packed fp32 pair helpers (Blackwell f32x2 instructions) ----
__device__ __forceinline__ uint64_t f2(float lo, float hi) {
  return ((uint64_t)__float_as_uint(hi) << 32) | __float_as_uint(lo);
}
__device__ __forceinline__ float lo_f(uint64_t v) { return __uint_as_float((uint32_t)v); }
__device__ __forceinline__ float hi_f(uint64_t v) { return __uint_as_float((uint32_t)(v >> 32)); }
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}


struct Work {
  int b, hk, head[2], qbs[2];
  int valid[2];
  int n;     // union list length; -1 = no more tiles
  int len;   // tokens of sequence b (S, or its cu_seqlens length when packed)
  int row0;  // row of its first token in the K/V/Q/O tensors (0, or cu_seqlens[b] when packed)
};

template <int D>
struct Smem {
  static constexpr int kChunks = D / 64;                  // 64-element (128 B) swizzle atoms along D
  static constexpr int kQBytes = kChunks * 128 * 128;     // 128 rows x 128 B per chunk
  static constexpr int kKVTileBytes = kChunks * 64 * 128; // 64 rows x 128 B per chunk
  // K and V sit in separate 2-stage rings: K(g) is released as soon as S(g) has run,
  // long before P.V(g) releases V(g), so K loads run well ahead of their use.
  static constexpr int kKOff = 0;                          // within the ring area
  static constexpr int kVOff = 2 * kKVTileBytes;
  static constexpr int kQOff = 0;
  static constexpr int kStageOff = kQOff + kQBytes;
  static constexpr int kListOff = kStageOff + 4 * kKVTileBytes;  // [2][kMaxNB] int32
  static constexpr int kBitmapOff = kListOff + 2 * kMaxNB * 4;   // [2 slots][kWords] uint32
  static constexpr int kWorkOff = kBitmapOff + 2 * kWords * 4;   // [2] Work
  static constexpr int kBarOff = (kWorkOff + 2 * (int)sizeof(Work) + 7) / 8 * 8;
  static constexpr int kNumBars = 22;
  static constexpr int kMiscOff = kBarOff + kNumBars * 8;
  static constexpr int kBytes = kMiscOff + 16;
  static constexpr int kAlloc = kBytes + 1024;  // slack for 1024-byte alignment
};

// Tile id -> work. Ids run heavy (late) q-blocks first, over the q-block window [qlo, qhi)
// (all q-blocks unless the caller restricts it). With `cu` (packed sequences of different
// lengths) q-blocks past a sequence's end are marked invalid.
__device__ __forceinline__ Work decode_tile(const tasft_prefill_args& a, const int32_t* cu, int NB, int id, int qlo,
                                            int qhi) {
  const int grp = a.Hq / a.Hk;
  const int pairs = grp >= 2 ? (grp + 1) / 2 : 1;
  // slots: q-blocks (GQA) or pairs of q-blocks (MHA)
  const int slo = grp >= 2 ? qlo : qlo / 2, shi = grp >= 2 ? qhi : (qhi + 1) / 2;
  const int inner = a.B * a.Hk * pairs;
  const int qbo = id / inner;
  const int rem = id % inner;
  const int p = rem % pairs;
  Work w;
  w.hk = (rem / pairs) % a.Hk;
  w.b = rem / (pairs * a.Hk);
  const int qslot = shi - 1 - qbo;
  for (int s = 0; s < 2; ++s) {
    if (grp >= 2) {
      w.head[s] = w.hk * grp + 2 * p + s;
      w.qbs[s] = qslot;
      w.valid[s] = (2 * p + s) < grp;
    } else {
      w.head[s] = w.hk;
      w.qbs[s] = 2 * qslot + s;
      w.valid[s] = w.qbs[s] < NB && w.qbs[s] >= qlo && w.qbs[s] < qhi;
    }
  }
  (void)slo;
  w.n = 0;
  w.len = a.S;
  w.row0 = 0;
  if (cu) {
    w.row0 = cu[w.b];
    w.len = cu[w.b + 1] - w.row0;
    const int nbs = (w.len + kBlk - 1) / kBlk;
    for (int s = 0; s < 2; ++s) w.valid[s] = w.valid[s] && w.qbs[s] < nbs;
  }
  return w;
}

__host__ __device__ __forceinline__ int num_tiles(const tasft_prefill_args& a, int qlo, int qhi) {
  const int grp = a.Hq / a.Hk;
  const int pairs = grp >= 2 ? (grp + 1) / 2 : 1;
  const int nbp = grp >= 2 ? qhi - qlo : (qhi + 1) / 2 - qlo / 2;
  return a.B * a.Hk * pairs * nbp;
}

// Warp-wide bounded wait; every lane gets the same answer.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity) {
  return __all_sync(0xffffffffu, mbar_wait(bar, parity));
}

template <int D, bool kF16>
__global__ void __launch_bounds__(kThreads, 2)
    bsa_prefill_tc_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
                          const __grid_constant__ CUtensorMap tmv, const tasft_prefill_args a, const int NB,
                          const int32_t* cu, float* bmax, const int emulate_bf16, const int wait_pv, const int qlo,
                          const int qhi) {
  using L = Smem<D>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint8_t* sQ = smem + L::kQOff;
  int32_t* lists = reinterpret_cast<int32_t*>(smem + L::kListOff);
  uint32_t* bitmap = reinterpret_cast<uint32_t*>(smem + L::kBitmapOff);
  Work* works = reinterpret_cast<Work*>(smem + L::kWorkOff);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* q_full = bars + 0;      // per tile: Q landed
  uint64_t* q_empty = bars + 1;     // per tile: every S of the tile has run (Q reusable)
  uint64_t* k_full = bars + 2;      // [2] per block
  uint64_t* k_empty = bars + 4;     // [2] per block: S(g) has run
  uint64_t* v_full = bars + 18;     // [2] per block
  uint64_t* v_empty = bars + 20;    // [2] per block: P.V(g) has run
  uint64_t* s_full = bars + 6;      // [2] per block
  uint64_t* p_ready = bars + 8;     // [2] per block (128 arrivals)
  // P.V completion, alternating by block parity: a single barrier could be two phases
  // ahead of a waiter at a tile boundary (P.V of block g-1 in flight while S(g) waits for
  // g-2), which a parity wait cannot see.
  uint64_t* pv_done = bars + 10;    // [2] per block
  uint64_t* o_final = bars + 12;    // per tile: O complete
  uint64_t* o_free = bars + 13;     // per tile: epilogue has read O (128 arrivals)
  uint64_t* list_full = bars + 14;  // [2] per tile
  uint64_t* list_empty = bars + 16; // [2] per tile (128 arrivals)
  uint32_t* misc = reinterpret_cast<uint32_t*>(smem + L::kMiscOff);  // [0] tmem base

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles = num_tiles(a, qlo, qhi);
  const int words = (NB + 31) / 32;

  if (warp == 0 && lane == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_ready[i], 128);
      mbar_init(&list_full[i], 1);
      mbar_init(&list_empty[i], 128);
      mbar_init(&pv_done[i], 1);
    }
    mbar_init(o_final, 1);
    mbar_init(o_free, 128);
    fence_barrier_init();
  }
  if (warp == 1) {
    tc::tmem_alloc(&misc[0], kTmemCols);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = misc[0];
  const uint32_t tS0 = tmem;       // S buffers: columns [0,64) and [64,128)
  const uint32_t tO = tmem + 128;  // O: columns [128, 128 + D)

  if (warp == 0) {
    // ================= producer =================
    if (lane == 0) {
      tc::prefetch_tmap(&tmq);
      tc::prefetch_tmap(&tmk);
      tc::prefetch_tmap(&tmv);
    }
    const int grp_m = a.Hq / a.Hm;
    int gk = 0;  // global block counter (ring position)
    bool ok = true;
    for (int u = 0; ok; ++u) {
      // tiles run heaviest first; the CTA order snakes (0..G-1, then G-1..0, ...) so every
      // CTA's sum of tile sizes comes out about equal
      const int tile = u * gridDim.x + ((u & 1) ? (int)gridDim.x - 1 - (int)blockIdx.x : (int)blockIdx.x);
      const int lb = u & 1;
      if (u >= 2 && !warp_wait(&list_empty[lb], ((u >> 1) - 1) & 1)) {
        set_err(a.err, TASFT_DEVERR_TIMEOUT | (1 << (8 + 1)));
        ok = false;
        break;
      }
      Work w;
      int* list = lists + lb * kMaxNB;
      if (tile >= tiles) {
        w.n = -1;
      } else {
        // ---- union of the two slots' kept lists (warp 0 only) ----
        w = decode_tile(a, cu, NB, tile, qlo, qhi);
        for (int i = lane; i < 2 * words; i += 32) bitmap[(i / words) * kWords + i % words] = 0;
        __syncwarp();
        for (int s = 0; s < 2; ++s) {
          if (!w.valid[s]) continue;
          const int hm = w.head[s] / grp_m;
          const int64_t lrow = ((int64_t)w.b * a.Hm + hm) * NB + w.qbs[s];
          const int cnt = min(a.kept_cnt[lrow], NB);
          const int32_t* idx = a.kept_idx + lrow * NB;
          for (int t = lane; t < cnt; t += 32) {
            const int kb = idx[t];
            if (kb < 0 || kb >= NB) {
              set_err(a.err, TASFT_DEVERR_INDEX);
              continue;
            }
            if (a.causal && kb > w.qbs[s]) continue;
            atomicOr(&bitmap[s * kWords + (kb >> 5)], 1u << (kb & 31));
          }
        }
        __syncwarp();
        int n = 0;
        for (int wd = 0; wd < words; ++wd) {
          const uint32_t m0 = bitmap[wd], m1 = bitmap[kWords + wd];
          const uint32_t bit = 1u << lane;
          const bool any = ((m0 | m1) & bit) != 0;
          const unsigned bal = __ballot_sync(0xffffffffu, any);
          if (any) {
            const int slots = ((m0 & bit) ? 1 : 0) | ((m1 & bit) ? 2 : 0);
            list[n + __popc(bal & (bit - 1u))] = (wd * 32 + lane) | (slots << 16);
          }
          n += __popc(bal);
        }
        w.n = n;
        __syncwarp();
      }
      if (lane == 0) {
        works[lb] = w;
        mbar_arrive(&list_full[lb]);  // release: the list and the work record
      }
      if (w.n < 0) break;
      if (lane == 0) {
        // ---- Q once the previous tile's S MMAs have run ----
        if (u >= 1 && !mbar_wait(q_empty, (u - 1) & 1)) {
          set_err(a.err, TASFT_DEVERR_TIMEOUT | (1 << (8 + 2)));
          ok = false;
        }
        if (ok) {
          // a tile that keeps nothing (e.g. q-blocks outside this rank's range) needs no Q:
          // its phase completes on the arrival alone
          const bool need_q = w.n > 0;
          const int nvalid = need_q ? (w.valid[0] ? 1 : 0) + (w.valid[1] ? 1 : 0) : 0;
          mbar_arrive_expect_tx(q_full, nvalid * L::kChunks * 64 * 128);
          for (int s = 0; s < 2; ++s) {
            if (!w.valid[s] || !need_q) continue;
            for (int c = 0; c < L::kChunks; ++c)
              tc::tma_load_4d(sQ + c * 128 * 128 + s * 64 * 128, &tmq, c * 64, w.row0 + w.qbs[s] * kBlk, w.head[s],
                              cu ? 0 : w.b,
                              q_full);
          }
        }
        // ---- K(j) then V(j-1): the order the MMA warp consumes them ----
        auto load_k = [&](int gi, int kb) -> bool {
          const int st = gi & 1;
          if (gi >= 2 && !mbar_wait(&k_empty[st], ((gi >> 1) - 1) & 1)) return false;
          uint8_t* dst = smem + L::kStageOff + L::kKOff + st * L::kKVTileBytes;
          mbar_arrive_expect_tx(&k_full[st], L::kKVTileBytes);
          for (int c = 0; c < L::kChunks; ++c)
            tc::tma_load_4d(dst + c * 64 * 128, &tmk, c * 64, w.row0 + kb * kBlk, w.hk, cu ? 0 : w.b, &k_full[st]);
          return true;
        };
        auto load_v = [&](int gi, int kb) -> bool {
          const int st = gi & 1;
          if (gi >= 2 && !mbar_wait(&v_empty[st], ((gi >> 1) - 1) & 1)) return false;
          uint8_t* dst = smem + L::kStageOff + L::kVOff + st * L::kKVTileBytes;
          mbar_arrive_expect_tx(&v_full[st], L::kKVTileBytes);
          for (int c = 0; c < L::kChunks; ++c)
            tc::tma_load_4d(dst + c * 64 * 128, &tmv, c * 64, w.row0 + kb * kBlk, w.hk, cu ? 0 : w.b, &v_full[st]);
          return true;
        };
        for (int j = 0; ok && j <= w.n && w.n > 0; ++j) {
          if (j < w.n && !load_k(gk + j, list[j] & 0xffff)) ok = false;
          if (ok && j >= 1 && !load_v(gk + j - 1, list[j - 1] & 0xffff)) ok = false;
        }
        if (!ok) set_err(a.err, TASFT_DEVERR_TIMEOUT | (1 << (8 + 3)));
        if (w.n > 0) gk += w.n;
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      gk = __shfl_sync(0xffffffffu, gk, 0);
    }
    // do not leave while copies into shared memory are in flight
    if (lane == 0) {
      for (int i = max(0, gk - 2); i < gk; ++i) {
        mbar_wait(&k_full[i & 1], (i >> 1) & 1);
        mbar_wait(&v_full[i & 1], (i >> 1) & 1);
      }
    }
  } else if (warp == 1) {
    // ================= MMA issuer =================
    if (lane == 0) {
      constexpr uint32_t fmt = kF16 ? 0u : 1u;
      constexpr uint32_t idesc_s = tc::make_idesc(128, 64, fmt, false);
      constexpr uint32_t idesc_o = tc::make_idesc(128, D, fmt, true);
      const uint32_t q_addr = smem_u32(sQ);
      int g = 0;  // global block counter
      bool ok = true;
      int where = 0;  // wait site that gave up (reported in the error word)
      auto issue_s = [&](int gi) {
        const int st = gi & 1;
        const uint32_t k_addr = smem_u32(smem + L::kStageOff + L::kKOff + st * L::kKVTileBytes);
        const uint32_t dst = tS0 + st * 64;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint64_t ad = tc::make_sdesc(q_addr + (kk >> 2) * 128 * 128 + (kk & 3) * 32, 16, 1024);
          const uint64_t bd = tc::make_sdesc(k_addr + (kk >> 2) * 64 * 128 + (kk & 3) * 32, 16, 1024);
          tc::mma_ss(dst, ad, bd, idesc_s, kk > 0 ? 1u : 0u);
        }
        tc::mma_commit(&s_full[st]);
        tc::mma_commit(&k_empty[st]);
      };
      // S(gi) may overwrite S buffer gi & 1 once P.V of block gi - 2 has run
      auto ready_s = [&](int gi) -> bool {
        if (!mbar_wait(&k_full[gi & 1], (gi >> 1) & 1)) { where = 4; return false; }
        // S(gi) overwrites P(gi - 2) in TMEM. P.V(gi - 2) was issued earlier by this thread, and
        // MMAs issued by one thread run through the tensor pipe in issue order (CUTLASS's sm100
        // FMHA mainloop writes its next Q K^T over the P its last P V reads the same way), so
        // no wait is needed; wait_pv restores the completion wait (a checking aid).
        if (wait_pv && gi >= 2 && !mbar_wait(&pv_done[gi & 1], ((gi - 2) >> 1) & 1)) { where = 5; return false; }
        tc::tc_fence_after();
        return true;
      };
      for (int u = 0; ok; ++u) {
        const int lb = u & 1;
        if (!mbar_wait(&list_full[lb], (u >> 1) & 1)) { where = 6; ok = false; break; }
        const int n = works[lb].n;
        if (n < 0) break;
        if (!mbar_wait(q_full, u & 1)) { where = 7; ok = false; break; }
        tc::tc_fence_after();
        if (n > 0) {
          ok = ready_s(g);
          if (ok) issue_s(g);
        }
        if (n <= 1) tc::mma_commit(q_empty);  // no further S of this tile reads Q
        for (int j = 0; ok && j < n; ++j) {
          const int gi = g + j;
          if (j + 1 < n) {
            ok = ready_s(gi + 1);
            if (!ok) break;
            issue_s(gi + 1);
            if (j + 2 == n) tc::mma_commit(q_empty);
          }
          if (!mbar_wait(&p_ready[gi & 1], (gi >> 1) & 1)) { where = 8; ok = false; break; }
          // O is reused: the previous tile's epilogue must have read it
          if (j == 0 && u >= 1 && !mbar_wait(o_free, (u - 1) & 1)) { where = 9; ok = false; break; }
          if (!mbar_wait(&v_full[gi & 1], (gi >> 1) & 1)) { where = 15; ok = false; break; }
          tc::tc_fence_after();
          const uint32_t v_addr = smem_u32(smem + L::kStageOff + L::kVOff + (gi & 1) * L::kKVTileBytes);
          const uint32_t p_tmem = tS0 + (gi & 1) * 64;
#pragma unroll
          for (int kk = 0; kk < kBlk / 16; ++kk) {
            const uint64_t bd = tc::make_sdesc(v_addr + kk * 16 * 128, 64 * 128, 1024);
            tc::mma_ts(tO, p_tmem + kk * 8, bd, idesc_o, (j > 0 || kk > 0) ? 1u : 0u);
          }
          tc::mma_commit(&v_empty[gi & 1]);
          tc::mma_commit(&pv_done[gi & 1]);
        }
        if (!ok) break;
        if (n == 0 && u >= 1 && !mbar_wait(o_free, (u - 1) & 1)) { where = 10; ok = false; break; }
        tc::mma_commit(o_final);
        g += n;
      }
      if (!ok) set_err(a.err, TASFT_DEVERR_TIMEOUT | (1 << (8 + where)));
    }
  } else {
    // ================= softmax + epilogue (warps 2..5) =================
    const int quarter = warp & 3;            // TMEM lanes [32*quarter, 32*quarter + 32)
    const int r = quarter * 32 + lane;       // tile row
    const int slot = r >> 6;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const float sl2 = a.scale * kLog2e;
    using T = typename std::conditional<kF16, __half, __nv_bfloat16>::type;
    int g = 0;
    bool ok = true;
    int where = 0;
    for (int u = 0; ok; ++u) {
      const int lb = u & 1;
      if (!warp_wait(&list_full[lb], (u >> 1) & 1)) { where = 11; ok = false; break; }
      const Work w = works[lb];
      if (w.n < 0) break;
      const int* list = lists + lb * kMaxNB;
      const int qpos = w.qbs[slot] * kBlk + (r & 63);
      float m = -INFINITY, l = 0.f;
      for (int j = 0; j < w.n; ++j) {
        const int gi = g + j;
        if (!warp_wait(&s_full[gi & 1], (gi >> 1) & 1)) { where = 12; ok = false; break; }
        tc::tc_fence_after();
        const int entry = list[j];
        const int kb = entry & 0xffff;
        const bool active = w.valid[slot] && ((entry >> (16 + slot)) & 1);
        uint32_t sraw[64];
        tc::tmem_ld64_sync(tS0 + (gi & 1) * 64 + lane_off, sraw);
        const int kbase = kb * kBlk;
        // keys valid for this row: inside its sequence, and <= qpos when causal (rows of
        // the next packed sequence that a block overlaps are masked here)
        int lim = w.len - kbase;
        if (a.causal) lim = min(lim, qpos - kbase + 1);
        if (!active) lim = 0;
        lim = max(0, min(lim, kBlk));
        float sv[64];
#pragma unroll
        for (int c = 0; c < 64; ++c) sv[c] = __uint_as_float(sraw[c]);
        if (__any_sync(0xffffffffu, lim < kBlk)) {  // diagonal / ragged / inactive rows
#pragma unroll
          for (int c = 0; c < 64; ++c)
            if (c >= lim) sv[c] = -INFINITY;
        }
        // max of the raw (unscaled) scores, four independent chains; the scale is > 0
        float mq[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
        for (int c = 0; c < 64; c += 8) {
#pragma unroll
          for (int qd = 0; qd < 4; ++qd) mq[qd] = max3(mq[qd], sv[c + 2 * qd], sv[c + 2 * qd + 1]);
        }
        const float mb = max3(mq[0], mq[1], fmaxf(mq[2], mq[3]));
        if (bmax) {
          // training-forward gate target: max of this 64 x 64 tile's scores (masked entries are
          // -inf, as in the reference's triu(-inf) scores); rows of a slot span two warps, whose
          // maxima meet in a float atomic max. Rounded as the reference's bf16 (Q K^T) * scale
          // when asked (monotone rounding commutes with max).
          float wm = warp_max(qpos < w.len ? mb : -INFINITY);  // padding rows past S do not count
          if (lane == 0 && active && wm != -INFINITY) {
            wm = emulate_bf16 ? __bfloat162float(__float2bfloat16_rn(__bfloat162float(__float2bfloat16_rn(wm)) * a.scale))
                              : wm * a.scale;
            float* dst = bmax + (((int64_t)w.b * a.Hq + w.head[slot]) * NB + w.qbs[slot]) * NB + kb;
            if (wm >= 0.f) atomicMax(reinterpret_cast<int*>(dst), __float_as_int(wm));
            else atomicMin(reinterpret_cast<unsigned*>(dst), __float_as_uint(wm));
          }
        }
        const float m_new = fmaxf(m, mb * sl2);
        const bool need = (m != -INFINITY) && (m_new > m + kRescaleThreshold);
        if (m == -INFINITY) m = m_new;  // O row is still exactly zero: no rescale
        if (__any_sync(0xffffffffu, need)) {
          // O must hold every earlier P.V of this tile before it is rescaled
          if (!warp_wait(&pv_done[(gi - 1) & 1], ((gi - 1) >> 1) & 1)) { where = 13; ok = false; break; }
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
        if (m == -INFINITY) {  // nothing valid in this row yet: p = 0
#pragma unroll
          for (int c = 0; c < 32; ++c) pk[c] = 0u;
        } else {
          const uint64_t sc2 = f2(sl2, sl2), nm2 = f2(-m, -m);
          uint64_t rs2 = 0;
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            const uint64_t x2 = fma2(f2(sv[2 * c], sv[2 * c + 1]), sc2, nm2);  // s * scale - m
            // all on MUFU ex2: measured faster than moving part of 2^x to the FMA pipe,
            // which the packed arithmetic around it already keeps busy
            const uint64_t p2 = f2(ex2(lo_f(x2)), ex2(hi_f(x2)));
            rs2 = add2(rs2, p2);
            pk[c] = kF16 ? tc::pack_f16x2(lo_f(p2), hi_f(p2)) : tc::pack_bf16x2(lo_f(p2), hi_f(p2));
          }
          rs = lo_f(rs2) + hi_f(rs2);
        }
        l += rs;
        tc::tmem_st32(tS0 + (gi & 1) * 64 + lane_off, pk);
        tc::tmem_wait_st();
        tc::tc_fence_before();
        mbar_arrive(&p_ready[gi & 1]);
      }
      if (!ok) break;
      if (!warp_wait(o_final, u & 1)) { where = 14; ok = false; break; }
      tc::tc_fence_after();
      // ---- epilogue: O / l -> global (rows >= S and invalid slots are not stored) ----
      const bool store = w.valid[slot] && qpos < w.len;
      T* orow = reinterpret_cast<T*>(a.out) + (cu ? 0 : w.b * a.o_stride[0]) + (int64_t)w.head[slot] * a.o_stride[1] +
                (int64_t)(w.row0 + qpos) * a.o_stride[2];
      const float inv = (l > 0.f) ? 1.0f / l : 0.f;
      for (int c0 = 0; c0 < D; c0 += 32) {
        uint32_t o[32];
        if (w.n > 0) {
          tc::tmem_ld32_sync(tO + c0 + lane_off, o);
        } else {
#pragma unroll
          for (int c = 0; c < 32; ++c) o[c] = 0u;
        }
        if (store) {
          uint32_t pk[16];
#pragma unroll
          for (int c = 0; c < 16; ++c) {
            const float v0 = __uint_as_float(o[2 * c]) * inv;
            const float v1 = __uint_as_float(o[2 * c + 1]) * inv;
            pk[c] = kF16 ? tc::pack_f16x2(v0, v1) : tc::pack_bf16x2(v0, v1);
          }
          uint4* dst = reinterpret_cast<uint4*>(orow + c0);
#pragma unroll
          for (int v = 0; v < 4; ++v) dst[v] = make_uint4(pk[4 * v], pk[4 * v + 1], pk[4 * v + 2], pk[4 * v + 3]);
        }
      }
      tc::tc_fence_before();
      mbar_arrive(o_free);
      mbar_arrive(&list_empty[lb]);
      g += w.n;
    }
    if (!ok) set_err(a.err, TASFT_DEVERR_TIMEOUT | (1 << (8 + where)));
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
int launch_tc(const tasft_prefill_args& a, const int32_t* cu, int total, cudaStream_t st, float* bmax,
              int emulate_bf16) {
  const int es = 2;
  const int NB = (a.S + kBlk - 1) / kBlk;
  // packed sequences: one [1, H, total, D] tensor, rows offset by cu_seqlens in the kernel
  const int mb = cu ? 1 : a.B, ms = cu ? total : a.S;
  CUtensorMap mq, mk, mv;
  if (!make_tmap_bhsd(&mq, a.q, mb, a.Hq, ms, D, a.q_stride, es, 64)) return TASFT_ERR_UNSUPPORTED;
  if (!make_tmap_bhsd(&mk, a.k, mb, a.Hk, ms, D, a.k_stride, es, 64)) return TASFT_ERR_UNSUPPORTED;
  if (!make_tmap_bhsd(&mv, a.v, mb, a.Hk, ms, D, a.v_stride, es, 64)) return TASFT_ERR_UNSUPPORTED;
  // q-block window (qb_hi <= 0: every q-block)
  const int qlo = a.qb_hi > 0 ? a.qb_lo : 0, qhi = a.qb_hi > 0 ? a.qb_hi : NB;
  const int64_t tiles = num_tiles(a, qlo, qhi);
  auto kern = bsa_prefill_tc_kernel<D, kF16>;
  const int smem = Smem<D>::kAlloc;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return TASFT_ERR_CUDA;
  cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  int64_t grid = 2LL * sms;  // persistent: two CTAs per SM
  if (const char* cap = std::getenv("TASFT_PREFILL_GRID")) {  // debugging aid: fewer CTAs, more tiles each
    const long long c = std::atoll(cap);
    if (c > 0 && c < grid) grid = c;
  }
  if (grid > tiles) grid = tiles;
  if (debug_enabled()) debug_log("prefill_tc D=%d tiles=%lld grid=%lld smem=%d", D, (long long)tiles, (long long)grid, smem);
  const int wait_pv = std::getenv("TASFT_PREFILL_WAIT_PV") != nullptr;
  if (tiles <= 0) return TASFT_OK;
  kern<<<(unsigned)grid, kThreads, smem, st>>>(mq, mk, mv, a, NB, cu, bmax, emulate_bf16, wait_pv, qlo, qhi);
  count_launch();
  return launch_status();
}

}  // namespace

int prefill_tc(const tasft_prefill_args& a, cudaStream_t st, const int32_t* cu, int total, float* bmax,
               int emulate_bf16) {
  if (a.block != kBlk) return TASFT_ERR_UNSUPPORTED;
  if (a.dtype != TASFT_BF16 && a.dtype != TASFT_F16) return TASFT_ERR_UNSUPPORTED;
  if (a.D != 64 && a.D != 128) return TASFT_ERR_UNSUPPORTED;
  const int NB = (a.S + kBlk - 1) / kBlk;
  if (NB > kMaxNB) return TASFT_ERR_UNSUPPORTED;
  // vectorised epilogue stores: 16-byte aligned rows
  if (!aligned16(a.out) || (a.o_stride[0] % 8) || (a.o_stride[1] % 8) || (a.o_stride[2] % 8))
    return TASFT_ERR_UNSUPPORTED;
  const bool f16 = a.dtype == TASFT_F16;
  if (bmax && cu) return TASFT_ERR_UNSUPPORTED;  // block maxima only for the padded layout
  if (a.qb_hi > 0 && (cu || a.qb_lo < 0 || a.qb_lo >= a.qb_hi || a.qb_hi > NB)) return TASFT_ERR_INVALID_ARG;
  if (a.D == 128)
    return f16 ? launch_tc<128, true>(a, cu, total, st, bmax, emulate_bf16)
               : launch_tc<128, false>(a, cu, total, st, bmax, emulate_bf16);
  return f16 ? launch_tc<64, true>(a, cu, total, st, bmax, emulate_bf16)
             : launch_tc<64, false>(a, cu, total, st, bmax, emulate_bf16);
}

}  // namespace tasft
