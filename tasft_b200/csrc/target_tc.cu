// Gate-target tile maxima on the 5th-generation tensor cores (sm_100a).
//
// Reference: tasft/modules/tasft_attention.py:427-458 builds S = (Q K^T) * scale with a
// causal -inf fill; tasft/training/objectives.py:170-178 max-pools S over 64 x 64 tiles.
// Here S never leaves the chip: each 128 x 64 score tile lands in TMEM and is reduced to
// two 64 x 64 tile maxima right there; only the [B, Hq, NB, NB] maxima reach HBM.
//
// Unit = (b, kv-head, pair of q-heads of that kv-head, 128-row M tile = q-blocks 2mt and
// 2mt+1). Both q-heads of the pair share every K tile of the kv-head, so one 64-key K
// stage feeds two M128 x N64 MMAs. A unit visits k-blocks 0 .. 2mt+1 (the causal
// triangle of its two q-blocks; the one tile above the diagonal comes out as -inf).
//
// Persistent CTAs (1 per SM, 320 threads) take units in a snake order over a
// heavy-first list. Warp roles:
//   warp 0     producer: Q of the unit (both heads, double-buffered per unit, loaded one
//              K stage into the previous unit), K tiles through a 4-stage ring (TMA,
//              128-byte swizzle)
//   warp 1     MMA issuer: S_t = Q_t K^T for both heads into one of 4 TMEM buffers
//              (128 columns each), commit to the K stage and to the buffer
//   warps 2-9  two epilogue groups taking alternate buffers: tcgen05.ld a row of 64
//              scores per head, causal mask, row max, warp max, then the two warps of a
//              q-block combine through shared memory and one thread writes the maximum.
// Every ring has one producer and one consumer, so every parity wait is at most one phase
// behind; every wait is bounded (TASFT_DEVERR_TIMEOUT).
#include "tc.cuh"

namespace tasft {

namespace {

constexpr int kThreads = 320;
constexpr int kBlk = 64;
constexpr int kStages = 4;      // K ring depth
constexpr int kBufs = 4;        // TMEM score buffers (128 columns each)
constexpr uint32_t kTmemCols = 512;

template <int D>
struct TSmem {
  static constexpr int kChunks = D / 64;
  static constexpr int kQHead = kChunks * 128 * 128;     // one head: 128 rows x 128 B per chunk
  static constexpr int kQUnit = 2 * kQHead;              // both heads of a unit
  static constexpr int kKStage = kChunks * 64 * 128;     // 64 keys x 128 B per chunk
  static constexpr int kQOff = 0;
  static constexpr int kKOff = kQOff + 2 * kQUnit;
  static constexpr int kRedOff = kKOff + kStages * kKStage;  // [kBufs][2 heads][4 warps] float
  static constexpr int kBarOff = kRedOff + kBufs * 2 * 4 * 4;
  static constexpr int kNumBars = 2 + 2 + kStages * 2 + kBufs * 2;
  static constexpr int kMiscOff = kBarOff + kNumBars * 8;
  static constexpr int kBytes = kMiscOff + 16;
  // 512 TMEM columns per CTA: ask for enough shared memory that two CTAs never share an SM
  static constexpr int kAlloc = (kBytes + 1024) > 120 * 1024 ? (kBytes + 1024) : 120 * 1024;
};

struct Unit {
  int b, hk, h0, h1, mt;  // h1 < 0: single head
};

__host__ __device__ inline int64_t num_units(int B, int Hk, int pairs, int nmt) {
  return (int64_t)B * Hk * pairs * nmt;
}

// i-th unit of this CTA: snake over rounds of gridDim units, rounds in heavy-first order.
__device__ inline bool unit_of(const tasft_target_args& a, int pairs, int nmt, int i, Unit& u) {
  const int64_t per_mt = (int64_t)a.B * a.Hk * pairs;
  const int64_t total = per_mt * nmt;
  const int64_t g = gridDim.x;
  const int64_t r = i;
  const int64_t pos = (r & 1) ? (r + 1) * g - 1 - blockIdx.x : r * g + blockIdx.x;
  if (pos >= total) return false;
  u.mt = nmt - 1 - (int)(pos / per_mt);
  int64_t rest = pos % per_mt;
  const int p = (int)(rest % pairs);
  rest /= pairs;
  u.hk = (int)(rest % a.Hk);
  u.b = (int)(rest / a.Hk);
  const int grp = a.Hq / a.Hk;
  u.h0 = u.hk * grp + 2 * p;
  u.h1 = (2 * p + 1 < grp) ? u.h0 + 1 : -1;
  return true;
}

__device__ __forceinline__ float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

__device__ __forceinline__ void named_sync(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }

template <int D, bool kF16>
__global__ void __launch_bounds__(kThreads, 1)
    target_tc_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
                     tasft_target_args a, float* bm, int NB, int pairs, int nmt) {
  using L = TSmem<D>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  float* red = reinterpret_cast<float*>(smem + L::kRedOff);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* q_full = bars + 0;                   // [2] per unit
  uint64_t* q_empty = bars + 2;                  // [2] per unit: its last MMA has run
  uint64_t* k_full = bars + 4;                   // [kStages]
  uint64_t* k_empty = k_full + kStages;          // [kStages]
  uint64_t* s_full = k_empty + kStages;          // [kBufs]
  uint64_t* s_empty = s_full + kBufs;            // [kBufs] (4 warp arrivals)
  uint32_t* misc = reinterpret_cast<uint32_t*>(smem + L::kMiscOff);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp == 0 && lane == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
    }
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
    }
    for (int i = 0; i < kBufs; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], 4);
    }
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

  if (warp == 0) {
    // ================= producer =================
    if (lane == 0) {
      tc::prefetch_tmap(&tmq);
      tc::prefetch_tmap(&tmk);
      bool ok = true;
      int g = 0;  // global K stage counter
      Unit u, nu;
      bool have = unit_of(a, pairs, nmt, 0, u);
      auto load_q = [&](const Unit& x, int ul) -> bool {
        const int qb = ul & 1;
        if (ul >= 2 && !mbar_wait(&q_empty[qb], ((ul >> 1) - 1) & 1)) return false;
        const int heads = x.h1 >= 0 ? 2 : 1;
        // the second q-block of the last M tile may lie wholly past S: not loaded, its
        // rows are masked in the epilogue
        const int halves = x.mt * 128 + 64 < a.S ? 2 : 1;
        mbar_arrive_expect_tx(&q_full[qb], heads * halves * L::kChunks * 64 * 128);
        uint8_t* base = smem + L::kQOff + qb * L::kQUnit;
        for (int t = 0; t < heads; ++t) {
          const int h = t ? x.h1 : x.h0;
          for (int c = 0; c < L::kChunks; ++c)
            for (int half = 0; half < halves; ++half)
              tc::tma_load_4d(base + t * L::kQHead + c * 128 * 128 + half * 64 * 128, &tmq, c * 64,
                              x.mt * 128 + half * 64, h, x.b, &q_full[qb]);
        }
        return true;
      };
      if (have) ok = load_q(u, 0);
      for (int ul = 0; have && ok; ++ul) {
        const int nk = min(2 * u.mt + 2, NB);
        const bool next = unit_of(a, pairs, nmt, ul + 1, nu);
        for (int kb = 0; kb < nk && ok; ++kb, ++g) {
          const int s = g % kStages;
          if (g >= kStages && !mbar_wait(&k_empty[s], ((g / kStages) - 1) & 1)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&k_full[s], L::kKStage);
          uint8_t* dst = smem + L::kKOff + s * L::kKStage;
          for (int c = 0; c < L::kChunks; ++c)
            tc::tma_load_4d(dst + c * 64 * 128, &tmk, c * 64, kb * kBlk, u.hk, u.b, &k_full[s]);
          if (kb == 0 && next) ok = load_q(nu, ul + 1);  // next unit's Q behind the first K stage
        }
        if (nk == 0 && next && ok) ok = load_q(nu, ul + 1);
        u = nu;
        have = next;
      }
      if (!ok) set_err(a.err, TASFT_DEVERR_TIMEOUT | (1 << (8 + 0)));
    }
  } else if (warp == 1) {
    // ================= MMA issuer =================
    if (lane == 0) {
      constexpr uint32_t idesc = tc::make_idesc(128, 64, kF16 ? 0u : 1u, false);
      bool ok = true;
      int g = 0;
      Unit u;
      for (int ul = 0; ok && unit_of(a, pairs, nmt, ul, u); ++ul) {
        const int qb = ul & 1;
        if (!mbar_wait(&q_full[qb], (ul >> 1) & 1)) {
          ok = false;
          break;
        }
        const int nk = min(2 * u.mt + 2, NB);
        const int heads = u.h1 >= 0 ? 2 : 1;
        const uint32_t q_addr = smem_u32(smem + L::kQOff + qb * L::kQUnit);
        for (int kb = 0; kb < nk; ++kb, ++g) {
          const int s = g % kStages, bf = g % kBufs;
          if (!mbar_wait(&k_full[s], (g / kStages) & 1) ||
              (g >= kBufs && !mbar_wait(&s_empty[bf], ((g / kBufs) - 1) & 1))) {
            ok = false;
            break;
          }
          tc::tc_fence_after();
          const uint32_t k_addr = smem_u32(smem + L::kKOff + s * L::kKStage);
          for (int t = 0; t < heads; ++t) {
            const uint32_t dst = tmem + bf * 128 + t * 64;
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk) {
              const uint64_t ad =
                  tc::make_sdesc(q_addr + t * L::kQHead + (kk >> 2) * 128 * 128 + (kk & 3) * 32, 16, 1024);
              const uint64_t bd = tc::make_sdesc(k_addr + (kk >> 2) * 64 * 128 + (kk & 3) * 32, 16, 1024);
              tc::mma_ss(dst, ad, bd, idesc, kk > 0 ? 1u : 0u);
            }
          }
          tc::mma_commit(&k_empty[s]);
          tc::mma_commit(&s_full[bf]);
        }
        if (ok) tc::mma_commit(&q_empty[qb]);
      }
      if (!ok) set_err(a.err, TASFT_DEVERR_TIMEOUT | (1 << (8 + 1)));
    }
  } else {
    // ================= epilogue groups =================
    const int eg = (warp - 2) >> 2;          // 0: warps 2-5, 1: warps 6-9
    const int quarter = warp & 3;            // TMEM lane quarter this warp may access
    const int row = quarter * 32 + lane;     // row of the 128-row M tile
    const int gt = threadIdx.x - 64 - eg * 128;  // 0..127 within the group
    const bool emu = a.emulate_bf16_scores != 0;
    bool ok = true;
    int g = 0;
    Unit u;
    for (int ul = 0; ok && unit_of(a, pairs, nmt, ul, u); ++ul) {
      const int nk = min(2 * u.mt + 2, NB);
      const int heads = u.h1 >= 0 ? 2 : 1;
      const int qpos = u.mt * 128 + row;
      // tiles above the unit's reach: -inf (group of the unit's parity writes them)
      if ((ul & 1) == eg) {
        const int first = 2 * u.mt + 2, span = NB - first;
        if (span > 0) {
          for (int i = gt; i < heads * 2 * span; i += 128) {
            const int t = i / (2 * span), rem = i % (2 * span), qbl = rem / span, kb = first + rem % span;
            const int qb = 2 * u.mt + qbl;
            if (qb >= NB) continue;
            const int h = t ? u.h1 : u.h0;
            bm[(((int64_t)u.b * a.Hq + h) * NB + qb) * NB + kb] = -INFINITY;
          }
        }
      }
      for (int kb = 0; kb < nk; ++kb, ++g) {
        if ((g & 1) != eg) continue;
        const int bf = g % kBufs;
        if (!mbar_wait(&s_full[bf], (g / kBufs) & 1)) {
          ok = false;
          break;
        }
        tc::tc_fence_after();
        // valid key columns of this row: key <= qpos (causal) and key < S
        const int lim = (qpos < a.S ? qpos : -1) - kb * kBlk;  // last valid column
        float m[2] = {-INFINITY, -INFINITY};
        for (int t = 0; t < heads; ++t) {
          uint32_t r[64];
          tc::tmem_ld64_sync(tmem + ((uint32_t)(quarter * 32) << 16) + bf * 128 + t * 64, r);
          float mx = -INFINITY;
          if (lim >= 63) {
#pragma unroll
            for (int c = 0; c < 64; c += 2) mx = max3(mx, __uint_as_float(r[c]), __uint_as_float(r[c + 1]));
          } else {
#pragma unroll
            for (int c = 0; c < 64; ++c) mx = c <= lim ? fmaxf(mx, __uint_as_float(r[c])) : mx;
          }
          m[t] = mx;
        }
        tc::tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s_empty[bf]);
        float* rb = red + bf * 8;
        for (int t = 0; t < heads; ++t) {
          const float w = warp_max(m[t]);
          if (lane == 0) rb[t * 4 + quarter] = w;
        }
        named_sync(1 + eg, 128);
        if (gt < 2 * heads) {
          const int t = gt >> 1, qbl = gt & 1;
          const int qb = 2 * u.mt + qbl;
          if (qb < NB) {
            const float mx = fmaxf(rb[t * 4 + 2 * qbl], rb[t * 4 + 2 * qbl + 1]);
            float v;
            if (emu) {
              // reference: bf16(bf16(q.k) * scale); both roundings are monotone, so max commutes
              v = __bfloat162float(__float2bfloat16_rn(__bfloat162float(__float2bfloat16_rn(mx)) * a.scale));
            } else {
              v = mx * a.scale;
            }
            const int h = t ? u.h1 : u.h0;
            bm[(((int64_t)u.b * a.Hq + h) * NB + qb) * NB + kb] = v;
          }
        }
      }
    }
    if (!ok) set_err(a.err, TASFT_DEVERR_TIMEOUT | (1 << (8 + 2)));
  }
  __syncwarp();
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, kTmemCols);
  }
}

template <int D, bool kF16>
int launch(const tasft_target_args& a, float* bm, cudaStream_t st) {
  const int NB = (a.S + kBlk - 1) / kBlk;
  CUtensorMap mq, mk;
  if (!make_tmap_bhsd(&mq, a.q, a.B, a.Hq, a.S, D, a.q_stride, 2, 64)) return TASFT_ERR_UNSUPPORTED;
  if (!make_tmap_bhsd(&mk, a.k, a.B, a.Hk, a.S, D, a.k_stride, 2, 64)) return TASFT_ERR_UNSUPPORTED;
  const int grp = a.Hq / a.Hk;
  const int pairs = (grp + 1) / 2;
  const int nmt = (NB + 1) / 2;
  const int64_t units = num_units(a.B, a.Hk, pairs, nmt);
  auto kern = target_tc_kernel<D, kF16>;
  const int smem = TSmem<D>::kAlloc;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return TASFT_ERR_CUDA;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  int64_t grid = sms;
  if (grid > units) grid = units;
  if (debug_enabled()) debug_log("target_tc D=%d units=%lld grid=%lld smem=%d", D, (long long)units, (long long)grid, smem);
  kern<<<(unsigned)grid, kThreads, smem, st>>>(mq, mk, a, bm, NB, pairs, nmt);
  count_launch();
  return launch_status();
}

}  // namespace

int gate_target_blockmax_tc(const tasft_target_args& a, float* bm, cudaStream_t st) {
  if (a.block != kBlk) return TASFT_ERR_UNSUPPORTED;
  if (a.dtype != TASFT_BF16 && a.dtype != TASFT_F16) return TASFT_ERR_UNSUPPORTED;
  if (a.D != 64 && a.D != 128) return TASFT_ERR_UNSUPPORTED;
  const bool f16 = a.dtype == TASFT_F16;
  if (a.D == 128) return f16 ? launch<128, true>(a, bm, st) : launch<128, false>(a, bm, st);
  return f16 ? launch<64, true>(a, bm, st) : launch<64, false>(a, bm, st);
}

}  // namespace tasft
