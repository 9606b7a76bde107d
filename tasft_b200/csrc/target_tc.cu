// Gate-target tile maxima on the 5th-generation tensor cores (sm_100a).
//
// Reference: tasft/modules/tasft_attention.py:427-458 builds S = (Q K^T) * scale with a
// causal -inf fill; tasft/training/objectives.py:170-178 max-pools S over 64 x 64 tiles.
// Here S never leaves the chip: each 128 x 64 score tile lands in TMEM and is reduced to
// two 64 x 64 tile maxima right there; only the [B, Hq, NB, NB] maxima reach HBM.
//
// Unit = (b, kv-head, pair of q-heads of that kv-head, 128-row M tile = q-blocks 2mt and
// 2mt+1). The transposed tile S^T = K Q^T is formed: keys are the MMA's M (a 128-key K
// stage = k-blocks 2j, 2j+1) and the 256 q-rows of both heads are its N, so one
// M128 x N256 MMA per 16-deep slice reads 12 KB of operands from shared memory per 1 MFLOP
// (an M128 x N64 tile per head would need twice the shared-memory bandwidth the SM has).
// A unit visits key stages j = 0 .. mt (the causal triangle of its two q-blocks; tiles
// above the diagonal come out as -inf).
//
// Persistent CTAs (1 per SM, 320 threads) take units in a snake order over a
// heavy-first list. Warp roles:
//   warp 0     producer: Q of the unit (both heads, double-buffered per unit, loaded one
//              K stage into the previous unit), K stages through a 3-deep ring (TMA,
//              128-byte swizzle)
//   warp 1     MMA issuer: S^T into one of two TMEM buffers (256 columns each), commit to
//              the K stage and to the buffer
//   warps 2-9  two epilogue groups, one per TMEM buffer: each thread owns one key (TMEM
//              lane) and reduces the 64 q-rows of each (head, q-block) with the causal
//              mask, a warp max covers 32 keys, and the two warps of a k-block combine
//              through shared memory before one thread writes the tile maximum.
// Every ring has one producer and one consumer, so every parity wait is at most one phase
// behind; every wait is bounded (TASFT_DEVERR_TIMEOUT).
#include "tc.cuh"

namespace tasft {

namespace {

constexpr int kThreads = 320;
constexpr int kBlk = 64;
constexpr int kStages = 3;      // K ring depth (128 keys per stage)
constexpr uint32_t kTmemCols = 512;  // two 256-column score buffers

template <int D>
struct TSmem {
  static constexpr int kChunks = D / 64;                 // 64-element (128 B) swizzle atoms along D
  static constexpr int kQUnit = kChunks * 256 * 128;     // [chunk][head][128 rows] x 128 B
  static constexpr int kKStage = kChunks * 128 * 128;    // [chunk][128 keys] x 128 B
  static constexpr int kQOff = 0;
  static constexpr int kKOff = kQOff + 2 * kQUnit;
  static constexpr int kRedOff = kKOff + kStages * kKStage;  // [2 bufs][4 quarters][4 (head, q-block)] float
  static constexpr int kBarOff = kRedOff + 2 * 4 * 4 * 4;
  static constexpr int kNumBars = 2 + 2 + kStages * 2 + 2 * 2;
  static constexpr int kMiscOff = kBarOff + kNumBars * 8;
  static constexpr int kBytes = kMiscOff + 16;
  // 512 TMEM columns per CTA: ask for enough shared memory that two CTAs never share an SM
  static constexpr int kAlloc = (kBytes + 1024) > 120 * 1024 ? (kBytes + 1024) : 120 * 1024;
};

struct Unit {
  int b, hk, h0, h1, mt;  // h1 < 0: single head
};

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

__device__ __forceinline__ void named_sync(int id, int n) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

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
  uint64_t* s_full = k_empty + kStages;          // [2] per TMEM buffer
  uint64_t* s_empty = s_full + 2;                // [2] (4 warp arrivals)
  uint32_t* misc = reinterpret_cast<uint32_t*>(smem + L::kMiscOff);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp == 0 && lane == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], 4);
    }
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
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
        // the second q-block of the last M tile may lie wholly past S: not loaded (its
        // columns are masked in the epilogue)
        const int halves = x.mt * 128 + 64 < a.S ? 2 : 1;
        mbar_arrive_expect_tx(&q_full[qb], heads * halves * L::kChunks * 64 * 128);
        uint8_t* base = smem + L::kQOff + qb * L::kQUnit;
        for (int t = 0; t < heads; ++t) {
          const int h = t ? x.h1 : x.h0;
          for (int c = 0; c < L::kChunks; ++c)
            for (int half = 0; half < halves; ++half)
              tc::tma_load_4d(base + c * 256 * 128 + t * 128 * 128 + half * 64 * 128, &tmq, c * 64,
                              x.mt * 128 + half * 64, h, x.b, &q_full[qb]);
        }
        return true;
      };
      if (have) ok = load_q(u, 0);
      for (int ul = 0; have && ok; ++ul) {
        const int nst = u.mt + 1;  // key stages 0 .. mt
        const bool next = unit_of(a, pairs, nmt, ul + 1, nu);
        for (int j = 0; j < nst && ok; ++j, ++g) {
          const int s = g % kStages;
          if (g >= kStages && !mbar_wait(&k_empty[s], ((g / kStages) - 1) & 1)) {
            ok = false;
            break;
          }
          // the second k-block of the stage may lie wholly past S (NB odd): not loaded,
          // its keys exceed every valid query and are masked
          const int halves = j * 128 + 64 < a.S ? 2 : 1;
          mbar_arrive_expect_tx(&k_full[s], halves * L::kChunks * 64 * 128);
          uint8_t* dst = smem + L::kKOff + s * L::kKStage;
          for (int c = 0; c < L::kChunks; ++c)
            for (int half = 0; half < halves; ++half)
              tc::tma_load_4d(dst + c * 128 * 128 + half * 64 * 128, &tmk, c * 64, j * 128 + half * 64, u.hk,
                              u.b, &k_full[s]);
          if (j == 0 && next) ok = load_q(nu, ul + 1);  // next unit's Q behind the first K stage
        }
        u = nu;
        have = next;
      }
      if (!ok) set_err(a.err, TASFT_DEVERR_TIMEOUT | (1 << (8 + 0)));
    }
  } else if (warp == 1) {
    // ================= MMA issuer =================
    if (lane == 0) {
      constexpr uint32_t fmt = kF16 ? 0u : 1u;
      constexpr uint32_t idesc2 = tc::make_idesc(128, 256, fmt, false);
      constexpr uint32_t idesc1 = tc::make_idesc(128, 128, fmt, false);
      bool ok = true;
      int g = 0;
      Unit u;
      for (int ul = 0; ok && unit_of(a, pairs, nmt, ul, u); ++ul) {
        const int qb = ul & 1;
        if (!mbar_wait(&q_full[qb], (ul >> 1) & 1)) {
          ok = false;
          break;
        }
        const int nst = u.mt + 1;
        const uint32_t idesc = u.h1 >= 0 ? idesc2 : idesc1;
        const uint32_t q_addr = smem_u32(smem + L::kQOff + qb * L::kQUnit);
        for (int j = 0; j < nst; ++j, ++g) {
          const int s = g % kStages, bf = g & 1;
          if (!mbar_wait(&k_full[s], (g / kStages) & 1) || (g >= 2 && !mbar_wait(&s_empty[bf], ((g >> 1) - 1) & 1))) {
            ok = false;
            break;
          }
          tc::tc_fence_after();
          const uint32_t k_addr = smem_u32(smem + L::kKOff + s * L::kKStage);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint64_t ad = tc::make_sdesc(k_addr + (kk >> 2) * 128 * 128 + (kk & 3) * 32, 16, 1024);
            const uint64_t bd = tc::make_sdesc(q_addr + (kk >> 2) * 256 * 128 + (kk & 3) * 32, 16, 1024);
            tc::mma_ss(tmem + bf * 256, ad, bd, idesc, kk > 0 ? 1u : 0u);
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
    const int eg = (warp - 2) >> 2;              // 0: warps 2-5, 1: warps 6-9; group eg owns buffer eg
    const int quarter = warp & 3;                // TMEM lane quarter this warp may access
    const int gt = threadIdx.x - 64 - eg * 128;  // 0..127 within the group
    const bool emu = a.emulate_bf16_scores != 0;
    const uint32_t taddr = tmem + ((uint32_t)(quarter * 32) << 16) + eg * 256;
    float* rb = red + eg * 16;
    bool ok = true;
    int g = 0;
    Unit u;
    for (int ul = 0; ok && unit_of(a, pairs, nmt, ul, u); ++ul) {
      const int nst = u.mt + 1;
      const int heads = u.h1 >= 0 ? 2 : 1;
      // tiles above the unit's reach: -inf (the group of the unit's parity writes them)
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
      const int qrows = min(a.S - u.mt * 128, 128);  // valid q-rows (columns) of the tile
      for (int j = 0; j < nst; ++j, ++g) {
        if ((g & 1) != eg) continue;
        if (!mbar_wait(&s_full[eg], (g >> 1) & 1)) {
          ok = false;
          break;
        }
        tc::tc_fence_after();
        // this thread's key; column r (q-row mt*128 + r) is valid for r >= lo and r < qrows
        const int key = j * 128 + quarter * 32 + lane;
        const int lo = key - u.mt * 128;
        const bool full = lo <= 0 && qrows == 128;
        float m[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {  // i = head * 2 + q-block
          if ((i >> 1) >= heads) {
            m[i] = -INFINITY;
            continue;
          }
          uint32_t r[64];
          tc::tmem_ld64_sync(taddr + i * 64, r);
          float a0 = -INFINITY, a1 = -INFINITY, a2 = -INFINITY, a3 = -INFINITY;  // four short chains
          if (full) {
#pragma unroll
            for (int c = 0; c < 64; c += 8) {
              a0 = max3(a0, __uint_as_float(r[c]), __uint_as_float(r[c + 1]));
              a1 = max3(a1, __uint_as_float(r[c + 2]), __uint_as_float(r[c + 3]));
              a2 = max3(a2, __uint_as_float(r[c + 4]), __uint_as_float(r[c + 5]));
              a3 = max3(a3, __uint_as_float(r[c + 6]), __uint_as_float(r[c + 7]));
            }
          } else {
            const int c0 = (i & 1) * 64;
#pragma unroll
            for (int c = 0; c < 64; c += 4) {
              const int rr = c0 + c;
              a0 = (rr >= lo && rr < qrows) ? fmaxf(a0, __uint_as_float(r[c])) : a0;
              a1 = (rr + 1 >= lo && rr + 1 < qrows) ? fmaxf(a1, __uint_as_float(r[c + 1])) : a1;
              a2 = (rr + 2 >= lo && rr + 2 < qrows) ? fmaxf(a2, __uint_as_float(r[c + 2])) : a2;
              a3 = (rr + 3 >= lo && rr + 3 < qrows) ? fmaxf(a3, __uint_as_float(r[c + 3])) : a3;
            }
          }
          m[i] = fmaxf(max3(a0, a1, a2), a3);
        }
        tc::tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s_empty[eg]);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float w = warp_max(m[i]);
          if (lane == 0) rb[quarter * 4 + i] = w;
        }
        named_sync(1 + eg, 128);
        if (gt < 8) {
          const int kbl = gt >> 2, i = gt & 3;
          const int t = i >> 1, qb = 2 * u.mt + (i & 1), kb = 2 * j + kbl;
          if (t < heads && qb < NB && kb < NB) {
            const float mx = fmaxf(rb[(2 * kbl) * 4 + i], rb[(2 * kbl + 1) * 4 + i]);
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
        named_sync(1 + eg, 128);  // rb is rewritten by this group's next buffer
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
  const int64_t units = (int64_t)a.B * a.Hk * pairs * nmt;
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
