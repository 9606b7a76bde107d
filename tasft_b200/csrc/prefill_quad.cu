// Block-sparse causal GQA prefill, quad-tile variant for kv-head-granular kept lists.
//
// Same contract as the reference kernel (tasft/kernels/block_sparse_fa.py:108-269):
// per q-block, the kept k-blocks in ascending order, fp32 online softmax, p cast to the
// value dtype before P.V, rows with nothing kept give 0.
//
// When the kept lists are per kv-head (one list shared by the q-heads of a GQA group),
// four q-heads of a group at the same q-block ("a quad": 4 slots of 64 rows) walk the
// same list and read the same K/V. One CTA per SM owns a quad at a time as two 128-row
// M tiles (A = slots 0,1, B = slots 2,3) that share every K/V stage:
//   * a stage holds TWO kept 64-key blocks (128 keys), so S = Q K^T is one M128 x N128
//     MMA chain per tile and O += P V one M128 x N=D chain with K = 128 keys;
//   * TMEM (512 columns): S_A, S_B (128 each; P overwrites the first 64 as packed
//     16-bit pairs), O_A, O_B (128 each);
//   * the MMA warp issues P.V_A, S_A(next), P.V_B, S_B(next) per stage: tile B's MMAs run
//     while tile A's softmax works and the other way round;
//   * softmax: one warpgroup per tile, one thread per row, 2^x on MUFU;
//   * K and V stream through separate 2-stage TMA rings (128B swizzle).
// A lone last block (odd list length) runs as an N64 S chain and a K = 64 P.V chain.
// Every wait is bounded (TASFT_DEVERR_TIMEOUT); phases are indexed by a per-CTA stage
// counter (one S, one P and one P.V per tile per stage) or by the quad counter.
#include <cstdlib>
#include <type_traits>

#include "tc.cuh"

namespace tasft {

namespace {

// Warpgroup 0: warp 0 TMA, warp 1 MMA (warps 2-3 idle); warpgroups 1 and 2: softmax and
// epilogue of tiles A and B. Launched at 168 registers a thread (three warps per SM
// sub-partition share its 16K registers); warpgroup 0 then gives registers to the softmax
// warpgroups: 384 x 168 = 128 x 56 + 256 x 224.
constexpr int kThreads = 384;
constexpr int kRegsLow = 56, kRegsSoftmax = 224;
constexpr int kBlk = 64;
constexpr int kMaxNB = 1024;
constexpr int kWords = kMaxNB / 32;
constexpr uint32_t kTmemCols = 512;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescaleThreshold = 8.0f;  // log2 units
// 2^x of the softmax: kExpF32 = ex2.approx.f32 on MUFU for every element; kExpF16x2 =
// ex2.approx.f16x2 (two results per MUFU operation; the argument is rounded to f16,
// relative error <= 2^-11 * |x| * ln 2 in p, which matters only for small p); kExpPoly =
// kPolyPairs of every 64 pairs on the FMA pipe (exp2_poly2), the rest as kExpF32.
enum : int { kExpF32 = 0, kExpF16x2 = 1, kExpPoly = 2 };
constexpr int kExpDefault = kExpF32;
constexpr int kPolyPairs = 16;

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
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
__device__ __forceinline__ uint64_t sub2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("sub.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint32_t ex2_h2(uint32_t x) {
  uint32_t y;
  asm("ex2.approx.f16x2 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}
__device__ __forceinline__ float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// 2^x for a pair, on the FMA pipe: x = j + f with j = round(x), f in [-1/2, 1/2];
// 2^f by a degree-3 polynomial (coefficients: least-squares fit of 2^f on [-1/2, 1/2]
// weighted to relative error, max relative error 7.8e-5, far below the 2^-9 rounding of
// the 16-bit p that P.V uses), then j added to the exponent field. x is clamped at -125
// so the result stays a normal number (the true value is below 2^-125 anyway).
__device__ __forceinline__ uint64_t exp2_poly2(uint64_t x2) {
  const float xl = fmaxf(lo_f(x2), -125.f), xh = fmaxf(hi_f(x2), -125.f);
  const uint64_t x = f2(xl, xh);
  const uint64_t magic = f2(12582912.f, 12582912.f);  // 1.5 * 2^23: adding it rounds to an integer
  const uint64_t t = add2(x, magic);
  const uint64_t j = sub2(t, magic);
  const uint64_t f = sub2(x, j);
  uint64_t p = fma2(f2(0.05508881653277375f, 0.05508881653277375f), f, f2(0.24260436174225863f, 0.24260436174225863f));
  p = fma2(p, f, f2(0.6932762437639659f, 0.6932762437639659f));
  p = fma2(p, f, f2(0.9999289212634266f, 0.9999289212634266f));
  const uint32_t lo = (uint32_t)p + ((uint32_t)t << 23);
  const uint32_t hi = (uint32_t)(p >> 32) + ((uint32_t)(t >> 32) << 23);
  return ((uint64_t)hi << 32) | lo;
}

struct Quad {
  int b, hk, qb;
  int head[4];
  int valid[4];
  int n;  // kept blocks in the list; -1 = no more work
};

template <int D>
struct Smem {
  static constexpr int kChunks = D / 64;                // 128-byte swizzle atoms along D
  static constexpr int kTileBytes = kChunks * 128 * 128;  // 128 rows x D (a Q tile or a K/V stage)
  static constexpr int kQOff = 0;                         // Q_A, Q_B
  static constexpr int kKOff = 2 * kTileBytes;            // K ring [2]
  static constexpr int kVOff = 4 * kTileBytes;            // V ring [2]
  static constexpr int kListOff = 6 * kTileBytes;         // [2][kMaxNB] int32
  static constexpr int kBitmapOff = kListOff + 2 * kMaxNB * 4;
  static constexpr int kWorkOff = kBitmapOff + kWords * 4;
  static constexpr int kBarOff = (kWorkOff + 2 * (int)sizeof(Quad) + 7) / 8 * 8;
  static constexpr int kNumBars = 28;
  static constexpr int kMiscOff = kBarOff + kNumBars * 8;
  static constexpr int kBytes = kMiscOff + 16;
  static constexpr int kAlloc = kBytes + 1024;
};

__device__ __forceinline__ Quad decode_quad(const tasft_prefill_args& a, int NB, int id) {
  const int grp = a.Hq / a.Hk;
  const int P = (grp + 3) / 4;
  const int inner = a.B * a.Hk * P;
  const int qbo = id / inner, rem = id % inner;
  Quad w;
  const int p = rem % P;
  w.hk = (rem / P) % a.Hk;
  w.b = rem / (P * a.Hk);
  w.qb = NB - 1 - qbo;  // heavy (late) q-blocks first
#pragma unroll
  for (int s = 0; s < 4; ++s) {
    w.valid[s] = 4 * p + s < grp;
    w.head[s] = w.hk * grp + min(4 * p + s, grp - 1);
  }
  w.n = 0;
  return w;
}

__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity) {
  return __all_sync(0xffffffffu, mbar_wait(bar, parity));
}

template <int D, bool kF16, int kExp>
__global__ void __launch_bounds__(kThreads, 1)
    bsa_prefill_quad_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
                            const __grid_constant__ CUtensorMap tmv, const tasft_prefill_args a, const int NB,
                            const int wait_pv, const int order_exp) {
  using L = Smem<D>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  int32_t* lists = reinterpret_cast<int32_t*>(smem + L::kListOff);
  uint32_t* bitmap = reinterpret_cast<uint32_t*>(smem + L::kBitmapOff);
  Quad* works = reinterpret_cast<Quad*>(smem + L::kWorkOff);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* q_full = bars + 0;       // [2 tiles]
  uint64_t* q_empty = bars + 2;      // [2 tiles]
  uint64_t* k_full = bars + 4;       // [2]
  uint64_t* k_empty = bars + 6;      // [2]
  uint64_t* v_full = bars + 8;       // [2]
  uint64_t* v_empty = bars + 10;     // [2]
  uint64_t* s_full = bars + 12;      // [2 tiles]
  uint64_t* p_ready = bars + 14;     // [2 tiles] (128 arrivals)
  uint64_t* pv_done = bars + 16;     // [2 tiles]
  uint64_t* o_final = bars + 18;     // [2 tiles]
  uint64_t* o_free = bars + 20;      // [2 tiles] (128 arrivals)
  uint64_t* list_full = bars + 22;   // [2]
  uint64_t* list_empty = bars + 24;  // [2] (256 arrivals: the softmax threads)
  uint64_t* exp_turn = bars + 26;    // [2] (128 arrivals): tiles take turns for their exponentials
  uint32_t* misc = reinterpret_cast<uint32_t*>(smem + L::kMiscOff);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int grp = a.Hq / a.Hk;
  const int tiles = a.B * a.Hk * ((grp + 3) / 4) * NB;
  const int words = (NB + 31) / 32;

  if (warp == 0 && lane == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_ready[i], 128);
      mbar_init(&pv_done[i], 1);
      mbar_init(&o_final[i], 1);
      mbar_init(&o_free[i], 128);
      mbar_init(&list_full[i], 1);
      mbar_init(&list_empty[i], 256);
      mbar_init(&exp_turn[i], 128);
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
  // columns: S_A [0,128), S_B [128,256), O_A [256, 256+D), O_B [384, 384+D)

  if (warp == 0) {
    // ================= producer =================
    tc::reg_dealloc<kRegsLow>();
    if (lane == 0) {
      tc::prefetch_tmap(&tmq);
      tc::prefetch_tmap(&tmk);
      tc::prefetch_tmap(&tmv);
    }
    int gk = 0;  // stage counter
    bool ok = true;
    for (int u = 0; ok; ++u) {
      // quads run heaviest first; the CTA order snakes (0..G-1, then G-1..0, ...) so every
      // CTA's sum of quad sizes comes out about equal
      const int tile = u * gridDim.x + ((u & 1) ? (int)gridDim.x - 1 - (int)blockIdx.x : (int)blockIdx.x);
      const int lb = u & 1;
      if (u >= 2 && !warp_wait(&list_empty[lb], ((u >> 1) - 1) & 1)) {
        set_err(a.err, TASFT_DEVERR_TIMEOUT | (1 << (8 + 1)));
        ok = false;
        break;
      }
      Quad w;
      int* list = lists + lb * kMaxNB;
      if (tile >= tiles) {
        w.n = -1;
      } else {
        w = decode_quad(a, NB, tile);
        // the kv-head list of this q-block, filtered (range, causal) and sorted through a bitmap
        for (int i = lane; i < words; i += 32) bitmap[i] = 0;
        __syncwarp();
        const int64_t lrow = ((int64_t)w.b * a.Hm + w.hk) * NB + w.qb;
        const int cnt = min(a.kept_cnt[lrow], NB);
        const int32_t* idx = a.kept_idx + lrow * NB;
        for (int t = lane; t < cnt; t += 32) {
          const int kb = idx[t];
          if (kb < 0 || kb >= NB) {
            set_err(a.err, TASFT_DEVERR_INDEX);
            continue;
          }
          if (a.causal && kb > w.qb) continue;
          atomicOr(&bitmap[kb >> 5], 1u << (kb & 31));
        }
        __syncwarp();
        int n = 0;
        for (int wd = 0; wd < words; ++wd) {
          const uint32_t bit = 1u << lane;
          const bool any = (bitmap[wd] & bit) != 0;
          const unsigned bal = __ballot_sync(0xffffffffu, any);
          if (any) list[n + __popc(bal & (bit - 1u))] = wd * 32 + lane;
          n += __popc(bal);
        }
        w.n = n;
        __syncwarp();
      }
      if (lane == 0) {
        works[lb] = w;
        mbar_arrive(&list_full[lb]);
      }
      if (w.n < 0) break;
      if (lane == 0) {
        // Q of each tile as soon as the previous quad's last S of that tile has run
        for (int x = 0; ok && x < 2; ++x) {
          if (u >= 1 && !mbar_wait(&q_empty[x], (u - 1) & 1)) {
            set_err(a.err, TASFT_DEVERR_TIMEOUT | (1 << (8 + 2)));
            ok = false;
            break;
          }
          const int nvalid = (w.valid[2 * x] ? 1 : 0) + (w.valid[2 * x + 1] ? 1 : 0);
          mbar_arrive_expect_tx(&q_full[x], nvalid * L::kChunks * 64 * 128);
          for (int s = 2 * x; s < 2 * x + 2; ++s) {
            if (!w.valid[s]) continue;
            uint8_t* dst = smem + L::kQOff + x * L::kTileBytes + (s & 1) * 64 * 128;
            for (int c = 0; c < L::kChunks; ++c)
              tc::tma_load_4d(dst + c * 128 * 128, &tmq, c * 64, w.qb * kBlk, w.head[s], w.b, &q_full[x]);
          }
        }
        const int T = (w.n + 1) / 2;
        auto load_stage = [&](const CUtensorMap* map, uint64_t* full, uint64_t* empty, int off, int gi, int t) -> bool {
          const int st = gi & 1;
          if (gi >= 2 && !mbar_wait(&empty[st], ((gi >> 1) - 1) & 1)) return false;
          const int nb = (2 * t + 1 < w.n) ? 2 : 1;
          uint8_t* dst = smem + off + st * L::kTileBytes;
          mbar_arrive_expect_tx(&full[st], nb * L::kChunks * 64 * 128);
          for (int h = 0; h < nb; ++h) {
            const int kb = list[2 * t + h];
            for (int c = 0; c < L::kChunks; ++c)
              tc::tma_load_4d(dst + c * 128 * 128 + h * 64 * 128, map, c * 64, kb * kBlk, w.hk, w.b, &full[st]);
          }
          return true;
        };
        for (int t = 0; ok && t <= T && T > 0; ++t) {
          if (t < T && !load_stage(&tmk, k_full, k_empty, L::kKOff, gk + t, t)) ok = false;
          if (ok && t >= 1 && !load_stage(&tmv, v_full, v_empty, L::kVOff, gk + t - 1, t - 1)) ok = false;
        }
        if (!ok) set_err(a.err, TASFT_DEVERR_TIMEOUT | (1 << (8 + 3)));
        gk += T;
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      gk = __shfl_sync(0xffffffffu, gk, 0);
    }
    if (lane == 0) {  // do not leave while copies into shared memory are in flight
      for (int i = max(0, gk - 2); i < gk; ++i) {
        mbar_wait(&k_full[i & 1], (i >> 1) & 1);
        mbar_wait(&v_full[i & 1], (i >> 1) & 1);
      }
    }
  } else if (warp == 1) {
    // ================= MMA issuer =================
    tc::reg_dealloc<kRegsLow>();
    if (lane == 0) {
      constexpr uint32_t fmt = kF16 ? 0u : 1u;
      constexpr uint32_t idesc_s128 = tc::make_idesc(128, 128, fmt, false);
      constexpr uint32_t idesc_s64 = tc::make_idesc(128, 64, fmt, false);
      constexpr uint32_t idesc_o = tc::make_idesc(128, D, fmt, true);
      const uint32_t q_addr = smem_u32(smem + L::kQOff);
      int g = 0;
      bool ok = true;
      int where = 0;
      auto issue_s = [&](int tile, int gi, bool single) {
        const uint32_t qa = q_addr + tile * L::kTileBytes;
        const uint32_t ka = smem_u32(smem + L::kKOff + (gi & 1) * L::kTileBytes);
        const uint32_t dst = tmem + tile * 128;
        const uint32_t idesc = single ? idesc_s64 : idesc_s128;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint64_t ad = tc::make_sdesc(qa + (kk >> 2) * 128 * 128 + (kk & 3) * 32, 16, 1024);
          const uint64_t bd = tc::make_sdesc(ka + (kk >> 2) * 128 * 128 + (kk & 3) * 32, 16, 1024);
          tc::mma_ss(dst, ad, bd, idesc, kk > 0 ? 1u : 0u);
        }
        tc::mma_commit(&s_full[tile]);
      };
      auto issue_pv = [&](int tile, int gi, bool single, bool first) {
        const uint32_t va = smem_u32(smem + L::kVOff + (gi & 1) * L::kTileBytes);
        const uint32_t p_tmem = tmem + tile * 128;
        const uint32_t o_tmem = tmem + 256 + tile * 128;
        const int ksteps = single ? kBlk / 16 : 2 * kBlk / 16;
        for (int kk = 0; kk < ksteps; ++kk) {
          const uint64_t bd = tc::make_sdesc(va + kk * 16 * 128, 128 * 128, 1024);
          tc::mma_ts(o_tmem, p_tmem + kk * 8, bd, idesc_o, (!first || kk > 0) ? 1u : 0u);
        }
        tc::mma_commit(&pv_done[tile]);
      };
      for (int u = 0; ok; ++u) {
        const int lb = u & 1;
        if (!mbar_wait(&list_full[lb], (u >> 1) & 1)) { where = 4; ok = false; break; }
        const int n = works[lb].n;
        if (n < 0) break;
        const int T = (n + 1) / 2;
        if (T == 0) {
          for (int x = 0; ok && x < 2; ++x) {
            if (!mbar_wait(&q_full[x], u & 1)) { where = 5; ok = false; break; }
            tc::mma_commit(&q_empty[x]);
            if (u >= 1 && !mbar_wait(&o_free[x], (u - 1) & 1)) { where = 6; ok = false; break; }
            tc::mma_commit(&o_final[x]);
          }
          continue;
        }
        // Issue order per stage: P.V_A(t), S_A(t+1), P.V_B(t), S_B(t+1). S_X(t+1) overwrites
        // the TMEM columns P.V_X(t) reads P_X(t) from. MMAs issued by one thread run through
        // the tensor pipe in issue order (CUTLASS's sm100 FMHA mainloop issues its next
        // Q K^T into the S/P columns right behind the P V that reads them, with no wait);
        // `wait_pv` instead waits for P.V_X(t) to complete first (a checking aid).
        if (!mbar_wait(&k_full[g & 1], (g >> 1) & 1)) { where = 7; ok = false; break; }
        for (int x = 0; x < 2 && ok; ++x) {
          if (!mbar_wait(&q_full[x], u & 1)) { where = 5; ok = false; break; }
          if (wait_pv && g >= 1 && !mbar_wait(&pv_done[x], (g - 1) & 1)) { where = 8; ok = false; break; }
          tc::tc_fence_after();
          issue_s(x, g, n == 1);
          if (T == 1) tc::mma_commit(&q_empty[x]);
        }
        if (!ok) break;
        tc::mma_commit(&k_empty[g & 1]);
        for (int t = 0; ok && t < T; ++t) {
          const int gi = g + t;
          const bool single = 2 * t + 1 == n;
          const bool has_next = t + 1 < T;
          const bool single_next = 2 * t + 3 == n;
          if (!mbar_wait(&v_full[gi & 1], (gi >> 1) & 1)) { where = 9; ok = false; break; }
          for (int x = 0; x < 2; ++x) {
            if (!mbar_wait(&p_ready[x], gi & 1)) { where = 10; ok = false; break; }
            // O_X is reused: the previous quad's epilogue must have read it
            if (t == 0 && u >= 1 && !mbar_wait(&o_free[x], (u - 1) & 1)) { where = 11; ok = false; break; }
            tc::tc_fence_after();
            issue_pv(x, gi, single, t == 0);
            if (t == T - 1) tc::mma_commit(&o_final[x]);
            if (x == 1) tc::mma_commit(&v_empty[gi & 1]);
            if (has_next) {
              if (x == 0 && !mbar_wait(&k_full[(gi + 1) & 1], ((gi + 1) >> 1) & 1)) { where = 7; ok = false; break; }
              if (wait_pv && !mbar_wait(&pv_done[x], gi & 1)) { where = 8; ok = false; break; }
              tc::tc_fence_after();
              issue_s(x, gi + 1, single_next);
              if (t + 2 == T) tc::mma_commit(&q_empty[x]);
              if (x == 1) tc::mma_commit(&k_empty[(gi + 1) & 1]);
            }
          }
        }
        if (!ok) break;
        g += T;
      }
      if (!ok) set_err(a.err, TASFT_DEVERR_TIMEOUT | (1 << (8 + where)));
    }
  } else if (warp < 4) {
    tc::reg_dealloc<kRegsLow>();  // idle warps of warpgroup 0
  } else {
    // ================= softmax + epilogue: warps 4-7 tile A, warps 8-11 tile B =================
    tc::reg_alloc<kRegsSoftmax>();
    const int tile = (warp - 4) >> 2;
    const int quarter = warp & 3;  // TMEM lane quarter this warp may access
    const int r = quarter * 32 + lane;
    const int slot = tile * 2 + (r >> 6);
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t tS = tmem + tile * 128 + lane_off;
    const uint32_t tO = tmem + 256 + tile * 128 + lane_off;
    const float sl2 = a.scale * kLog2e;
    int g = 0;
    bool ok = true;
    int where = 0;
    for (int u = 0; ok; ++u) {
      const int lb = u & 1;
      if (!warp_wait(&list_full[lb], (u >> 1) & 1)) { where = 12; ok = false; break; }
      const Quad& w = works[lb];  // read in place: a local copy indexed by slot would live in local memory
      const int wn = w.n;
      if (wn < 0) break;
      const int* list = lists + lb * kMaxNB;
      const int Tn = (wn + 1) / 2;
      const int qpos = w.qb * kBlk + (r & 63);
      const bool row_on = w.valid[slot] && qpos < a.S;
      float m = -INFINITY, l = 0.f;
      for (int t = 0; t < Tn; ++t) {
        const int gi = g + t;
        const bool single = 2 * t + 1 == wn;
        const int kb0 = list[2 * t], kb1 = single ? kb0 : list[2 * t + 1];
        if (!warp_wait(&s_full[tile], gi & 1)) { where = 13; ok = false; break; }
        tc::tc_fence_after();
        float sv[128];
        if (!single) {
          uint32_t raw[128];
          tc::tmem_ld128_sync(tS, raw);
#pragma unroll
          for (int c = 0; c < 128; ++c) sv[c] = __uint_as_float(raw[c]);
        } else {
          uint32_t raw[64];
          tc::tmem_ld64_sync(tS, raw);
#pragma unroll
          for (int c = 0; c < 64; ++c) sv[c] = __uint_as_float(raw[c]);
#pragma unroll
          for (int c = 64; c < 128; ++c) sv[c] = -INFINITY;
        }
        // valid keys of this row in each half: < S, and <= qpos when causal
        int lim0 = a.S - kb0 * kBlk, lim1 = a.S - kb1 * kBlk;
        if (a.causal) {
          lim0 = min(lim0, qpos - kb0 * kBlk + 1);
          lim1 = min(lim1, qpos - kb1 * kBlk + 1);
        }
        if (!row_on) lim0 = lim1 = 0;
        if (single) lim1 = 0;
        lim0 = max(0, min(lim0, kBlk));
        lim1 = max(0, min(lim1, kBlk));
        const bool masked = __any_sync(0xffffffffu, lim0 < kBlk || lim1 < kBlk);
        if (masked) {
#pragma unroll
          for (int c = 0; c < 64; ++c) {
            if (c >= lim0) sv[c] = -INFINITY;
            if (c >= lim1) sv[64 + c] = -INFINITY;
          }
        }
        float mq[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
        for (int c = 0; c < 128; c += 8) {
#pragma unroll
          for (int qd = 0; qd < 4; ++qd) mq[qd] = max3(mq[qd], sv[c + 2 * qd], sv[c + 2 * qd + 1]);
        }
        const float mb = max3(mq[0], mq[1], fmaxf(mq[2], mq[3]));
        const float m_new = fmaxf(m, mb * sl2);
        const bool need = (m != -INFINITY) && (m_new > m + kRescaleThreshold);
        if (m == -INFINITY) m = m_new;  // O row still exactly zero: no rescale
        if (__any_sync(0xffffffffu, need)) {
          // O holds every earlier P.V of this quad: P.V_X(gi - 1) was issued before S_X(gi),
          // and the commit that signalled s_full tracks every MMA issued before it
          tc::tc_fence_after();
          const float alpha = need ? ex2(m - m_new) : 1.0f;
          for (int c0 = 0; c0 < D; c0 += 32) {
            uint32_t o[32];
            tc::tmem_ld32_sync(tO + c0, o);
#pragma unroll
            for (int c = 0; c < 32; ++c) o[c] = __float_as_uint(__uint_as_float(o[c]) * alpha);
            tc::tmem_st32(tO + c0, o);
          }
          tc::tmem_wait_st();
          if (need) {
            l *= alpha;
            m = m_new;
          }
        }
        const uint64_t sc2 = f2(sl2, sl2), nm2 = f2(-m, -m);
        uint64_t rs2 = 0;
        // one half (64 columns) of the row: p = 2^(s * scale - m), packed to 16 bits into TMEM
        auto half = [&](auto hc) {
          constexpr int h = decltype(hc)::value;
          uint32_t pk[32];
          if (m == -INFINITY) {
#pragma unroll
            for (int c = 0; c < 32; ++c) pk[c] = 0u;
          } else if (masked) {
            // masked entries are -inf: MUFU ex2 gives exact zeros
#pragma unroll
            for (int c = 0; c < 32; ++c) {
              const uint64_t x2 = fma2(f2(sv[64 * h + 2 * c], sv[64 * h + 2 * c + 1]), sc2, nm2);
              const uint64_t p2 = f2(ex2(lo_f(x2)), ex2(hi_f(x2)));
              rs2 = add2(rs2, p2);
              pk[c] = kF16 ? tc::pack_f16x2(lo_f(p2), hi_f(p2)) : tc::pack_bf16x2(lo_f(p2), hi_f(p2));
            }
          } else {
#pragma unroll
            for (int c = 0; c < 32; ++c) {
              const uint64_t x2 = fma2(f2(sv[64 * h + 2 * c], sv[64 * h + 2 * c + 1]), sc2, nm2);
              if constexpr (kExp == kExpF16x2) {
                const uint32_t ph = ex2_h2(tc::pack_f16x2(lo_f(x2), hi_f(x2)));
                const float2 pf = __half22float2(*reinterpret_cast<const __half2*>(&ph));
                rs2 = add2(rs2, f2(pf.x, pf.y));
                pk[c] = kF16 ? ph : tc::pack_bf16x2(pf.x, pf.y);
              } else {
                // poly pairs spread over the row so MUFU and FMA work interleave
                const int pi = c * 2 + h;  // pair index over the row, halves interleaved
                const bool poly = kExp == kExpPoly && (pi * kPolyPairs) / 64 != ((pi + 1) * kPolyPairs) / 64;
                const uint64_t p2 = poly ? exp2_poly2(x2) : f2(ex2(lo_f(x2)), ex2(hi_f(x2)));
                rs2 = add2(rs2, p2);
                pk[c] = kF16 ? tc::pack_f16x2(lo_f(p2), hi_f(p2)) : tc::pack_bf16x2(lo_f(p2), hi_f(p2));
              }
            }
          }
          tc::tmem_st32(tS + 32 * h, pk);
        };
        // with order_exp the two tiles' exponential phases alternate (A(t), B(t), A(t+1), ...),
        // so the tile on the critical path gets the whole MUFU
        if (order_exp) {
          const bool mine = tile == 0 ? (gi == 0 || warp_wait(&exp_turn[0], (gi - 1) & 1)) : warp_wait(&exp_turn[1], gi & 1);
          if (!mine) { where = 16; ok = false; break; }
        }
        half(std::integral_constant<int, 0>{});
        if (!single) half(std::integral_constant<int, 1>{});
        if (order_exp) mbar_arrive(&exp_turn[tile ^ 1]);
        tc::tmem_wait_st();
        tc::tc_fence_before();
        mbar_arrive(&p_ready[tile]);
        l += lo_f(rs2) + hi_f(rs2);
      }
      if (!ok) break;
      if (!warp_wait(&o_final[tile], u & 1)) { where = 15; ok = false; break; }
      tc::tc_fence_after();
      // epilogue: O / l -> global (rows past S and invalid slots are not stored)
      using T = typename std::conditional<kF16, __half, __nv_bfloat16>::type;
      T* orow = reinterpret_cast<T*>(a.out) + w.b * a.o_stride[0] + (int64_t)w.head[slot] * a.o_stride[1] +
                (int64_t)qpos * a.o_stride[2];
      const float inv = (l > 0.f) ? 1.0f / l : 0.f;
      for (int c0 = 0; c0 < D; c0 += 32) {
        uint32_t o[32];
        if (Tn > 0) {
          tc::tmem_ld32_sync(tO + c0, o);
        } else {
#pragma unroll
          for (int c = 0; c < 32; ++c) o[c] = 0u;
        }
        if (row_on) {
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
      mbar_arrive(&o_free[tile]);
      mbar_arrive(&list_empty[lb]);
      g += Tn;
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

template <int D, bool kF16, int kExp = kExpDefault>
int launch_quad(const tasft_prefill_args& a, cudaStream_t st) {
  const int NB = (a.S + kBlk - 1) / kBlk;
  CUtensorMap mq, mk, mv;
  if (!make_tmap_bhsd(&mq, a.q, a.B, a.Hq, a.S, D, a.q_stride, 2, 64)) return TASFT_ERR_UNSUPPORTED;
  if (!make_tmap_bhsd(&mk, a.k, a.B, a.Hk, a.S, D, a.k_stride, 2, 64)) return TASFT_ERR_UNSUPPORTED;
  if (!make_tmap_bhsd(&mv, a.v, a.B, a.Hk, a.S, D, a.v_stride, 2, 64)) return TASFT_ERR_UNSUPPORTED;
  const int grp = a.Hq / a.Hk;
  const int64_t tiles = (int64_t)a.B * a.Hk * ((grp + 3) / 4) * NB;
  auto kern = bsa_prefill_quad_kernel<D, kF16, kExp>;
  const int smem = Smem<D>::kAlloc;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return TASFT_ERR_CUDA;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  int64_t grid = sms;  // persistent: one CTA per SM (it holds all 512 TMEM columns)
  if (const char* cap = std::getenv("TASFT_PREFILL_GRID")) {  // testing aid: fewer CTAs, more quads each
    const long long c = std::atoll(cap);
    if (c > 0 && c < grid) grid = c;
  }
  if (grid > tiles) grid = tiles;
  if (debug_enabled()) debug_log("prefill_quad D=%d tiles=%lld grid=%lld smem=%d", D, (long long)tiles, (long long)grid, smem);
  const int wait_pv = std::getenv("TASFT_QUAD_WAIT_PV") != nullptr;
  const int order_exp = std::getenv("TASFT_QUAD_ORDER") != nullptr;
  kern<<<(unsigned)grid, kThreads, smem, st>>>(mq, mk, mv, a, NB, wait_pv, order_exp);
  count_launch();
  return launch_status();
}

}  // namespace

// Quad kernel: bf16/fp16, block 64, D 64/128, GQA group >= 3 with per-kv-head lists
// (Hm == Hk), padded layout. Returns TASFT_ERR_UNSUPPORTED for anything else.
int prefill_quad(const tasft_prefill_args& a, cudaStream_t st) {
  if (a.block != kBlk || (a.dtype != TASFT_BF16 && a.dtype != TASFT_F16)) return TASFT_ERR_UNSUPPORTED;
  if (a.D != 64 && a.D != 128) return TASFT_ERR_UNSUPPORTED;
  if (a.Hk <= 0 || a.Hq % a.Hk || a.Hq / a.Hk < 3 || a.Hm != a.Hk) return TASFT_ERR_UNSUPPORTED;
  const int NB = (a.S + kBlk - 1) / kBlk;
  if (NB > kMaxNB) return TASFT_ERR_UNSUPPORTED;
  if (!aligned16(a.out) || (a.o_stride[0] % 8) || (a.o_stride[1] % 8) || (a.o_stride[2] % 8))
    return TASFT_ERR_UNSUPPORTED;
  if (std::getenv("TASFT_PREFILL_NO_QUAD")) return TASFT_ERR_UNSUPPORTED;  // comparison aid
  const bool f16 = a.dtype == TASFT_F16;
  if (const char* pp = std::getenv("TASFT_QUAD_EXP")) {  // tuning aid: how 2^x is computed (bf16, D 128)
    if (a.D == 128 && !f16) {
      switch (std::atoi(pp)) {
        case kExpF32: return launch_quad<128, false, kExpF32>(a, st);
        case kExpF16x2: return launch_quad<128, false, kExpF16x2>(a, st);
        case kExpPoly: return launch_quad<128, false, kExpPoly>(a, st);
        default: break;
      }
    }
  }
  if (a.D == 128) return f16 ? launch_quad<128, true>(a, st) : launch_quad<128, false>(a, st);
  return f16 ? launch_quad<64, true>(a, st) : launch_quad<64, false>(a, st);
}

}  // namespace tasft
