// Block-sparse decode for bf16/fp16 caches on tensor-core fragments (mma.sync).
//
// Decode is HBM-bound: every kept KV byte is read once and used by the few q-heads of
// its GQA group. The tensor cores are used only to keep the instruction count per byte
// small (CUDA-core dot products with shuffle reductions issued ~14K warp instructions
// per 32 KB block; this path issues a few hundred).
//
//   CTA = (sequence, kv-head, split); 2 warps: warp 1 = TMA producer, warp 0 = the one
//   consumer, 3 CTAs per SM. K/V tiles arrive through a 2-stage ring of 128B-swizzled
//   TMA boxes (64 rows x 64 elements), so ldmatrix reads are conflict free. A single
//   in-order consumer per ring keeps every mbarrier parity wait exact: with several
//   consumers taking turns on a shared ring, a fast one can reach a stage two phases
//   ahead of its barrier, where a parity wait cannot tell the phases apart.
//   Per block and warp:  S[16 x 64] = Qpad[16 x D] K^T (q-heads in rows, zero padded),
//   fp32 online softmax in base 2, P rounded to the value dtype as the reference kernel
//   does (tasft/kernels/block_sparse_fa.py:252), O[16 x D] += P V.
//   Splits of one (sequence, kv-head) merge via decode_finish.
#include "decode.cuh"
#include "tc.cuh"

namespace tasft {
namespace {

constexpr int kConsumers = 1;
constexpr int kThreadsM = (kConsumers + 1) * 32;
constexpr int kStages = 2;
constexpr int kBlkM = 64;
constexpr float kLog2eM = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
template <bool kF16>
__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  if constexpr (kF16) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
}
__device__ __forceinline__ float ex2f(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
template <bool kF16>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  return kF16 ? tc::pack_f16x2(lo, hi) : tc::pack_bf16x2(lo, hi);
}

// byte offset of 16-byte chunk `c` (0 .. D/8-1) of tile row `r` in a 128B-swizzled tile
// made of D/64 regions of [64 rows x 128 B]
__device__ __forceinline__ uint32_t swz(int r, int c) {
  return (uint32_t)((c >> 3) * (kBlkM * 128) + r * 128 + (((c & 7) ^ (r & 7)) << 4));
}

template <int D, bool kF16>
__global__ void __launch_bounds__(kThreadsM, 3)
    bsa_decode_mma_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
                          const tasft_decode_args a, const DecodeWs ws, const int nsplit) {
  using T = typename std::conditional<kF16, __half, __nv_bfloat16>::type;
  constexpr int kTile = (D / 64) * kBlkM * 128;  // bytes of one K (or V) tile
  constexpr int kStage = 2 * kTile;
  constexpr int NT = kBlkM / 8;   // key n-tiles per block
  constexpr int KS = D / 16;      // k-steps over D
  constexpr int DT = D / 8;       // dim n-tiles of O
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * kStage);
  uint64_t* empty = full + kStages;
  __shared__ int s_last;

  const int unit = blockIdx.x / nsplit;
  const int split = blockIdx.x % nsplit;
  const int b = unit / a.Hk, hk = unit % a.Hk;
  const int grp = a.Hq / a.Hk;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cnt_all = a.kept_cnt[(int64_t)b * a.Hk + hk];
  const int t0 = (int)((int64_t)split * cnt_all / nsplit);
  const int t1 = (int)((int64_t)(split + 1) * cnt_all / nsplit);
  const int n = t1 - t0;
  const int32_t* list = a.kept_idx + ((int64_t)b * a.Hk + hk) * a.nb_max + t0;
  const int kvlen = min(a.kv_len[b], a.L);
  const int NBk = (a.L + kBlkM - 1) / kBlkM;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == kConsumers) {
    // ---------------- producer ----------------
    if (lane == 0) {
      tc::prefetch_tmap(&tmk);
      tc::prefetch_tmap(&tmv);
      int issued = 0;
      for (int i = 0; i < n; ++i) {
        const int s = i % kStages;
        if (i >= kStages && !mbar_wait(&empty[s], ((i / kStages) - 1) & 1)) {
          set_err(a.err, TASFT_DEVERR_TIMEOUT);
          break;
        }
        const int kb = list[i];
        if (kb >= 0 && kb < NBk) {
          uint8_t* sk = smem + s * kStage;
          mbar_arrive_expect_tx(&full[s], kStage);
#pragma unroll
          for (int c = 0; c < D / 64; ++c) {
            tc::tma_load_4d(sk + c * kBlkM * 128, &tmk, c * 64, kb * kBlkM, hk, b, &full[s]);
            tc::tma_load_4d(sk + kTile + c * kBlkM * 128, &tmv, c * 64, kb * kBlkM, hk, b, &full[s]);
          }
        } else {
          mbar_arrive(&full[s]);
        }
        ++issued;
      }
      for (int i = max(0, issued - kStages); i < issued; ++i) mbar_wait(&full[i % kStages], (i / kStages) & 1);
    }
  } else {
    // ---------------- consumers ----------------
    const int g = lane >> 2, tig = lane & 3;
    // Q as the A operand: rows = q-heads of the group (g and g + 8), zero padded
    uint32_t qa[KS][4];
    {
      const T* Q = reinterpret_cast<const T*>(a.q) + b * a.q_stride[0];
      const bool r0 = g < grp, r1 = g + 8 < grp;
      const T* q0 = Q + (int64_t)(hk * grp + g) * a.q_stride[1];
      const T* q1 = Q + (int64_t)(hk * grp + g + 8) * a.q_stride[1];
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
        const int d0 = ks * 16 + 2 * tig;
        qa[ks][0] = r0 ? *reinterpret_cast<const uint32_t*>(q0 + d0) : 0u;
        qa[ks][1] = r1 ? *reinterpret_cast<const uint32_t*>(q1 + d0) : 0u;
        qa[ks][2] = r0 ? *reinterpret_cast<const uint32_t*>(q0 + d0 + 8) : 0u;
        qa[ks][3] = r1 ? *reinterpret_cast<const uint32_t*>(q1 + d0 + 8) : 0u;
      }
    }
    const float sl2 = a.scale * kLog2eM;
    float o[DT][4];
#pragma unroll
    for (int t = 0; t < DT; ++t) o[t][0] = o[t][1] = o[t][2] = o[t][3] = 0.f;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;  // rows g, g + 8 (base 2)
    bool ok = true;
    for (int i = warp; i < n; i += kConsumers) {
      const int s = i % kStages;
      if (!__all_sync(0xffffffffu, mbar_wait(&full[s], (i / kStages) & 1))) {
        ok = false;
        set_err(a.err, TASFT_DEVERR_TIMEOUT);
        break;
      }
      const int kb = list[i];
      const bool kb_ok = kb >= 0 && kb < NBk;
      if (!kb_ok) {
        if (lane == 0) {
          set_err(a.err, TASFT_DEVERR_INDEX);
          mbar_arrive(&empty[s]);
        }
        continue;
      }
      const uint32_t kbase = smem_u32(smem + s * kStage);
      const uint32_t vbase = kbase + kTile;
      // ---- S = Q K^T ----
      float sc[NT][4];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
        const int row = nt * 8 + (lane & 7);
#pragma unroll
        for (int kp = 0; kp < KS / 2; ++kp) {
          uint32_t b0, b1, b2, b3;
          ldsm_x4(kbase + swz(row, kp * 4 + (lane >> 3)), b0, b1, b2, b3);
          mma16816<kF16>(sc[nt], qa[2 * kp], b0, b1);
          mma16816<kF16>(sc[nt], qa[2 * kp + 1], b2, b3);
        }
      }
      // ---- mask, scale, block max ----
      const int kp0 = kb * kBlkM;
      float mb0 = -INFINITY, mb1 = -INFINITY;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const bool valid = kp0 + nt * 8 + 2 * tig + e < kvlen;
          sc[nt][e] = valid ? sc[nt][e] * sl2 : -INFINITY;
          sc[nt][2 + e] = valid ? sc[nt][2 + e] * sl2 : -INFINITY;
          mb0 = fmaxf(mb0, sc[nt][e]);
          mb1 = fmaxf(mb1, sc[nt][2 + e]);
        }
      }
      mb0 = fmaxf(mb0, __shfl_xor_sync(0xffffffffu, mb0, 1));
      mb0 = fmaxf(mb0, __shfl_xor_sync(0xffffffffu, mb0, 2));
      mb1 = fmaxf(mb1, __shfl_xor_sync(0xffffffffu, mb1, 1));
      mb1 = fmaxf(mb1, __shfl_xor_sync(0xffffffffu, mb1, 2));
      const float mn0 = fmaxf(m0, mb0), mn1 = fmaxf(m1, mb1);
      const float al0 = mn0 == -INFINITY ? 1.f : ex2f(m0 - mn0);
      const float al1 = mn1 == -INFINITY ? 1.f : ex2f(m1 - mn1);
      m0 = mn0;
      m1 = mn1;
      l0 *= al0;
      l1 *= al1;
#pragma unroll
      for (int t = 0; t < DT; ++t) {
        o[t][0] *= al0;
        o[t][1] *= al0;
        o[t][2] *= al1;
        o[t][3] *= al1;
      }
      // ---- P (rounded to the value dtype) as A fragments ----
      uint32_t pa[KS > 0 ? kBlkM / 16 : 1][4];
#pragma unroll
      for (int ks = 0; ks < kBlkM / 16; ++ks) {
        float p[2][4];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int nt = 2 * ks + h;
          p[h][0] = mn0 == -INFINITY ? 0.f : ex2f(sc[nt][0] - mn0);
          p[h][1] = mn0 == -INFINITY ? 0.f : ex2f(sc[nt][1] - mn0);
          p[h][2] = mn1 == -INFINITY ? 0.f : ex2f(sc[nt][2] - mn1);
          p[h][3] = mn1 == -INFINITY ? 0.f : ex2f(sc[nt][3] - mn1);
          l0 += p[h][0] + p[h][1];
          l1 += p[h][2] + p[h][3];
        }
        pa[ks][0] = pack2<kF16>(p[0][0], p[0][1]);
        pa[ks][1] = pack2<kF16>(p[0][2], p[0][3]);
        pa[ks][2] = pack2<kF16>(p[1][0], p[1][1]);
        pa[ks][3] = pack2<kF16>(p[1][2], p[1][3]);
      }
      // ---- O += P V ----
#pragma unroll
      for (int ks = 0; ks < kBlkM / 16; ++ks) {
        const int row = ks * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
#pragma unroll
        for (int tp = 0; tp < DT / 2; ++tp) {
          uint32_t b0, b1, b2, b3;
          ldsm_x4_t(vbase + swz(row, 2 * tp + (lane >> 4)), b0, b1, b2, b3);
          mma16816<kF16>(o[2 * tp], pa[ks], b0, b1);
          mma16816<kF16>(o[2 * tp + 1], pa[ks], b2, b3);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
    // quad-reduce l (each thread summed its own columns)
    l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
    l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
    // ---- merge the two consumer warps in shared memory (reuses the ring) ----
    named_bar(1, kConsumers * 32);
    float* wbuf = reinterpret_cast<float*>(smem);  // [warps][16 rows][D + 2] : O (unnormalised), m, l
    float* res = wbuf + kConsumers * 16 * (D + 2);  // [grp][D + 2]
#pragma unroll
    for (int t = 0; t < DT; ++t) {
      const int c = t * 8 + 2 * tig;
      wbuf[(warp * 16 + g) * (D + 2) + c] = o[t][0];
      wbuf[(warp * 16 + g) * (D + 2) + c + 1] = o[t][1];
      wbuf[(warp * 16 + g + 8) * (D + 2) + c] = o[t][2];
      wbuf[(warp * 16 + g + 8) * (D + 2) + c + 1] = o[t][3];
    }
    if (tig == 0) {
      wbuf[(warp * 16 + g) * (D + 2) + D] = ok ? m0 : -INFINITY;
      wbuf[(warp * 16 + g) * (D + 2) + D + 1] = ok ? l0 : 0.f;
      wbuf[(warp * 16 + g + 8) * (D + 2) + D] = ok ? m1 : -INFINITY;
      wbuf[(warp * 16 + g + 8) * (D + 2) + D + 1] = ok ? l1 : 0.f;
    }
    named_bar(1, kConsumers * 32);
    const int tid = threadIdx.x;
    for (int x = tid; x < grp * (D + 2); x += kConsumers * 32) {
      const int r = x / (D + 2), d = x % (D + 2);
      float mt = -INFINITY;
#pragma unroll
      for (int w = 0; w < kConsumers; ++w) {
        const float* row = wbuf + (w * 16 + r) * (D + 2);
        if (row[D + 1] > 0.f) mt = fmaxf(mt, row[D]);
      }
      float num = 0.f, den = 0.f;
#pragma unroll
      for (int w = 0; w < kConsumers; ++w) {
        const float* row = wbuf + (w * 16 + r) * (D + 2);
        if (row[D + 1] > 0.f) {
          const float sc = ex2f(row[D] - mt);
          den += row[D + 1] * sc;
          if (d < D) num += row[d] * sc;
        }
      }
      float v;
      if (d < D) v = den > 0.f ? num / den : 0.f;
      else if (d == D) v = mt * kLn2;  // base-2 max -> base-e for the shared finish
      else v = den;
      res[x] = v;
    }
    named_bar(1, kConsumers * 32);
    decode_finish<T>(a, ws, nsplit, split, unit, b, hk, grp, res, tid, kConsumers * 32, 1, &s_last);
  }
  __syncwarp();
}

template <int D, bool kF16>
int launch_mma(const tasft_decode_args& a, const DecodeWs& ws, int nsplit, cudaStream_t st) {
  CUtensorMap mk, mv;
  if (!make_tmap_bhsd(&mk, a.k_cache, a.B, a.Hk, a.L, D, a.k_stride, 2, kBlkM) ||
      !make_tmap_bhsd(&mv, a.v_cache, a.B, a.Hk, a.L, D, a.v_stride, 2, kBlkM)) {
    if (debug_enabled()) debug_log("decode: tensor map rejected, using the CUDA-core kernel");
    return TASFT_ERR_UNSUPPORTED;
  }
  constexpr int kStage = 2 * (D / 64) * kBlkM * 128;
  const int wbuf = (kConsumers * 16 + 16) * (D + 2) * 4;
  const int ring = kStages * kStage;
  const int smem = 1024 + (ring > wbuf ? ring : wbuf) + 2 * kStages * 8;
  auto kern = bsa_decode_mma_kernel<D, kF16>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return TASFT_ERR_CUDA;
  cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
  const int64_t grid = (int64_t)a.B * a.Hk * nsplit;
  if (debug_enabled()) debug_log("decode_mma D=%d f16=%d grid=%lld smem=%d splits=%d", D, (int)kF16, (long long)grid, smem, nsplit);
  kern<<<(unsigned)grid, kThreadsM, smem, st>>>(mk, mv, a, ws, nsplit);
  count_launch();
  return launch_status();
}

}  // namespace

int decode_mma(const tasft_decode_args& a, const DecodeWs& ws, int nsplit, cudaStream_t st) {
  if (a.dtype != TASFT_BF16 && a.dtype != TASFT_F16) return TASFT_ERR_UNSUPPORTED;
  if (a.block != kBlkM || (a.D != 64 && a.D != 128)) return TASFT_ERR_UNSUPPORTED;
  if (a.Hq / a.Hk > 16) return TASFT_ERR_UNSUPPORTED;
  // Q fragments are read as aligned 32-bit pairs
  if ((reinterpret_cast<uintptr_t>(a.q) & 3u) || (a.q_stride[0] & 1) || (a.q_stride[1] & 1)) return TASFT_ERR_UNSUPPORTED;
  const bool f16 = a.dtype == TASFT_F16;
  if (a.D == 128) return f16 ? launch_mma<128, true>(a, ws, nsplit, st) : launch_mma<128, false>(a, ws, nsplit, st);
  return f16 ? launch_mma<64, true>(a, ws, nsplit, st) : launch_mma<64, false>(a, ws, nsplit, st);
}

}  // namespace tasft
