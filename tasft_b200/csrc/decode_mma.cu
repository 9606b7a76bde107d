// Block-sparse decode for bf16/fp16 caches on tensor-core fragments (mma.sync).
//
// Decode is HBM-bound: every kept KV byte is read once and used by the few q-heads of
// its GQA group. The tensor cores are used only to keep the instruction count per byte
// small (CUDA-core dot products with shuffle reductions issued ~14K warp instructions
// per 32 KB block; this path issues a few hundred).
//
//   Persistent CTAs (every resident slot, 6 per SM), 2 warps each: warp 1 = TMA
//   producer, warp 0 = the one consumer. Work items are (sequence, kv-head, split)
//   slices of the kept lists; the producer claims them from a counter in the workspace
//   (dynamic balance; a static stride when there is no workspace), tags every ring entry
//   with (item, half-block) and streams all items through one ring, so the pipeline never
//   drains between items. K/V half-blocks (32 keys) arrive in a 2-stage ring of
//   128B-swizzled TMA boxes, so ldmatrix reads are conflict free. A single in-order
//   consumer per ring keeps every mbarrier parity wait exact: with several consumers
//   taking turns on a shared ring, a fast one can reach a stage two phases ahead of its
//   barrier, where a parity wait cannot tell the phases apart.
//   Per stage: S^T[32 keys x 8 heads] = K Q^T (keys in the MMA's M, the group's q-heads
//   in N), fp32 online softmax in base 2, P rounded to the value dtype as the reference
//   kernel does (tasft/kernels/block_sparse_fa.py:252) and turned into the B operand with
//   movmatrix.trans, O^T[D x 8] += V^T P^T. Splits of one (sequence, kv-head) merge
//   through an atomic ticket: the last split to finish merges all partials.
#include "decode.cuh"
#include "tc.cuh"
#include "peer.cuh"

namespace tasft {
namespace {

constexpr int kThreadsM = 64;    // warp 0 consumer, warp 1 producer
constexpr int kStages = 2;
constexpr int kBlkM = 64;        // kv block (list granularity)
constexpr int kSub = 32;         // keys per ring stage (half a block)
constexpr int kCtasPerSm = 6;
// up to this many splits the last split of a unit merges them (one warp); above it a
// separate merge kernel does (decode_merge_kernel)
constexpr int kInlineMergeMaxSplits = 16;
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
// made of D/64 regions of [32 rows x 128 B]
__device__ __forceinline__ uint32_t swz32(int r, int c) {
  return (uint32_t)((c >> 3) * (kSub * 128) + r * 128 + (((c & 7) ^ (r & 7)) << 4));
}

// Ring-entry tag written by the producer before it arms the stage's barrier; the
// mbarrier arrive (release) / wait (acquire) pair makes it visible to the consumer.
struct Tag {
  int item;  // work item (unit * nsplit + split); -1 = no more work
  int j;     // stage index within the item (two 32-key halves per kept block)
  int n;     // stages in the item (0: empty item, finish only)
  int kb;    // kv block index; the half is j & 1
};

// Claim the next work item: a global counter when the workspace provides one (dynamic
// balance), else a static stride over the grid.
__device__ __forceinline__ int next_item(int32_t* ctr, int& k, int items) {
  int it;
  if (ctr) {
    it = atomicAdd(ctr, 1);
    if (it >= items) {
      // the last CTA to run out resets both counters for the next launch
      if (atomicAdd(ctr + 1, 1) == (int)gridDim.x - 1) {
        atomicExch(ctr, 0);
        atomicExch(ctr + 1, 0);
      }
      return -1;
    }
    return it;
  }
  it = blockIdx.x + (k++) * gridDim.x;
  return it < items ? it : -1;
}

// Page-pool geometry of a paged cache (unused by the contiguous kernel).
struct PagedInfo {
  const int32_t* table;  // [B, max_pages] physical page of each logical page
  int max_pages, page_size, num_pages;
};

__device__ __forceinline__ uint32_t movm_t(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}

template <int D, bool kF16, bool kPaged>
__global__ void __launch_bounds__(kThreadsM, kCtasPerSm)
    bsa_decode_mma_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
                          const tasft_decode_args a, const DecodeWs ws, const int nsplit, const PagedInfo pg,
                          const int merge_inline) {
  using T = typename std::conditional<kF16, __half, __nv_bfloat16>::type;
  constexpr int kTile = (D / 64) * kSub * 128;  // bytes of one K (or V) half-block tile
  constexpr int kStage = 2 * kTile;
  constexpr int KS = D / 16;   // k-steps over D (S^T = K Q^T)
  constexpr int MD = D / 16;   // m-tiles over D (O^T = V^T P^T)
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * kStage);
  uint64_t* empty = full + kStages;
  Tag* tags = reinterpret_cast<Tag*>(empty + kStages);

  const int grp = a.Hq / a.Hk;
  const int items = a.B * a.Hk * nsplit;
  const int NBk = (a.L + kBlkM - 1) / kBlkM;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // dynamic claiming only pays when there are more items than resident CTAs
  int32_t* ctr = (ws.ticket && items > (int)gridDim.x) ? ws.ticket + (int64_t)a.B * a.Hk : nullptr;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    fence_barrier_init();
  }
  __syncthreads();
  // a merge kernel launched behind this one (wide splits) may start its CTAs now; they
  // wait for this grid to complete before reading the partials
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  if (warp == 1) {
    // ---------------- producer: streams every claimed item's half-blocks ----------------
    if (lane == 0) {
      tc::prefetch_tmap(&tmk);
      tc::prefetch_tmap(&tmv);
      int r = 0, k = 0;
      bool alive = true;
      auto push = [&](const Tag& t) -> bool {
        const int s = r % kStages;
        if (r >= kStages && !mbar_wait(&empty[s], ((r / kStages) - 1) & 1)) {
          set_err(a.err, TASFT_DEVERR_TIMEOUT);
          return false;
        }
        Tag tt = t;
        bool load = t.item >= 0 && t.n > 0 && t.kb >= 0 && t.kb < NBk;
        const int unit = t.item >= 0 ? t.item / nsplit : 0;
        const int b = unit / a.Hk, hk = unit % a.Hk;
        const int row = t.kb * kBlkM + (t.j & 1) * kSub;  // logical token of the stage's first key
        int pages[2] = {0, 0};                            // physical page(s) of the stage (paged)
        if constexpr (kPaged) {
          if (load) {
            // a 32-key stage spans one page (page_size >= 32) or two 16-token pages
            const int np = pg.page_size >= kSub ? 1 : kSub / pg.page_size;
            for (int i = 0; i < np; ++i) {
              const int lp = (row + i * pg.page_size) / pg.page_size;
              const int ph = lp < pg.max_pages ? pg.table[(int64_t)b * pg.max_pages + lp] : -1;
              if (ph < 0 || ph >= pg.num_pages) load = false;
              pages[i] = ph;
            }
            if (!load) {
              set_err(a.err, TASFT_DEVERR_INDEX);
              tt.kb = -1;  // the consumer skips the stage
            }
          }
        }
        tags[s] = tt;
        if (load) {
          uint8_t* sk = smem + s * kStage;
          mbar_arrive_expect_tx(&full[s], kStage);
#pragma unroll
          for (int c = 0; c < D / 64; ++c) {
            if constexpr (kPaged) {
              if (pg.page_size >= kSub) {
                const int off = row % pg.page_size;
                tc::tma_load_4d(sk + c * kSub * 128, &tmk, c * 64, hk, off, pages[0], &full[s]);
                tc::tma_load_4d(sk + kTile + c * kSub * 128, &tmv, c * 64, hk, off, pages[0], &full[s]);
              } else {
#pragma unroll
                for (int i = 0; i < 2; ++i) {
                  tc::tma_load_4d(sk + c * kSub * 128 + i * 16 * 128, &tmk, c * 64, hk, 0, pages[i], &full[s]);
                  tc::tma_load_4d(sk + kTile + c * kSub * 128 + i * 16 * 128, &tmv, c * 64, hk, 0, pages[i],
                                  &full[s]);
                }
              }
            } else {
              tc::tma_load_4d(sk + c * kSub * 128, &tmk, c * 64, row, hk, b, &full[s]);
              tc::tma_load_4d(sk + kTile + c * kSub * 128, &tmv, c * 64, row, hk, b, &full[s]);
            }
          }
        } else {
          mbar_arrive(&full[s]);
        }
        ++r;
        return true;
      };
      // claim one item ahead so the counter's round trip overlaps the current pushes
      int nxt = next_item(ctr, k, items);
      while (alive) {
        const int it = nxt;
        if (it < 0) {
          push(Tag{-1, 0, 0, -1});
          break;
        }
        nxt = next_item(ctr, k, items);
        const int unit = it / nsplit, split = it % nsplit;
        const int cnt_all = a.kept_cnt[unit];
        const int t0 = (int)((int64_t)split * cnt_all / nsplit);
        const int n = (int)((int64_t)(split + 1) * cnt_all / nsplit) - t0;
        const int32_t* list = a.kept_idx + (int64_t)unit * a.nb_max + t0;
        if (n == 0) {
          alive = push(Tag{it, 0, 0, -1});
        } else {
          for (int j = 0; j < 2 * n && alive; ++j) alive = push(Tag{it, j, 2 * n, list[j >> 1]});
        }
      }
      for (int i = max(0, r - kStages); i < r; ++i) mbar_wait(&full[i % kStages], (i / kStages) & 1);
    }
  } else {
    // ---------------- consumer: follows the tags ----------------
    // Thread (g, tig) = (lane / 4, lane % 4) owns q-heads 2 tig and 2 tig + 1 (columns of
    // S^T and O^T), keys g and g + 8 of each 16-key m-tile, dims g and g + 8 of each
    // 16-dim m-tile of O^T.
    const int g = lane >> 2, tig = lane & 3;
    const float sl2 = a.scale * kLog2eM;
    uint32_t qb[KS][2];   // Q^T as the B operand: [D x 8 heads]
    float o[MD][4];       // O^T accumulators
    float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
    int cur = -1, kvlen = 0;
    for (int r = 0;; ++r) {
      const int s = r % kStages;
      if (!__all_sync(0xffffffffu, mbar_wait(&full[s], (r / kStages) & 1))) {
        set_err(a.err, TASFT_DEVERR_TIMEOUT);
        break;
      }
      const Tag t = tags[s];
      if (t.item < 0) break;
      const int unit = t.item / nsplit, split = t.item % nsplit;
      const int b = unit / a.Hk, hk = unit % a.Hk;
      if (t.item != cur) {
        cur = t.item;
        kvlen = max(0, min(a.kv_len[b] - a.kv_offset, a.L));
        const T* qh = reinterpret_cast<const T*>(a.q) + b * a.q_stride[0] + (int64_t)(hk * grp + g) * a.q_stride[1];
        const bool hv = g < grp;
#pragma unroll
        for (int ks = 0; ks < KS; ++ks) {
          qb[ks][0] = hv ? *reinterpret_cast<const uint32_t*>(qh + ks * 16 + 2 * tig) : 0u;
          qb[ks][1] = hv ? *reinterpret_cast<const uint32_t*>(qh + ks * 16 + 8 + 2 * tig) : 0u;
        }
#pragma unroll
        for (int x = 0; x < MD; ++x) o[x][0] = o[x][1] = o[x][2] = o[x][3] = 0.f;
        m[0] = m[1] = -INFINITY;
        l[0] = l[1] = 0.f;
      }
      const bool kb_ok = t.n > 0 && t.kb >= 0 && t.kb < NBk;
      if (t.n > 0 && !kb_ok && lane == 0 && (t.j & 1) == 0) set_err(a.err, TASFT_DEVERR_INDEX);
      if (kb_ok) {
        const uint32_t kbase = smem_u32(smem + s * kStage);
        const uint32_t vbase = kbase + kTile;
        // ---- S^T [32 keys x 8 heads] = K Q^T ----
        float sc[2][4];
#pragma unroll
        for (int mt = 0; mt < 2; ++mt) {
          sc[mt][0] = sc[mt][1] = sc[mt][2] = sc[mt][3] = 0.f;
          const int row = mt * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
#pragma unroll
          for (int ks = 0; ks < KS; ++ks) {
            uint32_t af[4];
            ldsm_x4(kbase + swz32(row, 2 * ks + (lane >> 4)), af[0], af[1], af[2], af[3]);
            mma16816<kF16>(sc[mt], af, qb[ks][0], qb[ks][1]);
          }
        }
        // ---- mask, scale, per-head max over the 32 keys ----
        const int key0 = t.kb * kBlkM + (t.j & 1) * kSub;
        float mb[2] = {-INFINITY, -INFINITY};
#pragma unroll
        for (int mt = 0; mt < 2; ++mt) {
#pragma unroll
          for (int h = 0; h < 2; ++h) {  // h: key g (c0, c1) or key g + 8 (c2, c3)
            const bool valid = key0 + mt * 16 + g + 8 * h < kvlen;
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              float& v = sc[mt][2 * h + e];
              v = valid ? v * sl2 : -INFINITY;
              mb[e] = fmaxf(mb[e], v);
            }
          }
        }
#pragma unroll
        for (int e = 0; e < 2; ++e) {
#pragma unroll
          for (int off = 4; off < 32; off <<= 1) mb[e] = fmaxf(mb[e], __shfl_xor_sync(0xffffffffu, mb[e], off));
        }
        float mn[2], al[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          mn[e] = fmaxf(m[e], mb[e]);
          al[e] = mn[e] == -INFINITY ? 1.f : ex2f(m[e] - mn[e]);
          m[e] = mn[e];
          l[e] *= al[e];
        }
#pragma unroll
        for (int x = 0; x < MD; ++x) {
          o[x][0] *= al[0];
          o[x][1] *= al[1];
          o[x][2] *= al[0];
          o[x][3] *= al[1];
        }
        // ---- P^T (rounded to the value dtype) as B fragments via 8x8 transposes ----
        uint32_t pb[2][2];
#pragma unroll
        for (int mt = 0; mt < 2; ++mt) {
          float p[4];
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4) {
            const int e = q4 & 1;
            p[q4] = mn[e] == -INFINITY ? 0.f : ex2f(sc[mt][q4] - mn[e]);
            l[e] += p[q4];
          }
          pb[mt][0] = movm_t(pack2<kF16>(p[0], p[1]));  // keys 0-7 of the m-tile
          pb[mt][1] = movm_t(pack2<kF16>(p[2], p[3]));  // keys 8-15
        }
        // ---- O^T [D x 8 heads] += V^T P^T ----
#pragma unroll
        for (int md = 0; md < MD; ++md) {
#pragma unroll
          for (int kk = 0; kk < 2; ++kk) {
            const int row = kk * 16 + (lane & 7) + (lane >> 4) * 8;
            uint32_t af[4];
            ldsm_x4_t(vbase + swz32(row, 2 * md + ((lane >> 3) & 1)), af[0], af[1], af[2], af[3]);
            mma16816<kF16>(o[md], af, pb[kk][0], pb[kk][1]);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
      if (t.n > 0 && t.j != t.n - 1) continue;
      // ---- item done: warp-level finish (no shared memory) ----
      float L[2], inv[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        L[e] = l[e];
#pragma unroll
        for (int off = 4; off < 32; off <<= 1) L[e] += __shfl_xor_sync(0xffffffffu, L[e], off);
        inv[e] = L[e] > 0.f ? 1.f / L[e] : 0.f;
      }
      if (nsplit == 1) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int hh = 2 * tig + e;
          if (hh >= grp) continue;
          const int hq = hk * grp + hh;
          const int64_t row = (int64_t)b * a.Hq + hq;
#pragma unroll
          for (int md = 0; md < MD; ++md) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const int d = md * 16 + g + 8 * h;
              const float v = o[md][2 * h + e] * inv[e];
              if (a.out) reinterpret_cast<T*>(a.out)[b * a.o_stride[0] + hq * a.o_stride[1] + d] = from_f<T>(v);
              if (a.part_o) a.part_o[row * D + d] = v;
            }
          }
          if (a.part_ml && g == 0) {
            a.part_ml[row * 2] = m[e] * kLn2;
            a.part_ml[row * 2 + 1] = L[e];
          }
        }
        continue;
      }
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int hh = 2 * tig + e;
        if (hh >= grp) continue;
        float* pr = ws.part + (((int64_t)b * a.Hq + hk * grp + hh) * ws.max_splits + split) * (D + 2);
#pragma unroll
        for (int md = 0; md < MD; ++md) {
          pr[md * 16 + g] = o[md][e] * inv[e];
          pr[md * 16 + g + 8] = o[md][2 + e] * inv[e];
        }
        if (g == 0) {
          pr[D] = m[e] * kLn2;
          pr[D + 1] = L[e];
        }
      }
      if (!merge_inline) continue;  // wide splits: decode_merge_kernel merges after this grid
      __threadfence();
      __syncwarp();
      int last = 0;
      if (lane == 0) {
        last = atomicAdd(&ws.ticket[unit], 1) == nsplit - 1;
        if (last) ws.ticket[unit] = 0;  // ready for the next call
      }
      last = __shfl_sync(0xffffffffu, last, 0);
      if (!last) continue;
      __threadfence();
      // merge, per q-head row: the max over the splits (lanes over splits), then chunks
      // of 16 splits whose partial rows are all loaded before any is used (independent
      // 8-byte loads, lane -> d = 2 lane + 64 i), weighted by shuffle
      for (int gg = 0; gg < grp; ++gg) {
        const int64_t row = (int64_t)b * a.Hq + hk * grp + gg;
        const float* pr = ws.part + row * ws.max_splits * (D + 2);
        float mt = -INFINITY;
        for (int sp = lane; sp < nsplit; sp += 32)
          if (__ldcg(pr + sp * (D + 2) + D + 1) > 0.f) mt = fmaxf(mt, __ldcg(pr + sp * (D + 2) + D));
        mt = warp_max(mt);
        constexpr int DP = D / 64;  // float2 per lane per split
        float2 num[DP];
#pragma unroll
        for (int i = 0; i < DP; ++i) num[i] = make_float2(0.f, 0.f);
        float den = 0.f;
        for (int base = 0; base < nsplit; base += 16) {
          const int nb = min(16, nsplit - base);
          float w = 0.f;  // lane j (< nb) holds split base + j's weight
          if (lane < nb) {
            const float lv = __ldcg(pr + (base + lane) * (D + 2) + D + 1);
            if (lv > 0.f) w = lv * __expf(__ldcg(pr + (base + lane) * (D + 2) + D) - mt);
          }
          den += w;
          float2 v[16][DP];
#pragma unroll
          for (int j = 0; j < 16; ++j)
#pragma unroll
            for (int i = 0; i < DP; ++i)
              v[j][i] = j < nb ? __ldcg(reinterpret_cast<const float2*>(pr + (base + j) * (D + 2) + i * 64) + lane)
                               : make_float2(0.f, 0.f);
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const float wj = __shfl_sync(0xffffffffu, w, j);
#pragma unroll
            for (int i = 0; i < DP; ++i) {
              num[i].x = fmaf(wj, v[j][i].x, num[i].x);
              num[i].y = fmaf(wj, v[j][i].y, num[i].y);
            }
          }
        }
        den = warp_sum(den);
        const float inv_den = den > 0.f ? 1.f / den : 0.f;
#pragma unroll
        for (int i = 0; i < DP; ++i) {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int d = i * 64 + 2 * lane + h;
            const float ov = (h ? num[i].y : num[i].x) * inv_den;
            if (a.out) reinterpret_cast<T*>(a.out)[b * a.o_stride[0] + (hk * grp + gg) * a.o_stride[1] + d] = from_f<T>(ov);
            if (a.part_o) a.part_o[row * D + d] = ov;
          }
        }
        if (a.part_ml && lane == 0) {
          a.part_ml[row * 2] = mt;
          a.part_ml[row * 2 + 1] = den;
        }
      }
    }
  }
  __syncwarp();
}

// Merge of wide splits: one CTA per q-head row, launched behind the decode grid with
// programmatic dependent launch (its CTAs are resident early and wait on the grid). Warp w
// takes splits w, w + 4, ...; lane l holds d = 64 i + 2 l + {0, 1} (8-byte loads: a
// partial row is D + 2 floats, so rows are only 8-byte aligned). A warp loads up to 16 of
// its partial rows at once, merges them against its own running max, and the four warps'
// results are rescaled to the common max in shared memory, so the row costs one round
// trip to L2 per 64 splits. Same maths as the in-kernel merge:
// o = sum_s l_s e^(m_s - m) o_s / sum_s l_s e^(m_s - m).
constexpr int kMergeThreads = 128;
constexpr int kMaxPeerWorld = 8;  // ranks of one NVLink node (tasft_bsa_decode_peer_fwd checks)

template <int D, bool kF16>
__global__ void __launch_bounds__(kMergeThreads) decode_merge_kernel(const tasft_decode_args a, const DecodeWs ws,
                                                                      const int nsplit, const PeerMode pm) {
  using T = typename std::conditional<kF16, __half, __nv_bfloat16>::type;
  constexpr int kW = kMergeThreads / 32;
  constexpr int DP = D / 64;  // float2 per lane
  constexpr int kBatch = 16;  // partial rows a warp has in flight
  __shared__ float s_max[kW];
  __shared__ float s_num[kW][D];
  __shared__ float s_den[kW];
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int64_t row = blockIdx.x;  // b * Hq + hq
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float* pr = ws.part + row * ws.max_splits * (D + 2);
  float mw = -INFINITY, den = 0.f;
  float2 num[DP];
#pragma unroll
  for (int i = 0; i < DP; ++i) num[i] = make_float2(0.f, 0.f);
  for (int s0 = warp; s0 < nsplit; s0 += kBatch * kW) {
    float lv[kBatch], mv[kBatch];
    float2 v[kBatch][DP];
#pragma unroll
    for (int k = 0; k < kBatch; ++k) {
      const int sp = s0 + k * kW;
      lv[k] = 0.f;
      mv[k] = -INFINITY;
      if (sp < nsplit) {
        const float* ps = pr + sp * (D + 2);
        lv[k] = __ldcg(ps + D + 1);
        mv[k] = __ldcg(ps + D);
#pragma unroll
        for (int i = 0; i < DP; ++i) v[k][i] = __ldcg(reinterpret_cast<const float2*>(ps + i * 64) + lane);
      }
    }
    float mb = mw;
#pragma unroll
    for (int k = 0; k < kBatch; ++k)
      if (lv[k] > 0.f) mb = fmaxf(mb, mv[k]);
    if (mb == -INFINITY) continue;  // nothing kept in these splits yet
    const float sc = mw == -INFINITY ? 0.f : __expf(mw - mb);  // rescale what came before
    den *= sc;
#pragma unroll
    for (int i = 0; i < DP; ++i) {
      num[i].x *= sc;
      num[i].y *= sc;
    }
    mw = mb;
#pragma unroll
    for (int k = 0; k < kBatch; ++k) {
      if (!(lv[k] > 0.f)) continue;
      const float w = lv[k] * __expf(mv[k] - mw);
      den += w;
#pragma unroll
      for (int i = 0; i < DP; ++i) {
        num[i].x = fmaf(w, v[k][i].x, num[i].x);
        num[i].y = fmaf(w, v[k][i].y, num[i].y);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < DP; ++i) {
    s_num[warp][i * 64 + 2 * lane] = num[i].x;
    s_num[warp][i * 64 + 2 * lane + 1] = num[i].y;
  }
  if (lane == 0) {
    s_max[warp] = mw;
    s_den[warp] = den;
  }
  __syncthreads();
  float mt = -INFINITY;
#pragma unroll
  for (int w = 0; w < kW; ++w) mt = fmaxf(mt, s_max[w]);
  float scw[kW];
  float dt = 0.f;
#pragma unroll
  for (int w = 0; w < kW; ++w) {
    scw[w] = s_max[w] == -INFINITY ? 0.f : __expf(s_max[w] - mt);
    dt += scw[w] * s_den[w];
  }
  const float inv = dt > 0.f ? 1.f / dt : 0.f;
  const int b = (int)(row / a.Hq), hq = (int)(row % a.Hq);
  if (pm.world == 0) {
    for (int d = threadIdx.x; d < D; d += kMergeThreads) {
      float t = 0.f;
#pragma unroll
      for (int w = 0; w < kW; ++w) t += scw[w] * s_num[w][d];
      const float ov = t * inv;
      if (a.out) reinterpret_cast<T*>(a.out)[b * a.o_stride[0] + hq * a.o_stride[1] + d] = from_f<T>(ov);
      if (a.part_o) a.part_o[row * D + d] = ov;
    }
    if (a.part_ml && threadIdx.x == 0) {
      a.part_ml[row * 2] = mt;
      a.part_ml[row * 2 + 1] = dt;
    }
    return;
  }
  // ---- cross-GPU exchange of this row (tasft_bsa_decode_peer_fwd; mailbox layout in
  //      peer.cuh): every value of the row's (o, m, l) goes to slot [parity][rank][row] of
  //      every rank's mailbox as one 8-byte word (value | epoch << 32); then each thread
  //      spins (bounded) on the words it needs in this rank's mailbox until they carry this
  //      call's epoch, and merges as tasft_bsa_decode_combine does. No fence, no flag: a word
  //      is published by the store that writes it ----
  const int world = pm.world, rank = pm.rank;
  const int64_t rows = (int64_t)a.B * a.Hq;
  const uint32_t e = *pm.epoch + 1u;
  const int par = (int)(e & 1u);
  const int64_t woff = peer_word_off(world);
  const uint64_t tag = (uint64_t)e << 32;
  for (int d = threadIdx.x; d < D + 2; d += kMergeThreads) {
    float v;
    if (d < D) {
      float t = 0.f;
#pragma unroll
      for (int w = 0; w < kW; ++w) t += scw[w] * s_num[w][d];
      v = t * inv;
    } else {
      v = d == D ? mt : dt;
    }
    const uint64_t word = tag | __float_as_uint(v);
    for (int p = 0; p < world; ++p)
      st_relaxed_sys_u64(reinterpret_cast<uint64_t*>(pm.mailboxes[p]) + woff +
                             (((int64_t)par * world + rank) * rows + row) * (D + 2) + d,
                         word);
  }
  const uint64_t* box = reinterpret_cast<const uint64_t*>(pm.mailboxes[rank]) + woff;
  const uint64_t t0 = globaltimer_ns();
  bool timed_out = false;
  // a word of this call, spinning until it arrives (0 after the bound)
  auto fetch = [&](int g, int d) -> float {
    const uint64_t* src = box + (((int64_t)par * world + g) * rows + row) * (D + 2) + d;
    uint64_t v = ld_relaxed_sys_u64(src);
    while ((uint32_t)(v >> 32) != e) {
      if (timed_out || globaltimer_ns() - t0 > pm.timeout_ns) {
        timed_out = true;
        return 0.f;
      }
      v = ld_relaxed_sys_u64(src);
    }
    return __uint_as_float((uint32_t)v);
  };
  float gm[kMaxPeerWorld], gl[kMaxPeerWorld];
  float gmax = -INFINITY;
  for (int g = 0; g < world; ++g) {
    gm[g] = fetch(g, D);
    gl[g] = fetch(g, D + 1);
    if (gl[g] > 0.f) gmax = fmaxf(gmax, gm[g]);
  }
  for (int d = threadIdx.x; d < D; d += kMergeThreads) {
    float num = 0.f, den = 0.f;
    for (int g = 0; g < world; ++g) {
      const float ov = fetch(g, d);
      if (gl[g] > 0.f) {
        const float w = gl[g] * __expf(gm[g] - gmax);
        num = fmaf(w, ov, num);
        den += w;
      }
    }
    if (a.out) reinterpret_cast<T*>(a.out)[b * a.o_stride[0] + hq * a.o_stride[1] + d] = from_f<T>(den > 0.f ? num / den : 0.f);
  }
  if (timed_out) set_err(a.err, TASFT_DEVERR_TIMEOUT);
  // the last row's CTA to finish advances the epoch (every CTA read it on entry)
  __syncthreads();
  if (threadIdx.x == 0) {
    int* done = reinterpret_cast<int*>(pm.mailboxes[rank]) + world;  // call flags' spare word
    if (atomicAdd(done, 1) == (int)gridDim.x - 1) {
      *done = 0;
      __threadfence();
      *pm.epoch = e;
    }
  }
}

template <int D, bool kF16, bool kPaged>
int launch_mma(const tasft_decode_args& a, const DecodeWs& ws, int nsplit, const PagedInfo& pg, cudaStream_t st,
               const PeerMode& pm) {
  CUtensorMap mk, mv;
  bool maps;
  if constexpr (kPaged) {
    const int rows = pg.page_size >= kSub ? kSub : pg.page_size;
    maps = make_tmap_paged(&mk, a.k_cache, pg.num_pages, pg.page_size, a.Hk, D, a.k_stride, rows) &&
           make_tmap_paged(&mv, a.v_cache, pg.num_pages, pg.page_size, a.Hk, D, a.v_stride, rows);
  } else {
    maps = make_tmap_bhsd(&mk, a.k_cache, a.B, a.Hk, a.L, D, a.k_stride, 2, kSub) &&
           make_tmap_bhsd(&mv, a.v_cache, a.B, a.Hk, a.L, D, a.v_stride, 2, kSub);
  }
  if (!maps) {
    if (debug_enabled()) debug_log("decode: tensor map rejected");
    return TASFT_ERR_UNSUPPORTED;
  }
  constexpr int kStage = 2 * (D / 64) * kSub * 128;
  const int smem = 1024 + kStages * kStage + 2 * kStages * 8 + kStages * (int)sizeof(Tag);
  auto kern = bsa_decode_mma_kernel<D, kF16, kPaged>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return TASFT_ERR_CUDA;
  cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
  // persistent grid: every resident CTA slot, never more CTAs than work items
  int dev = 0, sms = 148, per_sm = 1;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreadsM, smem);
  const int64_t items = (int64_t)a.B * a.Hk * nsplit;
  int64_t grid = (int64_t)sms * (per_sm > 0 ? per_sm : 1);
  if (grid > items) grid = items;
  if (debug_enabled())
    debug_log("decode_mma D=%d f16=%d paged=%d grid=%lld smem=%d splits=%d", D, (int)kF16, (int)kPaged,
              (long long)grid, smem, nsplit);
  const int inline_merge = nsplit <= kInlineMergeMaxSplits && pm.world == 0;
  kern<<<(unsigned)grid, kThreadsM, smem, st>>>(mk, mv, a, ws, nsplit, pg, inline_merge);
  count_launch();
  if (inline_merge) return launch_status();
  // wide splits: the merge kernel, its launch overlapped with the decode grid
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(a.B * a.Hq));
  cfg.blockDim = dim3(kMergeThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, decode_merge_kernel<D, kF16>, a, ws, nsplit, pm) != cudaSuccess) return launch_status();
  count_launch();
  return launch_status();
}

bool mma_ok(const tasft_decode_args& a) {
  if (a.dtype != TASFT_BF16 && a.dtype != TASFT_F16) return false;
  if (a.block != kBlkM || (a.D != 64 && a.D != 128)) return false;
  if (a.Hq / a.Hk > 8) return false;  // q-heads of a group fill the MMA's N = 8
  // Q fragments are read as aligned 32-bit pairs
  if ((reinterpret_cast<uintptr_t>(a.q) & 3u) || (a.q_stride[0] & 1) || (a.q_stride[1] & 1)) return false;
  return true;
}

template <bool kPaged>
int dispatch(const tasft_decode_args& a, const DecodeWs& ws, int nsplit, const PagedInfo& pg, cudaStream_t st,
             const PeerMode& pm) {
  if (!mma_ok(a)) return TASFT_ERR_UNSUPPORTED;
  const bool f16 = a.dtype == TASFT_F16;
  if (a.D == 128)
    return f16 ? launch_mma<128, true, kPaged>(a, ws, nsplit, pg, st, pm)
               : launch_mma<128, false, kPaged>(a, ws, nsplit, pg, st, pm);
  return f16 ? launch_mma<64, true, kPaged>(a, ws, nsplit, pg, st, pm)
             : launch_mma<64, false, kPaged>(a, ws, nsplit, pg, st, pm);
}

}  // namespace

bool decode_mma_ok(const tasft_decode_args& a) { return mma_ok(a); }

int decode_mma(const tasft_decode_args& a, const DecodeWs& ws, int nsplit, cudaStream_t st, const PeerMode& pm) {
  return dispatch<false>(a, ws, nsplit, PagedInfo{nullptr, 0, 0, 0}, st, pm);
}

int decode_mma_paged(const tasft_decode_args& a, const DecodeWs& ws, int nsplit, const int32_t* table, int max_pages,
                     int page_size, int num_pages, cudaStream_t st) {
  return dispatch<true>(a, ws, nsplit, PagedInfo{table, max_pages, page_size, num_pages}, st,
                       PeerMode{nullptr, nullptr, 0, 0, 0});
}

}  // namespace tasft
