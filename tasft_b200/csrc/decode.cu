// Block-sparse decode: one query token per sequence attends over the kept KV blocks
// of its kv-head. New capability (the reference has no sparse decode; it delegates
// decode to vLLM's dense forward, tasft/inference/vllm_patch.py:189-196).
//
// HBM-bound design. One CTA = one (sequence, kv-head, split) unit: a contiguous
// slice of that kv-head's kept-block list. A producer warp streams each kept block's
// K and V rows (contiguous in the [B, Hk, L, D] cache) into a shared-memory ring with
// cp.async.bulk (one instruction per tensor per block, completion on an mbarrier);
// four consumer warps score all q-heads of the GQA group against the block
// (16-byte vector reads, half-warp per key at D=128 bf16), take the block max, then
// accumulate p.V. All consumer warps share the running max, so their partial sums add
// without rescaling. Splits of one unit are merged by the last CTA to finish
// (an atomic ticket; no CTA ever waits on another).
#include "decode.cuh"

namespace tasft {

constexpr int kDecConsumerWarps = 4;
constexpr int kDecThreads = (kDecConsumerWarps + 1) * 32;
constexpr int kGmax = 8;  // max q-heads per kv-head handled by one CTA

template <typename T, int D>
__global__ void __launch_bounds__(kDecThreads) bsa_decode_simt_kernel(tasft_decode_args a, DecodeWs ws, int nsplit,
                                                                 int nst) {
  constexpr int EPL = 16 / sizeof(T);   // elements per 16-byte lane load
  constexpr int LPK = D / EPL;          // lanes per key row
  constexpr int KPW = 32 / LPK;         // keys per warp step
  static_assert(LPK >= 1 && LPK <= 32 && 32 % LPK == 0, "bad D");
  extern __shared__ __align__(128) uint8_t smem_raw[];
  const int BLK = a.block;
  const int stage_elems = BLK * D;
  T* stages = reinterpret_cast<T*>(smem_raw);  // [nst][2][BLK][D]
  float* S_sm = reinterpret_cast<float*>(smem_raw + (size_t)nst * 2 * stage_elems * sizeof(T));  // [kGmax][BLK]
  uint64_t* full = reinterpret_cast<uint64_t*>(S_sm + kGmax * BLK);
  uint64_t* empty = full + nst;
  __shared__ int s_last;

  const int unit = blockIdx.x / nsplit;
  const int split = blockIdx.x % nsplit;
  const int b = unit / a.Hk, hk = unit % a.Hk;
  const int grp = a.Hq / a.Hk;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cnt_all = a.kept_cnt[(int64_t)b * a.Hk + hk];
  const int t0 = (int)((int64_t)split * cnt_all / nsplit);
  const int t1 = (int)((int64_t)(split + 1) * cnt_all / nsplit);
  const int32_t* list = a.kept_idx + ((int64_t)b * a.Hk + hk) * a.nb_max;
  const int kvlen = max(0, min(a.kv_len[b] - a.kv_offset, a.L));
  const int NBk = (a.L + BLK - 1) / BLK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < nst; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kDecConsumerWarps);
    }
    fence_barrier_init();
  }
  __syncthreads();

  const T* Kb = reinterpret_cast<const T*>(a.k_cache) + b * a.k_stride[0] + hk * a.k_stride[1];
  const T* Vb = reinterpret_cast<const T*>(a.v_cache) + b * a.v_stride[0] + hk * a.v_stride[1];
  bool timed_out = false;

  if (warp == kDecConsumerWarps) {
    // ---------------- producer ----------------
    if (lane == 0) {
      for (int t = t0; t < t1; ++t) {
        const int i = t - t0;
        const int s = i % nst;
        if (i >= nst) {
          if (!mbar_wait(&empty[s], ((i / nst) - 1) & 1)) { timed_out = true; break; }
        }
        int kb = list[t];
        int rows = 0;
        if (kb >= 0 && kb < NBk) rows = min(BLK, a.L - kb * BLK);
        const uint32_t bytes = (uint32_t)rows * D * sizeof(T);
        T* dst = stages + (size_t)s * 2 * stage_elems;
        if (rows > 0) {
          mbar_arrive_expect_tx(&full[s], 2 * bytes);
          bulk_g2s(dst, Kb + (int64_t)kb * BLK * D, bytes, &full[s]);
          bulk_g2s(dst + stage_elems, Vb + (int64_t)kb * BLK * D, bytes, &full[s]);
        } else {
          mbar_arrive(&full[s]);
        }
      }
      if (timed_out) {
        set_err(a.err, TASFT_DEVERR_TIMEOUT);
        // let copies already issued land before the CTA exits
        const int issued = t1 - t0;
        for (int i = max(0, issued - nst); i < issued; ++i) mbar_wait(&full[i % nst], (i / nst) & 1);
      }
    }
    __syncwarp();
  } else {
    // ---------------- consumers ----------------
    const int kg = lane / LPK;   // key slot within the warp step
    const int ch = lane % LPK;   // 16-byte chunk of the row
    float q[kGmax][EPL];
    const T* Qb = reinterpret_cast<const T*>(a.q) + b * a.q_stride[0];
#pragma unroll
    for (int g = 0; g < kGmax; ++g) {
#pragma unroll
      for (int e = 0; e < EPL; ++e)
        q[g][e] = g < grp ? to_f<T>(Qb[(int64_t)(hk * grp + g) * a.q_stride[1] + ch * EPL + e]) : 0.f;
    }
    float acc[kGmax][EPL];
    float l_run[kGmax], m_run[kGmax];
#pragma unroll
    for (int g = 0; g < kGmax; ++g) {
      l_run[g] = 0.f;
      m_run[g] = -INFINITY;
#pragma unroll
      for (int e = 0; e < EPL; ++e) acc[g][e] = 0.f;
    }
    const int keys_per_step = kDecConsumerWarps * KPW;
    for (int t = t0; t < t1; ++t) {
      const int i = t - t0;
      const int s = i % nst;
      // A timeout never skips a named barrier: the loop keeps its shape and only the
      // work is skipped, so the four consumer warps cannot strand each other.
      if (!timed_out && !__all_sync(0xffffffffu, mbar_wait(&full[s], (i / nst) & 1))) {
        timed_out = true;
        set_err(a.err, TASFT_DEVERR_TIMEOUT);
      }
      const int kb = timed_out ? -1 : list[t];
      const bool kb_ok = kb >= 0 && kb < NBk;
      if (!kb_ok && !timed_out && threadIdx.x == 0) set_err(a.err, TASFT_DEVERR_INDEX);
      const T* Ks = stages + (size_t)s * 2 * stage_elems;
      const T* Vs = Ks + stage_elems;
      // pass 1: scores
      for (int j0 = warp * KPW; j0 < BLK; j0 += keys_per_step) {
        const int j = j0 + kg;
        const int kp = kb * BLK + j;
        const bool valid = kb_ok && j < BLK && kp < kvlen;
        float part[kGmax];
#pragma unroll
        for (int g = 0; g < kGmax; ++g) part[g] = 0.f;
        if (valid) {
          const uint4 u = *reinterpret_cast<const uint4*>(Ks + (size_t)j * D + ch * EPL);
          float f[EPL];
          Vec16<T>::unpack(u, f);
#pragma unroll
          for (int g = 0; g < kGmax; ++g) {
            if (g < grp) {
#pragma unroll
              for (int e = 0; e < EPL; ++e) part[g] = fmaf(q[g][e], f[e], part[g]);
            }
          }
        }
#pragma unroll
        for (int g = 0; g < kGmax; ++g) {
          if (g < grp) {
#pragma unroll
            for (int o = LPK / 2; o > 0; o >>= 1) part[g] += __shfl_xor_sync(0xffffffffu, part[g], o);
          }
        }
        if (ch == 0 && j < BLK) {
#pragma unroll
          for (int g = 0; g < kGmax; ++g)
            if (g < grp) S_sm[g * BLK + j] = valid ? part[g] * a.scale : -INFINITY;
        }
      }
      named_bar(1, kDecConsumerWarps * 32);
      // block max per head, shared by all consumer warps
      float alpha[kGmax], m_new[kGmax];
#pragma unroll
      for (int g = 0; g < kGmax; ++g) {
        float mb = -INFINITY;
        if (g < grp) {
          for (int j = lane; j < BLK; j += 32) mb = fmaxf(mb, S_sm[g * BLK + j]);
          mb = warp_max(mb);
        }
        m_new[g] = fmaxf(m_run[g], mb);
        alpha[g] = (m_new[g] == -INFINITY) ? 1.f : __expf(m_run[g] - m_new[g]);
        l_run[g] *= alpha[g];
#pragma unroll
        for (int e = 0; e < EPL; ++e) acc[g][e] *= alpha[g];
        m_run[g] = m_new[g];
      }
      // pass 2: p.V
      for (int j0 = warp * KPW; j0 < BLK; j0 += keys_per_step) {
        const int j = j0 + kg;
        const int kp = kb * BLK + j;
        const bool valid = kb_ok && j < BLK && kp < kvlen;
        if (valid) {
          const uint4 u = *reinterpret_cast<const uint4*>(Vs + (size_t)j * D + ch * EPL);
          float f[EPL];
          Vec16<T>::unpack(u, f);
#pragma unroll
          for (int g = 0; g < kGmax; ++g) {
            if (g < grp) {
              const float p = __expf(S_sm[g * BLK + j] - m_new[g]);
              if (ch == 0) l_run[g] += p;
#pragma unroll
              for (int e = 0; e < EPL; ++e) acc[g][e] = fmaf(p, f[e], acc[g][e]);
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0 && !timed_out) mbar_arrive(&empty[s]);
      named_bar(1, kDecConsumerWarps * 32);  // S_sm is rewritten by the next block
    }
    // reduce over the key slots of this warp: lanes with equal `ch`
#pragma unroll
    for (int g = 0; g < kGmax; ++g) {
      if (g < grp) {
#pragma unroll
        for (int o = LPK; o < 32; o <<= 1) {
          l_run[g] += __shfl_xor_sync(0xffffffffu, l_run[g], o);
#pragma unroll
          for (int e = 0; e < EPL; ++e) acc[g][e] += __shfl_xor_sync(0xffffffffu, acc[g][e], o);
        }
      }
    }
    // warp partials -> shared memory (reuses the stage ring: every copy has landed)
    named_bar(1, kDecConsumerWarps * 32);
    float* red = reinterpret_cast<float*>(smem_raw);  // [warps][kGmax][D + 1]
    if (!timed_out && kg == 0) {
#pragma unroll
      for (int g = 0; g < kGmax; ++g) {
        if (g < grp) {
#pragma unroll
          for (int e = 0; e < EPL; ++e) red[(warp * kGmax + g) * (D + 1) + ch * EPL + e] = acc[g][e];
          if (ch == 0) red[(warp * kGmax + g) * (D + 1) + D] = l_run[g];
        }
      }
    }
    named_bar(1, kDecConsumerWarps * 32);
    // CTA result per q-head: o (unnormalised sum), l, m (same for all warps)
    const int tid = threadIdx.x;
    for (int x = tid; x < grp * (D + 1); x += kDecConsumerWarps * 32) {
      const int g = x / (D + 1), d = x % (D + 1);
      float v = 0.f;
      for (int w = 0; w < kDecConsumerWarps; ++w) v += red[(w * kGmax + g) * (D + 1) + d];
      red[(kDecConsumerWarps * kGmax + g) * (D + 1) + d] = v;
    }
    named_bar(1, kDecConsumerWarps * 32);
    const float* tot = red + kDecConsumerWarps * kGmax * (D + 1);
    // per-head (o / l, m, l) for the shared finish (m is already in base-e units here)
    float* res = red + (kDecConsumerWarps + 1) * kGmax * (D + 1);
    for (int x = tid; x < grp * (D + 2); x += kDecConsumerWarps * 32) {
      const int g = x / (D + 2), d = x % (D + 2);
      const float l = tot[g * (D + 1) + D];
      float v;
      if (d < D) v = l > 0.f ? tot[g * (D + 1) + d] / l : 0.f;
      else if (d == D) {
        float mm = -INFINITY;
#pragma unroll
        for (int gg = 0; gg < kGmax; ++gg) if (gg == g) mm = m_run[gg];
        v = mm;
      } else v = l;
      res[x] = v;
    }
    named_bar(1, kDecConsumerWarps * 32);
    decode_finish<T>(a, ws, nsplit, split, unit, b, hk, grp, res, tid, kDecConsumerWarps * 32, 1, &s_last);
  }
}

// Merge G partial (o, m, l) sets, e.g. gathered from G GPUs, into the output.
template <typename T>
__global__ void decode_combine_kernel(tasft_combine_args a) {
  const int64_t row = blockIdx.x;
  float mt = -INFINITY;
  for (int g = 0; g < a.G; ++g) {
    const float l = a.part_ml[((int64_t)g * a.rows + row) * 2 + 1];
    if (l > 0.f) mt = fmaxf(mt, a.part_ml[((int64_t)g * a.rows + row) * 2]);
  }
  for (int d = threadIdx.x; d < a.D; d += blockDim.x) {
    float num = 0.f, den = 0.f;
    for (int g = 0; g < a.G; ++g) {
      const float l = a.part_ml[((int64_t)g * a.rows + row) * 2 + 1];
      if (l > 0.f) {
        const float w = l * __expf(a.part_ml[((int64_t)g * a.rows + row) * 2] - mt);
        num = fmaf(w, a.part_o[((int64_t)g * a.rows + row) * a.D + d], num);
        den += w;
      }
    }
    reinterpret_cast<T*>(a.out)[row * a.D + d] = from_f<T>(den > 0.f ? num / den : 0.f);
  }
}

static int decode_stages(int block, int D, int esize) {
  const int stage = 2 * block * D * esize;
  int n = (96 * 1024) / stage;
  return n < 2 ? 2 : (n > 4 ? 4 : n);
}

static size_t decode_smem(int block, int D, int esize, int nst) {
  size_t s = (size_t)nst * 2 * block * D * esize + (size_t)kGmax * block * 4;
  s = (s + 15) / 16 * 16 + (size_t)2 * nst * 8;
  const size_t red = ((size_t)(kDecConsumerWarps + 1) * kGmax * (D + 1) + (size_t)kGmax * (D + 2)) * 4;
  const size_t ring = (size_t)nst * 2 * block * D * esize;
  if (red > ring) s += red - ring;  // reduction buffer aliases the ring
  return s;
}

template <typename T, int D>
static int launch_decode_t(const tasft_decode_args& a, DecodeWs ws, int nsplit, cudaStream_t st) {
  const int nst = decode_stages(a.block, D, sizeof(T));
  const size_t smem = decode_smem(a.block, D, sizeof(T), nst);
  auto kern = bsa_decode_simt_kernel<T, D>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return TASFT_ERR_CUDA;
  const int64_t grid = (int64_t)a.B * a.Hk * nsplit;
  kern<<<(unsigned)grid, kDecThreads, smem, st>>>(a, ws, nsplit, nst);
  count_launch();
  return launch_status();
}

template <typename T>
static int launch_decode_dt(const tasft_decode_args& a, DecodeWs ws, int nsplit, cudaStream_t st) {
  switch (a.D) {
    case 64: return launch_decode_t<T, 64>(a, ws, nsplit, st);
    case 128: return launch_decode_t<T, 128>(a, ws, nsplit, st);
    default: return TASFT_ERR_UNSUPPORTED;
  }
}

}  // namespace tasft

using namespace tasft;

extern "C" int64_t tasft_decode_workspace_size(int32_t B, int32_t Hq, int32_t Hk, int32_t D, int32_t max_splits) {
  if (B <= 0 || Hq <= 0 || Hk <= 0 || D <= 0 || max_splits <= 0) return -1;
  const int64_t tick = ((int64_t)(B * Hk + 2) * 4 + 255) / 256 * 256;
  const int64_t part = (int64_t)B * Hq * max_splits * (D + 2) * 4;
  return tick + (part + 255) / 256 * 256;
}

namespace tasft {
int decode_check_args(const tasft_decode_args& a);
int decode_pick_splits(const tasft_decode_args& a);
int decode_run(const tasft_decode_args& a, const DecodeWs& ws, int nsplit, cudaStream_t st);
}  // namespace tasft

// Workspace layout: [tickets: B*Hk int32 + 2 work counters, padded to 256 B][partials: B*Hq x nsplit x (D+2) fp32].
// Tickets sit first so their place does not depend on the split count; every split call
// clears them before its launch.
static int decode_ws_from(const tasft_decode_args& a, int nsplit, DecodeWs* ws) {
  const int64_t tick = ((int64_t)(a.B * a.Hk + 2) * 4 + 255) / 256 * 256;
  const int64_t need = tick + (int64_t)a.B * a.Hq * nsplit * (a.D + 2) * 4;
  if (a.workspace_bytes < need) return TASFT_ERR_WORKSPACE;
  ws->max_splits = nsplit;
  ws->ticket = reinterpret_cast<int32_t*>(a.workspace);
  ws->part = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(a.workspace) + tick);
  return TASFT_OK;
}

// Tickets and work counters are cleared on the caller's stream at the start of every
// split call, so a call that follows one whose bounded wait gave up (and therefore left
// its tickets behind) starts from a clean state.
static int decode_clear_tickets(const tasft_decode_args& a, const DecodeWs& ws, cudaStream_t st) {
  const size_t tick = (size_t)(a.B * a.Hk + 2) * 4;
  return cudaMemsetAsync(ws.ticket, 0, tick, st) == cudaSuccess ? TASFT_OK : TASFT_ERR_CUDA;
}

extern "C" int tasft_bsa_decode_fwd(const tasft_decode_args* ap, tasft_stream_t stream) {
  if (!ap) return TASFT_ERR_INVALID_ARG;
  const tasft_decode_args& a = *ap;
  int rc = decode_check_args(a);
  if (rc != TASFT_OK) return rc;
  const int nsplit = decode_pick_splits(a);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  DecodeWs ws{nullptr, nullptr, 0};
  if (nsplit > 1) {
    if (!a.workspace) return TASFT_ERR_WORKSPACE;
    rc = decode_ws_from(a, nsplit, &ws);
    if (rc != TASFT_OK) return rc;
    rc = decode_clear_tickets(a, ws, st);
    if (rc != TASFT_OK) return rc;
  }
  return decode_run(a, ws, nsplit, st);
}

extern "C" int tasft_bsa_decode_peer_fwd(const tasft_decode_args* ap, const tasft_decode_peer_args* pp,
                                         tasft_stream_t stream) {
  if (!ap || !pp) return TASFT_ERR_INVALID_ARG;
  const tasft_decode_args& a = *ap;
  int rc = decode_check_args(a);
  if (rc != TASFT_OK) return rc;
  if (!a.out || !pp->mailboxes || !pp->epoch) return TASFT_ERR_INVALID_ARG;
  if (pp->world <= 0 || pp->world > 8 || pp->rank < 0 || pp->rank >= pp->world) return TASFT_ERR_INVALID_ARG;
  if (!decode_mma_ok(a)) return TASFT_ERR_UNSUPPORTED;
  int nsplit = decode_pick_splits(a);
  if (nsplit < 2) nsplit = 2;  // the exchange runs in the separate merge kernel
  if (!a.workspace) return TASFT_ERR_WORKSPACE;
  DecodeWs ws{nullptr, nullptr, 0};
  rc = decode_ws_from(a, nsplit, &ws);
  if (rc != TASFT_OK) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  rc = decode_clear_tickets(a, ws, st);
  if (rc != TASFT_OK) return rc;
  return decode_mma(a, ws, nsplit, st, PeerMode{pp->mailboxes, pp->epoch, pp->world, pp->rank, pp->timeout_ns});
}

extern "C" int tasft_bsa_decode_combine(const tasft_combine_args* ap, tasft_stream_t stream) {
  if (!ap || !ap->part_o || !ap->part_ml || !ap->out || ap->G <= 0 || ap->rows <= 0 || ap->D <= 0)
    return TASFT_ERR_INVALID_ARG;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const unsigned grid = (unsigned)ap->rows;
  switch (ap->dtype) {
    case TASFT_F32: decode_combine_kernel<float><<<grid, 128, 0, st>>>(*ap); break;
    case TASFT_BF16: decode_combine_kernel<__nv_bfloat16><<<grid, 128, 0, st>>>(*ap); break;
    case TASFT_F16: decode_combine_kernel<__half><<<grid, 128, 0, st>>>(*ap); break;
    default: return TASFT_ERR_UNSUPPORTED;
  }
  count_launch();
  return launch_status();
}

// ---------------------------------------------------------------------------
// Argument checks, split choice and kernel dispatch, shared by tasft_bsa_decode_fwd and
// the entry point that brings its own scratch (decode_noalloc.cu).
// ---------------------------------------------------------------------------
namespace tasft {

int decode_check_args(const tasft_decode_args& a) {
  if (!a.q || !a.k_cache || !a.v_cache || !a.kv_len || !a.kept_idx || !a.kept_cnt) return TASFT_ERR_INVALID_ARG;
  if (!a.out && !a.part_o) return TASFT_ERR_INVALID_ARG;
  if (a.B <= 0 || a.Hq <= 0 || a.Hk <= 0 || a.L <= 0 || a.block <= 0 || a.nb_max <= 0) return TASFT_ERR_INVALID_ARG;
  if (a.Hq % a.Hk != 0 || a.Hq / a.Hk > kGmax) return TASFT_ERR_UNSUPPORTED;
  if (a.block > 128 || a.block % 8 != 0) return TASFT_ERR_UNSUPPORTED;
  const int es = elem_size(a.dtype);
  if (a.k_stride[3] != 1 || a.v_stride[3] != 1 || a.k_stride[2] != a.D || a.v_stride[2] != a.D ||
      a.q_stride[2] != 1 || (a.out && a.o_stride[2] != 1))
    return TASFT_ERR_INVALID_ARG;
  if (!aligned16(a.k_cache) || !aligned16(a.v_cache) || !aligned16(a.q) || (a.k_stride[1] * es) % 16 ||
      (a.v_stride[1] * es) % 16 || (a.k_stride[0] * es) % 16 || (a.v_stride[0] * es) % 16 ||
      (a.q_stride[1] * es) % 16 || (a.q_stride[0] * es) % 16)
    return TASFT_ERR_INVALID_ARG;
  return TASFT_OK;
}

int decode_pick_splits(const tasft_decode_args& a) {
  int nsplit = a.num_splits;
  if (nsplit <= 0) {
    const int units = a.B * a.Hk;
    nsplit = (6 * 148) / units;  // items within the resident CTA slots
    int cap = a.nb_max / 4 > 1 ? a.nb_max / 4 : 1;
    // the scalar path merges in the last split (one warp, up to 16); the tensor-core path
    // merges wide splits in a separate kernel, so few units (one long sequence) can still
    // spread over the SMs
    const int most = decode_mma_ok(a) ? 64 : 16;
    if (cap > most) cap = most;
    if (nsplit > cap) nsplit = cap;
    if (nsplit < 1) nsplit = 1;
  }
  return nsplit;
}

int decode_run(const tasft_decode_args& a, const DecodeWs& ws, int nsplit, cudaStream_t st) {
  if (a.dtype != TASFT_F32) {
    const int rc = decode_mma(a, ws, nsplit, st);
    if (rc != TASFT_ERR_UNSUPPORTED) return rc;
  }
  switch (a.dtype) {
    case TASFT_F32: return launch_decode_dt<float>(a, ws, nsplit, st);
    case TASFT_BF16: return launch_decode_dt<__nv_bfloat16>(a, ws, nsplit, st);
    case TASFT_F16: return launch_decode_dt<__half>(a, ws, nsplit, st);
    default: return TASFT_ERR_UNSUPPORTED;
  }
}

}  // namespace tasft

using namespace tasft;

// Paged KV cache: the same tensor-core decode, with K/V loaded through the block table.
extern "C" int tasft_bsa_decode_paged_fwd(const tasft_paged_decode_args* pp, tasft_stream_t stream) {
  if (!pp) return TASFT_ERR_INVALID_ARG;
  const tasft_decode_args& a = pp->base;
  if (!a.q || !a.k_cache || !a.v_cache || !a.kv_len || !a.kept_idx || !a.kept_cnt || !pp->block_table)
    return TASFT_ERR_INVALID_ARG;
  if (!a.out && !a.part_o) return TASFT_ERR_INVALID_ARG;
  if (a.B <= 0 || a.Hq <= 0 || a.Hk <= 0 || a.D <= 0 || a.block <= 0 || a.nb_max <= 0 || a.Hq % a.Hk)
    return TASFT_ERR_INVALID_ARG;
  const int ps = pp->page_size;
  if (ps != 16 && ps != 32 && ps != 64 && ps != 128) return TASFT_ERR_UNSUPPORTED;
  if (pp->max_pages <= 0 || pp->num_pages <= 0 || (int64_t)pp->max_pages * ps != a.L) return TASFT_ERR_INVALID_ARG;
  if (a.dtype != TASFT_BF16 && a.dtype != TASFT_F16) return TASFT_ERR_UNSUPPORTED;
  // page pools [num_pages, page_size, Hk, D], D contiguous; TMA wants 16-byte strides and base
  if (a.k_stride[3] != 1 || a.v_stride[3] != 1 || a.q_stride[2] != 1 || (a.out && a.o_stride[2] != 1))
    return TASFT_ERR_INVALID_ARG;
  for (int i = 0; i < 3; ++i)
    if ((a.k_stride[i] * 2) % 16 || (a.v_stride[i] * 2) % 16) return TASFT_ERR_INVALID_ARG;
  if (!aligned16(a.k_cache) || !aligned16(a.v_cache)) return TASFT_ERR_INVALID_ARG;
  const int nsplit = decode_pick_splits(a);
  DecodeWs ws{nullptr, nullptr, 0};
  if (nsplit > 1) {
    if (!a.workspace) return TASFT_ERR_WORKSPACE;
    int rc = decode_ws_from(a, nsplit, &ws);
    if (rc != TASFT_OK) return rc;
    rc = decode_clear_tickets(a, ws, reinterpret_cast<cudaStream_t>(stream));
    if (rc != TASFT_OK) return rc;
  }
  return decode_mma_paged(a, ws, nsplit, pp->block_table, pp->max_pages, ps, pp->num_pages,
                          reinterpret_cast<cudaStream_t>(stream));
}
