// AttnGate mask builder: fused block pooling + gate projection, pair scores,
// threshold and kept-block list emission.
//
// Reference: tasft/modules/attn_gate.py:351-485 (AttnGate._pool_to_blocks / forward).
// The reference materialises every (q-block, k-block) pair [q_i; k_j] and runs
// Linear(2D->hid) on it. Here the first layer is split by linearity:
//   W_in [q_i; k_j] + b = (W_q q_i + b) + W_k k_j =: a_i + c_j
// so a_i and c_j are computed once per block while pooling (one HBM pass over Q and
// K), and the pair kernel only evaluates w_out . relu(a_i + c_j). Same maths; the fp32
// summation order differs from the reference's single 2D-long dot product.
#include "common.cuh"

namespace tasft {

// ---------------------------------------------------------------------------
// Kernel 1: pool `block` rows of Q or K to their mean and project it.
//   A  [B, Hq, NBq, hid]  = W_q qbar + b        (row-major, hid fastest)
//   Ct [B, Hk, hid, NBk]  = W_k kbar            (transposed: j fastest, for coalesced pair reads)
// One CTA per (tensor, b, head, block). Padding rows count as zeros in the mean
// (attn_gate.py:366-375), so the divisor is always `block`.
// ---------------------------------------------------------------------------
constexpr int kPoolThreads = 256;

template <typename T, int EPV>
__global__ void __launch_bounds__(kPoolThreads) gate_pool_project_kernel(tasft_gate_args a, float* A, float* Ct,
                                                                        int NBq, int NBk) {
  extern __shared__ float sm[];  // [rowgroups][D] partial sums, then mean[D]
  const int D = a.D;
  const int hid = a.hidden;
  int64_t bid = blockIdx.x;
  const int64_t nq = (int64_t)a.B * a.Hq * NBq;
  const bool isq = bid < nq;
  if (!isq) bid -= nq;
  const int H = isq ? a.Hq : a.Hk;
  const int NB = isq ? NBq : NBk;
  const int S = isq ? a.Sq : a.Sk;
  const int blk = (int)(bid % NB);
  const int h = (int)((bid / NB) % H);
  const int b = (int)(bid / ((int64_t)NB * H));
  const T* base = reinterpret_cast<const T*>(isq ? a.q : a.k);
  const int64_t* st = isq ? a.q_stride : a.k_stride;
  base += b * st[0] + h * st[1];

  const int row0 = blk * a.block;
  const int rows = min(a.block, S - row0);
  const int CV = D / EPV;                      // vectors per row
  const int RG = kPoolThreads / CV;            // row groups (CV <= 256 guaranteed by host)
  const int c = threadIdx.x % CV;
  const int rg = threadIdx.x / CV;
  float acc[EPV];
#pragma unroll
  for (int e = 0; e < EPV; ++e) acc[e] = 0.f;
  if (rg < RG) {
#pragma unroll 4
    for (int r = rg; r < rows; r += RG) {
      const T* p = base + (int64_t)(row0 + r) * st[2] + c * EPV;
      if constexpr (EPV * sizeof(T) == 16) {
        uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
        float f[EPV];
        Vec16<T>::unpack(u, f);
#pragma unroll
        for (int e = 0; e < EPV; ++e) acc[e] += f[e];
      } else {
#pragma unroll
        for (int e = 0; e < EPV; ++e) acc[e] += to_f<T>(p[e]);
      }
    }
  }
  if (rg < RG) {
    if constexpr (EPV % 4 == 0) {
#pragma unroll
      for (int e = 0; e < EPV; e += 4)
        *reinterpret_cast<float4*>(&sm[rg * D + c * EPV + e]) = make_float4(acc[e], acc[e + 1], acc[e + 2], acc[e + 3]);
    } else {
#pragma unroll
      for (int e = 0; e < EPV; ++e) sm[rg * D + c * EPV + e] = acc[e];
    }
  }
  __syncthreads();
  float* mean = sm + RG * D;
  const float inv = 1.0f / (float)a.block;
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float s = 0.f;
    for (int g = 0; g < RG; ++g) s += sm[g * D + d];
    mean[d] = s * inv;
  }
  __syncthreads();
  float* pooled = isq ? a.pooled_q : a.pooled_k;
  const int64_t prow = ((int64_t)b * H + h) * NB + blk;
  if (pooled) {
    for (int d = threadIdx.x; d < D; d += blockDim.x) pooled[prow * D + d] = mean[d];
  }
  // projection: one warp per hidden unit, lanes over D (coalesced weight rows)
  const int off = isq ? 0 : D;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int j = warp; j < hid; j += kPoolThreads / 32) {
    const float* w = a.w_in + (int64_t)j * 2 * D + off;
    float s = 0.f;
    for (int d = lane; d < D; d += 32) s = fmaf(__ldg(w + d), mean[d], s);
    s = warp_sum(s);
    if (lane == 0) {
      if (isq) {
        A[prow * hid + j] = s + a.b_in[j];
      } else {
        Ct[(((int64_t)b * H + h) * hid + j) * NB + blk] = s;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Kernel 2: one warp per (b, q-head, q-block) row of the score grid.
//   soft[j] = sigmoid(w_out . relu(a_i + c_j)), zeroed for j > i when causal and NBq == NBk
//   hard[j] = soft[j] >= tau                                        (attn_gate.py:475)
//   kept list = ascending j with hard[j] (and j <= i when causal), -1 padded
// ---------------------------------------------------------------------------
constexpr int kRowsPerCta = 8;

__device__ __forceinline__ void emit_row(float s, int j, int NBk, bool in_range, bool list_ok, float tau,
                                         int64_t row, uint8_t* hard, int32_t* kept_idx, int& base_cnt) {
  const bool keep = in_range && (s >= tau);
  if (hard && in_range) hard[row * NBk + j] = keep ? 1 : 0;
  const bool lk = keep && list_ok;
  const unsigned bal = __ballot_sync(0xffffffffu, lk);
  const int lane = threadIdx.x & 31;
  if (kept_idx) {
    const int pos = base_cnt + __popc(bal & ((1u << lane) - 1u));
    if (lk) kept_idx[row * NBk + pos] = j;
  }
  base_cnt += __popc(bal);
}

__global__ void __launch_bounds__(kRowsPerCta * 32) gate_pair_kernel(tasft_gate_args a, const float* A, const float* Ct,
                                                                     int NBq, int NBk) {
  extern __shared__ float sm[];  // [kRowsPerCta][hid] a-rows, then w_out[hid]
  const int hid = a.hidden;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* wout = sm + kRowsPerCta * hid;
  for (int j = threadIdx.x; j < hid; j += blockDim.x) wout[j] = a.w_out[j];
  const int64_t rows = (int64_t)a.B * a.Hq * NBq;
  const int64_t row = (int64_t)blockIdx.x * kRowsPerCta + warp;
  float* arow = sm + warp * hid;
  if (row < rows) {
    for (int j = lane; j < hid; j += 32) arow[j] = A[row * hid + j];
  }
  __syncthreads();
  if (row >= rows) return;
  const int i = (int)(row % NBq);
  const int hq = (int)((row / NBq) % a.Hq);
  const int b = (int)(row / ((int64_t)NBq * a.Hq));
  const int hk = hq / (a.Hq / a.Hk);
  const float* ct = Ct + ((int64_t)b * a.Hk + hk) * hid * NBk;
  const bool causal = a.causal && (NBq == NBk);
  int cnt = 0;
  int kept_total = 0;
  for (int j0 = 0; j0 < NBk; j0 += 32) {
    const int j = j0 + lane;
    const bool in_range = j < NBk;
    float s = 0.f;
    if (in_range) {
      float logit = 0.f;
      for (int h = 0; h < hid; ++h) logit = fmaf(wout[h], fmaxf(arow[h] + ct[(int64_t)h * NBk + j], 0.f), logit);
      s = 1.0f / (1.0f + __expf(-logit));
      if (causal && j > i) s = 0.f;
      a.soft[row * NBk + j] = s;
    }
    const bool keep = in_range && (s >= a.tau);
    kept_total += __popc(__ballot_sync(0xffffffffu, keep));
    emit_row(s, j, NBk, in_range, !(causal && j > i), a.tau, row, a.hard, a.kept_idx, cnt);
  }
  if (a.kept_idx) {
    for (int j = cnt + lane; j < NBk; j += 32) a.kept_idx[row * NBk + j] = -1;
  }
  if (lane == 0) {
    if (a.kept_cnt) a.kept_cnt[row] = cnt;
    if (a.num_kept) atomicAdd(a.num_kept, kept_total);
  }
}

// ---------------------------------------------------------------------------
// Threshold from given fp32 scores (bit-exact `soft >= tau`).
// ---------------------------------------------------------------------------
__global__ void threshold_kernel(tasft_threshold_args a) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + warp;
  if (row >= a.rows) return;
  const int i = (int)(row % a.NBq);
  int cnt = 0, total = 0;
  for (int j0 = 0; j0 < a.NBk; j0 += 32) {
    const int j = j0 + lane;
    const bool in_range = j < a.NBk;
    const float s = in_range ? a.soft[row * a.NBk + j] : 0.f;
    const bool keep = in_range && (s >= a.tau);
    total += __popc(__ballot_sync(0xffffffffu, keep));
    emit_row(s, j, a.NBk, in_range, !(a.causal && j > i), a.tau, row, a.hard, a.kept_idx, cnt);
  }
  if (a.kept_idx) {
    for (int j = cnt + lane; j < a.NBk; j += 32) a.kept_idx[row * a.NBk + j] = -1;
  }
  if (lane == 0) {
    if (a.kept_cnt) a.kept_cnt[row] = cnt;
    if (a.num_kept) atomicAdd(a.num_kept, total);
  }
}

// Bool mask -> kept lists (block_sparse_fa.py:497-508 + the kernel's ascending visit).
__global__ void mask_to_kept_kernel(tasft_mask_args a) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + warp;
  if (row >= a.rows) return;
  const int i = (int)(row % a.NBq);
  int cnt = 0;
  for (int j0 = 0; j0 < a.NBk; j0 += 32) {
    const int j = j0 + lane;
    const bool keep = j < a.NBk && a.mask[row * a.NBk + j] != 0 && !(a.causal && j > i);
    const unsigned bal = __ballot_sync(0xffffffffu, keep);
    if (keep) a.kept_idx[row * a.NBk + cnt + __popc(bal & ((1u << lane) - 1u))] = j;
    cnt += __popc(bal);
  }
  for (int j = cnt + lane; j < a.NBk; j += 32) a.kept_idx[row * a.NBk + j] = -1;
  if (lane == 0) {
    a.kept_cnt[row] = cnt;
    if (a.num_kept) atomicAdd(a.num_kept, cnt);
  }
}

}  // namespace tasft

using namespace tasft;

extern "C" int64_t tasft_gate_workspace_size(int32_t B, int32_t Hq, int32_t Hk, int32_t Sq, int32_t Sk, int32_t block,
                                             int32_t hidden) {
  if (B <= 0 || Hq <= 0 || Hk <= 0 || Sq <= 0 || Sk <= 0 || block <= 0 || hidden <= 0) return -1;
  const int64_t NBq = ceil_div(Sq, block), NBk = ceil_div(Sk, block);
  const int64_t floats = (int64_t)B * Hq * NBq * hidden + (int64_t)B * Hk * NBk * hidden;
  return ((floats * 4 + 255) / 256) * 256;
}

template <typename T>
static int launch_pool(const tasft_gate_args& a, float* A, float* Ct, int NBq, int NBk, cudaStream_t st) {
  constexpr int EPV = 16 / sizeof(T);
  const bool vec_ok = (a.D % EPV == 0) && aligned16(a.q) && aligned16(a.k) && (a.q_stride[0] % EPV == 0) &&
                      (a.q_stride[1] % EPV == 0) && (a.q_stride[2] % EPV == 0) && (a.k_stride[0] % EPV == 0) &&
                      (a.k_stride[1] % EPV == 0) && (a.k_stride[2] % EPV == 0) && (a.D / EPV <= kPoolThreads);
  const int64_t grid = (int64_t)a.B * a.Hq * NBq + (int64_t)a.B * a.Hk * NBk;
  if (vec_ok) {
    const int RG = kPoolThreads / (a.D / EPV);
    const size_t smem = (size_t)(RG + 1) * a.D * sizeof(float);
    gate_pool_project_kernel<T, EPV><<<(unsigned)grid, kPoolThreads, smem, st>>>(a, A, Ct, NBq, NBk);
  } else {
    if (a.D > kPoolThreads) return TASFT_ERR_UNSUPPORTED;
    const int RG = kPoolThreads / a.D;
    const size_t smem = (size_t)(RG + 1) * a.D * sizeof(float);
    gate_pool_project_kernel<T, 1><<<(unsigned)grid, kPoolThreads, smem, st>>>(a, A, Ct, NBq, NBk);
  }
  count_launch();
  return launch_status();
}

extern "C" int tasft_gate_mask_build(const tasft_gate_args* ap, tasft_stream_t stream) {
  if (!ap) return TASFT_ERR_INVALID_ARG;
  const tasft_gate_args& a = *ap;
  if (!a.q || !a.k || !a.w_in || !a.b_in || !a.w_out || !a.soft) return TASFT_ERR_INVALID_ARG;
  if (a.B <= 0 || a.Hq <= 0 || a.Hk <= 0 || a.Sq <= 0 || a.Sk <= 0 || a.D <= 0 || a.block <= 0)
    return TASFT_ERR_INVALID_ARG;
  if (a.Hq % a.Hk != 0) return TASFT_ERR_INVALID_ARG;
  if (a.hidden <= 0 || a.hidden > 256) return TASFT_ERR_UNSUPPORTED;
  if (a.D > 1024) return TASFT_ERR_UNSUPPORTED;
  if ((a.kept_idx == nullptr) != (a.kept_cnt == nullptr)) return TASFT_ERR_INVALID_ARG;
  if (a.q_stride[3] != 1 || a.k_stride[3] != 1) return TASFT_ERR_INVALID_ARG;
  const int64_t need = tasft_gate_workspace_size(a.B, a.Hq, a.Hk, a.Sq, a.Sk, a.block, a.hidden);
  if (!a.workspace || a.workspace_bytes < need) return TASFT_ERR_WORKSPACE;
  const int NBq = ceil_div(a.Sq, a.block), NBk = ceil_div(a.Sk, a.block);
  float* A = reinterpret_cast<float*>(a.workspace);
  float* Ct = A + (int64_t)a.B * a.Hq * NBq * a.hidden;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  int rc;
  switch (a.dtype) {
    case TASFT_F32: rc = launch_pool<float>(a, A, Ct, NBq, NBk, st); break;
    case TASFT_BF16: rc = launch_pool<__nv_bfloat16>(a, A, Ct, NBq, NBk, st); break;
    case TASFT_F16: rc = launch_pool<__half>(a, A, Ct, NBq, NBk, st); break;
    default: return TASFT_ERR_UNSUPPORTED;
  }
  if (rc != TASFT_OK) return rc;
  const int64_t rows = (int64_t)a.B * a.Hq * NBq;
  const size_t smem = (size_t)(kRowsPerCta + 1) * a.hidden * sizeof(float);
  gate_pair_kernel<<<ceil_div(rows, kRowsPerCta), kRowsPerCta * 32, smem, st>>>(a, A, Ct, NBq, NBk);
  count_launch();
  return launch_status();
}

extern "C" int tasft_mask_from_scores(const tasft_threshold_args* ap, tasft_stream_t stream) {
  if (!ap || !ap->soft || ap->rows < 0 || ap->NBq <= 0 || ap->NBk <= 0) return TASFT_ERR_INVALID_ARG;
  if ((ap->kept_idx == nullptr) != (ap->kept_cnt == nullptr)) return TASFT_ERR_INVALID_ARG;
  if (ap->rows == 0) return TASFT_OK;
  threshold_kernel<<<ceil_div(ap->rows, 8), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(*ap);
  count_launch();
  return launch_status();
}

extern "C" int tasft_mask_to_kept(const tasft_mask_args* ap, tasft_stream_t stream) {
  if (!ap || !ap->mask || !ap->kept_idx || !ap->kept_cnt || ap->rows < 0 || ap->NBq <= 0 || ap->NBk <= 0)
    return TASFT_ERR_INVALID_ARG;
  if (ap->rows == 0) return TASFT_OK;
  mask_to_kept_kernel<<<ceil_div(ap->rows, 8), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(*ap);
  count_launch();
  return launch_status();
}
