// Training-time gate target, gate losses and the gate backward.
//
// Reference path (tasft/modules/tasft_attention.py:427-458 -> tasft/training/objectives.py):
//   scores = (Q K^T) * scale (+ causal -inf), 2-D max-pool over 64x64 tiles
//   (objectives.py:170-178), softmax over the flattened NB x NB grid (:180-185),
//   KL(target || soft / sum soft) batchmean (:187-221), (mean(soft) - tau)^2 (:223-241).
// Here the S x S score matrix is never stored: each tile's max is reduced on chip.
#include <algorithm>

#include "common.cuh"

namespace tasft {

int gate_target_blockmax_tc(const tasft_target_args& a, float* block_max, cudaStream_t st);
int prefill_tc(const tasft_prefill_args& a, cudaStream_t st, const int32_t* cu, int total, float* bmax,
               int emulate_bf16);

__global__ void fill_kernel(float* p, int64_t n, float v) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) p[i] = v;
}

// ---------------------------------------------------------------------------
// CUDA-core tile max: one CTA per (q-block, k-block <= q-block, b*h).
// ---------------------------------------------------------------------------
template <typename T, int D>
__global__ void __launch_bounds__(256) blockmax_simt_kernel(tasft_target_args a, float* bm, int NB) {
  const int qb = blockIdx.x, kb = blockIdx.y, bh = blockIdx.z;
  const int b = bh / a.Hq, hq = bh % a.Hq;
  const int blk = a.block;
  float* dst = bm + ((int64_t)bh * NB + qb) * NB + kb;
  if (kb > qb) {
    if (threadIdx.x == 0) *dst = -INFINITY;
    return;
  }
  extern __shared__ float sm[];
  float* Qs = sm;                  // [blk][D+1]
  float* Ks = sm + blk * (D + 1);  // [blk][D+1]
  const int hk = hq / (a.Hq / a.Hk);
  const T* Q = reinterpret_cast<const T*>(a.q) + b * a.q_stride[0] + hq * a.q_stride[1];
  const T* K = reinterpret_cast<const T*>(a.k) + b * a.k_stride[0] + hk * a.k_stride[1];
  for (int x = threadIdx.x; x < blk * D; x += blockDim.x) {
    const int r = x / D, d = x % D;
    const int qp = qb * blk + r, kp = kb * blk + r;
    Qs[r * (D + 1) + d] = qp < a.S ? to_f<T>(Q[(int64_t)qp * a.q_stride[2] + d]) : 0.f;
    Ks[r * (D + 1) + d] = kp < a.S ? to_f<T>(K[(int64_t)kp * a.k_stride[2] + d]) : 0.f;
  }
  __syncthreads();
  float mx = -INFINITY;
  for (int e = threadIdx.x; e < blk * blk; e += blockDim.x) {
    const int r = e / blk, c = e % blk;
    const int qp = qb * blk + r, kp = kb * blk + c;
    if (qp >= a.S || kp >= a.S || kp > qp) continue;
    float s = 0.f;
#pragma unroll 8
    for (int d = 0; d < D; ++d) s = fmaf(Qs[r * (D + 1) + d], Ks[c * (D + 1) + d], s);
    mx = fmaxf(mx, s);
  }
  mx = warp_max(mx);
  __shared__ float red[8];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
  __syncthreads();
  if (threadIdx.x == 0) {
    float m = red[0];
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) m = fmaxf(m, red[w]);
    float v;
    if (a.emulate_bf16_scores) {
      // reference: bf16(bf16(q.k) * scale); both roundings are monotone, so max commutes
      v = __bfloat162float(__float2bfloat16_rn(__bfloat162float(__float2bfloat16_rn(m)) * a.scale));
    } else {
      v = m * a.scale;
    }
    *dst = v;
  }
}

// ---------------------------------------------------------------------------
// Block max of a given score tensor (objectives.py:128-185: -inf padding, 2-D max-pool
// over block x block tiles). HBM-bound streaming read: one CTA per (b*h, q-block,
// window of kpc k-blocks); warp w reads rows w, w+8, ... of the q-block, each thread a
// VEC-wide (16-byte when aligned) column slice, so a warp row load is 32 x 16 B
// contiguous. Per-warp column maxima meet in shared memory, then one warp per k-block
// reduces its columns. NaN and +inf are flagged (the reference raises on them).
// ---------------------------------------------------------------------------
template <typename T, int VEC>
__global__ void __launch_bounds__(256) scores_blockmax_kernel(tasft_scores_target_args a, float* bm, int NBq,
                                                              int NBk, int kpc) {
  extern __shared__ float colmax[];  // [8][W]
  const int W = kpc * a.block;
  const int kb0 = blockIdx.x * kpc;
  const int qb = blockIdx.y;
  const int bh = blockIdx.z;
  const int b = bh / a.H, h = bh % a.H;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const T* base = reinterpret_cast<const T*>(a.scores) + b * a.stride[0] + h * a.stride[1];
  const int r0 = qb * a.block;
  const int rows = min(a.block, a.Sq - r0);
  const int c0 = kb0 * a.block;
  bool bad_nan = false, bad_inf = false;
  for (int cc = lane * VEC; cc < W; cc += 32 * VEC) {
    float m[VEC];
#pragma unroll
    for (int j = 0; j < VEC; ++j) m[j] = -INFINITY;
    const int col = c0 + cc;
    if (col < a.Sk) {
      const T* p = base + (int64_t)col * a.stride[3];
#pragma unroll 4
      for (int r = warp; r < rows; r += 8) {
        const T* pr = p + (int64_t)(r0 + r) * a.stride[2];
        if (VEC > 1) {
          // VEC > 1 only when Sk % VEC == 0 and the rows are 16-byte aligned
          uint4 raw = __ldcs(reinterpret_cast<const uint4*>(pr));
          const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
          for (int j = 0; j < VEC; ++j) {
            const float x = to_f<T>(e[j]);
            bad_nan |= x != x;
            bad_inf |= x == INFINITY;
            m[j] = fmaxf(m[j], x);
          }
        } else {
          const float x = to_f<T>(pr[0]);
          bad_nan |= x != x;
          bad_inf |= x == INFINITY;
          m[0] = fmaxf(m[0], x);
        }
      }
    }
#pragma unroll
    for (int j = 0; j < VEC; ++j) colmax[warp * W + cc + j] = m[j];
  }
  __syncthreads();
  for (int kl = warp; kl < kpc; kl += 8) {
    const int kb = kb0 + kl;
    if (kb >= NBk) break;
    float mx = -INFINITY;
    for (int c = lane; c < a.block; c += 32) {
      const int cc = kl * a.block + c;
#pragma unroll
      for (int w = 0; w < 8; ++w) mx = fmaxf(mx, colmax[w * W + cc]);
    }
    mx = warp_max(mx);
    if (lane == 0) bm[((int64_t)bh * NBq + qb) * NBk + kb] = mx;
  }
  if (a.flags) {
    const unsigned any_nan = __ballot_sync(0xffffffffu, bad_nan), any_inf = __ballot_sync(0xffffffffu, bad_inf);
    if (lane == 0 && (any_nan | any_inf)) atomicOr(a.flags, (any_nan ? 1 : 0) | (any_inf ? 2 : 0));
  }
}

// Softmax over each (b, h) grid of NB*NB block maxima (objectives.py:180-185), with the
// alternate target's clamp and temperature (tasft_attention.py:278-289) as options.
__global__ void target_softmax_kernel(const float* bm, float* target, int64_t n, float inv_temp, float clamp) {
  const int64_t base = (int64_t)blockIdx.x * n;
  __shared__ float red[32];
  auto val = [&](int64_t i) {
    float x = bm[base + i];
    if (clamp > 0.f && isfinite(x)) x = fminf(fmaxf(x, -clamp), clamp);
    return x * inv_temp;
  };
  float mx = -INFINITY;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) mx = fmaxf(mx, val(i));
  mx = warp_max(mx);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
  __syncthreads();
  if (threadIdx.x < 32) {
    float m = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : -INFINITY;
    m = warp_max(m);
    if (threadIdx.x == 0) red[0] = m;
  }
  __syncthreads();
  mx = red[0];
  __syncthreads();
  float s = 0.f;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) s += __expf(val(i) - mx);
  s = warp_sum(s);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    t = warp_sum(t);
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  const float inv = 1.0f / red[0];
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) target[base + i] = __expf(val(i) - mx) * inv;
}

// ---------------------------------------------------------------------------
// Loss forward + gradient w.r.t. the soft scores.
// ---------------------------------------------------------------------------
constexpr float kEps = 1e-8f;

__device__ __forceinline__ double block_sum_d(double v, double* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  double t = 0.0;
  for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += red[w];
  return t;
}

// one CTA per (b, h): partial KL, partial sum, and w_kl * dKL/dsoft
__global__ void loss_rows_kernel(tasft_loss_args a, double* part) {
  const int64_t n = (int64_t)a.NBq * a.NBk;
  const int64_t base = (int64_t)blockIdx.x * n;
  __shared__ double red[32];
  double s = 0.0;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) s += a.soft[base + i];
  const double S = block_sum_d(s, red);
  const float denom = (float)S + kEps;
  double kl = 0.0, cross = 0.0;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
    const float t = a.target[base + i];
    const float g = a.soft[base + i] / denom;
    if (t > 0.f) kl += (double)t * ((double)logf(t) - (double)logf(g + kEps));
    cross += (double)t * a.soft[base + i] / (g + kEps);
  }
  const double KL = block_sum_d(kl, red);
  const double X = block_sum_d(cross, red);
  if (a.d_soft) {
    const float invB = 1.0f / (float)a.B;
    const float c2 = (float)(X / ((double)denom * denom));
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
      const float t = a.target[base + i];
      const float g = a.soft[base + i] / denom;
      const float d = -invB * (t / ((g + kEps) * denom) - c2);
      a.d_soft[base + i] = a.w_kl * d;
    }
  }
  if (threadIdx.x == 0) {
    part[2 * blockIdx.x] = KL;
    part[2 * blockIdx.x + 1] = S;
  }
}

__global__ void loss_final_kernel(tasft_loss_args a, const double* part, int rows, float* gsp) {
  __shared__ double red[32];
  double kl = 0.0, s = 0.0;
  for (int i = threadIdx.x; i < rows; i += blockDim.x) {
    kl += part[2 * i];
    s += part[2 * i + 1];
  }
  const double KL = block_sum_d(kl, red);
  const double Ssum = block_sum_d(s, red);
  if (threadIdx.x == 0) {
    const double N = (double)a.B * a.H * a.NBq * a.NBk;
    const double mean = Ssum / N;
    const double dev = mean - (double)a.tau_target;
    if (a.kl) *a.kl = (float)(KL / a.B);
    if (a.sparse) *a.sparse = (float)(dev * dev);
    *gsp = (float)(a.w_sparse * 2.0 * dev / N);
  }
}

__global__ void loss_add_kernel(float* d, int64_t n, const float* gsp) {
  const float g = *gsp;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    d[i] += g;
}

// ---------------------------------------------------------------------------
// Gate backward: soft = sigmoid(w_out . relu(a_i + c_j)) (zeroed above the diagonal)
// ---------------------------------------------------------------------------
// A [rows_q, hid] = W_q pq + b ; Ct [B*Hk, hid, NBk] = W_k pk
// A = W_q pq + b, Ct = W_k pk (transposed) recomputed from the block means: one warp per
// row, lanes over d (coalesced reads of the means row and of each W_in row, which stays in
// L1), a warp sum per hidden unit.
__global__ void bwd_project_kernel(tasft_gate_bwd_args a, float* A, float* Ct) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t rq = (int64_t)a.B * a.Hq * a.NBq, rk = (int64_t)a.B * a.Hk * a.NBk;
  int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + warp;
  if (r >= rq + rk) return;
  const bool isq = r < rq;
  if (!isq) r -= rq;
  const float* x = (isq ? a.pooled_q : a.pooled_k) + r * a.D;
  const int off = isq ? 0 : a.D;
  float xv[8];  // D <= 256: lane holds x[lane + 32 k]
#pragma unroll
  for (int k = 0; k < 8; ++k) xv[k] = lane + 32 * k < a.D ? x[lane + 32 * k] : 0.f;
  for (int h = 0; h < a.hidden; ++h) {
    const float* w = a.w_in + (int64_t)h * 2 * a.D + off;
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k)
      if (lane + 32 * k < a.D) s = fmaf(__ldg(w + lane + 32 * k), xv[k], s);
    s = warp_sum(s);
    if (lane == 0) {
      if (isq) {
        A[r * a.hidden + h] = s + a.b_in[h];
      } else {
        const int64_t bh = r / a.NBk, j = r % a.NBk;
        Ct[(bh * a.hidden + h) * a.NBk + j] = s;
      }
    }
  }
}

__device__ __forceinline__ float dlogit_of(const tasft_gate_bwd_args& a, int64_t idx) {
  const float s = a.soft[idx];
  return a.d_soft[idx] * s * (1.f - s);
}

// rows: one warp per (b, hq, i); dA[row][h], dwo[row][h]
__global__ void bwd_rows_kernel(tasft_gate_bwd_args a, const float* A, const float* Ct, float* dA, float* dwo) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + warp;
  const int64_t rows = (int64_t)a.B * a.Hq * a.NBq;
  if (row >= rows) return;
  const int hq = (int)((row / a.NBq) % a.Hq), b = (int)(row / ((int64_t)a.NBq * a.Hq));
  const int hk = hq / (a.Hq / a.Hk);
  const float* ct = Ct + ((int64_t)b * a.Hk + hk) * a.hidden * a.NBk;
  // this lane's d logit for its first k-blocks (the rest recomputed when NBk > 256)
  float dlv[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) dlv[k] = lane + 32 * k < a.NBk ? dlogit_of(a, row * a.NBk + lane + 32 * k) : 0.f;
  for (int h = 0; h < a.hidden; ++h) {
    const float ai = A[row * a.hidden + h];
    const float wh = a.w_out[h];
    float da = 0.f, dw = 0.f;
    for (int j = lane, k = 0; j < a.NBk; j += 32, ++k) {
      const float dl = k < 8 ? dlv[k & 7] : dlogit_of(a, row * a.NBk + j);
      const float pre = ai + ct[(int64_t)h * a.NBk + j];
      if (pre > 0.f) {
        da = fmaf(dl, wh, da);
        dw = fmaf(dl, pre, dw);
      }
    }
    da = warp_sum(da);
    dw = warp_sum(dw);
    if (lane == 0) {
      dA[row * a.hidden + h] = da;
      dwo[row * a.hidden + h] = dw;
    }
  }
}

// rows, hidden 32 / 64: lanes take k-blocks and keep per-unit sums in registers over all of
// them (the d logit of a (row, k-block) computed once); a butterfly reduce-scatter over the
// warp then leaves unit h's totals in lane h % 32 (HID / 32 units per lane), so the row
// costs about 2 HID shuffles instead of 10 per unit.
template <int HID>
__global__ void bwd_rows_rs_kernel(tasft_gate_bwd_args a, const float* A, const float* Ct, float* dA, float* dwo) {
  constexpr int U = HID / 32;  // units per lane after the reduction
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + warp;
  const int64_t rows = (int64_t)a.B * a.Hq * a.NBq;
  if (row >= rows) return;
  const int hq = (int)((row / a.NBq) % a.Hq), b = (int)(row / ((int64_t)a.NBq * a.Hq));
  const int hk = hq / (a.Hq / a.Hk);
  const float* ct = Ct + ((int64_t)b * a.Hk + hk) * HID * a.NBk;
  float ai[HID], da[HID], dw[HID];
#pragma unroll
  for (int h = 0; h < HID; ++h) {
    ai[h] = A[row * HID + h];
    da[h] = 0.f;
    dw[h] = 0.f;
  }
  for (int j = lane; j < a.NBk; j += 32) {
    const float dl = dlogit_of(a, row * a.NBk + j);
#pragma unroll
    for (int h = 0; h < HID; ++h) {
      const float pre = ai[h] + ct[(int64_t)h * a.NBk + j];
      if (pre > 0.f) {
        da[h] += dl;  // times w_out[h] after the reduction
        dw[h] = fmaf(dl, pre, dw[h]);
      }
    }
  }
  // reduce-scatter: after the step with offset d, lane l keeps the half of the units whose
  // bit d matches its own
  int n = HID;
#pragma unroll
  for (int d = 16; d >= 1; d >>= 1) {
    const bool upper = (lane & d) != 0;
    n >>= 1;
#pragma unroll
    for (int i = 0; i < HID / 2; ++i) {
      if (i < n) {
        const float sa = upper ? da[i] : da[i + n], ka = upper ? da[i + n] : da[i];
        const float sw = upper ? dw[i] : dw[i + n], kw = upper ? dw[i + n] : dw[i];
        da[i] = ka + __shfl_xor_sync(0xffffffffu, sa, d);
        dw[i] = kw + __shfl_xor_sync(0xffffffffu, sw, d);
      }
    }
  }
  // lane l now holds units l * U .. l * U + U - 1
#pragma unroll
  for (int i = 0; i < U; ++i) {
    const int h = lane * U + i;
    dA[row * HID + h] = da[i] * a.w_out[h];
    dwo[row * HID + h] = dw[i];
  }
}

// cols: one warp per (b, hk, j); dC[col][h] summed over the group's q-heads and rows.
// Lanes take rows; a lane computes its row's d logit once and runs over the hidden units
// with its row of A (contiguous) against c_j (in registers); per-unit warp sums at the end.
template <int HID>
__global__ void bwd_cols_kernel(tasft_gate_bwd_args a, const float* A, const float* Ct, float* dC) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t col = (int64_t)blockIdx.x * (blockDim.x >> 5) + warp;
  const int64_t cols = (int64_t)a.B * a.Hk * a.NBk;
  if (col >= cols) return;
  const int j = (int)(col % a.NBk);
  const int64_t bhk = col / a.NBk;
  const int hk = (int)(bhk % a.Hk), b = (int)(bhk / a.Hk);
  const int grp = a.Hq / a.Hk;
  const int rows = grp * a.NBq;
  float cj[HID], wo[HID], dc[HID];
#pragma unroll
  for (int h = 0; h < HID; ++h) {
    cj[h] = Ct[(bhk * HID + h) * a.NBk + j];
    wo[h] = a.w_out[h];
    dc[h] = 0.f;
  }
  for (int t = lane; t < rows; t += 32) {
    const int g = t / a.NBq, i = t % a.NBq;
    const int64_t row = ((int64_t)b * a.Hq + hk * grp + g) * a.NBq + i;
    const float dl = dlogit_of(a, row * a.NBk + j);
    const float4* ar = reinterpret_cast<const float4*>(A + row * HID);
#pragma unroll
    for (int h4 = 0; h4 < HID / 4; ++h4) {
      const float4 av = ar[h4];
      const float pv[4] = {av.x, av.y, av.z, av.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int h = 4 * h4 + e;
        if (pv[e] + cj[h] > 0.f) dc[h] = fmaf(dl, wo[h], dc[h]);
      }
    }
  }
#pragma unroll
  for (int h = 0; h < HID; ++h) {
    const float v = warp_sum(dc[h]);
    if (lane == 0) dC[col * HID + h] = v;
  }
}

// Any hidden width: one unit at a time.
__global__ void bwd_cols_any_kernel(tasft_gate_bwd_args a, const float* A, const float* Ct, float* dC) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t col = (int64_t)blockIdx.x * (blockDim.x >> 5) + warp;
  const int64_t cols = (int64_t)a.B * a.Hk * a.NBk;
  if (col >= cols) return;
  const int j = (int)(col % a.NBk);
  const int64_t bhk = col / a.NBk;
  const int hk = (int)(bhk % a.Hk), b = (int)(bhk / a.Hk);
  const int grp = a.Hq / a.Hk;
  const int rows = grp * a.NBq;
  for (int h = 0; h < a.hidden; ++h) {
    const float cjh = Ct[(bhk * a.hidden + h) * a.NBk + j];
    const float wh = a.w_out[h];
    float dc = 0.f;
    for (int t = lane; t < rows; t += 32) {
      const int g = t / a.NBq, i = t % a.NBq;
      const int64_t row = ((int64_t)b * a.Hq + hk * grp + g) * a.NBq + i;
      const float pre = A[row * a.hidden + h] + cjh;
      if (pre > 0.f) dc = fmaf(dlogit_of(a, row * a.NBk + j), wh, dc);
    }
    dc = warp_sum(dc);
    if (lane == 0) dC[col * a.hidden + h] = dc;
  }
}

// Weight gradients dW_q = dA^T pq, dW_k = dC^T pk, db = sum dA, dw_out = sum dwo, as two
// deterministic stages: each CTA reduces one chunk of kWChunk rows into partials (the
// rows staged in shared memory), then one thread per output sums the chunks in order.
constexpr int kWChunk = 64;

__global__ void bwd_wpart_kernel(tasft_gate_bwd_args a, const float* dA, const float* dwo, const float* dC,
                                 int chunks_q, float* part, float* part_b) {
  extern __shared__ float sh[];
  const int hid = a.hidden, D = a.D;
  const bool isq = (int)blockIdx.x < chunks_q;
  const int chunk = isq ? blockIdx.x : blockIdx.x - chunks_q;
  const int64_t n = isq ? (int64_t)a.B * a.Hq * a.NBq : (int64_t)a.B * a.Hk * a.NBk;
  const int64_t r0 = (int64_t)chunk * kWChunk;
  const int rows = (int)(n - r0 < kWChunk ? n - r0 : kWChunk);
  const float* g = (isq ? dA : dC) + r0 * hid;
  const float* x = (isq ? a.pooled_q : a.pooled_k) + r0 * D;
  float* sg = sh;                  // [kWChunk][hid]
  float* sx = sh + kWChunk * hid;  // [kWChunk][D]
  for (int i = threadIdx.x; i < rows * hid; i += blockDim.x) sg[i] = g[i];
  for (int i = threadIdx.x; i < rows * D; i += blockDim.x) sx[i] = x[i];
  __syncthreads();
  float* out = part + (int64_t)blockIdx.x * hid * D;
  for (int o = threadIdx.x; o < hid * D; o += blockDim.x) {
    const int h = o / D, d = o % D;
    float s = 0.f;
    for (int r = 0; r < rows; ++r) s = fmaf(sg[r * hid + h], sx[r * D + d], s);
    out[o] = s;
  }
  if (isq) {
    for (int h = threadIdx.x; h < hid; h += blockDim.x) {
      float sb = 0.f, sw = 0.f;
      for (int r = 0; r < rows; ++r) {
        sb += sg[r * hid + h];
        sw += dwo[(r0 + r) * hid + h];
      }
      part_b[((int64_t)chunk * hid + h) * 2] = sb;
      part_b[((int64_t)chunk * hid + h) * 2 + 1] = sw;
    }
  }
}

__global__ void bwd_wsum_kernel(tasft_gate_bwd_args a, int chunks_q, int chunks_k, const float* part,
                                const float* part_b) {
  const int hid = a.hidden, D = a.D;
  const int64_t nw = (int64_t)hid * 2 * D;
  const int64_t o = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (o < nw) {
    const int h = (int)(o / (2 * D)), c = (int)(o % (2 * D));
    const bool isq = c < D;
    const int d = isq ? c : c - D;
    const int c0 = isq ? 0 : chunks_q, nc = isq ? chunks_q : chunks_k;
    float s = 0.f;
    for (int k = 0; k < nc; ++k) s += part[((int64_t)(c0 + k) * hid + h) * D + d];
    a.d_w_in[o] = s;
  } else if (o < nw + 2 * hid) {
    const int t = (int)(o - nw), h = t >> 1, which = t & 1;
    float s = 0.f;
    for (int k = 0; k < chunks_q; ++k) s += part_b[((int64_t)k * hid + h) * 2 + which];
    (which ? a.d_w_out : a.d_b_in)[h] = s;
  }
}

// input grads: d_pooled[r][d] = sum_h g[r][h] W[h][off + d]
__global__ void bwd_inputs_kernel(tasft_gate_bwd_args a, const float* dA, const float* dC) {
  const int64_t rq = (int64_t)a.B * a.Hq * a.NBq;
  int64_t r = blockIdx.x;
  const bool isq = r < rq;
  if (!isq) r -= rq;
  float* out = isq ? a.d_pooled_q : a.d_pooled_k;
  if (!out) return;
  const float* g = (isq ? dA : dC) + r * a.hidden;
  const int off = isq ? 0 : a.D;
  for (int d = threadIdx.x; d < a.D; d += blockDim.x) {
    float s = 0.f;
    for (int h = 0; h < a.hidden; ++h) s = fmaf(g[h], a.w_in[(int64_t)h * 2 * a.D + off + d], s);
    out[r * a.D + d] = s;
  }
}

template <typename T, int D>
static int launch_bm_simt(const tasft_target_args& a, float* bm, int NB, cudaStream_t st) {
  const size_t smem = (size_t)2 * a.block * (D + 1) * sizeof(float);
  auto kern = blockmax_simt_kernel<T, D>;
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return TASFT_ERR_CUDA;
  dim3 grid(NB, NB, a.B * a.Hq);
  kern<<<grid, 256, smem, st>>>(a, bm, NB);
  count_launch();
  return launch_status();
}

template <typename T>
static int launch_bm_simt_dt(const tasft_target_args& a, float* bm, int NB, cudaStream_t st) {
  switch (a.D) {
    case 32: return launch_bm_simt<T, 32>(a, bm, NB, st);
    case 64: return launch_bm_simt<T, 64>(a, bm, NB, st);
    case 128: return launch_bm_simt<T, 128>(a, bm, NB, st);
    default: return TASFT_ERR_UNSUPPORTED;
  }
}

}  // namespace tasft

using namespace tasft;

extern "C" int64_t tasft_gate_target_workspace_size(int32_t B, int32_t Hq, int32_t S, int32_t block) {
  if (B <= 0 || Hq <= 0 || S <= 0 || block <= 0) return -1;
  const int64_t NB = ceil_div(S, block);
  return ((int64_t)B * Hq * NB * NB * 4 + 255) / 256 * 256;
}

extern "C" int tasft_gate_target_fwd(const tasft_target_args* ap, tasft_stream_t stream) {
  if (!ap) return TASFT_ERR_INVALID_ARG;
  const tasft_target_args& a = *ap;
  if (!a.q || !a.k || !a.target) return TASFT_ERR_INVALID_ARG;
  if (a.B <= 0 || a.Hq <= 0 || a.Hk <= 0 || a.S <= 0 || a.D <= 0 || a.block <= 0 || a.Hq % a.Hk)
    return TASFT_ERR_INVALID_ARG;
  if (a.q_stride[3] != 1 || a.k_stride[3] != 1) return TASFT_ERR_INVALID_ARG;
  if (a.block > 128) return TASFT_ERR_UNSUPPORTED;
  const int NB = ceil_div(a.S, a.block);
  float* bm = a.block_max;
  if (!bm) {
    if (!a.workspace || a.workspace_bytes < tasft_gate_target_workspace_size(a.B, a.Hq, a.S, a.block))
      return TASFT_ERR_WORKSPACE;
    bm = reinterpret_cast<float*>(a.workspace);
  }
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  int rc = TASFT_ERR_UNSUPPORTED;
  if (!a.force_simt) rc = gate_target_blockmax_tc(a, bm, st);
  if (rc == TASFT_ERR_UNSUPPORTED) {
    switch (a.dtype) {
      case TASFT_F32: rc = launch_bm_simt_dt<float>(a, bm, NB, st); break;
      case TASFT_BF16: rc = launch_bm_simt_dt<__nv_bfloat16>(a, bm, NB, st); break;
      case TASFT_F16: rc = launch_bm_simt_dt<__half>(a, bm, NB, st); break;
      default: return TASFT_ERR_UNSUPPORTED;
    }
  }
  if (rc != TASFT_OK) return rc;
  const float inv_t = a.temperature > 0.f ? 1.0f / a.temperature : 1.0f;
  target_softmax_kernel<<<a.B * a.Hq, 512, 0, st>>>(bm, a.target, (int64_t)NB * NB, inv_t, a.clamp);
  count_launch();
  return launch_status();
}

template <typename T, int VEC>
static int launch_scores_bm(const tasft_scores_target_args& a, float* bm, int NBq, int NBk, cudaStream_t st) {
  const int kpc = a.block >= 256 ? 1 : 256 / a.block;
  const size_t smem = (size_t)8 * kpc * a.block * sizeof(float);
  auto kern = scores_blockmax_kernel<T, VEC>;
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return TASFT_ERR_CUDA;
  dim3 grid((unsigned)ceil_div(NBk, kpc), (unsigned)NBq, (unsigned)(a.B * a.H));
  kern<<<grid, 256, smem, st>>>(a, bm, NBq, NBk, kpc);
  count_launch();
  return launch_status();
}

template <typename T>
static int launch_scores_bm_dt(const tasft_scores_target_args& a, float* bm, int NBq, int NBk, cudaStream_t st) {
  constexpr int V = 16 / sizeof(T);
  const bool vec = a.stride[3] == 1 && a.block % V == 0 && a.Sk % V == 0 && aligned16(a.scores) &&
                   (a.stride[2] * (int64_t)sizeof(T)) % 16 == 0 && (a.stride[1] * (int64_t)sizeof(T)) % 16 == 0 &&
                   (a.stride[0] * (int64_t)sizeof(T)) % 16 == 0;
  return vec ? launch_scores_bm<T, V>(a, bm, NBq, NBk, st) : launch_scores_bm<T, 1>(a, bm, NBq, NBk, st);
}

extern "C" int64_t tasft_scores_target_workspace_size(int32_t B, int32_t H, int32_t Sq, int32_t Sk, int32_t block) {
  if (B <= 0 || H <= 0 || Sq <= 0 || Sk <= 0 || block <= 0) return -1;
  return ((int64_t)B * H * ceil_div(Sq, block) * ceil_div(Sk, block) * 4 + 255) / 256 * 256;
}

extern "C" int tasft_gate_target_from_scores(const tasft_scores_target_args* ap, tasft_stream_t stream) {
  if (!ap) return TASFT_ERR_INVALID_ARG;
  const tasft_scores_target_args& a = *ap;
  if (!a.scores || !a.target || a.B <= 0 || a.H <= 0 || a.Sq <= 0 || a.Sk <= 0 || a.block <= 0)
    return TASFT_ERR_INVALID_ARG;
  if (a.block > 1024) return TASFT_ERR_UNSUPPORTED;
  const int NBq = ceil_div(a.Sq, a.block), NBk = ceil_div(a.Sk, a.block);
  if ((int64_t)a.B * a.H > 65535 || NBq > 65535) return TASFT_ERR_UNSUPPORTED;
  float* bm = a.block_max;
  if (!bm) {
    if (!a.workspace || a.workspace_bytes < tasft_scores_target_workspace_size(a.B, a.H, a.Sq, a.Sk, a.block))
      return TASFT_ERR_WORKSPACE;
    bm = reinterpret_cast<float*>(a.workspace);
  }
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  int rc;
  switch (a.dtype) {
    case TASFT_F32: rc = launch_scores_bm_dt<float>(a, bm, NBq, NBk, st); break;
    case TASFT_BF16: rc = launch_scores_bm_dt<__nv_bfloat16>(a, bm, NBq, NBk, st); break;
    case TASFT_F16: rc = launch_scores_bm_dt<__half>(a, bm, NBq, NBk, st); break;
    default: return TASFT_ERR_UNSUPPORTED;
  }
  if (rc != TASFT_OK) return rc;
  const float inv_t = a.temperature > 0.f ? 1.0f / a.temperature : 1.0f;
  target_softmax_kernel<<<a.B * a.H, 512, 0, st>>>(bm, a.target, (int64_t)NBq * NBk, inv_t, a.clamp);
  count_launch();
  return launch_status();
}

// Training forward: attention (through the tcgen05 prefill kernel, which is dense when the
// lists hold every causal block) and, from the same S tiles, the gate target's block maxima
// and softmax. Replaces TASFTAttention._training_forward's score matrix + softmax + P V
// (tasft/modules/tasft_attention.py:427-466) followed by compute_gate_target.
extern "C" int tasft_attention_train_fwd(const tasft_train_fwd_args* ap, tasft_stream_t stream) {
  if (!ap || !ap->block_max) return TASFT_ERR_INVALID_ARG;
  const tasft_prefill_args& a = ap->base;
  if (!a.q || !a.k || !a.v || !a.out || !a.kept_idx || !a.kept_cnt) return TASFT_ERR_INVALID_ARG;
  if (a.B <= 0 || a.Hq <= 0 || a.Hk <= 0 || a.S <= 0 || a.D <= 0 || a.Hm <= 0 || a.Hq % a.Hk || a.Hq % a.Hm)
    return TASFT_ERR_INVALID_ARG;
  if (a.q_stride[3] != 1 || a.k_stride[3] != 1 || a.v_stride[3] != 1 || a.o_stride[3] != 1)
    return TASFT_ERR_INVALID_ARG;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int NB = ceil_div(a.S, a.block);
  const int64_t n = (int64_t)a.B * a.Hq * NB * NB;
  fill_kernel<<<(unsigned)std::min<int64_t>(ceil_div(n, 256), 4096), 256, 0, st>>>(ap->block_max, n, -INFINITY);
  count_launch();
  int rc = launch_status();
  if (rc != TASFT_OK) return rc;
  rc = prefill_tc(a, st, nullptr, 0, ap->block_max, ap->emulate_bf16_scores);
  if (rc != TASFT_OK) return rc;  // TASFT_ERR_UNSUPPORTED: not a tcgen05 shape
  if (ap->target) {
    const float inv_t = ap->temperature > 0.f ? 1.0f / ap->temperature : 1.0f;
    target_softmax_kernel<<<a.B * a.Hq, 512, 0, st>>>(ap->block_max, ap->target, (int64_t)NB * NB, inv_t, ap->clamp);
    count_launch();
    rc = launch_status();
  }
  return rc;
}

extern "C" int64_t tasft_gate_loss_workspace_size(int32_t B, int32_t H) {
  if (B <= 0 || H <= 0) return -1;
  return ((int64_t)B * H * 16 + 256 + 255) / 256 * 256;
}

extern "C" int tasft_gate_loss_fwd_bwd(const tasft_loss_args* ap, tasft_stream_t stream) {
  if (!ap) return TASFT_ERR_INVALID_ARG;
  const tasft_loss_args& a = *ap;
  if (!a.soft || !a.target || a.B <= 0 || a.H <= 0 || a.NBq <= 0 || a.NBk <= 0) return TASFT_ERR_INVALID_ARG;
  if (!a.workspace || a.workspace_bytes < tasft_gate_loss_workspace_size(a.B, a.H)) return TASFT_ERR_WORKSPACE;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  double* part = reinterpret_cast<double*>(a.workspace);
  float* gsp = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(a.workspace) + (int64_t)a.B * a.H * 16);
  const int rows = a.B * a.H;
  loss_rows_kernel<<<rows, 256, 0, st>>>(a, part);
  loss_final_kernel<<<1, 256, 0, st>>>(a, part, rows, gsp);
  count_launch(2);
  if (a.d_soft) {
    const int64_t n = (int64_t)rows * a.NBq * a.NBk;
    loss_add_kernel<<<ceil_div(n, 256) > 4096 ? 4096 : ceil_div(n, 256), 256, 0, st>>>(a.d_soft, n, gsp);
    count_launch();
  }
  return launch_status();
}

extern "C" int64_t tasft_gate_bwd_workspace_size(int32_t B, int32_t Hq, int32_t Hk, int32_t NBq, int32_t NBk,
                                                 int32_t hidden) {
  if (B <= 0 || Hq <= 0 || Hk <= 0 || NBq <= 0 || NBk <= 0 || hidden <= 0) return -1;
  const int64_t rq = (int64_t)B * Hq * NBq, rk = (int64_t)B * Hk * NBk;
  const int64_t floats = rq * hidden * 3 + rk * hidden * 2;  // A, dA, dwo, Ct, dC
  // weight-gradient partials: one [hidden, D] slab per row chunk + (db, dw_out) per q chunk
  // (D is not an argument here; the partials are sized for the largest supported D, 256)
  const int64_t cq = (rq + 63) / 64, ck = (rk + 63) / 64;
  const int64_t part = (cq + ck) * hidden * 256 + cq * hidden * 2;
  return ((floats + part) * 4 + 1023) / 256 * 256;
}

extern "C" int tasft_gate_bwd(const tasft_gate_bwd_args* ap, tasft_stream_t stream) {
  if (!ap) return TASFT_ERR_INVALID_ARG;
  const tasft_gate_bwd_args& a = *ap;
  if (!a.pooled_q || !a.pooled_k || !a.d_soft || !a.soft || !a.w_in || !a.b_in || !a.w_out || !a.d_w_in ||
      !a.d_b_in || !a.d_w_out)
    return TASFT_ERR_INVALID_ARG;
  if (a.B <= 0 || a.Hq <= 0 || a.Hk <= 0 || a.NBq <= 0 || a.NBk <= 0 || a.D <= 0 || a.hidden <= 0 || a.Hq % a.Hk)
    return TASFT_ERR_INVALID_ARG;
  if (a.D > 256 || a.hidden > 256) return TASFT_ERR_UNSUPPORTED;
  const int64_t need = tasft_gate_bwd_workspace_size(a.B, a.Hq, a.Hk, a.NBq, a.NBk, a.hidden);
  if (!a.workspace || a.workspace_bytes < need) return TASFT_ERR_WORKSPACE;
  const int64_t rq = (int64_t)a.B * a.Hq * a.NBq, rk = (int64_t)a.B * a.Hk * a.NBk;
  float* A = reinterpret_cast<float*>(a.workspace);
  float* dA = A + rq * a.hidden;
  float* dwo = dA + rq * a.hidden;
  float* Ct = dwo + rq * a.hidden;
  float* dC = Ct + rk * a.hidden;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  bwd_project_kernel<<<(unsigned)ceil_div(rq + rk, 8), 256, 0, st>>>(a, A, Ct);
  if (a.hidden == 32)
    bwd_rows_rs_kernel<32><<<ceil_div(rq, 8), 256, 0, st>>>(a, A, Ct, dA, dwo);
  else if (a.hidden == 64)
    bwd_rows_rs_kernel<64><<<ceil_div(rq, 8), 256, 0, st>>>(a, A, Ct, dA, dwo);
  else
    bwd_rows_kernel<<<ceil_div(rq, 8), 256, 0, st>>>(a, A, Ct, dA, dwo);
  if (a.hidden == 32)
    bwd_cols_kernel<32><<<ceil_div(rk, 8), 256, 0, st>>>(a, A, Ct, dC);
  else if (a.hidden == 64)
    bwd_cols_kernel<64><<<ceil_div(rk, 8), 256, 0, st>>>(a, A, Ct, dC);
  else
    bwd_cols_any_kernel<<<ceil_div(rk, 8), 256, 0, st>>>(a, A, Ct, dC);
  const int cq = (int)ceil_div(rq, kWChunk), ck = (int)ceil_div(rk, kWChunk);
  float* part = dC + rk * a.hidden;
  float* part_b = part + (int64_t)(cq + ck) * a.hidden * a.D;
  const size_t wsm = (size_t)kWChunk * (a.hidden + a.D) * sizeof(float);
  if (wsm > 48 * 1024 && cudaFuncSetAttribute(bwd_wpart_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              (int)wsm) != cudaSuccess)
    return TASFT_ERR_CUDA;
  bwd_wpart_kernel<<<cq + ck, 256, wsm, st>>>(a, dA, dwo, dC, cq, part, part_b);
  const int64_t nout = (int64_t)a.hidden * 2 * a.D + 2 * a.hidden;
  bwd_wsum_kernel<<<(unsigned)ceil_div(nout, 256), 256, 0, st>>>(a, cq, ck, part, part_b);
  bwd_inputs_kernel<<<(unsigned)(rq + rk), 128, 0, st>>>(a, dA, dC);
  count_launch(6);
  return launch_status();
}
