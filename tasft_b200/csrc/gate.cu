// AttnGate mask builder: block pooling, gate projection, pair scores, threshold and
// kept-block list emission.
//
// Reference: tasft/modules/attn_gate.py:351-485 (AttnGate._pool_to_blocks / forward).
// The reference materialises every (q-block, k-block) pair [q_i; k_j] and runs
// Linear(2D->hid) on it. Here the first layer is split by linearity:
//   W_in [q_i; k_j] + b = (W_q q_i + b) + W_k k_j =: a_i + c_j
// so a_i and c_j are computed once per block (one HBM pass over Q and K pools them; a
// small kernel projects the means), and the pair kernel only evaluates
// w_out . relu(a_i + c_j). Same maths; the fp32 summation order differs from the
// reference's single 2D-long dot product.
#include <algorithm>
#include <cstdlib>
#include <type_traits>

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

// Programmatic dependent launch: a CTA whose streaming is done lets the next kernel on the
// stream (the pair kernel, which waits with griddepcontrol.wait) start launching.
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---------------------------------------------------------------------------
// Kernel 1 fast path, two passes.
// 1a: one thread per (tensor, b, head, block, 16-byte column vector) sums that column over
//     the block's rows by itself: no cross-thread reduction, few registers, many loads in
//     flight; a warp reads two rows' 256 contiguous bytes per step. The fp32 means go to
//     the caller's pooled outputs when given, else to the workspace.
// 1b: the projection of 64 pooled rows per CTA through one half of W_in, as a small
//     matrix product out of shared memory: W transposed (hidden fastest), the 64 means
//     row-major; thread (row octet, hidden unit) accumulates 8 outputs, reading its weight
//     once per d and the means as warp-wide broadcasts.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint64_t pack_f2(float lo, float hi) {
  return ((uint64_t)__float_as_uint(hi) << 32) | __float_as_uint(lo);
}

__device__ __forceinline__ void add_bf16x8(const uint4& u, uint64_t (&acc)[4]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    // bf16 -> fp32 is the 16-bit pattern in the high half of the word
    const uint64_t pair = ((uint64_t)(w[i] & 0xffff0000u) << 32) | (uint64_t)(w[i] << 16);
    asm("add.f32x2 %0, %0, %1;" : "+l"(acc[i]) : "l"(pair));
  }
}

template <typename T, int EPV>
__global__ void __launch_bounds__(kPoolThreads, 6) gate_pool_kernel(tasft_gate_args a, float* mq, float* mk, int NBq,
                                                                int NBk, int lcv) {
  const int CV = 1 << lcv;
  const int D = a.D;
  int t = blockIdx.x * kPoolThreads + threadIdx.x;
  const int nq = a.B * a.Hq * NBq * CV;
  const int nk = a.B * a.Hk * NBk * CV;
  if (t >= nq + nk) return;
  const bool isq = t < nq;
  if (!isq) t -= nq;
  const int c = t & (CV - 1);
  const int row = t >> lcv;  // (b * H + h) * NB + blk
  const int H = isq ? a.Hq : a.Hk, NB = isq ? NBq : NBk, S = isq ? a.Sq : a.Sk;
  const int blk = row % NB, bh = row / NB;
  const int h = bh % H, b = bh / H;
  const int64_t* st = isq ? a.q_stride : a.k_stride;
  const T* p = reinterpret_cast<const T*>(isq ? a.q : a.k) + b * st[0] + h * st[1] +
               (int64_t)blk * a.block * st[2] + c * EPV;
  const int rows = min(a.block, S - blk * a.block);  // padding rows count as zeros
  const int64_t rs = st[2];
  float f[EPV];
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    uint64_t acc[4] = {0, 0, 0, 0};
#pragma unroll 8
    for (int r = 0; r < rows; ++r) add_bf16x8(__ldg(reinterpret_cast<const uint4*>(p + r * rs)), acc);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      f[2 * i] = __uint_as_float((uint32_t)acc[i]);
      f[2 * i + 1] = __uint_as_float((uint32_t)(acc[i] >> 32));
    }
  } else {
#pragma unroll
    for (int e = 0; e < EPV; ++e) f[e] = 0.f;
#pragma unroll 8
    for (int r = 0; r < rows; ++r) {
      float g[EPV];
      Vec16<T>::unpack(__ldg(reinterpret_cast<const uint4*>(p + r * rs)), g);
#pragma unroll
      for (int e = 0; e < EPV; ++e) f[e] += g[e];
    }
  }
  const float inv = 1.0f / (float)a.block;
  float* out = (isq ? mq : mk) + (int64_t)row * D + c * EPV;
#pragma unroll
  for (int e = 0; e < EPV; e += 4)
    *reinterpret_cast<float4*>(out + e) = make_float4(f[e] * inv, f[e + 1] * inv, f[e + 2] * inv, f[e + 3] * inv);
}


// Pool and project in one pass. A block's column sums are split over CV * RS lanes of one
// warp: lane (rs, c) sums the 16-byte column c (EPV elements) over rows rs, rs + RS, ...
// (so a warp instruction reads RS whole consecutive rows), and shuffles over the RS row
// groups complete the sums. Then each lane forms the partial products of its EPV means with
// the HID / RS units of its row group's share of W_in (read through L1), and a butterfly
// reduce-scatter over the block's CV lanes sums them: lane (rs, c) ends with
// NOUT = HID / (RS * CV) units. Saves the means' round trip through HBM and a kernel boundary.
template <typename T, int EPV, int CV, int HID, int RS>
__global__ void __launch_bounds__(kPoolThreads, 3) gate_pool_project_fused_kernel(tasft_gate_args a, float* A,
                                                                                  float* Ct, int NBq, int NBk) {
  constexpr int D = EPV * CV;
  constexpr int HR = HID / RS;     // units per row group
  constexpr int NOUT = HR / CV;    // units per lane after the reduction
  static_assert(HR % CV == 0 && (CV & (CV - 1)) == 0 && (RS & (RS - 1)) == 0 && CV * RS <= 32, "shape");
  int t = blockIdx.x * kPoolThreads + threadIdx.x;
  const int nq = a.B * a.Hq * NBq * CV * RS;
  const int nk = a.B * a.Hk * NBk * CV * RS;
  const bool live = t < nq + nk;
  if (!live) t = nq + nk - 1;  // idle lanes shadow the last block so the shuffles stay full-warp
  const bool isq = t < nq;
  if (!isq) t -= nq;
  const int c = t % CV;
  const int rs = (t / CV) % RS;
  const int row = t / (CV * RS);  // (b * H + h) * NB + blk
  const int H = isq ? a.Hq : a.Hk, NB = isq ? NBq : NBk, S = isq ? a.Sq : a.Sk;
  const int blk = row % NB, bh = row / NB;
  const int h = bh % H, b = bh / H;
  const int64_t* st = isq ? a.q_stride : a.k_stride;
  const int64_t rstr = st[2];
  const T* p = reinterpret_cast<const T*>(isq ? a.q : a.k) + b * st[0] + h * st[1] +
               ((int64_t)blk * a.block + rs) * rstr + c * EPV;
  const int rows = min(a.block, S - blk * a.block);  // padding rows count as zeros
  const int64_t rs_step = RS * rstr;
  float f[EPV];
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    uint64_t acc[4] = {0, 0, 0, 0};
#pragma unroll 8
    for (int r = rs; r < rows; r += RS, p += rs_step) add_bf16x8(__ldg(reinterpret_cast<const uint4*>(p)), acc);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      f[2 * i] = __uint_as_float((uint32_t)acc[i]);
      f[2 * i + 1] = __uint_as_float((uint32_t)(acc[i] >> 32));
    }
  } else {
#pragma unroll
    for (int e = 0; e < EPV; ++e) f[e] = 0.f;
#pragma unroll 8
    for (int r = rs; r < rows; r += RS, p += rs_step) {
      float g[EPV];
      Vec16<T>::unpack(__ldg(reinterpret_cast<const uint4*>(p)), g);
#pragma unroll
      for (int e = 0; e < EPV; ++e) f[e] += g[e];
    }
  }
  // this CTA's streaming is done: the pair kernel may launch (it waits for this grid)
  pdl_trigger();
  // complete the column sums over the RS row groups (lanes CV apart)
#pragma unroll
  for (int e = 0; e < EPV; ++e)
#pragma unroll
    for (int d = CV; d < CV * RS; d <<= 1) f[e] += __shfl_xor_sync(0xffffffffu, f[e], d);
  const float inv = 1.0f / (float)a.block;
#pragma unroll
  for (int e = 0; e < EPV; ++e) f[e] *= inv;
  float* pooled = isq ? a.pooled_q : a.pooled_k;
  if (pooled && live && rs == 0) {
    float* out = pooled + (int64_t)row * D + c * EPV;
#pragma unroll
    for (int e = 0; e < EPV; e += 4) *reinterpret_cast<float4*>(out + e) = make_float4(f[e], f[e + 1], f[e + 2], f[e + 3]);
  }
  // partial products of this lane's EPV means with its row group's units [rs * HR, rs * HR + HR)
  float v[HR];
  const float* w = a.w_in + (int64_t)rs * HR * 2 * D + (isq ? 0 : D) + c * EPV;
#pragma unroll
  for (int j = 0; j < HR; ++j) {
    float s = 0.f;
#pragma unroll
    for (int e = 0; e < EPV; e += 4) {
      const float4 wv = __ldg(reinterpret_cast<const float4*>(w + (int64_t)j * 2 * D + e));
      s = fmaf(wv.x, f[e], fmaf(wv.y, f[e + 1], fmaf(wv.z, f[e + 2], fmaf(wv.w, f[e + 3], s))));
    }
    v[j] = s;
  }
  // butterfly reduce-scatter over the CV lanes of this row group
  int n = HR;
#pragma unroll
  for (int d = CV / 2; d >= 1; d >>= 1) {
    const bool upper = (c & d) != 0;
    n >>= 1;
#pragma unroll
    for (int i = 0; i < HR / 2; ++i) {
      if (i < n) {
        const float send = upper ? v[i] : v[i + n];
        const float keep = upper ? v[i + n] : v[i];
        v[i] = keep + __shfl_xor_sync(0xffffffffu, send, d);
      }
    }
  }
  if (!live) return;
  const int j0 = rs * HR + c * NOUT;  // lane (rs, c) holds units [j0, j0 + NOUT)
  if (isq) {
#pragma unroll
    for (int i = 0; i < NOUT; ++i) A[(int64_t)row * HID + j0 + i] = v[i] + a.b_in[j0 + i];
  } else {
#pragma unroll
    for (int i = 0; i < NOUT; ++i) Ct[((int64_t)bh * HID + j0 + i) * NB + blk] = v[i];
  }
}

// Persistent form of the fused kernel for bf16 (one warp per block as above): each warp
// walks blocks with a stride of the grid's warps and, before projecting a block, puts the
// first 8 row loads of its next block in flight, so the warp's reads do not stop while it
// computes the projection.
template <int CV, int HID, int RS>
__global__ void __launch_bounds__(kPoolThreads, 2) gate_pool_project_stream_kernel(tasft_gate_args a, float* A,
                                                                                  float* Ct, int NBq, int NBk) {
  constexpr int EPV = 8;
  constexpr int D = EPV * CV;
  constexpr int HR = HID / RS;
  constexpr int NOUT = HR / CV;
  constexpr int kPre = 8;  // rows per lane put in flight ahead
  static_assert(HR % CV == 0 && CV * RS == 32, "one warp per block");
  using T = __nv_bfloat16;
  const int lane = threadIdx.x & 31;
  const int c = lane % CV, rs = lane / CV;
  const int64_t nq = (int64_t)a.B * a.Hq * NBq, nk = (int64_t)a.B * a.Hk * NBk, total = nq + nk;
  const int64_t nw = (int64_t)gridDim.x * (blockDim.x >> 5);
  int64_t item = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  struct Blk {
    const T* p;  // this lane's first row (row rs, column c)
    int64_t rstr;
    int rows;
  };
  auto locate = [&](int64_t it) -> Blk {
    const bool isq = it < nq;
    const int64_t r = isq ? it : it - nq;
    const int H = isq ? a.Hq : a.Hk, NB = isq ? NBq : NBk, S = isq ? a.Sq : a.Sk;
    const int blk = (int)(r % NB);
    const int64_t bh = r / NB;
    const int h = (int)(bh % H), b = (int)(bh / H);
    const int64_t* st = isq ? a.q_stride : a.k_stride;
    Blk k;
    k.rstr = st[2];
    k.p = reinterpret_cast<const T*>(isq ? a.q : a.k) + b * st[0] + h * st[1] + ((int64_t)blk * a.block + rs) * k.rstr +
          c * EPV;
    k.rows = min(a.block, S - blk * a.block);
    return k;
  };
  uint4 pre[kPre];
  auto prefetch = [&](const Blk& k) {
#pragma unroll
    for (int i = 0; i < kPre; ++i)
      pre[i] = rs + RS * i < k.rows ? __ldg(reinterpret_cast<const uint4*>(k.p + (int64_t)RS * i * k.rstr))
                                    : make_uint4(0u, 0u, 0u, 0u);
  };
  Blk cur{};
  if (item < total) {
    cur = locate(item);
    prefetch(cur);
  }
  for (; item < total; item += nw) {
    uint64_t acc[4] = {0, 0, 0, 0};
#pragma unroll
    for (int i = 0; i < kPre; ++i) add_bf16x8(pre[i], acc);
    {
      const T* p = cur.p + (int64_t)RS * kPre * cur.rstr;
#pragma unroll 8
      for (int r = rs + RS * kPre; r < cur.rows; r += RS, p += RS * cur.rstr)
        add_bf16x8(__ldg(reinterpret_cast<const uint4*>(p)), acc);
    }
    // the next block's first rows go out now, ahead of this block's projection
    const int64_t nxt = item + nw;
    Blk nb{};
    if (nxt < total) {
      nb = locate(nxt);
      prefetch(nb);
    }
    float f[EPV];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      f[2 * i] = __uint_as_float((uint32_t)acc[i]);
      f[2 * i + 1] = __uint_as_float((uint32_t)(acc[i] >> 32));
    }
#pragma unroll
    for (int e = 0; e < EPV; ++e)
#pragma unroll
      for (int d = CV; d < 32; d <<= 1) f[e] += __shfl_xor_sync(0xffffffffu, f[e], d);
    const float inv = 1.0f / (float)a.block;
#pragma unroll
    for (int e = 0; e < EPV; ++e) f[e] *= inv;
    const bool isq = item < nq;
    const int64_t row = isq ? item : item - nq;  // (b * H + h) * NB + blk
    float* pooled = isq ? a.pooled_q : a.pooled_k;
    if (pooled && rs == 0) {
      float* out = pooled + row * D + c * EPV;
#pragma unroll
      for (int e = 0; e < EPV; e += 4) *reinterpret_cast<float4*>(out + e) = make_float4(f[e], f[e + 1], f[e + 2], f[e + 3]);
    }
    float v[HR];
    const float* w = a.w_in + (int64_t)rs * HR * 2 * D + (isq ? 0 : D) + c * EPV;
#pragma unroll
    for (int j = 0; j < HR; ++j) {
      float sacc = 0.f;
#pragma unroll
      for (int e = 0; e < EPV; e += 4) {
        const float4 wv = __ldg(reinterpret_cast<const float4*>(w + (int64_t)j * 2 * D + e));
        sacc = fmaf(wv.x, f[e], fmaf(wv.y, f[e + 1], fmaf(wv.z, f[e + 2], fmaf(wv.w, f[e + 3], sacc))));
      }
      v[j] = sacc;
    }
    int n = HR;
#pragma unroll
    for (int d = CV / 2; d >= 1; d >>= 1) {
      const bool upper = (c & d) != 0;
      n >>= 1;
#pragma unroll
      for (int i = 0; i < HR / 2; ++i) {
        if (i < n) {
          const float send = upper ? v[i] : v[i + n];
          const float keep = upper ? v[i + n] : v[i];
          v[i] = keep + __shfl_xor_sync(0xffffffffu, send, d);
        }
      }
    }
    const int j0 = rs * HR + c * NOUT;
    if (isq) {
#pragma unroll
      for (int i = 0; i < NOUT; ++i) A[row * HID + j0 + i] = v[i] + a.b_in[j0 + i];
    } else {
      const int64_t bh = row / NBk, blk = row % NBk;
#pragma unroll
      for (int i = 0; i < NOUT; ++i) Ct[(bh * HID + j0 + i) * NBk + blk] = v[i];
    }
    cur = nb;
  }
  pdl_trigger();
}

template <int HID>
__global__ void __launch_bounds__(kPoolThreads) gate_project_kernel(tasft_gate_args a, const float* mq,
                                                                   const float* mk, float* A, float* Ct, int NBq,
                                                                   int NBk) {
  extern __shared__ __align__(16) float psm[];  // w [HID][D + 1] (padded), then means [RPC][D]
  constexpr int RPT = 4;                       // rows per thread: each weight read feeds 4 FMAs
  constexpr int RPC = kPoolThreads / HID * RPT;  // rows per CTA
  const int D = a.D;
  const int rq = a.B * a.Hq * NBq, rk = a.B * a.Hk * NBk;
  const int tq = (rq + RPC - 1) / RPC;
  const bool isq = (int)blockIdx.x < tq;
  const int r0 = (isq ? blockIdx.x : blockIdx.x - tq) * RPC;
  const int nrows = min(RPC, (isq ? rq : rk) - r0);
  const int DP = D + 1;  // row pitch: lanes (units j) reading one d hit distinct banks
  float* wt = psm;
  float* ms = psm + ((HID * DP + 3) & ~3);
  const int off = isq ? 0 : D;
  // 16-byte reads, unrolled so a thread's loads are in flight together (a rolled loop
  // waits one L2 round trip per element before the compute can start)
#pragma unroll 8
  for (int x = threadIdx.x; x < HID * D / 4; x += kPoolThreads) {
    const int j = x / (D / 4), d = (x % (D / 4)) * 4;
    const float4 v = __ldg(reinterpret_cast<const float4*>(a.w_in + (int64_t)j * 2 * D + off + d));
    float* w = wt + j * DP + d;
    w[0] = v.x;
    w[1] = v.y;
    w[2] = v.z;
    w[3] = v.w;
  }
  const float4* src = reinterpret_cast<const float4*>((isq ? mq : mk) + (int64_t)r0 * D);
  for (int x = threadIdx.x; x < nrows * D / 4; x += kPoolThreads) reinterpret_cast<float4*>(ms)[x] = src[x];
  __syncthreads();
  const int j = threadIdx.x % HID, rg = threadIdx.x / HID;  // rows rg + i * (RPC / RPT)
  constexpr int kStride = RPC / RPT;
  if (rg >= nrows) return;
  const float* w = wt + j * DP;
  float acc[RPT];
#pragma unroll
  for (int i = 0; i < RPT; ++i) acc[i] = 0.f;
  for (int d = 0; d < D; d += 4) {
    const float w0 = w[d], w1 = w[d + 1], w2 = w[d + 2], w3 = w[d + 3];
#pragma unroll
    for (int i = 0; i < RPT; ++i) {
      const int r = min(rg + i * kStride, nrows - 1);
      const float4 mv = *reinterpret_cast<const float4*>(ms + r * D + d);  // broadcast within the warp
      acc[i] = fmaf(mv.x, w0, fmaf(mv.y, w1, fmaf(mv.z, w2, fmaf(mv.w, w3, acc[i]))));
    }
  }
#pragma unroll
  for (int i = 0; i < RPT; ++i) {
    const int r = rg + i * kStride;
    if (r >= nrows) break;
    const int rr = r0 + r;
    if (isq) {
      A[(int64_t)rr * HID + j] = acc[i] + a.b_in[j];
    } else {
      const int blk = rr % NBk, bh = rr / NBk;
      Ct[((int64_t)bh * HID + j) * NBk + blk] = acc[i];
    }
  }
}

template <int HID>
static void launch_project(const tasft_gate_args& a, const float* mq, const float* mk, float* A, float* Ct, int NBq,
                           int NBk, cudaStream_t st) {
  constexpr int RPC = kPoolThreads / HID * 4;
  const int rq = a.B * a.Hq * NBq, rk = a.B * a.Hk * NBk;
  const int grid = ceil_div(rq, RPC) + ceil_div(rk, RPC);
  const size_t smem = (size_t)(((HID * (a.D + 1) + 3) & ~3) + RPC * a.D) * sizeof(float);
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(gate_project_kernel<HID>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  gate_project_kernel<HID><<<grid, kPoolThreads, smem, st>>>(a, mq, mk, A, Ct, NBq, NBk);
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

// The same row computation with the kv-head's projected K rows (Ct slab, hid x NBk)
// staged in shared memory once per CTA: a CTA takes 8 q-rows of one (b, kv-head) (the
// group's q-heads read the same slab), one warp per row, lanes over k-blocks.
constexpr int kSlabRowsDefault = 16;  // q-rows per CTA (4 per warp): the Ct slab staging is amortised

// HID = hidden width when it is 32 or 64 (a_i and w_out then live in registers), 0 otherwise.
template <int HID>
__global__ void __launch_bounds__(kRowsPerCta * 32) gate_pair_slab_kernel(tasft_gate_args a, const float* A,
                                                                          const float* Ct, int NBq, int NBk,
                                                                          int kSlabRows) {
  extern __shared__ float sm[];  // ct [hid][NBk], arows [kSlabRows][hid], wout [hid]
  const int hid = a.hidden;
  const int grp = a.Hq / a.Hk;
  const int per_bk = grp * NBq;  // q-rows of one (b, kv-head)
  const int chunks = (per_bk + kSlabRows - 1) / kSlabRows;
  const int bk = blockIdx.x / chunks;  // b * Hk + hk
  const int lr0 = (blockIdx.x % chunks) * kSlabRows;
  const int nrows = min(kSlabRows, per_bk - lr0);
  const int b = bk / a.Hk, hk = bk % a.Hk;
  float* ct = sm;
  float* arows = sm + hid * NBk;
  float* wout = arows + kSlabRows * hid;
  const float* src = Ct + (int64_t)bk * hid * NBk;
  // launched early (programmatic dependent launch) behind the pooling kernel: wait for its
  // results; a no-op when launched normally
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if constexpr (HID > 0) {
    // [unit pair][k-block][2]: a lane's two units of one k-block are one 8-byte word, and the
    // lanes of a warp (consecutive k-blocks) read consecutive words
#pragma unroll 8
    for (int x = threadIdx.x; x < hid * NBk; x += blockDim.x) {
      const int h = x / NBk, j = x % NBk;
      ct[((h >> 1) * NBk + j) * 2 + (h & 1)] = __ldg(src + x);
    }
  } else {
#pragma unroll 8
    for (int x = threadIdx.x; x < hid * NBk; x += blockDim.x) ct[x] = __ldg(src + x);
  }
  for (int x = threadIdx.x; x < nrows * hid; x += blockDim.x) {
    const int r = x / hid, lr = lr0 + r;
    const int64_t row = ((int64_t)b * a.Hq + hk * grp + lr / NBq) * NBq + lr % NBq;
    arows[x] = A[row * hid + x % hid];
  }
  for (int j = threadIdx.x; j < hid; j += blockDim.x) wout[j] = a.w_out[j];
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool causal = a.causal && (NBq == NBk);
  // kept blocks of the whole CTA, added to the global counter once (a counter hit by every
  // row serialises at one L2 slice)
  __shared__ int cta_kept;
  if (threadIdx.x == 0) cta_kept = 0;
  __syncthreads();
  int warp_kept = 0;
  for (int r = warp; r < nrows; r += kRowsPerCta) {
    const int lr = lr0 + r;
    const int i = lr % NBq;
    const int64_t row = ((int64_t)b * a.Hq + hk * grp + lr / NBq) * NBq + i;
    const float* ar = arows + r * hid;
    int cnt = 0, kept_total = 0;
    uint64_t arr2[HID > 0 ? HID / 2 : 1];  // this row's a_i, and w_out, in registers (HID known),
    uint64_t wr2[HID > 0 ? HID / 2 : 1];   // as (unit h, unit h + 1) pairs
    if constexpr (HID > 0) {
#pragma unroll
      for (int h = 0; h < HID; h += 4) {
        const float4 av = *reinterpret_cast<const float4*>(ar + h);
        const float4 wv = *reinterpret_cast<const float4*>(wout + h);
        arr2[h >> 1] = pack_f2(av.x, av.y);
        arr2[(h >> 1) + 1] = pack_f2(av.z, av.w);
        wr2[h >> 1] = pack_f2(wv.x, wv.y);
        wr2[(h >> 1) + 1] = pack_f2(wv.z, wv.w);
      }
    }
    for (int j0 = 0; j0 < NBk; j0 += 32) {
      const int j = j0 + lane;
      const bool in_range = j < NBk;
      float s = 0.f;
      if (in_range) {
        float l0 = 0.f, l1 = 0.f;
        if constexpr (HID > 0) {
          // units h (even chain) and h + 1 (odd chain) side by side in packed f32x2 ops: the same
          // per-lane roundings as two scalar chains
          uint64_t acc = 0;
          const float2* c2 = reinterpret_cast<const float2*>(ct) + j;
#pragma unroll
          for (int h = 0; h < HID; h += 2) {
            const float2 cv = c2[(h >> 1) * NBk];
            uint64_t pre;
            asm("add.f32x2 %0, %1, %2;" : "=l"(pre) : "l"(arr2[h >> 1]), "l"(pack_f2(cv.x, cv.y)));
            const uint64_t rl = pack_f2(fmaxf(__uint_as_float((uint32_t)pre), 0.f),
                                        fmaxf(__uint_as_float((uint32_t)(pre >> 32)), 0.f));
            asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(acc) : "l"(wr2[h >> 1]), "l"(rl));
          }
          l0 = __uint_as_float((uint32_t)acc);
          l1 = __uint_as_float((uint32_t)(acc >> 32));
        } else {
          int h = 0;
          for (; h + 1 < hid; h += 2) {
            l0 = fmaf(wout[h], fmaxf(ar[h] + ct[h * NBk + j], 0.f), l0);
            l1 = fmaf(wout[h + 1], fmaxf(ar[h + 1] + ct[(h + 1) * NBk + j], 0.f), l1);
          }
          if (h < hid) l0 = fmaf(wout[h], fmaxf(ar[h] + ct[h * NBk + j], 0.f), l0);
        }
        s = 1.0f / (1.0f + __expf(-(l0 + l1)));
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
    if (lane == 0 && a.kept_cnt) a.kept_cnt[row] = cnt;
    warp_kept += kept_total;
  }
  if (lane == 0 && warp_kept) atomicAdd(&cta_kept, warp_kept);
  __syncthreads();
  if (threadIdx.x == 0 && a.num_kept && cta_kept) atomicAdd(a.num_kept, cta_kept);
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
                                             int32_t hidden, int32_t D) {
  if (B <= 0 || Hq <= 0 || Hk <= 0 || Sq <= 0 || Sk <= 0 || block <= 0 || hidden <= 0 || D <= 0) return -1;
  const int64_t NBq = ceil_div(Sq, block), NBk = ceil_div(Sk, block);
  const int64_t rows = (int64_t)B * Hq * NBq + (int64_t)B * Hk * NBk;
  // [projected rows: A then Ct] [fp32 block means: Q rows then K rows, 256-byte aligned]
  const int64_t floats = (rows * hidden + 63) / 64 * 64 + rows * D;
  return ((floats * 4 + 255) / 256) * 256;
}

template <typename T>
static int launch_pool(const tasft_gate_args& a, float* A, float* Ct, float* mq, float* mk, int NBq, int NBk,
                       cudaStream_t st) {
  constexpr int EPV = 16 / sizeof(T);
  const bool vec_ok = (a.D % EPV == 0) && aligned16(a.q) && aligned16(a.k) && (a.q_stride[0] % EPV == 0) &&
                      (a.q_stride[1] % EPV == 0) && (a.q_stride[2] % EPV == 0) && (a.k_stride[0] % EPV == 0) &&
                      (a.k_stride[1] % EPV == 0) && (a.k_stride[2] % EPV == 0) && (a.D / EPV <= kPoolThreads);
  const int64_t grid = (int64_t)a.B * a.Hq * NBq + (int64_t)a.B * a.Hk * NBk;
  // fast path: hidden 32 or 64 (the gate's default is max(32, D/4)) and D <= 128, so the
  // projection's shared memory (D * (hidden + 256 / hidden) floats) stays under 48 KB
  const int CV = a.D / EPV;
  const int64_t nthreads = ((int64_t)a.B * a.Hq * NBq + (int64_t)a.B * a.Hk * NBk) * CV;
  const bool pooled_ok = (!a.pooled_q || aligned16(a.pooled_q)) && (!a.pooled_k || aligned16(a.pooled_k)) &&
                         aligned16(a.w_in);
  // row groups per block in the fused kernel: a block takes a whole warp (CV * RS = 32)
  const int RS = 32 / (CV > 0 ? CV : 1);
  if (std::is_same<T, __nv_bfloat16>::value && vec_ok && (a.D == 64 || a.D == 128) &&
      (a.hidden == 32 || a.hidden == 64) && pooled_ok && !std::getenv("TASFT_GATE_UNFUSED")) {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int64_t items = (int64_t)a.B * a.Hq * NBq + (int64_t)a.B * a.Hk * NBk;
    int64_t blocks = (int64_t)sms * 2;
    if (blocks * (kPoolThreads / 32) > items) blocks = ceil_div(items, kPoolThreads / 32);
    auto go = [&](auto kern) { kern<<<(unsigned)blocks, kPoolThreads, 0, st>>>(a, A, Ct, NBq, NBk); };
    if (a.D == 128) {
      if (a.hidden == 32) go(gate_pool_project_stream_kernel<16, 32, 2>);
      else go(gate_pool_project_stream_kernel<16, 64, 2>);
    } else {
      if (a.hidden == 32) go(gate_pool_project_stream_kernel<8, 32, 4>);
      else go(gate_pool_project_stream_kernel<8, 64, 4>);
    }
  } else   if (vec_ok && EPV == 8 && (a.D == 64 || a.D == 128) && (a.hidden == 32 || a.hidden == 64) && pooled_ok &&
      nthreads * RS < (1LL << 31) - kPoolThreads && !std::getenv("TASFT_GATE_UNFUSED")) {
    const unsigned blocks = (unsigned)ceil_div(nthreads * RS, kPoolThreads);
    auto go = [&](auto kern) { kern<<<blocks, kPoolThreads, 0, st>>>(a, A, Ct, NBq, NBk); };
    if (a.D == 128) {
      if (a.hidden == 32) go(gate_pool_project_fused_kernel<T, 8, 16, 32, 2>);
      else go(gate_pool_project_fused_kernel<T, 8, 16, 64, 2>);
    } else {
      if (a.hidden == 32) go(gate_pool_project_fused_kernel<T, 8, 8, 32, 4>);
      else go(gate_pool_project_fused_kernel<T, 8, 8, 64, 4>);
    }
  } else if (vec_ok && (CV & (CV - 1)) == 0 && a.D % 4 == 0 && a.D <= 128 && (a.hidden == 32 || a.hidden == 64) &&
      nthreads < (1LL << 31) - kPoolThreads && aligned16(mq) && aligned16(mk)) {
    int lcv = 0;
    while ((1 << lcv) < CV) ++lcv;
    gate_pool_kernel<T, EPV><<<ceil_div(nthreads, kPoolThreads), kPoolThreads, 0, st>>>(a, mq, mk, NBq, NBk, lcv);
    if (a.hidden == 32) launch_project<32>(a, mq, mk, A, Ct, NBq, NBk, st);
    else launch_project<64>(a, mq, mk, A, Ct, NBq, NBk, st);
    count_launch();
  } else if (vec_ok) {
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
  const bool pooled_in = !a.q && !a.k;  // block means given (tasft_qkv_rope_pool)
  if (pooled_in && (!a.pooled_q || !a.pooled_k)) return TASFT_ERR_INVALID_ARG;
  if ((!pooled_in && (!a.q || !a.k)) || !a.w_in || !a.b_in || !a.w_out || !a.soft) return TASFT_ERR_INVALID_ARG;
  if (a.B <= 0 || a.Hq <= 0 || a.Hk <= 0 || a.Sq <= 0 || a.Sk <= 0 || a.D <= 0 || a.block <= 0)
    return TASFT_ERR_INVALID_ARG;
  if (a.Hq % a.Hk != 0) return TASFT_ERR_INVALID_ARG;
  if (a.hidden <= 0 || a.hidden > 256) return TASFT_ERR_UNSUPPORTED;
  if (a.D > 1024) return TASFT_ERR_UNSUPPORTED;
  if ((a.kept_idx == nullptr) != (a.kept_cnt == nullptr)) return TASFT_ERR_INVALID_ARG;
  if (!pooled_in && (a.q_stride[3] != 1 || a.k_stride[3] != 1)) return TASFT_ERR_INVALID_ARG;
  const int64_t need = tasft_gate_workspace_size(a.B, a.Hq, a.Hk, a.Sq, a.Sk, a.block, a.hidden, a.D);
  if (!a.workspace || a.workspace_bytes < need) return TASFT_ERR_WORKSPACE;
  const int NBq = ceil_div(a.Sq, a.block), NBk = ceil_div(a.Sk, a.block);
  float* A = reinterpret_cast<float*>(a.workspace);
  float* Ct = A + (int64_t)a.B * a.Hq * NBq * a.hidden;
  // block means: the caller's pooled outputs when given, else the workspace's tail
  float* means = A + ((int64_t)a.B * a.Hq * NBq * a.hidden + (int64_t)a.B * a.Hk * NBk * a.hidden + 63) / 64 * 64;
  float* mq = a.pooled_q ? a.pooled_q : means;
  float* mk = a.pooled_k ? a.pooled_k : means + (int64_t)a.B * a.Hq * NBq * a.D;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  int rc;
  if (pooled_in) {
    if ((a.hidden != 32 && a.hidden != 64) || a.D % 4 || !aligned16(mq) || !aligned16(mk))
      return TASFT_ERR_UNSUPPORTED;
    if (a.hidden == 32) launch_project<32>(a, mq, mk, A, Ct, NBq, NBk, st);
    else launch_project<64>(a, mq, mk, A, Ct, NBq, NBk, st);
    count_launch();
    rc = launch_status();
  } else switch (a.dtype) {
    case TASFT_F32: rc = launch_pool<float>(a, A, Ct, mq, mk, NBq, NBk, st); break;
    case TASFT_BF16: rc = launch_pool<__nv_bfloat16>(a, A, Ct, mq, mk, NBq, NBk, st); break;
    case TASFT_F16: rc = launch_pool<__half>(a, A, Ct, mq, mk, NBq, NBk, st); break;
    default: return TASFT_ERR_UNSUPPORTED;
  }
  if (rc != TASFT_OK) return rc;
  int kSlabRows = kSlabRowsDefault;
  if (const char* e = std::getenv("TASFT_GATE_SLAB_ROWS")) kSlabRows = std::max(1, std::atoi(e));  // tuning aid
  const size_t slab = (size_t)(a.hidden * NBk + kSlabRows * a.hidden + a.hidden) * sizeof(float);
  if (slab <= 96 * 1024) {
    auto kern = a.hidden == 32 ? gate_pair_slab_kernel<32> : a.hidden == 64 ? gate_pair_slab_kernel<64>
                                                                                : gate_pair_slab_kernel<0>;
    if (slab > 48 * 1024 &&
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)slab) != cudaSuccess)
      return TASFT_ERR_CUDA;
    const int64_t grid = (int64_t)a.B * a.Hk * ceil_div((int64_t)(a.Hq / a.Hk) * NBq, kSlabRows);
    // programmatic dependent launch: the pair kernel's launch overlaps the pooling tail
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(kRowsPerCta * 32);
    cfg.dynamicSmemBytes = slab;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = std::getenv("TASFT_GATE_NO_PDL") ? 0 : 1;  // comparison aid
    if (cudaLaunchKernelEx(&cfg, kern, a, (const float*)A, (const float*)Ct, NBq, NBk, kSlabRows) != cudaSuccess)
      return launch_status();
  } else {
    const int64_t rows = (int64_t)a.B * a.Hq * NBq;
    const size_t smem = (size_t)(kRowsPerCta + 1) * a.hidden * sizeof(float);
    gate_pair_kernel<<<ceil_div(rows, kRowsPerCta), kRowsPerCta * 32, smem, st>>>(a, A, Ct, NBq, NBk);
  }
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
