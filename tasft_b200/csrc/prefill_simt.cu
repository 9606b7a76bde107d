// CUDA-core block-sparse prefill kernel: every dtype, block size 32/64/128 and
// head_dim <= 256. It is the exact-fp32 path (tensor cores cannot meet the 1e-5 fp32
// tolerance) and the comparator for the tcgen05 kernel in prefill_tc.cu.
//
// Follows the reference kernel loop (tasft/kernels/block_sparse_fa.py:169-269): per
// (b, q-head, q-block) visit the kept k-blocks in ascending order with an fp32 online
// softmax, cast p to the value dtype before P.V (:252), zero rows that kept nothing
// (:257-258). K/V are read through the GQA group (no repeat_interleave copy). With `cu`
// (cu_seqlens) the tensors hold packed sequences: rows are offset by the sequence's start
// and bounded by its own length.
#include "common.cuh"

namespace tasft {

constexpr int kTPR = 4;  // threads per query row; thread slice c owns d = e*4 + c

template <typename T, int D, int BLK>
__global__ void __launch_bounds__(BLK* kTPR) bsa_prefill_simt_kernel(tasft_prefill_args a, const int32_t* cu) {
  extern __shared__ float sm[];
  float* Ks = sm;            // [BLK][D]
  float* Vs = sm + BLK * D;  // [BLK][D]
  constexpr int DS = D / kTPR;
  const int qb = blockIdx.x, hq = blockIdx.y, b = blockIdx.z;
  const int NB = (a.S + BLK - 1) / BLK;
  const int row0 = cu ? cu[b] : 0;
  const int len = cu ? cu[b + 1] - row0 : a.S;  // tokens of this sequence
  if (qb * BLK >= len) return;                   // q-block past the sequence's end
  const int64_t bo = cu ? 0 : b;                 // batch index into the strided tensors
  const int hk = hq / (a.Hq / a.Hk);
  const int hm = hq / (a.Hq / a.Hm);
  const int r = threadIdx.x / kTPR, c = threadIdx.x % kTPR;
  const int qp = qb * BLK + r;
  const T* Q = reinterpret_cast<const T*>(a.q) + bo * a.q_stride[0] + hq * a.q_stride[1] + row0 * a.q_stride[2];
  const T* K = reinterpret_cast<const T*>(a.k) + bo * a.k_stride[0] + hk * a.k_stride[1] + row0 * a.k_stride[2];
  const T* V = reinterpret_cast<const T*>(a.v) + bo * a.v_stride[0] + hk * a.v_stride[1] + row0 * a.v_stride[2];
  float q[DS], acc[DS];
#pragma unroll
  for (int e = 0; e < DS; ++e) {
    q[e] = qp < len ? to_f<T>(Q[(int64_t)qp * a.q_stride[2] + e * kTPR + c]) : 0.f;
    acc[e] = 0.f;
  }
  float m_i = -INFINITY, l_i = 0.f;
  const int64_t lrow = (((int64_t)b * a.Hm + hm) * NB + qb);
  const int cnt = a.kept_cnt[lrow];
  const int32_t* idx = a.kept_idx + lrow * NB;
  int prev = -1;
  for (int t = 0; t < cnt; ++t) {
    const int kb = idx[t];
    if (kb < 0 || kb >= NB) {
      if (threadIdx.x == 0) set_err(a.err, TASFT_DEVERR_INDEX);
      continue;
    }
    if (kb <= prev && threadIdx.x == 0) set_err(a.err, TASFT_DEVERR_ORDER);
    prev = kb;
    if (a.causal && kb > qb) continue;
    __syncthreads();
    for (int x = threadIdx.x; x < BLK * D; x += blockDim.x) {
      const int j = x / D, d = x % D;
      const int kp = kb * BLK + j;
      Ks[x] = kp < len ? to_f<T>(K[(int64_t)kp * a.k_stride[2] + d]) : 0.f;
      Vs[x] = kp < len ? to_f<T>(V[(int64_t)kp * a.v_stride[2] + d]) : 0.f;
    }
    __syncthreads();
    // pass 1: row max of the masked scores in this block
    float mb = -INFINITY;
    for (int j = 0; j < BLK; ++j) {
      float s = 0.f;
#pragma unroll
      for (int e = 0; e < DS; ++e) s = fmaf(q[e], Ks[j * D + e * kTPR + c], s);
      s += __shfl_xor_sync(0xffffffffu, s, 1);
      s += __shfl_xor_sync(0xffffffffu, s, 2);
      const int kp = kb * BLK + j;
      const bool ok = kp < len && qp < len && (!a.causal || kp <= qp);
      if (ok) mb = fmaxf(mb, s * a.scale);
    }
    const float m_new = fmaxf(m_i, mb);
    const bool live = m_new != -INFINITY;  // false while nothing valid was seen by this row
    const float alpha = live ? expf(m_i - m_new) : 1.0f;
    l_i *= alpha;
#pragma unroll
    for (int e = 0; e < DS; ++e) acc[e] *= alpha;
    // pass 2: p = exp(s - m_new), l += p, acc += round(p) v
    for (int j = 0; j < BLK; ++j) {
      float s = 0.f;
#pragma unroll
      for (int e = 0; e < DS; ++e) s = fmaf(q[e], Ks[j * D + e * kTPR + c], s);
      s += __shfl_xor_sync(0xffffffffu, s, 1);
      s += __shfl_xor_sync(0xffffffffu, s, 2);
      const int kp = kb * BLK + j;
      const bool ok = kp < len && qp < len && (!a.causal || kp <= qp);
      if (!ok || !live) continue;
      const float p = expf(s * a.scale - m_new);
      l_i += p;
      const float pr = round_through<T>(p);
#pragma unroll
      for (int e = 0; e < DS; ++e) acc[e] = fmaf(pr, Vs[j * D + e * kTPR + c], acc[e]);
    }
    m_i = m_new;
  }
  if (qp < len) {
    const float inv = l_i > 0.f ? 1.0f / l_i : 1.0f;
    T* O = reinterpret_cast<T*>(a.out) + bo * a.o_stride[0] + hq * a.o_stride[1] + (int64_t)(row0 + qp) * a.o_stride[2];
#pragma unroll
    for (int e = 0; e < DS; ++e) O[e * kTPR + c] = from_f<T>(acc[e] * inv);
  }
}

template <typename T, int D, int BLK>
static int launch_simt_t(const tasft_prefill_args& a, cudaStream_t st, const int32_t* cu) {
  const int NB = (a.S + BLK - 1) / BLK;
  const size_t smem = (size_t)2 * BLK * D * sizeof(float);
  auto kern = bsa_prefill_simt_kernel<T, D, BLK>;
  if (smem > 48 * 1024) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return TASFT_ERR_CUDA;
  }
  dim3 grid(NB, a.Hq, a.B);
  kern<<<grid, BLK * kTPR, smem, st>>>(a, cu);
  count_launch();
  return launch_status();
}

template <typename T, int D>
static int launch_simt_d(const tasft_prefill_args& a, cudaStream_t st, const int32_t* cu) {
  switch (a.block) {
    case 32: return launch_simt_t<T, D, 32>(a, st, cu);
    case 64: return launch_simt_t<T, D, 64>(a, st, cu);
    case 128: return launch_simt_t<T, D, 128>(a, st, cu);
    default: return TASFT_ERR_UNSUPPORTED;
  }
}

template <typename T>
static int launch_simt_dt(const tasft_prefill_args& a, cudaStream_t st, const int32_t* cu) {
  switch (a.D) {
    case 32: return launch_simt_d<T, 32>(a, st, cu);
    case 64: return launch_simt_d<T, 64>(a, st, cu);
    case 128: return launch_simt_d<T, 128>(a, st, cu);
    default: return TASFT_ERR_UNSUPPORTED;
  }
}

int prefill_simt(const tasft_prefill_args& a, cudaStream_t st, const int32_t* cu) {
  switch (a.dtype) {
    case TASFT_F32: return launch_simt_dt<float>(a, st, cu);
    case TASFT_BF16: return launch_simt_dt<__nv_bfloat16>(a, st, cu);
    case TASFT_F16: return launch_simt_dt<__half>(a, st, cu);
    default: return TASFT_ERR_UNSUPPORTED;
  }
}

}  // namespace tasft
