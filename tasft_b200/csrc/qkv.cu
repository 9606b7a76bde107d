// Q/K/V projection epilogue: head split, rotary embedding and the gate's block pooling in
// one pass over the projection outputs.
//
// Reference (tasft/modules/tasft_attention.py:615-742, _prepare_qkv): the q/k/v projection
// outputs [B, S, H*D] are viewed as [B, S, H, D], transposed to [B, H, S, D], rotated
// (_apply_rotary_pos_emb, :872-908: x * cos + rotate_half(x) * sin, each op in the model
// dtype) and, before attention, pooled again by AttnGate (attn_gate.py:351-375: zero-padded
// block means). Here one kernel reads each projection output once, writes the rotated
// [B, H, S, D] tensors and, for Q and K, the fp32 block means the gate consumes
// (tasft_gate_mask_build in pooled-input mode), so the gate does not re-read Q and K. K/V
// stay at their own head count (the reference repeats them per q-head, :725-729; the
// kernels here are GQA-native).
//
// Rounding follows the reference's element-wise ops in the model dtype: x * cos and
// rotate_half(x) * sin are each rounded to the dtype, then their sum.
#include "common.cuh"

namespace tasft {
namespace {

constexpr int kQkvThreads = 256;

template <typename T>
__device__ __forceinline__ float rnd(float x) {
  return round_through<T>(x);
}

// grid (ceil(S / block), Hq + 2 Hk, B). Thread (row group g, pair p) handles element pair
// p of the row: columns [p * V, p * V + V) of the first half and the same of the second
// half (V = 16 bytes of T), rows g, g + G, ... of the block.
template <typename T>
__global__ void __launch_bounds__(kQkvThreads) qkv_rope_pool_kernel(tasft_qkv_args a) {
  constexpr int V = 16 / sizeof(T);
  extern __shared__ float psum[];  // [G][D] partial column sums (Q and K heads)
  const int D = a.D, half = D / 2;
  const int P = half / V;  // thread pairs per row
  const int G = kQkvThreads / P;
  const int p = threadIdx.x % P, g = threadIdx.x / P;
  const int blk = blockIdx.x, hh = blockIdx.y, b = blockIdx.z;
  int kind, h, H;  // 0 = q, 1 = k, 2 = v
  if (hh < a.Hq) {
    kind = 0; h = hh; H = a.Hq;
  } else if (hh < a.Hq + a.Hk) {
    kind = 1; h = hh - a.Hq; H = a.Hk;
  } else {
    kind = 2; h = hh - a.Hq - a.Hk; H = a.Hk;
  }
  const T* in = reinterpret_cast<const T*>(kind == 0 ? a.q_in : kind == 1 ? a.k_in : a.v_in);
  const int64_t* ist = kind == 0 ? a.q_in_stride : kind == 1 ? a.k_in_stride : a.v_in_stride;
  T* out = reinterpret_cast<T*>(kind == 0 ? a.q_out : kind == 1 ? a.k_out : a.v_out);
  float* pooled = kind == 0 ? a.pooled_q : kind == 1 ? a.pooled_k : nullptr;
  const bool rope = a.rope && kind < 2;
  const int r0 = blk * a.block;
  const int rows = min(a.block, a.S - r0);
  float acc[2 * V];
#pragma unroll
  for (int e = 0; e < 2 * V; ++e) acc[e] = 0.f;
  if (g < G) {
    // read-only loads (ld.global.nc) so the two rows' loads can be in flight together
#pragma unroll 2
    for (int r = g; r < rows; r += G) {
      const int s = r0 + r;
      const T* src = in + b * ist[0] + (int64_t)s * ist[1] + (int64_t)h * D;
      uint4 u1 = __ldg(reinterpret_cast<const uint4*>(src + p * V));
      uint4 u2 = __ldg(reinterpret_cast<const uint4*>(src + half + p * V));
      T* x1 = reinterpret_cast<T*>(&u1);
      T* x2 = reinterpret_cast<T*>(&u2);
      if (rope) {
        const T* cs = reinterpret_cast<const T*>(a.cos) + b * a.cs_stride[0] + (int64_t)s * a.cs_stride[1];
        const T* sn = reinterpret_cast<const T*>(a.sin) + b * a.cs_stride[0] + (int64_t)s * a.cs_stride[1];
        const uint4 c1u = __ldg(reinterpret_cast<const uint4*>(cs + p * V));
        const uint4 c2u = __ldg(reinterpret_cast<const uint4*>(cs + half + p * V));
        const uint4 s1u = __ldg(reinterpret_cast<const uint4*>(sn + p * V));
        const uint4 s2u = __ldg(reinterpret_cast<const uint4*>(sn + half + p * V));
        const T* c1 = reinterpret_cast<const T*>(&c1u);
        const T* c2 = reinterpret_cast<const T*>(&c2u);
        const T* s1 = reinterpret_cast<const T*>(&s1u);
        const T* s2 = reinterpret_cast<const T*>(&s2u);
#pragma unroll
        for (int e = 0; e < V; ++e) {
          const float a1 = to_f<T>(x1[e]), a2 = to_f<T>(x2[e]);
          // rotate_half(x) = [-x2, x1]
          // explicit _rn ops: no fused multiply-add, so each product is rounded like the
          // reference's separate element-wise multiplications
          const float o1 = rnd<T>(__fadd_rn(rnd<T>(__fmul_rn(a1, to_f<T>(c1[e]))), rnd<T>(__fmul_rn(-a2, to_f<T>(s1[e])))));
          const float o2 = rnd<T>(__fadd_rn(rnd<T>(__fmul_rn(a2, to_f<T>(c2[e]))), rnd<T>(__fmul_rn(a1, to_f<T>(s2[e])))));
          x1[e] = from_f<T>(o1);
          x2[e] = from_f<T>(o2);
        }
      }
      T* dst = out + (((int64_t)b * H + h) * a.S + s) * D;
      *reinterpret_cast<uint4*>(dst + p * V) = u1;
      *reinterpret_cast<uint4*>(dst + half + p * V) = u2;
      if (pooled) {
#pragma unroll
        for (int e = 0; e < V; ++e) {
          acc[e] += to_f<T>(x1[e]);
          acc[V + e] += to_f<T>(x2[e]);
        }
      }
    }
  }
  if (!pooled) return;
  if (g < G) {
#pragma unroll
    for (int e = 0; e < V; ++e) {
      psum[g * D + p * V + e] = acc[e];
      psum[g * D + half + p * V + e] = acc[V + e];
    }
  }
  __syncthreads();
  const int NB = (a.S + a.block - 1) / a.block;
  const float inv = 1.0f / (float)a.block;  // padding rows count as zeros (attn_gate.py:366-375)
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float t = 0.f;
    for (int q = 0; q < G; ++q) t += psum[q * D + d];
    pooled[(((int64_t)b * H + h) * NB + blk) * D + d] = t * inv;
  }
}

}  // namespace
}  // namespace tasft

using namespace tasft;

extern "C" int tasft_qkv_rope_pool(const tasft_qkv_args* ap, tasft_stream_t stream) {
  if (!ap) return TASFT_ERR_INVALID_ARG;
  const tasft_qkv_args& a = *ap;
  if (!a.q_in || !a.k_in || !a.v_in || !a.q_out || !a.k_out || !a.v_out) return TASFT_ERR_INVALID_ARG;
  if (a.B <= 0 || a.Hq <= 0 || a.Hk <= 0 || a.S <= 0 || a.D <= 0 || a.block <= 0) return TASFT_ERR_INVALID_ARG;
  if (a.rope && (!a.cos || !a.sin)) return TASFT_ERR_INVALID_ARG;
  const int es = elem_size(a.dtype);
  const int V = 16 / es;
  if (a.D % (2 * V) || (a.D / 2) / V > kQkvThreads) return TASFT_ERR_UNSUPPORTED;
  // 16-byte vectors: aligned bases and strides
  const void* ptrs[] = {a.q_in, a.k_in, a.v_in, a.q_out, a.k_out, a.v_out};
  for (const void* p : ptrs)
    if (!aligned16(p)) return TASFT_ERR_INVALID_ARG;
  const int64_t* strides[] = {a.q_in_stride, a.k_in_stride, a.v_in_stride};
  for (const int64_t* st : strides)
    if ((st[0] * es) % 16 || (st[1] * es) % 16) return TASFT_ERR_INVALID_ARG;
  if (a.rope && (!aligned16(a.cos) || !aligned16(a.sin) || (a.cs_stride[0] * es) % 16 || (a.cs_stride[1] * es) % 16))
    return TASFT_ERR_INVALID_ARG;
  if (a.Hq + 2 * a.Hk > 65535 || a.B > 65535) return TASFT_ERR_UNSUPPORTED;
  const int P = (a.D / 2) / V, G = kQkvThreads / P;
  const size_t smem = (size_t)G * a.D * sizeof(float);
  dim3 grid((unsigned)ceil_div(a.S, a.block), (unsigned)(a.Hq + 2 * a.Hk), (unsigned)a.B);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  switch (a.dtype) {
    case TASFT_F32: qkv_rope_pool_kernel<float><<<grid, kQkvThreads, smem, st>>>(a); break;
    case TASFT_BF16: qkv_rope_pool_kernel<__nv_bfloat16><<<grid, kQkvThreads, smem, st>>>(a); break;
    case TASFT_F16: qkv_rope_pool_kernel<__half><<<grid, kQkvThreads, smem, st>>>(a); break;
    default: return TASFT_ERR_UNSUPPORTED;
  }
  count_launch();
  return launch_status();
}
