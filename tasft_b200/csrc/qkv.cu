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

// grid (ceil(S / block), ceil((Hq + 2 Hk) / kHeadsPerCta), B). Thread (row group g, pair p)
// handles element pair p of a row: columns [p * V, p * V + V) of the first half and the
// same of the second half (V = 16 bytes of T), rows g, g + G, ... of the block, for each
// of the CTA's heads in turn; its rows' cos / sin are loaded once and reused across heads.
constexpr int kHeadsPerCta = 8;
// R = rows per thread: block <= G * R (chosen on the host: 2 for the usual 64-token block)
template <typename T, int kMaxRowsPerThread>
__global__ void __launch_bounds__(kQkvThreads) qkv_rope_pool_kernel(tasft_qkv_args a) {
  constexpr int V = 16 / sizeof(T);
  extern __shared__ float psum[];  // [G][D] partial column sums of one head
  const int D = a.D, half = D / 2;
  const int P = half / V;  // thread pairs per row
  const int G = kQkvThreads / P;
  const int p = threadIdx.x % P, g = threadIdx.x / P;
  const int blk = blockIdx.x, b = blockIdx.z;
  const int r0 = blk * a.block;
  const int rows = min(a.block, a.S - r0);
  const int nh = a.Hq + 2 * a.Hk;
  const int NB = (a.S + a.block - 1) / a.block;
  // this thread's rows' rotary tables, shared by every head of the CTA
  uint4 c1u[kMaxRowsPerThread], c2u[kMaxRowsPerThread], s1u[kMaxRowsPerThread], s2u[kMaxRowsPerThread];
  if (a.rope) {
#pragma unroll
    for (int i = 0; i < kMaxRowsPerThread; ++i) {
      const int r = g + i * G;
      if (g < G && r < rows) {
        const int s = r0 + r;
        const T* cs = reinterpret_cast<const T*>(a.cos) + b * a.cs_stride[0] + (int64_t)s * a.cs_stride[1];
        const T* sn = reinterpret_cast<const T*>(a.sin) + b * a.cs_stride[0] + (int64_t)s * a.cs_stride[1];
        c1u[i] = *reinterpret_cast<const uint4*>(cs + p * V);
        c2u[i] = *reinterpret_cast<const uint4*>(cs + half + p * V);
        s1u[i] = *reinterpret_cast<const uint4*>(sn + p * V);
        s2u[i] = *reinterpret_cast<const uint4*>(sn + half + p * V);
      }
    }
  }
  const int h_end = min(nh, (int)(blockIdx.y + 1) * kHeadsPerCta);
  for (int hh = blockIdx.y * kHeadsPerCta; hh < h_end; ++hh) {
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
    float acc[2 * V];
#pragma unroll
    for (int e = 0; e < 2 * V; ++e) acc[e] = 0.f;
    // loads of all this thread's rows first (in flight together), then the math and stores
    uint4 u1[kMaxRowsPerThread], u2[kMaxRowsPerThread];
#pragma unroll
    for (int i = 0; i < kMaxRowsPerThread; ++i) {
      const int r = g + i * G;
      if (g < G && r < rows) {
        const T* src = in + b * ist[0] + (int64_t)(r0 + r) * ist[1] + (int64_t)h * D;
        u1[i] = *reinterpret_cast<const uint4*>(src + p * V);
        u2[i] = *reinterpret_cast<const uint4*>(src + half + p * V);
      }
    }
#pragma unroll
    for (int i = 0; i < kMaxRowsPerThread; ++i) {
      const int r = g + i * G;
      if (!(g < G && r < rows)) continue;
      T* x1 = reinterpret_cast<T*>(&u1[i]);
      T* x2 = reinterpret_cast<T*>(&u2[i]);
      if (rope) {
        const T* c1 = reinterpret_cast<const T*>(&c1u[i]);
        const T* c2 = reinterpret_cast<const T*>(&c2u[i]);
        const T* s1 = reinterpret_cast<const T*>(&s1u[i]);
        const T* s2 = reinterpret_cast<const T*>(&s2u[i]);
#pragma unroll
        for (int e = 0; e < V; ++e) {
          const float a1 = to_f<T>(x1[e]), a2 = to_f<T>(x2[e]);
          // rotate_half(x) = [-x2, x1]; explicit _rn ops: no fused multiply-add, so each
          // product is rounded like the reference's separate element-wise multiplications
          const float o1 = rnd<T>(__fadd_rn(rnd<T>(__fmul_rn(a1, to_f<T>(c1[e]))), rnd<T>(__fmul_rn(-a2, to_f<T>(s1[e])))));
          const float o2 = rnd<T>(__fadd_rn(rnd<T>(__fmul_rn(a2, to_f<T>(c2[e]))), rnd<T>(__fmul_rn(a1, to_f<T>(s2[e])))));
          x1[e] = from_f<T>(o1);
          x2[e] = from_f<T>(o2);
        }
      }
      T* dst = out + (((int64_t)b * H + h) * a.S + r0 + r) * D;
      *reinterpret_cast<uint4*>(dst + p * V) = u1[i];
      *reinterpret_cast<uint4*>(dst + half + p * V) = u2[i];
      if (pooled) {
#pragma unroll
        for (int e = 0; e < V; ++e) {
          acc[e] += to_f<T>(x1[e]);
          acc[V + e] += to_f<T>(x2[e]);
        }
      }
    }
    if (!pooled) continue;  // uniform over the CTA
    if (g < G) {
#pragma unroll
      for (int e = 0; e < V; ++e) {
        psum[g * D + p * V + e] = acc[e];
        psum[g * D + half + p * V + e] = acc[V + e];
      }
    }
    __syncthreads();
    const float inv = 1.0f / (float)a.block;  // padding rows count as zeros (attn_gate.py:366-375)
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
      float t = 0.f;
      for (int q = 0; q < G; ++q) t += psum[q * D + d];
      pooled[(((int64_t)b * H + h) * NB + blk) * D + d] = t * inv;
    }
    __syncthreads();
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
  if (a.B > 65535) return TASFT_ERR_UNSUPPORTED;
  const int P = (a.D / 2) / V, G = kQkvThreads / P;
  if (a.block > G * 8) return TASFT_ERR_UNSUPPORTED;
  const bool r2 = a.block <= G * 2;
  const size_t smem = (size_t)G * a.D * sizeof(float);
  dim3 grid((unsigned)ceil_div(a.S, a.block), (unsigned)ceil_div(a.Hq + 2 * a.Hk, kHeadsPerCta), (unsigned)a.B);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  switch (a.dtype) {
    case TASFT_F32:
      if (r2) qkv_rope_pool_kernel<float, 2><<<grid, kQkvThreads, smem, st>>>(a);
      else qkv_rope_pool_kernel<float, 8><<<grid, kQkvThreads, smem, st>>>(a);
      break;
    case TASFT_BF16:
      if (r2) qkv_rope_pool_kernel<__nv_bfloat16, 2><<<grid, kQkvThreads, smem, st>>>(a);
      else qkv_rope_pool_kernel<__nv_bfloat16, 8><<<grid, kQkvThreads, smem, st>>>(a);
      break;
    case TASFT_F16:
      if (r2) qkv_rope_pool_kernel<__half, 2><<<grid, kQkvThreads, smem, st>>>(a);
      else qkv_rope_pool_kernel<__half, 8><<<grid, kQkvThreads, smem, st>>>(a);
      break;
    default: return TASFT_ERR_UNSUPPORTED;
  }
  count_launch();
  return launch_status();
}
