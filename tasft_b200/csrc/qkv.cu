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
// rotate_half(x) * sin are each rounded to the dtype, then their sum (rotate_pair).
#include "common.cuh"

namespace tasft {
namespace {

constexpr int kQkvThreads = 128;

// Rotary embedding of one 16-byte column pair of a row: x1 = columns [c, c + V) of the first
// half, x2 the same columns of the second half. rotate_half(x) = [-x2, x1], so
//   y1 = x1 * cos1 - x2 * sin1,  y2 = x2 * cos2 + x1 * sin2,
// each product rounded to T, then the sum, like the reference's separate element-wise ops in
// the model dtype. For bf16 / f16 the ops run as packed two-lane instructions with
// round-to-nearest (mul.rn / add.rn / sub.rn .bf16x2 / .f16x2: the correctly rounded
// result, which is what rounding the fp32 result gives, since fp32 carries more than twice
// the significand bits plus two of either type, so the double rounding is innocuous); fp32
// uses explicit _rn ops so nothing fuses into a multiply-add.
template <typename T>
struct Packed;
template <>
struct Packed<__nv_bfloat16> {
  __device__ __forceinline__ static uint32_t mul(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
  }
  __device__ __forceinline__ static uint32_t add(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
  }
  __device__ __forceinline__ static uint32_t sub(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
  }
  // the two lanes as fp32 (bf16 is the top half of an fp32)
  __device__ __forceinline__ static float lo(uint32_t v) { return __uint_as_float(v << 16); }
  __device__ __forceinline__ static float hi(uint32_t v) { return __uint_as_float(v & 0xffff0000u); }
};
template <>
struct Packed<__half> {
  __device__ __forceinline__ static uint32_t mul(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
  }
  __device__ __forceinline__ static uint32_t add(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("add.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
  }
  __device__ __forceinline__ static uint32_t sub(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
  }
  __device__ __forceinline__ static float lo(uint32_t v) { return __half2float(__ushort_as_half((unsigned short)(v & 0xffffu))); }
  __device__ __forceinline__ static float hi(uint32_t v) { return __half2float(__ushort_as_half((unsigned short)(v >> 16))); }
};

template <typename T>
__device__ __forceinline__ void rotate_pair(uint4& u1, uint4& u2, const uint4& c1u, const uint4& c2u, const uint4& s1u,
                                            const uint4& s2u) {
  if constexpr (sizeof(T) == 2) {
    using Pk = Packed<T>;
    const uint32_t* x1 = &u1.x;
    const uint32_t* x2 = &u2.x;
    const uint32_t* c1 = &c1u.x;
    const uint32_t* c2 = &c2u.x;
    const uint32_t* s1 = &s1u.x;
    const uint32_t* s2 = &s2u.x;
    uint4 n1, n2;
    uint32_t* y1 = &n1.x;
    uint32_t* y2 = &n2.x;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      y1[w] = Pk::sub(Pk::mul(x1[w], c1[w]), Pk::mul(x2[w], s1[w]));
      y2[w] = Pk::add(Pk::mul(x2[w], c2[w]), Pk::mul(x1[w], s2[w]));
    }
    u1 = n1;
    u2 = n2;
  } else {
    constexpr int V = 16 / sizeof(T);
    const float* x1 = reinterpret_cast<const float*>(&u1);
    const float* x2 = reinterpret_cast<const float*>(&u2);
    const float* c1 = reinterpret_cast<const float*>(&c1u);
    const float* c2 = reinterpret_cast<const float*>(&c2u);
    const float* s1 = reinterpret_cast<const float*>(&s1u);
    const float* s2 = reinterpret_cast<const float*>(&s2u);
    uint4 n1, n2;
    float* y1 = reinterpret_cast<float*>(&n1);
    float* y2 = reinterpret_cast<float*>(&n2);
#pragma unroll
    for (int e = 0; e < V; ++e) {
      y1[e] = __fsub_rn(__fmul_rn(x1[e], c1[e]), __fmul_rn(x2[e], s1[e]));
      y2[e] = __fadd_rn(__fmul_rn(x2[e], c2[e]), __fmul_rn(x1[e], s2[e]));
    }
    u1 = n1;
    u2 = n2;
  }
}

// acc[0, V) += the first-half vector, acc[V, 2V) += the second-half vector, in fp32.
template <typename T>
__device__ __forceinline__ void accumulate(float* acc, const uint4& u1, const uint4& u2) {
  if constexpr (sizeof(T) == 2) {
    using Pk = Packed<T>;
    const uint32_t* x1 = &u1.x;
    const uint32_t* x2 = &u2.x;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      acc[2 * w] += Pk::lo(x1[w]);
      acc[2 * w + 1] += Pk::hi(x1[w]);
      acc[8 + 2 * w] += Pk::lo(x2[w]);
      acc[8 + 2 * w + 1] += Pk::hi(x2[w]);
    }
  } else {
    const float* x1 = reinterpret_cast<const float*>(&u1);
    const float* x2 = reinterpret_cast<const float*>(&u2);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      acc[e] += x1[e];
      acc[4 + e] += x2[e];
    }
  }
}

// grid (ceil(S / block), Hq + 2 Hk, B). Thread (row group g, pair p) handles element pair
// p of the row: columns [p * V, p * V + V) of the first half and the same of the second
// half (V = 16 bytes of T), rows g, g + G, ... of the block.
template <typename T>
__global__ void __launch_bounds__(kQkvThreads, 8) qkv_rope_pool_kernel(tasft_qkv_args a) {
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
    for (int r = g; r < rows; r += G) {
      const int s = r0 + r;
      const T* src = in + b * ist[0] + (int64_t)s * ist[1] + (int64_t)h * D;
      uint4 u1 = __ldg(reinterpret_cast<const uint4*>(src + p * V));
      uint4 u2 = __ldg(reinterpret_cast<const uint4*>(src + half + p * V));
      if (rope) {
        const int64_t cso = b * a.cs_stride[0] + (int64_t)s * a.cs_stride[1];
        const T* cs = reinterpret_cast<const T*>(a.cos) + cso;
        const T* sn = reinterpret_cast<const T*>(a.sin) + cso;
        rotate_pair<T>(u1, u2, __ldg(reinterpret_cast<const uint4*>(cs + p * V)),
                       __ldg(reinterpret_cast<const uint4*>(cs + half + p * V)),
                       __ldg(reinterpret_cast<const uint4*>(sn + p * V)),
                       __ldg(reinterpret_cast<const uint4*>(sn + half + p * V)));
      }
      T* dst = out + (((int64_t)b * H + h) * a.S + s) * D;
      *reinterpret_cast<uint4*>(dst + p * V) = u1;
      *reinterpret_cast<uint4*>(dst + half + p * V) = u2;
      if (pooled) accumulate<T>(acc, u1, u2);
    }
  }
  if (!pooled) return;
  const int NB = (a.S + a.block - 1) / a.block;
  const float inv = 1.0f / (float)a.block;  // padding rows count as zeros (attn_gate.py:366-375)
  float* dst = pooled + (((int64_t)b * H + h) * NB + blk) * D;
  if ((P & (P - 1)) == 0 && P <= 32) {
    // lane = (row group within the warp) * P + p: fold the warp's row groups with shuffles,
    // then one partial row per warp through shared memory
#pragma unroll
    for (int e = 0; e < 2 * V; ++e)
      for (int off = P; off < 32; off <<= 1) acc[e] += __shfl_xor_sync(0xffffffffu, acc[e], off);
    const int wid = threadIdx.x >> 5, ln = threadIdx.x & 31;
    if (ln < P) {
#pragma unroll
      for (int e = 0; e < V; ++e) {
        psum[wid * D + p * V + e] = acc[e];
        psum[wid * D + half + p * V + e] = acc[V + e];
      }
    }
    __syncthreads();
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
      float t = 0.f;
#pragma unroll
      for (int w = 0; w < kQkvThreads / 32; ++w) t += psum[w * D + d];
      dst[d] = t * inv;
    }
    return;
  }
  if (g < G) {
#pragma unroll
    for (int e = 0; e < V; ++e) {
      psum[g * D + p * V + e] = acc[e];
      psum[g * D + half + p * V + e] = acc[V + e];
    }
  }
  __syncthreads();
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float t = 0.f;
    for (int q = 0; q < G; ++q) t += psum[q * D + d];
    dst[d] = t * inv;
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
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int P = (a.D / 2) / V;
  const int G = kQkvThreads / P;
  const size_t smem = (size_t)G * a.D * sizeof(float);
  dim3 grid((unsigned)ceil_div(a.S, a.block), (unsigned)(a.Hq + 2 * a.Hk), (unsigned)a.B);
  switch (a.dtype) {
    case TASFT_F32: qkv_rope_pool_kernel<float><<<grid, kQkvThreads, smem, st>>>(a); break;
    case TASFT_BF16: qkv_rope_pool_kernel<__nv_bfloat16><<<grid, kQkvThreads, smem, st>>>(a); break;
    case TASFT_F16: qkv_rope_pool_kernel<__half><<<grid, kQkvThreads, smem, st>>>(a); break;
    default: return TASFT_ERR_UNSUPPORTED;
  }
  count_launch();
  return launch_status();
}
