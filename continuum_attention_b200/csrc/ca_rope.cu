// ca_rope.cu -- input/output layout of the CA-S decoder's attention block:
// rotary position embedding fused with the unpacking of the QKV projection.
//
// The reference block (cuda/continuum_attention.py:848-854) reshapes the
// projection output [B,T,3*H*D] to [B,T,3,H,D], permutes it to three [B,H,T,D]
// views, applies apply_rope (:825-835) to q and k through about a dozen
// elementwise kernels over strided temporaries, and makes every operand
// contiguous for the attention op.  Here one pass reads the projection output
// once and writes contiguous q, k (rotated) and v; the backward pass reads dq,
// dk, dv once, applies the inverse rotation and writes the projection-output
// gradient [B,T,3,H,D].
//
// Rotation of the interleaved pair (x_{2p}, x_{2p+1}) at position t, as in the
// reference: with (c, s) = (cos, sin)(t * theta^(-2p/D)),
//   y_{2p} = x_{2p} c - x_{2p+1} s,   y_{2p+1} = x_{2p+1} c + x_{2p} s,
// and its transpose for the gradient.  The caller passes the (c, s) table as
// float32 [T][D/2][2]; arithmetic is fp32 with one rounding per output.
//
// Work unit: one thread per 8-element chunk of a token's [3][H][D] projection row;
// a block takes one token forward, G consecutive tokens backward.  HBM-bound:
// 2 x 3*B*T*H*D elements per pass.
#include "ca_common.cuh"
#include "ca_internal.h"

namespace ca {
namespace rope {

template <typename T>
__device__ __forceinline__ void load8(const T* p, float (&x)[8]);
template <typename T>
__device__ __forceinline__ void store8(T* p, const float (&x)[8]);

template <>
__device__ __forceinline__ void load8<float>(const float* p, float (&x)[8]) {
  const float4 a = reinterpret_cast<const float4*>(p)[0], b = reinterpret_cast<const float4*>(p)[1];
  x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
  x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
}
template <>
__device__ __forceinline__ void store8<float>(float* p, const float (&x)[8]) {
  reinterpret_cast<float4*>(p)[0] = make_float4(x[0], x[1], x[2], x[3]);
  reinterpret_cast<float4*>(p)[1] = make_float4(x[4], x[5], x[6], x[7]);
}

template <typename T>
__device__ __forceinline__ void load8_16(const T* p, float (&x)[8]) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
  for (int i = 0; i < 8; ++i) x[i] = to_f32<T>(e[i]);
}
template <typename T>
__device__ __forceinline__ void store8_16(T* p, const float (&x)[8]) {
  uint4 u;
  T* e = reinterpret_cast<T*>(&u);
#pragma unroll
  for (int i = 0; i < 8; ++i) e[i] = from_f32<T>(x[i]);
  *reinterpret_cast<uint4*>(p) = u;
}
template <>
__device__ __forceinline__ void load8<__nv_bfloat16>(const __nv_bfloat16* p, float (&x)[8]) { load8_16(p, x); }
template <>
__device__ __forceinline__ void store8<__nv_bfloat16>(__nv_bfloat16* p, const float (&x)[8]) { store8_16(p, x); }
template <>
__device__ __forceinline__ void load8<__half>(const __half* p, float (&x)[8]) { load8_16(p, x); }
template <>
__device__ __forceinline__ void store8<__half>(__half* p, const float (&x)[8]) { store8_16(p, x); }

// Forward: one block per token (b, t); thread j of the token's 3*H*D/8 chunks takes
// chunk c = j % (D/8) of head h = (j / (D/8)) % H of q, k or v (j / (H*D/8)), so a
// warp reads one contiguous run of the projection row.  Backward: a block of G =
// 32 / (D/8) consecutive tokens; element j of its [3][H][G][D/8] chunk grid is
// chunk c of head h for token tt, so a warp reads G consecutive [B,H,T,D] rows of
// one head.  Reading contiguously measured faster than writing contiguously, each
// way.  32-bit index arithmetic once per chunk.

// tokens per backward block for head dim D
__host__ __device__ __forceinline__ unsigned tokens_per_block(unsigned D) {
  const unsigned chunks = D / 8;
  if (chunks == 0 || 32 % chunks) return 1;
  const unsigned g = 32 / chunks;
  return g > 8 ? 8 : g;
}

// qkv [B][T][3][H][D] -> q, k (rotated), v [B][H][T][D]
template <typename T>
__global__ void pack_fwd_kernel(const T* __restrict__ qkv, const float2* __restrict__ cs, T* __restrict__ q,
                                T* __restrict__ k, T* __restrict__ v, int Tn, int H, int D) {
  pdl_wait();
  pdl_launch_dependents();
  const unsigned chunks = (unsigned)D / 8, per_head = chunks, per_which = (unsigned)H * chunks;
  const unsigned token = blockIdx.x, t = token % (unsigned)Tn, b = token / (unsigned)Tn;
  const T* src = qkv + (size_t)token * 3 * per_which * 8;
  for (unsigned j = threadIdx.x; j < 3 * per_which; j += blockDim.x) {
    const unsigned which = j / per_which, rem = j - which * per_which;
    const unsigned h = rem / per_head, c = rem - h * per_head;
    float x[8];
    load8<T>(src + (size_t)j * 8, x);
    if (which < 2) {
      const float2* row = cs + (size_t)t * (D / 2) + 4 * c;
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        const float2 w = row[p];
        const float e = x[2 * p], o = x[2 * p + 1];
        x[2 * p] = fmaf(e, w.x, -o * w.y);
        x[2 * p + 1] = fmaf(o, w.x, e * w.y);
      }
    }
    T* dst = which == 0 ? q : (which == 1 ? k : v);
    store8<T>(dst + (((size_t)b * H + h) * Tn + t) * D + 8 * c, x);
  }
}

// dq, dk, dv [B][H][T][D] -> dqkv [B][T][3][H][D] (transposed rotation on dq, dk)
template <typename T>
__global__ void pack_bwd_kernel(const T* __restrict__ dq, const T* __restrict__ dk, const T* __restrict__ dv,
                                const float2* __restrict__ cs, T* __restrict__ dqkv, int ntok, int Tn, int H, int D,
                                int G) {
  pdl_wait();
  pdl_launch_dependents();
  const unsigned chunks = (unsigned)D / 8;
  const unsigned per_head = G * chunks, per_which = (unsigned)H * per_head;
  for (unsigned j = threadIdx.x; j < 3 * per_which; j += blockDim.x) {
    const unsigned which = j / per_which, rem = j - which * per_which;
    const unsigned h = rem / per_head, r2 = rem - h * per_head;
    const unsigned tt = r2 / chunks, c = r2 - tt * chunks;
    const unsigned token = blockIdx.x * (unsigned)G + tt;
    if (token >= (unsigned)ntok) continue;
    const unsigned t = token % (unsigned)Tn, b = token / (unsigned)Tn;
    const T* src = which == 0 ? dq : (which == 1 ? dk : dv);
    float x[8];
    load8<T>(src + (((size_t)b * H + h) * Tn + t) * D + 8 * c, x);
    if (which < 2) {
      const float2* row = cs + (size_t)t * (D / 2) + 4 * c;
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        const float2 w = row[p];
        const float e = x[2 * p], o = x[2 * p + 1];
        x[2 * p] = fmaf(e, w.x, o * w.y);
        x[2 * p + 1] = fmaf(o, w.x, -e * w.y);
      }
    }
    store8<T>(dqkv + ((size_t)token * 3 * H + which * H + h) * D + 8 * c, x);
  }
}

// threads per block of G tokens: the block's chunk count rounded up to whole warps, at most 512
static unsigned block_for(long long H, long long D, long long G) {
  const long long n = 3 * H * (D / 8) * G;
  const long long w = (n + 31) / 32 * 32;
  return (unsigned)(w < 512 ? w : 512);
}

template <typename T>
static cudaError_t fwd_t(const void* qkv, const float* cs, void* q, void* k, void* v, long long B, long long Tn,
                         long long H, long long D, cudaStream_t s) {
  return launch_pdl(pack_fwd_kernel<T>, dim3((unsigned)(B * Tn)), dim3(block_for(H, D, 1)), 0, s, (const T*)qkv,
                    (const float2*)cs, (T*)q, (T*)k, (T*)v, (int)Tn, (int)H, (int)D);
}

template <typename T>
static cudaError_t bwd_t(const void* dq, const void* dk, const void* dv, const float* cs, void* dqkv, long long B,
                         long long Tn, long long H, long long D, cudaStream_t s) {
  const long long G = tokens_per_block((unsigned)D);
  return launch_pdl(pack_bwd_kernel<T>, dim3((unsigned)((B * Tn + G - 1) / G)), dim3(block_for(H, D, G)), 0, s,
                    (const T*)dq, (const T*)dk, (const T*)dv, (const float2*)cs, (T*)dqkv, (int)(B * Tn), (int)Tn,
                    (int)H, (int)D, (int)G);
}

cudaError_t forward(const void* qkv, const float* cos_sin, void* q, void* k, void* v, long long B, long long T,
                    long long H, long long D, int dtype, cudaStream_t s) {
  switch (dtype) {
    case 0: return fwd_t<float>(qkv, cos_sin, q, k, v, B, T, H, D, s);
    case 1: return fwd_t<__nv_bfloat16>(qkv, cos_sin, q, k, v, B, T, H, D, s);
    default: return fwd_t<__half>(qkv, cos_sin, q, k, v, B, T, H, D, s);
  }
}

cudaError_t backward(const void* dq, const void* dk, const void* dv, const float* cos_sin, void* dqkv,
                     long long B, long long T, long long H, long long D, int dtype, cudaStream_t s) {
  switch (dtype) {
    case 0: return bwd_t<float>(dq, dk, dv, cos_sin, dqkv, B, T, H, D, s);
    case 1: return bwd_t<__nv_bfloat16>(dq, dk, dv, cos_sin, dqkv, B, T, H, D, s);
    default: return bwd_t<__half>(dq, dk, dv, cos_sin, dqkv, B, T, H, D, s);
  }
}

}  // namespace rope
}  // namespace ca
