// ca_gelu.cu -- the tanh-approximate GELU of the CA-S decoder's MLP
// (cuda/continuum_attention.py:866-867, F.gelu(fc1(x), approximate='tanh')),
// forward and backward, elementwise over a contiguous tensor.
//
//   u = sqrt(2/pi) (x + 0.044715 x^3),   gelu(x) = 0.5 x (1 + tanh u) = x s,
//   s = sigmoid(2u) = 1 / (1 + 2^(-2u log2 e)),
//   gelu'(x) = 0.5 (1 + tanh u) + 0.5 x (1 - tanh^2 u) du/dx = s + 2 x s (1 - s) du/dx,
//   du/dx = sqrt(2/pi) (1 + 3 * 0.044715 x^2).
// The sigmoid form avoids the cancellation in 1 + tanh u for x << 0 and costs one
// exp2 and one reciprocal on the MUFU pipe; arithmetic is fp32 for every storage
// type (the opmath of the reference's torch kernels).
// HBM-bound: the forward reads x and writes y, the backward reads x and dy and
// writes dx, 16 bytes per thread access, grid-stride over the SMs.
#include <algorithm>

#include "ca_common.cuh"
#include "ca_internal.h"

namespace ca {
namespace gelu {

constexpr float kSqrt2OverPi = 0.7978845608028654f;
constexpr float kCubic = 0.044715f;
constexpr int NT = 256;

// s = sigmoid(2u) and du/dx at x
__device__ __forceinline__ float sigmoid_2u(float x, float& du) {
  const float x2 = x * x;
  const float u = kSqrt2OverPi * fmaf(kCubic * x2, x, x);
  du = kSqrt2OverPi * fmaf(3.f * kCubic, x2, 1.f);
  return rcp_approx(1.f + ex2_approx(-2.f * kLog2e * u));
}

template <typename T> struct Vec { static constexpr int N = 16 / (int)sizeof(T); };

template <typename T> __device__ __forceinline__ void unpack(const uint4& u, float (&x)[Vec<T>::N]);
template <> __device__ __forceinline__ void unpack<float>(const uint4& u, float (&x)[4]) {
  x[0] = __uint_as_float(u.x); x[1] = __uint_as_float(u.y); x[2] = __uint_as_float(u.z); x[3] = __uint_as_float(u.w);
}
template <> __device__ __forceinline__ void unpack<__nv_bfloat16>(const uint4& u, float (&x)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    x[2 * i] = __uint_as_float(w[i] << 16);
    x[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}
template <> __device__ __forceinline__ void unpack<__half>(const uint4& u, float (&x)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
    x[2 * i] = f.x;
    x[2 * i + 1] = f.y;
  }
}

template <typename T> __device__ __forceinline__ uint4 pack(const float (&x)[Vec<T>::N]);
template <> __device__ __forceinline__ uint4 pack<float>(const float (&x)[4]) {
  return make_uint4(__float_as_uint(x[0]), __float_as_uint(x[1]), __float_as_uint(x[2]), __float_as_uint(x[3]));
}
template <> __device__ __forceinline__ uint4 pack<__nv_bfloat16>(const float (&x)[8]) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __nv_bfloat162 b = __floats2bfloat162_rn(x[2 * i], x[2 * i + 1]);
    w[i] = *reinterpret_cast<const uint32_t*>(&b);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}
template <> __device__ __forceinline__ uint4 pack<__half>(const float (&x)[8]) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __half2 b = __floats2half2_rn(x[2 * i], x[2 * i + 1]);
    w[i] = *reinterpret_cast<const uint32_t*>(&b);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

// nvec 16-byte vectors of T
template <typename T>
__global__ void __launch_bounds__(NT) fwd_kernel(const uint4* __restrict__ x, uint4* __restrict__ y, size_t nvec) {
  pdl_wait();
  pdl_launch_dependents();
  constexpr int N = Vec<T>::N;
  const size_t stride = (size_t)gridDim.x * NT;
  for (size_t i = (size_t)blockIdx.x * NT + threadIdx.x; i < nvec; i += stride) {
    float v[N];
    unpack<T>(__ldg(x + i), v);
#pragma unroll
    for (int j = 0; j < N; ++j) {
      float du;
      v[j] *= sigmoid_2u(v[j], du);
    }
    y[i] = pack<T>(v);
  }
}

template <typename T>
__global__ void __launch_bounds__(NT) bwd_kernel(const uint4* __restrict__ x, const uint4* __restrict__ dy,
                                                 uint4* __restrict__ dx, size_t nvec) {
  pdl_wait();
  pdl_launch_dependents();
  constexpr int N = Vec<T>::N;
  const size_t stride = (size_t)gridDim.x * NT;
  for (size_t i = (size_t)blockIdx.x * NT + threadIdx.x; i < nvec; i += stride) {
    float v[N], g[N];
    unpack<T>(__ldg(x + i), v);
    unpack<T>(__ldg(dy + i), g);
#pragma unroll
    for (int j = 0; j < N; ++j) {
      float du;
      const float s = sigmoid_2u(v[j], du);
      const float d = fmaf(2.f * v[j] * s * (1.f - s), du, s);
      g[j] *= d;
    }
    dx[i] = pack<T>(g);
  }
}

static unsigned grid_for(size_t nvec) {
  const size_t want = (nvec + NT - 1) / NT;
  return (unsigned)std::max<size_t>(1, std::min<size_t>(want, (size_t)num_sms_cached() * 8));
}

int vector_elems(int dtype) { return dtype == 0 ? 4 : 8; }

cudaError_t forward(const void* x, void* y, size_t n, int dtype, cudaStream_t stream) {
  const size_t nvec = n / vector_elems(dtype);
  const dim3 g(grid_for(nvec)), b(NT);
  const uint4* xv = static_cast<const uint4*>(x);
  uint4* yv = static_cast<uint4*>(y);
  switch (dtype) {
    case 0: return launch_pdl(fwd_kernel<float>, g, b, 0, stream, xv, yv, nvec);
    case 1: return launch_pdl(fwd_kernel<__nv_bfloat16>, g, b, 0, stream, xv, yv, nvec);
    default: return launch_pdl(fwd_kernel<__half>, g, b, 0, stream, xv, yv, nvec);
  }
}

cudaError_t backward(const void* x, const void* dy, void* dx, size_t n, int dtype, cudaStream_t stream) {
  const size_t nvec = n / vector_elems(dtype);
  const dim3 g(grid_for(nvec)), b(NT);
  const uint4* xv = static_cast<const uint4*>(x);
  const uint4* dyv = static_cast<const uint4*>(dy);
  uint4* dxv = static_cast<uint4*>(dx);
  switch (dtype) {
    case 0: return launch_pdl(bwd_kernel<float>, g, b, 0, stream, xv, dyv, dxv, nvec);
    case 1: return launch_pdl(bwd_kernel<__nv_bfloat16>, g, b, 0, stream, xv, dyv, dxv, nvec);
    default: return launch_pdl(bwd_kernel<__half>, g, b, 0, stream, xv, dyv, dxv, nvec);
  }
}

}  // namespace gelu
}  // namespace ca
