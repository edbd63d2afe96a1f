// ca_norm.cu -- the CA-S decoder block's RMSNorm (cuda/continuum_attention.py:815-821),
// y = w * x * rsqrt(mean(x^2) + eps) over the last axis, forward and backward.
//
// Forward: one warp per row; the row is read twice (sum of squares, then the
// scaled output; the second read hits L1), the output is written in the dtype
// the next matrix product consumes (bf16 under autocast), and rsqrt(mean + eps)
// is kept per row for the backward.
// Backward: with xh = x * r (r the saved rsqrt) and g = dy * w,
//   dx = r * (g - xh * mean(g * xh)),   dw = sum over rows of dy * xh.
// One warp per row again; each block accumulates its rows' dy * xh for the
// columns its lanes own in registers and writes one partial row, and a second
// kernel adds the partials in block order (deterministic).
// HBM-bound: forward reads x and writes y, backward reads x, dy and writes dx.
#include <algorithm>

#include "ca_common.cuh"
#include "ca_internal.h"

namespace ca {
namespace norm {

constexpr int WARPS = 8;          // rows in flight per block
constexpr int BWD_BLOCKS_PER_SM = 4;

template <typename T>
__device__ __forceinline__ void load4(const T* p, float (&x)[4]);
template <>
__device__ __forceinline__ void load4<float>(const float* p, float (&x)[4]) {
  const float4 a = *reinterpret_cast<const float4*>(p);
  x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
}
template <>
__device__ __forceinline__ void load4<__nv_bfloat16>(const __nv_bfloat16* p, float (&x)[4]) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  x[0] = __uint_as_float(u.x << 16); x[1] = __uint_as_float(u.x & 0xffff0000u);
  x[2] = __uint_as_float(u.y << 16); x[3] = __uint_as_float(u.y & 0xffff0000u);
}
template <typename T>
__device__ __forceinline__ void store4(T* p, const float (&x)[4]);
template <>
__device__ __forceinline__ void store4<float>(float* p, const float (&x)[4]) {
  *reinterpret_cast<float4*>(p) = make_float4(x[0], x[1], x[2], x[3]);
}
template <>
__device__ __forceinline__ void store4<__nv_bfloat16>(__nv_bfloat16* p, const float (&x)[4]) {
  const __nv_bfloat162 a = __floats2bfloat162_rn(x[0], x[1]), b = __floats2bfloat162_rn(x[2], x[3]);
  uint2 u;
  u.x = *reinterpret_cast<const uint32_t*>(&a);
  u.y = *reinterpret_cast<const uint32_t*>(&b);
  *reinterpret_cast<uint2*>(p) = u;
}

__device__ __forceinline__ float warp_sum(float s) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
  return s;
}

// lane l owns columns 128 c + 4 l .. +3 for c = 0 .. NC-1 (D = 128 NC)
template <typename TX, typename TY, int NC>
__global__ void __launch_bounds__(WARPS * 32) fwd_kernel(const TX* __restrict__ x, const float* __restrict__ w,
                                                         TY* __restrict__ y, float* __restrict__ rstd,
                                                         long long rows, float eps) {
  pdl_wait();
  pdl_launch_dependents();
  constexpr int D = 128 * NC;
  const int lane = threadIdx.x & 31;
  const long long row = (long long)blockIdx.x * WARPS + (threadIdx.x >> 5);
  if (row >= rows) return;
  const TX* xr = x + row * D;
  float v[NC][4];
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    load4<TX>(xr + 128 * c + 4 * lane, v[c]);
#pragma unroll
    for (int u = 0; u < 4; ++u) ss = fmaf(v[c][u], v[c][u], ss);
  }
  ss = warp_sum(ss);
  const float r = rsqrtf(ss * (1.f / D) + eps);
  TY* yr = y + row * D;
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    float wv[4], o[4];
    load4<float>(w + 128 * c + 4 * lane, wv);
#pragma unroll
    for (int u = 0; u < 4; ++u) o[u] = wv[u] * (v[c][u] * r);
    store4<TY>(yr + 128 * c + 4 * lane, o);
  }
  if (lane == 0) rstd[row] = r;
}

template <typename TX, typename TY, int NC>
__global__ void __launch_bounds__(WARPS * 32) bwd_kernel(const TX* __restrict__ x, const float* __restrict__ w,
                                                         const TY* __restrict__ dy, const float* __restrict__ rstd,
                                                         TX* __restrict__ dx, float* __restrict__ dw_part,
                                                         long long rows) {
  pdl_wait();
  pdl_launch_dependents();
  constexpr int D = 128 * NC;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float acc[NC][4];
#pragma unroll
  for (int c = 0; c < NC; ++c)
#pragma unroll
    for (int u = 0; u < 4; ++u) acc[c][u] = 0.f;
  for (long long row = (long long)blockIdx.x * WARPS + warp; row < rows; row += (long long)gridDim.x * WARPS) {
    const float r = rstd[row];
    const TX* xr = x + row * D;
    const TY* dr = dy + row * D;
    // pass 1: mean(g * xh); pass 2 re-reads the row (L1) for dx and the dw partial
    float dot = 0.f;
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      float xv[4], dv[4], wv[4];
      load4<TX>(xr + 128 * c + 4 * lane, xv);
      load4<TY>(dr + 128 * c + 4 * lane, dv);
      load4<float>(w + 128 * c + 4 * lane, wv);
#pragma unroll
      for (int u = 0; u < 4; ++u) dot = fmaf(dv[u] * wv[u], xv[u] * r, dot);
    }
    const float mean = warp_sum(dot) * (1.f / D);
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      float xv[4], dv[4], wv[4], o[4];
      load4<TX>(xr + 128 * c + 4 * lane, xv);
      load4<TY>(dr + 128 * c + 4 * lane, dv);
      load4<float>(w + 128 * c + 4 * lane, wv);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float xh = xv[u] * r;
        o[u] = r * fmaf(-xh, mean, dv[u] * wv[u]);
        acc[c][u] = fmaf(dv[u], xh, acc[c][u]);
      }
      store4<TX>(dx + row * D + 128 * c + 4 * lane, o);
    }
  }
  // the block's partial of dw: warps add their columns in warp order
  __shared__ float part[WARPS][128 * NC];
#pragma unroll
  for (int c = 0; c < NC; ++c)
#pragma unroll
    for (int u = 0; u < 4; ++u) part[warp][128 * c + 4 * lane + u] = acc[c][u];
  __syncthreads();
  for (int col = threadIdx.x; col < D; col += WARPS * 32) {
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < WARPS; ++k) s += part[k][col];
    dw_part[(size_t)blockIdx.x * D + col] = s;
  }
}

// dw[col] = sum of the blocks' partials.  A block of RW warps takes 32 columns
// (lane = column); warp k adds the partial rows k, k+RW, k+2RW, ... into eight
// accumulators (row k + RW(8i + a) into accumulator a, so eight independent loads
// are in flight), folds them in order, and warp 0 adds the RW warp sums in order:
// a fixed summation order, so dw is reproducible.
constexpr int RW = 32;
__global__ void __launch_bounds__(RW * 32) dw_reduce_kernel(const float* __restrict__ dw_part, float* __restrict__ dw,
                                                            int nblocks, int D) {
  pdl_wait();
  pdl_launch_dependents();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int col = blockIdx.x * 32 + lane;
  float s = 0.f;
  if (col < D) {
    float a[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) a[u] = 0.f;
    int b = warp;
    for (; b + 7 * RW < nblocks; b += 8 * RW) {
#pragma unroll
      for (int u = 0; u < 8; ++u) a[u] += dw_part[(size_t)(b + RW * u) * D + col];
    }
#pragma unroll
    for (int u = 0; u < 8; ++u)
      if (b + RW * u < nblocks) a[u] += dw_part[(size_t)(b + RW * u) * D + col];
#pragma unroll
    for (int u = 0; u < 8; ++u) s += a[u];
  }
  __shared__ float red[RW][32];
  red[warp][lane] = s;
  __syncthreads();
  if (warp == 0 && col < D) {
    float t = 0.f;
    for (int k = 0; k < RW; ++k) t += red[k][lane];
    dw[col] = t;
  }
}

// Residual add fused with the norm that follows it in a pre-norm block:
//   x_new = x + r,  y = w * x_new * rsqrt(mean(x_new^2) + eps)
// (x, x_new float32; r, y bfloat16: the residual stream and the branch output /
// next projection input under bf16 autocast).  Saves the separate add kernel and
// the norm's re-read of x_new.
template <int NC>
__global__ void __launch_bounds__(WARPS * 32) add_fwd_kernel(const float* __restrict__ x,
                                                             const __nv_bfloat16* __restrict__ r,
                                                             const float* __restrict__ w, float* __restrict__ xn,
                                                             __nv_bfloat16* __restrict__ y, float* __restrict__ rstd,
                                                             long long rows, float eps) {
  pdl_wait();
  pdl_launch_dependents();
  constexpr int D = 128 * NC;
  const int lane = threadIdx.x & 31;
  const long long row = (long long)blockIdx.x * WARPS + (threadIdx.x >> 5);
  if (row >= rows) return;
  float v[NC][4];
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    float xv[4], rv[4];
    const long long off = row * D + 128 * c + 4 * lane;
    load4<float>(x + off, xv);
    load4<__nv_bfloat16>(r + off, rv);
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      v[c][u] = xv[u] + rv[u];
      ss = fmaf(v[c][u], v[c][u], ss);
    }
    store4<float>(xn + off, v[c]);
  }
  ss = warp_sum(ss);
  const float rs = rsqrtf(ss * (1.f / D) + eps);
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    float wv[4], o[4];
    load4<float>(w + 128 * c + 4 * lane, wv);
#pragma unroll
    for (int u = 0; u < 4; ++u) o[u] = wv[u] * (v[c][u] * rs);
    store4<__nv_bfloat16>(y + row * D + 128 * c + 4 * lane, o);
  }
  if (lane == 0) rstd[row] = rs;
}

// Backward of add_fwd_kernel: with t = g_xnew + (the norm's input gradient), the
// gradients of x (float32) and of r (bfloat16) are both t; dw as in bwd_kernel.
// kG: g_xnew is given (x_new is used further on); otherwise it is zero.
template <int NC, bool kG>
__global__ void __launch_bounds__(WARPS * 32) add_bwd_kernel(const float* __restrict__ xn,
                                                             const float* __restrict__ w,
                                                             const __nv_bfloat16* __restrict__ dy,
                                                             const float* __restrict__ rstd,
                                                             const float* __restrict__ gxn, float* __restrict__ dx,
                                                             __nv_bfloat16* __restrict__ dr,
                                                             float* __restrict__ dw_part, long long rows) {
  pdl_wait();
  pdl_launch_dependents();
  constexpr int D = 128 * NC;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float acc[NC][4];
#pragma unroll
  for (int c = 0; c < NC; ++c)
#pragma unroll
    for (int u = 0; u < 4; ++u) acc[c][u] = 0.f;
  for (long long row = (long long)blockIdx.x * WARPS + warp; row < rows; row += (long long)gridDim.x * WARPS) {
    const float rs = rstd[row];
    float dot = 0.f;
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      float xv[4], dv[4], wv[4];
      const long long off = row * D + 128 * c + 4 * lane;
      load4<float>(xn + off, xv);
      load4<__nv_bfloat16>(dy + off, dv);
      load4<float>(w + 128 * c + 4 * lane, wv);
#pragma unroll
      for (int u = 0; u < 4; ++u) dot = fmaf(dv[u] * wv[u], xv[u] * rs, dot);
    }
    const float mean = warp_sum(dot) * (1.f / D);
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      float xv[4], dv[4], wv[4], gv[4], o[4];
      const long long off = row * D + 128 * c + 4 * lane;
      load4<float>(xn + off, xv);
      load4<__nv_bfloat16>(dy + off, dv);
      load4<float>(w + 128 * c + 4 * lane, wv);
      if (kG) load4<float>(gxn + off, gv);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float xh = xv[u] * rs;
        const float nd = rs * fmaf(-xh, mean, dv[u] * wv[u]);
        o[u] = kG ? gv[u] + nd : nd;
        acc[c][u] = fmaf(dv[u], xh, acc[c][u]);
      }
      store4<float>(dx + off, o);
      store4<__nv_bfloat16>(dr + off, o);
    }
  }
  __shared__ float part[WARPS][128 * NC];
#pragma unroll
  for (int c = 0; c < NC; ++c)
#pragma unroll
    for (int u = 0; u < 4; ++u) part[warp][128 * c + 4 * lane + u] = acc[c][u];
  __syncthreads();
  for (int col = threadIdx.x; col < D; col += WARPS * 32) {
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < WARPS; ++k) s += part[k][col];
    dw_part[(size_t)blockIdx.x * D + col] = s;
  }
}

int backward_blocks(long long rows) {
  const long long need = (rows + WARPS - 1) / WARPS;
  const long long cap = (long long)num_sms_cached() * BWD_BLOCKS_PER_SM;
  return (int)std::max<long long>(1, std::min(need, cap));
}

template <typename TX, typename TY, int NC>
static cudaError_t fwd_t(const void* x, const float* w, void* y, float* rstd, long long rows, float eps,
                         cudaStream_t s) {
  const unsigned blocks = (unsigned)((rows + WARPS - 1) / WARPS);
  return launch_pdl(fwd_kernel<TX, TY, NC>, dim3(blocks), dim3(WARPS * 32), 0, s, (const TX*)x, w, (TY*)y, rstd,
                    rows, eps);
}

template <typename TX, typename TY, int NC>
static cudaError_t bwd_t(const void* x, const float* w, const void* dy, const float* rstd, void* dx, float* dw,
                         float* dw_part, long long rows, cudaStream_t s) {
  const int nb = backward_blocks(rows);
  cudaError_t e = launch_pdl(bwd_kernel<TX, TY, NC>, dim3(nb), dim3(WARPS * 32), 0, s, (const TX*)x, w,
                             (const TY*)dy, rstd, (TX*)dx, dw_part, rows);
  if (e != cudaSuccess) return e;
  constexpr int D = 128 * NC;
  return launch_pdl(dw_reduce_kernel, dim3((D + 31) / 32), dim3(RW * 32), 0, s, (const float*)dw_part, dw, nb, D);
}

#define CA_NORM_DISPATCH(FN, ...)                                                          \
  switch (NCv) {                                                                           \
    case 1: return FN<TX, TY, 1>(__VA_ARGS__);                                             \
    case 2: return FN<TX, TY, 2>(__VA_ARGS__);                                             \
    case 4: return FN<TX, TY, 4>(__VA_ARGS__);                                             \
    case 8: return FN<TX, TY, 8>(__VA_ARGS__);                                             \
    default: return cudaErrorInvalidValue;                                                 \
  }

template <typename TX, typename TY>
static cudaError_t fwd_nc(int NCv, const void* x, const float* w, void* y, float* rstd, long long rows, float eps,
                          cudaStream_t s) {
  CA_NORM_DISPATCH(fwd_t, x, w, y, rstd, rows, eps, s)
}
template <typename TX, typename TY>
static cudaError_t bwd_nc(int NCv, const void* x, const float* w, const void* dy, const float* rstd, void* dx,
                          float* dw, float* dw_part, long long rows, cudaStream_t s) {
  CA_NORM_DISPATCH(bwd_t, x, w, dy, rstd, dx, dw, dw_part, rows, s)
}
#undef CA_NORM_DISPATCH

bool supported_dim(long long D) { return D == 128 || D == 256 || D == 512 || D == 1024; }

cudaError_t forward(const void* x, const float* w, void* y, float* rstd, long long rows, long long D, float eps,
                    int x_dtype, int y_dtype, cudaStream_t s) {
  const int nc = (int)(D / 128);
  if (x_dtype == 0 && y_dtype == 1) return fwd_nc<float, __nv_bfloat16>(nc, x, w, y, rstd, rows, eps, s);
  if (x_dtype == 0 && y_dtype == 0) return fwd_nc<float, float>(nc, x, w, y, rstd, rows, eps, s);
  if (x_dtype == 1 && y_dtype == 1) return fwd_nc<__nv_bfloat16, __nv_bfloat16>(nc, x, w, y, rstd, rows, eps, s);
  return fwd_nc<__nv_bfloat16, float>(nc, x, w, y, rstd, rows, eps, s);
}

cudaError_t backward(const void* x, const float* w, const void* dy, const float* rstd, void* dx, float* dw,
                     float* dw_part, long long rows, long long D, int x_dtype, int y_dtype, cudaStream_t s) {
  const int nc = (int)(D / 128);
  if (x_dtype == 0 && y_dtype == 1)
    return bwd_nc<float, __nv_bfloat16>(nc, x, w, dy, rstd, dx, dw, dw_part, rows, s);
  if (x_dtype == 0 && y_dtype == 0) return bwd_nc<float, float>(nc, x, w, dy, rstd, dx, dw, dw_part, rows, s);
  if (x_dtype == 1 && y_dtype == 1)
    return bwd_nc<__nv_bfloat16, __nv_bfloat16>(nc, x, w, dy, rstd, dx, dw, dw_part, rows, s);
  return bwd_nc<__nv_bfloat16, float>(nc, x, w, dy, rstd, dx, dw, dw_part, rows, s);
}

template <int NC>
static cudaError_t add_fwd_t(const float* x, const void* r, const float* w, float* xn, void* y, float* rstd,
                             long long rows, float eps, cudaStream_t s) {
  const unsigned blocks = (unsigned)((rows + WARPS - 1) / WARPS);
  return launch_pdl(add_fwd_kernel<NC>, dim3(blocks), dim3(WARPS * 32), 0, s, x, (const __nv_bfloat16*)r, w, xn,
                    (__nv_bfloat16*)y, rstd, rows, eps);
}

template <int NC>
static cudaError_t add_bwd_t(const float* xn, const float* w, const void* dy, const float* rstd, const float* gxn,
                             float* dx, void* dr, float* dw, float* dw_part, long long rows, cudaStream_t s) {
  const int nb = backward_blocks(rows);
  cudaError_t e = gxn ? launch_pdl(add_bwd_kernel<NC, true>, dim3(nb), dim3(WARPS * 32), 0, s, xn, w,
                                   (const __nv_bfloat16*)dy, rstd, gxn, dx, (__nv_bfloat16*)dr, dw_part, rows)
                      : launch_pdl(add_bwd_kernel<NC, false>, dim3(nb), dim3(WARPS * 32), 0, s, xn, w,
                                   (const __nv_bfloat16*)dy, rstd, gxn, dx, (__nv_bfloat16*)dr, dw_part, rows);
  if (e != cudaSuccess) return e;
  constexpr int D = 128 * NC;
  return launch_pdl(dw_reduce_kernel, dim3((D + 31) / 32), dim3(RW * 32), 0, s, (const float*)dw_part, dw, nb, D);
}

cudaError_t add_forward(const float* x, const void* r, const float* w, float* xn, void* y, float* rstd,
                        long long rows, long long D, float eps, cudaStream_t s) {
  switch (D / 128) {
    case 1: return add_fwd_t<1>(x, r, w, xn, y, rstd, rows, eps, s);
    case 2: return add_fwd_t<2>(x, r, w, xn, y, rstd, rows, eps, s);
    case 4: return add_fwd_t<4>(x, r, w, xn, y, rstd, rows, eps, s);
    case 8: return add_fwd_t<8>(x, r, w, xn, y, rstd, rows, eps, s);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t add_backward(const float* xn, const float* w, const void* dy, const float* rstd, const float* gxn,
                         float* dx, void* dr, float* dw, float* dw_part, long long rows, long long D, cudaStream_t s) {
  switch (D / 128) {
    case 1: return add_bwd_t<1>(xn, w, dy, rstd, gxn, dx, dr, dw, dw_part, rows, s);
    case 2: return add_bwd_t<2>(xn, w, dy, rstd, gxn, dx, dr, dw, dw_part, rows, s);
    case 4: return add_bwd_t<4>(xn, w, dy, rstd, gxn, dx, dr, dw, dw_part, rows, s);
    case 8: return add_bwd_t<8>(xn, w, dy, rstd, gxn, dx, dr, dw, dw_part, rows, s);
    default: return cudaErrorInvalidValue;
  }
}

size_t workspace_floats(long long rows, long long D) { return (size_t)backward_blocks(rows) * (size_t)D; }

}  // namespace norm
}  // namespace ca
