// ca_common.cuh -- element conversions and the per-segment moment math shared
// by every Continuum Attention kernel in this library.
//
// Notation (one query row, scores in natural-log units, m = reference max):
//   segment k runs from key k-1 (score a) to key k (score b), d = b - a,
//   Ea = e^{a-m}, Eb = e^{b-m},  M_n = e^{a-m} J_n(d),  J_n(d) = int_0^1 u^n e^{d u} du.
// Integration by parts gives the exact recurrences
//   M_0 = (Eb - Ea)/d,   M_n = (Eb - n M_{n-1})/d,
// which need one reciprocal per segment but cancel catastrophically as d -> 0
// (M_n loses about n+1 digits times log10(1/|d|)).  For |d| < kSeriesMax the
// highest moment needed comes from its power series
//   J_n(d) = sum_k d^k / (k! (k+n+1))
// and the lower ones from the downward form M_{n-1} = (Eb - d M_n)/n, which is
// stable for |d| < 1.  Ten series terms leave a truncation error below
// 1/(10! * 12) ~ 2.3e-8 relative at |d| = 1.
// Reference: the same moments appear as seg_L/seg_mu (cuda/continuum_attention.py:95-113)
// and moments() (:165-190); the float64 form is analytic_reference.py:12-49.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace ca {

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kSeriesMax = 1.0f;

// Where row r = bh*T + t of an activation in the [B,H,T,D] view (the output o or
// its gradient dO) is stored: row r itself when the tensor is stored [B,H,T,D]
// (bthd == 0), or row (b*T + t)*H + h when it is stored [B,T,H,D] (bthd != 0),
// the layout the attention output projection reads.  q, k, v, the fp32 output
// accumulator and the gradients dq, dk, dv are always [B,H,T,D].
__host__ __device__ __forceinline__ size_t act_row(size_t r, long long T, long long H, int bthd) {
  if (!bthd) return r;
  const size_t bh = r / (size_t)T, t = r - bh * (size_t)T;
  const size_t b = bh / (size_t)H, h = bh - b * (size_t)H;
  return (b * (size_t)T + t) * (size_t)H + h;
}

// 2^x on the MUFU pipe (relative error about 2^-22; flushes subnormal results to 0).
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// log2(x) on the MUFU pipe (absolute error about 2^-22 for x in [0.5, 2], relative elsewhere).
__device__ __forceinline__ float lg2_approx(float x) {
  float y;
  asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 1/x on the MUFU pipe (at most 1 ulp error).
__device__ __forceinline__ float rcp_approx(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Programmatic dependent launch: every kernel of this library is launched so that
// it may start while the previous kernel in the stream is finishing.  pdl_wait()
// blocks until that kernel has completed and its writes are visible (at once when
// there is no such kernel), so it precedes every global-memory access;
// pdl_launch_dependents() allows the next kernel to begin launching.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// e^x for x <= 0 relative to a row max (x = -inf gives 0).
__device__ __forceinline__ float exp_rel(float x) { return ex2_approx(x * kLog2e); }

template <typename T> __device__ __forceinline__ float to_f32(T x);
template <> __device__ __forceinline__ float to_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }
template <> __device__ __forceinline__ float to_f32<__half>(__half x) { return __half2float(x); }

template <typename T> __device__ __forceinline__ T from_f32(float x);
template <> __device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }
template <> __device__ __forceinline__ __half from_f32<__half>(float x) { return __float2half_rn(x); }

// Packed fp32 pairs (sm_100 f32x2 instructions): one instruction computes both
// lanes, each rounded exactly like its scalar counterpart.
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }
__device__ __forceinline__ float2 mul2(float2 a, float2 b) { return __fmul2_rn(a, b); }
__device__ __forceinline__ float2 add2(float2 a, float2 b) { return __fadd2_rn(a, b); }
__device__ __forceinline__ float2 splat2(float x) { return make_float2(x, x); }

// a - b on packed fp32 pairs, each lane rounded like its scalar counterpart
__device__ __forceinline__ float2 sub2(float2 a, float2 b) {
  uint64_t r;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(*reinterpret_cast<uint64_t*>(&a)), "l"(*reinterpret_cast<uint64_t*>(&b)));
  return *reinterpret_cast<float2*>(&r);
}

// max(a, b, c) in one instruction (three-input max, sm_100)
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// closed if |nd| >= thr, else ea * ps: the series branch of a moment select, as a
// compare and one predicated multiply (no separate product and select)
__device__ __forceinline__ float sel_series(float closed, float nd, float ea, float ps, float thr) {
  float r;
  asm("{\n\t.reg .pred p;\n\t.reg .f32 t;\n\tabs.f32 t, %2;\n\tsetp.lt.f32 p, t, %5;\n\t"
      "mov.f32 %0, %1;\n\t@p mul.f32 %0, %3, %4;\n\t}"
      : "=f"(r) : "f"(closed), "f"(nd), "f"(ea), "f"(ps), "f"(thr));
  return r;
}

// J_1(d) by its power series: sum_{k<10} d^k / (k! (k+2)).
__device__ __forceinline__ float series_j1(float d) {
  float p = 1.f / 3991680.f;
  p = fmaf(p, d, 1.f / 403200.f);
  p = fmaf(p, d, 1.f / 45360.f);
  p = fmaf(p, d, 1.f / 5760.f);
  p = fmaf(p, d, 1.f / 840.f);
  p = fmaf(p, d, 1.f / 144.f);
  p = fmaf(p, d, 1.f / 30.f);
  p = fmaf(p, d, 1.f / 8.f);
  p = fmaf(p, d, 1.f / 3.f);
  p = fmaf(p, d, 1.f / 2.f);
  return p;
}

// J_2(d) by its power series: sum_{k<10} d^k / (k! (k+3)).
__device__ __forceinline__ float series_j2(float d) {
  float p = 1.f / 4354560.f;
  p = fmaf(p, d, 1.f / 443520.f);
  p = fmaf(p, d, 1.f / 50400.f);
  p = fmaf(p, d, 1.f / 6480.f);
  p = fmaf(p, d, 1.f / 960.f);
  p = fmaf(p, d, 1.f / 168.f);
  p = fmaf(p, d, 1.f / 36.f);
  p = fmaf(p, d, 1.f / 10.f);
  p = fmaf(p, d, 1.f / 4.f);
  p = fmaf(p, d, 1.f / 3.f);
  return p;
}

// Forward moments of one segment: M0 = segment mass, M1 = right-endpoint share.
__device__ __forceinline__ void seg_moments01(float Ea, float Eb, float d, float& M0, float& M1) {
  if (fabsf(d) < kSeriesMax) {
    M1 = Ea * series_j1(d);
    M0 = fmaf(-d, M1, Eb);
  } else {
    const float r = rcp_approx(d);
    M0 = (Eb - Ea) * r;
    M1 = (Eb - M0) * r;
  }
}

// Backward moments of one segment: M0, M1, M2.
__device__ __forceinline__ void seg_moments012(float Ea, float Eb, float d, float& M0, float& M1,
                                               float& M2) {
  if (fabsf(d) < kSeriesMax) {
    M2 = Ea * series_j2(d);
    M1 = 0.5f * fmaf(-d, M2, Eb);
    M0 = fmaf(-d, M1, Eb);
  } else {
    const float r = rcp_approx(d);
    M0 = (Eb - Ea) * r;
    M1 = (Eb - M0) * r;
    M2 = fmaf(-2.f, M1, Eb) * r;
  }
}

// ---------------------------------------------------------------------------
// Branch-free variants for the bf16/f16 tensor-core kernels.  Both the closed
// form and a short series are evaluated and one is selected, so consecutive
// keys carry no divergent branch and the compiler can interleave them.  The
// thresholds trade closed-form cancellation against series length; their
// errors stay far inside the bf16/f16 budget.  The fp32 SIMT path keeps the
// more accurate threshold of 1 above.

// Forward-only threshold: M1 from the closed form loses ~2 eps / d^2 relative,
// 8e-6 at |d| = 0.125; four series terms then truncate below 4e-6, both far
// inside the precision of the bf16/f16 weights they produce.  Only M1 is
// selected; M0 = Eb - d M1 holds for both branches (exactly for the series, and
// for the closed form up to the rounding of M1).
constexpr float kSeriesMaxFwd = 0.125f;

// sum_{k<4} d^k / (k! (k+2))
__device__ __forceinline__ float series_j1_fwd(float d) {
  float p = 1.f / 30.f;
  p = fmaf(p, d, 1.f / 8.f);
  p = fmaf(p, d, 1.f / 3.f);
  p = fmaf(p, d, 1.f / 2.f);
  return p;
}

__device__ __forceinline__ void seg_moments01_sel(float Ea, float Eb, float d, float& M0, float& M1) {
  const float r = rcp_approx(d);
  const float m0c = (Eb - Ea) * r;
  const float m1c = (Eb - m0c) * r;
  const float m1s = Ea * series_j1_fwd(d);
  M1 = fabsf(d) < kSeriesMaxFwd ? m1s : m1c;
  M0 = fmaf(-d, M1, Eb);
}

// Backward threshold: M2 from the closed form loses ~1.4e-6 / |d|^3 relative
// (9e-5 at |d| = 0.25, on the few keys near the threshold); four series terms
// then truncate below 7e-5 relative, the same order and far below the bf16/f16
// rounding of the P and dS operands they feed.
constexpr float kSeriesMaxBwd = 0.25f;

// sum_{k<4} d^k / (k! (k+3))
__device__ __forceinline__ float series_j2_bwd(float d) {
  float p = 1.f / 36.f;
  p = fmaf(p, d, 1.f / 10.f);
  p = fmaf(p, d, 1.f / 4.f);
  p = fmaf(p, d, 1.f / 3.f);
  return p;
}

// Only M2 is selected; M1 and M0 follow from the downward recurrence, which is
// exact for the series and reproduces the closed form up to rounding.
__device__ __forceinline__ void seg_moments012_sel(float Ea, float Eb, float d, float& M0, float& M1,
                                                   float& M2) {
  const float r = rcp_approx(d);
  const float m0c = (Eb - Ea) * r;
  const float m1c = (Eb - m0c) * r;
  const float m2c = fmaf(-2.f, m1c, Eb) * r;
  M2 = sel_series(m2c, d, Ea, series_j2_bwd(d), kSeriesMaxBwd);
  M1 = 0.5f * fmaf(-d, M2, Eb);
  M0 = fmaf(-d, M1, Eb);
}

}  // namespace ca
