// ca_simt.cu -- CUDA-core (SIMT, fp32 arithmetic) Continuum Attention kernels.
//
// These kernels cover every dtype (f32/bf16/f16) and head dim D <= 128.  They
// are the float32 path (fp32 inputs need fp32-accurate scores, which the bf16
// tensor cores cannot give) and the semantic anchor for the tcgen05 kernels.
//
// Forward (flash style, one CTA per 64-row query tile): for each 64-key tile up
// to the diagonal, S = scale * Q K^T in shared memory, then per row an online
// max, the segment moments and the tile's P row, then O += P V.  Segment k
// (key k-1 -> key k) contributes A_k = M0-M1 to key k-1 and B_k = M1 to key k,
// so P column c of key tile j0 holds the weight of key j0-1+c:
//   P[c] = B_{j0+c-1} + A_{j0+c}
// with B_{j0-1} carried from the previous tile ("pending" weight) and V staged
// one row shifted (rows j0-1 .. j0+62).  The last pending weight and the two
// half-token caps are added in the epilogue.  Replaces the per-tile
// bmm -> ca_weights_kernel -> bmm chain of cuda/continuum_attention.py:670-690.
//
// Backward (one CTA per 64-key tile, looping over query tiles at or below the
// diagonal): recomputes S and dP = dO V^T over the tile plus one halo key on
// each side, forms dS from the analytic VJP with g = dP - D_i (D_i = dO_i.O_i,
// which equals sum_k w_ik dP_ik), and accumulates dV += P^T dO and
// dK += scale dS^T Q in registers; dQ += scale dS K goes to an fp32 buffer by
// atomics; sum dS*s is reduced per CTA for d log_gain.
// Replaces cuda/continuum_attention.py:713-764 and ca_backward_fused_kernel (:230-293).
#include "ca_common.cuh"
#include "ca_internal.h"

namespace ca {
namespace simt {

constexpr int BQ = 64;
constexpr int BK = 64;
constexpr int NT = 256;

// Shared tiles hold fp32 rows of stride DP + 4 floats: every row starts on a
// 16-byte boundary (float4 access), and rows r and r+1 start 4 banks apart, so
// one float4 column chunk read from 8 consecutive rows touches each bank once.
//
// The GEMM phases use register tiles of 4 rows x 4 keys (or 4 rows x DP/16
// columns) fed by float4 shared-memory reads along the reduction index; each
// sums its reduction index in increasing order, as a plain dot product does.

// 4 consecutive elements as fp32 (one 16-byte load for fp32, 8-byte for 16-bit types)
template <typename T> __device__ __forceinline__ float4 ld4(const T* p);
template <> __device__ __forceinline__ float4 ld4<float>(const float* p) {
  return __ldg(reinterpret_cast<const float4*>(p));
}
template <> __device__ __forceinline__ float4 ld4<__nv_bfloat16>(const __nv_bfloat16* p) {
  const uint2 raw = __ldg(reinterpret_cast<const uint2*>(p));
  const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.x));
  const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.y));
  return make_float4(a.x, a.y, b.x, b.y);
}
template <> __device__ __forceinline__ float4 ld4<__half>(const __half* p) {
  const uint2 raw = __ldg(reinterpret_cast<const uint2*>(p));
  const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&raw.x));
  const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&raw.y));
  return make_float4(a.x, a.y, b.x, b.y);
}

// 4 consecutive fp32 values stored as T (round to nearest)
template <typename T> __device__ __forceinline__ void st4(T* p, float4 x);
template <> __device__ __forceinline__ void st4<float>(float* p, float4 x) { *reinterpret_cast<float4*>(p) = x; }
template <> __device__ __forceinline__ void st4<__nv_bfloat16>(__nv_bfloat16* p, float4 x) {
  const __nv_bfloat162 a = __floats2bfloat162_rn(x.x, x.y), b = __floats2bfloat162_rn(x.z, x.w);
  *reinterpret_cast<uint2*>(p) = make_uint2(*reinterpret_cast<const uint32_t*>(&a), *reinterpret_cast<const uint32_t*>(&b));
}
template <> __device__ __forceinline__ void st4<__half>(__half* p, float4 x) {
  const __half2 a = __floats2half2_rn(x.x, x.y), b = __floats2half2_rn(x.z, x.w);
  *reinterpret_cast<uint2*>(p) = make_uint2(*reinterpret_cast<const uint32_t*>(&a), *reinterpret_cast<const uint32_t*>(&b));
}

// Rows row0 .. row0+n-1 of one head into tile rows 0 .. n-1 (fp32, stride DP + 4).
// Element (row, d) is src[off + row * rs + d]; rows outside [0, Tn) and columns
// d >= D read as 0.  vec: D == DP and 4-element chunks of src are aligned.
template <typename T, int DP>
__device__ __forceinline__ void load_tile(float* dst, const T* __restrict__ src, size_t off, size_t rs, int row0,
                                          int n, int Tn, int D, bool vec) {
  constexpr int LD = DP + 4;
  if (vec) {
    constexpr int C4 = DP / 4;
    for (int idx = threadIdx.x; idx < n * C4; idx += NT) {
      const int rr = idx / C4, c = (idx - rr * C4) * 4, row = row0 + rr;
      float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
      if (row >= 0 && row < Tn) x = ld4(src + off + (size_t)row * rs + c);
      *reinterpret_cast<float4*>(dst + rr * LD + c) = x;
    }
  } else {
    for (int idx = threadIdx.x; idx < n * DP; idx += NT) {
      const int rr = idx / DP, d = idx - rr * DP, row = row0 + rr;
      dst[rr * LD + d] = (row >= 0 && row < Tn && d < D) ? to_f32(src[off + (size_t)row * rs + d]) : 0.f;
    }
  }
}

// 16-byte global -> shared copy that bypasses registers (cp.async, L2 only);
// valid == false writes 16 zero bytes and reads nothing.
__device__ __forceinline__ void cp_async16(float* dst, const float* src, bool valid) {
  const uint32_t d = (uint32_t)__cvta_generic_to_shared(dst);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(src), "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// load_tile for fp32 with D == DP, issued as cp.async copies: the caller commits,
// waits (cp_async_wait_all) and then synchronises the CTA before reading.
template <int DP>
__device__ __forceinline__ void cp_async_tile(float* dst, const float* __restrict__ src, size_t off, size_t rs,
                                              int row0, int n, int Tn) {
  constexpr int LD = DP + 4, C4 = DP / 4;
  for (int idx = threadIdx.x; idx < n * C4; idx += NT) {
    const int rr = idx / C4, c = (idx - rr * C4) * 4, row = row0 + rr;
    const bool ok = row >= 0 && row < Tn;
    cp_async16(dst + rr * LD + c, ok ? src + off + (size_t)row * rs + c : src, ok);
  }
}

// CW consecutive floats of a shared row as CW/2 register pairs
template <int CW>
__device__ __forceinline__ void lds_pairs(float2 (&dst)[CW / 2], const float* p) {
  if constexpr (CW % 4 == 0) {
#pragma unroll
    for (int w = 0; w < CW; w += 4) {
      const float4 x = *reinterpret_cast<const float4*>(p + w);
      dst[w / 2] = make_float2(x.x, x.y);
      dst[w / 2 + 1] = make_float2(x.z, x.w);
    }
  } else {
    static_assert(CW == 2, "DP must be 32, 64 or 128");
    dst[0] = *reinterpret_cast<const float2*>(p);
  }
}

// S += A B^T over 4 reduction indices for a 4x4 tile, in packed pairs: lane x of
// acc[a][b] sums the even reduction indices, lane y the odd ones (the tile's
// result is x + y).
__device__ __forceinline__ void tile4x4_pairs(float2 (&acc)[4][4], const float4 (&qa)[4], const float4 (&kb)[4]) {
#pragma unroll
  for (int a = 0; a < 4; ++a)
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      acc[a][b] = fma2(make_float2(qa[a].x, qa[a].y), make_float2(kb[b].x, kb[b].y), acc[a][b]);
      acc[a][b] = fma2(make_float2(qa[a].z, qa[a].w), make_float2(kb[b].z, kb[b].w), acc[a][b]);
    }
}

// CW consecutive outputs of one row: columns col0 .. col0+CW-1 of a D-wide row
template <typename T, int CW>
__device__ __forceinline__ void store_cols(T* row, int col0, const float (&x)[CW], int D, bool vec) {
  if (vec && CW % 4 == 0) {
#pragma unroll
    for (int w = 0; w < CW; w += 4) st4<T>(row + col0 + w, make_float4(x[w], x[w + 1], x[w + 2], x[w + 3]));
  } else {
#pragma unroll
    for (int w = 0; w < CW; ++w)
      if (col0 + w < D) row[col0 + w] = from_f32<T>(x[w]);
  }
}

// ---------------------------------------------------------------------------
// forward

template <int DP>
struct FwdSmem {
  static constexpr int LD = DP + 4;      // Q / K / V' rows
  static constexpr int SLD = BK + 4;     // score row (keys j0 .. j0+63), then its P row in place
  static constexpr int kQ = 0;
  static constexpr int kK = kQ + BQ * LD;     // two K buffers (key tile kt in buffer kt & 1)
  static constexpr int kV = kK + 2 * BK * LD; // two V' buffers
  static constexpr int kS = kV + 2 * BK * LD;
  static constexpr int kRow = kS + BQ * SLD;   // per-row alpha, first, diag, w0, wi, 1/Z
  static constexpr int kFloats = kRow + 6 * BQ;
  static constexpr size_t bytes = sizeof(float) * kFloats;
};

template <typename T, int DP>
__global__ void __launch_bounds__(NT, DP <= 64 ? 2 : 1)
fwd_kernel(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
           const float* __restrict__ log_gain, T* __restrict__ o, float* __restrict__ o32,
           float* __restrict__ stats, int BH, int H, int Tn, int D, float inv_sqrt_d, int o_bthd, int vec) {
  pdl_wait();
  pdl_launch_dependents();
  using L = FwdSmem<DP>;
  constexpr int LD = L::LD, SLD = L::SLD;
  constexpr int CW = DP / 16;            // O columns per thread
  extern __shared__ __align__(16) float smem[];
  float* Qs = smem + L::kQ;
  float* Ks = smem + L::kK;
  float* Vs = smem + L::kV;
  float* Ss = smem + L::kS;
  float* sAlpha = smem + L::kRow;
  float* sFirst = sAlpha + BQ;
  float* sDiag = sFirst + BQ;
  float* sW0 = sDiag + BQ;
  float* sWi = sW0 + BQ;
  float* sInv = sWi + BQ;

  const int tid = threadIdx.x;
  const int nqt = (Tn + BQ - 1) / BQ;
  const int bh = blockIdx.x % BH;
  const int qt = nqt - 1 - blockIdx.x / BH;   // heaviest query tiles launch first
  const int h = bh % H;
  const int q0 = qt * BQ;
  const size_t base = (size_t)bh * Tn * D;
  const float scale = expf(log_gain[h]) * inv_sqrt_d;

  // fp32 tiles stream in by cp.async: key tile kt+1 is copied while tile kt is
  // computed; other element types convert through registers, tile by tile.
  const bool async = sizeof(T) == 4 && vec;
  if (async) {
    const float* qf = reinterpret_cast<const float*>(q);
    cp_async_tile<DP>(Qs, qf, base, D, q0, BQ, Tn);
    cp_async_tile<DP>(Ks, reinterpret_cast<const float*>(k), base, D, 0, BK, Tn);
    cp_async_tile<DP>(Vs, reinterpret_cast<const float*>(v), base, D, -1, BK, Tn);
    cp_async_commit();
  } else {
    load_tile<T, DP>(Qs, q, base, D, q0, BQ, Tn, D, vec);
  }

  // row phase: 4 consecutive lanes share query row r, keys 16*quad .. +15
  const int r = tid >> 2, quad = tid & 3;
  const int lane = tid & 31;
  const int i = q0 + r;
  const bool row_ok = i < Tn;
  float m_run = -INFINITY, z_part = 0.f, bpend = 0.f, sprev = 0.f;
  // tile phases: rows 4ty .. 4ty+3; keys tx + 16b (S) or O columns tx*CW .. (P V')
  const int ty = tid >> 4, tx = tid & 15;
  constexpr int CP = CW / 2;             // O column pairs per thread
  float2 acc[4][CP];
#pragma unroll
  for (int a = 0; a < 4; ++a)
#pragma unroll
    for (int w = 0; w < CP; ++w) acc[a][w] = make_float2(0.f, 0.f);

  const int last_row = min(q0 + BQ, Tn) - 1;
  const int nkt = last_row / BK + 1;

  for (int kt = 0; kt < nkt; ++kt) {
    const int j0 = kt * BK;
    float* Kb = Ks + (kt & 1) * BK * LD;
    float* Vb = Vs + (kt & 1) * BK * LD;     // V' row c = key j0-1+c
    if (async) {
      cp_async_wait_all();
      __syncthreads();   // tile kt visible; every thread is past tile kt-1, whose buffers refill now
      if (kt + 1 < nkt) {
        const int nb = ((kt + 1) & 1) * BK * LD;
        cp_async_tile<DP>(Ks + nb, reinterpret_cast<const float*>(k), base, D, j0 + BK, BK, Tn);
        cp_async_tile<DP>(Vs + nb, reinterpret_cast<const float*>(v), base, D, j0 + BK - 1, BK, Tn);
        cp_async_commit();
      }
    } else {
      __syncthreads();
      load_tile<T, DP>(Kb, k, base, D, j0, BK, Tn, D, vec);
      load_tile<T, DP>(Vb, v, base, D, j0 - 1, BK, Tn, D, vec);
      __syncthreads();
    }
    {
      float2 sacc[4][4];
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int b = 0; b < 4; ++b) sacc[a][b] = make_float2(0.f, 0.f);
#pragma unroll 2
      for (int d = 0; d < DP; d += 4) {
        float4 qa[4], kb[4];
#pragma unroll
        for (int a = 0; a < 4; ++a) qa[a] = *reinterpret_cast<const float4*>(Qs + (4 * ty + a) * LD + d);
#pragma unroll
        for (int b = 0; b < 4; ++b) kb[b] = *reinterpret_cast<const float4*>(Kb + (tx + 16 * b) * LD + d);
        tile4x4_pairs(sacc, qa, kb);
      }
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int b = 0; b < 4; ++b) Ss[(4 * ty + a) * SLD + tx + 16 * b] = (sacc[a][b].x + sacc[a][b].y) * scale;
    }
    __syncthreads();
    {
      float* srow = Ss + r * SLD;   // srow[c] = score of key j0 + c; becomes P[c] (key j0-1+c)
      const int nvis = row_ok ? min(max(i - j0 + 1, 0), BK) : 0;
      const int c0 = 16 * quad;
      float sv[16];
#pragma unroll
      for (int x = 0; x < 16; ++x) sv[x] = srow[c0 + x];
      const float sl2 = srow[max(c0 - 2, 0)], sl1 = srow[max(c0 - 1, 0)];
      const float slast = srow[BK - 1];
      if (j0 == 0 && quad == 0) sFirst[r] = sv[0];
      if (row_ok && i >= j0 + c0 && i < j0 + c0 + 16) sDiag[r] = srow[i - j0];
      __syncwarp();   // the row's four lanes have read their scores; P overwrites them

      float tmax = -INFINITY;
#pragma unroll
      for (int x = 0; x < 16; ++x)
        if (c0 + x < nvis) tmax = fmaxf(tmax, sv[x]);
      tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 1));
      tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 2));
      const float m_new = fmaxf(m_run, tmax);
      const float alpha = (m_new == -INFINITY) ? 1.f : exp_rel(m_run - m_new);
      m_run = m_new;
      z_part *= alpha;
      bpend *= alpha;
      if (quad == 0) sAlpha[r] = alpha;

      // left endpoint of segment j0+c0: key j0+c0-1
      float sa, ea, bprev;
      if (quad == 0) {
        sa = sprev;
        ea = (j0 >= 1 && nvis > 0) ? exp_rel(sprev - m_new) : 0.f;
        bprev = bpend;
      } else {
        // recompute segment j0+c0-1 (owned by the previous quad) for its right share
        const bool ok = (c0 - 1) < nvis;
        const float e2 = ok ? exp_rel(sl2 - m_new) : 0.f;
        const float e1 = ok ? exp_rel(sl1 - m_new) : 0.f;
        float M0, M1;
        seg_moments01(e2, e1, sl1 - sl2, M0, M1);
        bprev = ok ? M1 : 0.f;
        sa = sl1;
        ea = e1;
      }
#pragma unroll
      for (int x = 0; x < 16; ++x) {
        const int c = c0 + x;
        const bool vis = c < nvis;
        const bool seg_ok = vis && (j0 + c) >= 1;
        const float sb = sv[x];
        const float eb = vis ? exp_rel(sb - m_new) : 0.f;
        float A = 0.f, Bv = 0.f;
        if (seg_ok) {
          float M0, M1;
          seg_moments01(ea, eb, sb - sa, M0, M1);
          A = M0 - M1;
          Bv = M1;
          z_part += M0;
        }
        srow[c] = bprev + A;
        bprev = Bv;
        sa = sb;
        ea = eb;
      }
      bpend = __shfl_sync(0xffffffffu, bprev, (lane & ~3) | 3);
      sprev = slast;
    }
    __syncthreads();
    // O = alpha O + P V'  (rows 4ty+a, columns tx*CW ..)
    {
#pragma unroll
      for (int a = 0; a < 4; ++a) {
        const float2 al = splat2(sAlpha[4 * ty + a]);
#pragma unroll
        for (int w = 0; w < CP; ++w) acc[a][w] = mul2(acc[a][w], al);
      }
#pragma unroll 2
      for (int c = 0; c < BK; c += 4) {
        float4 pa[4];
        float2 vb[4][CP];
#pragma unroll
        for (int a = 0; a < 4; ++a) pa[a] = *reinterpret_cast<const float4*>(Ss + (4 * ty + a) * SLD + c);
#pragma unroll
        for (int u = 0; u < 4; ++u) lds_pairs<CW>(vb[u], Vb + (c + u) * LD + tx * CW);
#pragma unroll
        for (int a = 0; a < 4; ++a) {
          const float pu[4] = {pa[a].x, pa[a].y, pa[a].z, pa[a].w};
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const float2 pp = splat2(pu[u]);
#pragma unroll
            for (int w = 0; w < CP; ++w) acc[a][w] = fma2(pp, vb[u][w], acc[a][w]);
          }
        }
      }
    }
  }

  // epilogue: caps, last pending weight, normalisation
  z_part += __shfl_xor_sync(0xffffffffu, z_part, 1);
  z_part += __shfl_xor_sync(0xffffffffu, z_part, 2);
  if (quad == 0) {
    float w0 = 0.f, wi = 0.f, inv = 0.f;
    if (row_ok) {
      const float e0 = exp_rel(sFirst[r] - m_run);
      const float ei = exp_rel(sDiag[r] - m_run);
      const float Z = z_part + 0.5f * e0 + 0.5f * ei;
      w0 = 0.5f * e0;
      wi = bpend + 0.5f * ei;
      inv = 1.f / Z;
      if (stats) {   // stats == nullptr: inference, no backward follows
        stats[2 * ((size_t)bh * Tn + i)] = m_run;
        stats[2 * ((size_t)bh * Tn + i) + 1] = Z;
      }
    }
    sW0[r] = w0;
    sWi[r] = wi;
    sInv[r] = inv;
  }
  __syncthreads();
  const int col0 = tx * CW;
  float v0[CW];
#pragma unroll
  for (int w = 0; w < CW; ++w) v0[w] = (col0 + w < D) ? to_f32(v[base + col0 + w]) : 0.f;
#pragma unroll
  for (int a = 0; a < 4; ++a) {
    const int rr = 4 * ty + a, row = q0 + rr;
    if (row >= Tn) continue;
    const float w0 = sW0[rr], wi = sWi[rr], inv = sInv[rr];
    const T* vi = v + base + (size_t)row * D;
    float y[CW];
#pragma unroll
    for (int w = 0; w < CW; ++w) {
      const float vv = (col0 + w < D) ? to_f32(vi[col0 + w]) : 0.f;
      const float av = (w & 1) ? acc[a][w / 2].y : acc[a][w / 2].x;
      y[w] = (av + w0 * v0[w] + wi * vv) * inv;
    }
    store_cols<T, CW>(o + act_row((size_t)bh * Tn + row, Tn, H, o_bthd) * D, col0, y, D, vec);
    if (o32) store_cols<float, CW>(o32 + base + (size_t)row * D, col0, y, D, vec);
  }
}

// ---------------------------------------------------------------------------
// backward

template <int DP>
struct BwdSmem {
  static constexpr int LD = DP + 4;
  static constexpr int HK = BK + 2;      // keys j0-1 .. j0+64
  static constexpr int SLD = BK + 4;     // S / dP row over the HK keys, then P / scale*dS in place
  static constexpr int kK = 0;
  static constexpr int kV = kK + HK * LD;
  static constexpr int kQ = kV + HK * LD;
  static constexpr int kO = kQ + BQ * LD;
  static constexpr int kS = kO + BQ * LD;
  static constexpr int kDP = kS + BQ * SLD;
  static constexpr int kM = kDP + BQ * SLD;
  static constexpr int kIZ = kM + BQ;
  static constexpr int kDD = kIZ + BQ;
  static constexpr int kRed = kDD + BQ;
  static constexpr int kFloats = kRed + NT / 32;
  static constexpr size_t bytes = sizeof(float) * kFloats;
};

template <typename T, int DP>
__global__ void __launch_bounds__(NT, DP <= 64 ? 2 : 1)
bwd_kernel(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
           const T* __restrict__ dout, const float* __restrict__ log_gain,
           const float* __restrict__ stats, const float* __restrict__ rowdot,
           float* __restrict__ dq_acc, T* __restrict__ dk, T* __restrict__ dv,
           float* __restrict__ gain_part, int BH, int H, int Tn, int D, float inv_sqrt_d, int do_bthd, int vec) {
  pdl_wait();
  pdl_launch_dependents();
  using L = BwdSmem<DP>;
  constexpr int LD = L::LD, SLD = L::SLD, HK = L::HK;
  constexpr int CW = DP / 16;
  extern __shared__ __align__(16) float smem[];
  float* Ks = smem + L::kK;
  float* Vs = smem + L::kV;
  float* Qs = smem + L::kQ;
  float* Os = smem + L::kO;    // dO tile
  float* Ss = smem + L::kS;
  float* DPs = smem + L::kDP;
  float* sM = smem + L::kM;
  float* sIZ = smem + L::kIZ;
  float* sDD = smem + L::kDD;
  float* sRed = smem + L::kRed;

  const int tid = threadIdx.x;
  const int nkt = (Tn + BK - 1) / BK;
  const int bh = blockIdx.x % BH;
  const int kt = blockIdx.x / BH;          // low key tiles see the most queries: launch first
  const int h = bh % H;
  const int j0 = kt * BK;
  const size_t base = (size_t)bh * Tn * D;
  // dO row t of this head: [B,H,T,D] or [B,T,H,D]
  const size_t do_off = do_bthd ? ((size_t)(bh / H) * Tn * H + h) * D : base;
  const size_t do_rs = do_bthd ? (size_t)H * D : (size_t)D;
  const float scale = expf(log_gain[h]) * inv_sqrt_d;

  // stationary K and V with one halo key on each side (keys j0-1 .. j0+64)
  load_tile<T, DP>(Ks, k, base, D, j0 - 1, HK, Tn, D, vec);
  load_tile<T, DP>(Vs, v, base, D, j0 - 1, HK, Tn, D, vec);

  const int r = tid >> 2, quad = tid & 3;     // row phase: query row r, keys 16*quad .. +15
  const int ty = tid >> 4, tx = tid & 15;     // S/dP: rows 4ty.., keys tx+16b; dQ: rows 4ty.., columns tx*CW..
  const int kg = tid & 15, cg = tid >> 4;     // dK/dV: keys 4kg .. 4kg+3, columns cg*CW ..
  constexpr int CP = CW / 2;             // column pairs per thread
  float2 dk_acc[4][CP], dv_acc[4][CP];
#pragma unroll
  for (int u = 0; u < 4; ++u)
#pragma unroll
    for (int w = 0; w < CP; ++w) dk_acc[u][w] = dv_acc[u][w] = make_float2(0.f, 0.f);
  float gsum = 0.f;

  // fp32 query tiles stream in by cp.async: tile q0+BQ is copied during the dQ
  // product of tile q0 (which reads only dS and K); other element types convert
  // through registers, tile by tile.  Threads 0..63 fetch the row statistics of
  // the next tile into registers ahead of time as well.
  const bool async = sizeof(T) == 4 && vec;
  const int qfirst = j0 - (j0 % BQ);
  auto row_stats = [&](int q0, float& m, float& iz, float& dd) {
    const int row = q0 + tid;
    m = 0.f; iz = 0.f; dd = 0.f;
    if (row < Tn) {
      const size_t ri = (size_t)bh * Tn + row;
      m = stats[2 * ri];
      iz = 1.f / stats[2 * ri + 1];
      dd = rowdot[ri];
    }
  };
  float nM = 0.f, nIZ = 0.f, nDD = 0.f;
  if (tid < BQ) row_stats(qfirst, nM, nIZ, nDD);
  if (async) {
    cp_async_tile<DP>(Qs, reinterpret_cast<const float*>(q), base, D, qfirst, BQ, Tn);
    cp_async_tile<DP>(Os, reinterpret_cast<const float*>(dout), do_off, do_rs, qfirst, BQ, Tn);
    cp_async_commit();
  }

  for (int q0 = qfirst; q0 < Tn; q0 += BQ) {
    if (async) {
      cp_async_wait_all();
    } else {
      __syncthreads();
      load_tile<T, DP>(Qs, q, base, D, q0, BQ, Tn, D, vec);
      load_tile<T, DP>(Os, dout, do_off, do_rs, q0, BQ, Tn, D, vec);
    }
    if (tid < BQ) {   // the previous tile's readers of these passed two barriers since
      sM[tid] = nM;
      sIZ[tid] = nIZ;
      sDD[tid] = nDD;
    }
    __syncthreads();
    // S (scaled) and dP: keys j0 .. j0+63 (halo index 1 .. 64) as 4x4 register tiles
#pragma unroll
    for (int pass = 0; pass < 2; ++pass) {
      const float* A = pass ? Os : Qs;
      const float* Bm = pass ? Vs : Ks;
      float2 sacc[4][4];
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int b = 0; b < 4; ++b) sacc[a][b] = make_float2(0.f, 0.f);
#pragma unroll 2
      for (int d = 0; d < DP; d += 4) {
        float4 qa[4], kb[4];
#pragma unroll
        for (int a = 0; a < 4; ++a) qa[a] = *reinterpret_cast<const float4*>(A + (4 * ty + a) * LD + d);
#pragma unroll
        for (int b = 0; b < 4; ++b) kb[b] = *reinterpret_cast<const float4*>(Bm + (1 + tx + 16 * b) * LD + d);
        tile4x4_pairs(sacc, qa, kb);
      }
      float* dst = pass ? DPs : Ss;
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int b = 0; b < 4; ++b) {
          const float x = sacc[a][b].x + sacc[a][b].y;
          dst[(4 * ty + a) * SLD + 1 + tx + 16 * b] = pass ? x : x * scale;
        }
    }
    // the halo keys j0-1 and j0+64 (index 0 and HK-1): one dot product per thread
    {
      const int hr = tid & 63;
      const int hx = (tid & 64) ? HK - 1 : 0;
      const bool dpm = tid >= 128;
      const float* arow = (dpm ? Os : Qs) + hr * LD;
      const float* brow = (dpm ? Vs : Ks) + hx * LD;
      float2 s2 = make_float2(0.f, 0.f);   // even / odd d, summed like the tiles
#pragma unroll 4
      for (int d = 0; d < DP; d += 4) {
        const float4 a4 = *reinterpret_cast<const float4*>(arow + d);
        const float4 b4 = *reinterpret_cast<const float4*>(brow + d);
        s2 = fma2(make_float2(a4.x, a4.y), make_float2(b4.x, b4.y), s2);
        s2 = fma2(make_float2(a4.z, a4.w), make_float2(b4.z, b4.w), s2);
      }
      const float s = s2.x + s2.y;
      if (dpm)
        DPs[hr * SLD + hx] = s;
      else
        Ss[hr * SLD + hx] = s * scale;
    }
    __syncthreads();
    {
      // sv[y] / pv[y] hold key j0-1+c0+y (halo index c0+y)
      float* srow = Ss + r * SLD;
      float* prow = DPs + r * SLD;
      const int i = q0 + r;
      const bool row_ok = i < Tn;
      const float m = sM[r], iz = sIZ[r], dd = sDD[r];
      const int c0 = 16 * quad;
      float sv[18], pv[18];
#pragma unroll
      for (int y = 0; y < 18; ++y) {
        sv[y] = srow[c0 + y];
        pv[y] = prow[c0 + y];
      }
      __syncwarp();   // the row's four lanes have read S / dP; P / dS overwrite them
      // key j0-1+x visible iff it is >= 0 and <= i
      auto vis = [&](int x) { return row_ok && (j0 - 1 + x) >= 0 && (j0 - 1 + x) <= i; };
      float sa = sv[0];                       // key j0+c0-1
      float ea = vis(c0) ? exp_rel(sa - m) : 0.f;
      float ga = pv[0] - dd;
      float Rprev = 0.f, Bprev = 0.f;          // right shares of the segment into the current key
      {
        const int x = c0 + 1;                  // key j0+c0
        const float sb = sv[1];
        const bool ok = vis(x) && (j0 - 1 + x) >= 1;
        const float eb = vis(x) ? exp_rel(sb - m) : 0.f;
        const float gb = pv[1] - dd;
        if (ok) {
          float M0, M1, M2;
          seg_moments012(ea, eb, sb - sa, M0, M1, M2);
          const float G = gb - ga;
          Rprev = fmaf(ga, M1, G * M2);
          Bprev = M1;
        }
        sa = sb; ea = eb; ga = gb;
      }
#pragma unroll
      for (int xx = 0; xx < 16; ++xx) {
        const int x = c0 + 1 + xx;             // current key (halo index)
        const int key = j0 - 1 + x;
        // segment from key x to key x+1
        const float sb = sv[xx + 2];
        const bool okn = vis(x + 1);           // right key visible (and >= 1 automatically)
        const float eb = okn ? exp_rel(sb - m) : 0.f;
        const float gb = pv[xx + 2] - dd;
        float Lnext = 0.f, Anext = 0.f, Rn = 0.f, Bn = 0.f;
        if (okn) {
          float M0, M1, M2;
          seg_moments012(ea, eb, sb - sa, M0, M1, M2);
          const float G = gb - ga;
          const float A = M0 - M1;
          Lnext = fmaf(ga, A, G * (M1 - M2));
          Anext = A;
          Rn = fmaf(ga, M1, G * M2);
          Bn = M1;
        }
        float ds = 0.f, p = 0.f;
        if (vis(x)) {
          const float cap = 0.5f * ea * ((key == 0 ? 1.f : 0.f) + (key == i ? 1.f : 0.f));
          ds = (Rprev + Lnext + cap * ga) * iz;
          p = (Bprev + Anext + cap) * iz;
          gsum = fmaf(ds, sa, gsum);
        }
        prow[x - 1] = ds * scale;
        srow[x - 1] = p;
        Rprev = Rn; Bprev = Bn;
        sa = sb; ea = eb; ga = gb;
      }
    }
    __syncthreads();
    // dV += P^T dO, dK += (scale dS)^T Q  (keys 4kg+u, columns cg*CW ..)
    {
      const int cc = cg * CW;
#pragma unroll 2
      for (int rr = 0; rr < BQ; ++rr) {
        const float4 p4 = *reinterpret_cast<const float4*>(Ss + rr * SLD + 4 * kg);
        const float4 g4 = *reinterpret_cast<const float4*>(DPs + rr * SLD + 4 * kg);
        float2 ov[CP], qv[CP];
        lds_pairs<CW>(ov, Os + rr * LD + cc);
        lds_pairs<CW>(qv, Qs + rr * LD + cc);
        const float pp[4] = {p4.x, p4.y, p4.z, p4.w};
        const float gg[4] = {g4.x, g4.y, g4.z, g4.w};
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const float2 p2 = splat2(pp[u]), g2 = splat2(gg[u]);
#pragma unroll
          for (int w = 0; w < CP; ++w) {
            dv_acc[u][w] = fma2(p2, ov[w], dv_acc[u][w]);
            dk_acc[u][w] = fma2(g2, qv[w], dk_acc[u][w]);
          }
        }
      }
    }
    if (q0 + BQ < Tn) {
      if (tid < BQ) row_stats(q0 + BQ, nM, nIZ, nDD);
      if (async) {
        __syncthreads();   // every thread is done with this Q / dO tile
        cp_async_tile<DP>(Qs, reinterpret_cast<const float*>(q), base, D, q0 + BQ, BQ, Tn);
        cp_async_tile<DP>(Os, reinterpret_cast<const float*>(dout), do_off, do_rs, q0 + BQ, BQ, Tn);
        cp_async_commit();
      }
    }
    // dQ += (scale dS) K  (rows 4ty+a, columns tx*CW ..), fp32 atomics
    {
      float2 dq2[4][CP];
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int w = 0; w < CP; ++w) dq2[a][w] = make_float2(0.f, 0.f);
#pragma unroll 2
      for (int c = 0; c < BK; c += 4) {
        float4 g4[4];
        float2 kk[4][CP];
#pragma unroll
        for (int a = 0; a < 4; ++a) g4[a] = *reinterpret_cast<const float4*>(DPs + (4 * ty + a) * SLD + c);
#pragma unroll
        for (int u = 0; u < 4; ++u) lds_pairs<CW>(kk[u], Ks + (c + 1 + u) * LD + tx * CW);
#pragma unroll
        for (int a = 0; a < 4; ++a) {
          const float gu[4] = {g4[a].x, g4[a].y, g4[a].z, g4[a].w};
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const float2 g2 = splat2(gu[u]);
#pragma unroll
            for (int w = 0; w < CP; ++w) dq2[a][w] = fma2(g2, kk[u][w], dq2[a][w]);
          }
        }
      }
      float dqa[4][CW];
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int w = 0; w < CP; ++w) {
          dqa[a][2 * w] = dq2[a][w].x;
          dqa[a][2 * w + 1] = dq2[a][w].y;
        }
      const int col0 = tx * CW;
#pragma unroll
      for (int a = 0; a < 4; ++a) {
        const int row = q0 + 4 * ty + a;
        if (row >= Tn) continue;
        float* dst = dq_acc + base + (size_t)row * D + col0;
        if (vec) {
          if constexpr (CW % 4 == 0) {
#pragma unroll
            for (int w = 0; w < CW; w += 4)
              atomicAdd(reinterpret_cast<float4*>(dst + w),
                        make_float4(dqa[a][w], dqa[a][w + 1], dqa[a][w + 2], dqa[a][w + 3]));
          } else {
            atomicAdd(reinterpret_cast<float2*>(dst), make_float2(dqa[a][0], dqa[a][1]));
          }
        } else {
#pragma unroll
          for (int w = 0; w < CW; ++w)
            if (col0 + w < D) atomicAdd(dst + w, dqa[a][w]);
        }
      }
    }
  }

  {
    const int cc = cg * CW;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int key = j0 + 4 * kg + u;
      if (key < Tn) {
        float kx[CW], vx[CW];
#pragma unroll
        for (int w = 0; w < CP; ++w) {
          kx[2 * w] = dk_acc[u][w].x;
          kx[2 * w + 1] = dk_acc[u][w].y;
          vx[2 * w] = dv_acc[u][w].x;
          vx[2 * w + 1] = dv_acc[u][w].y;
        }
        store_cols<T, CW>(dk + base + (size_t)key * D, cc, kx, D, vec);
        store_cols<T, CW>(dv + base + (size_t)key * D, cc, vx, D, vec);
      }
    }
  }
  if (gain_part) {
    for (int off = 16; off > 0; off >>= 1) gsum += __shfl_xor_sync(0xffffffffu, gsum, off);
    if ((tid & 31) == 0) sRed[tid >> 5] = gsum;
    __syncthreads();
    if (tid == 0) {
      float t = 0.f;
      for (int w = 0; w < NT / 32; ++w) t += sRed[w];
      gain_part[(size_t)bh * nkt + kt] = t;
    }
  }
}

// D_i = dO_i . O_i  (one warp per row); O in the element type TO (dtype or its fp32 accumulator)
template <typename TO, typename T>
__global__ void rowdot_kernel(const TO* __restrict__ o, const T* __restrict__ dout,
                              float* __restrict__ rowdot, size_t rows, int D, int Tn, int H, int o_bthd,
                              int do_bthd) {
  pdl_wait();
  pdl_launch_dependents();
  const size_t row = (size_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  float s = 0.f;
  const TO* orow = o + act_row(row, Tn, H, o_bthd) * D;
  const T* drow = dout + act_row(row, Tn, H, do_bthd) * D;
  for (int d = lane; d < D; d += 32) s = fmaf(to_f32(orow[d]), to_f32(drow[d]), s);
  for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
  if (lane == 0) rowdot[row] = s;
}

// Backward preparation for D = 64, one pass: D_i = dO_i . O_i and zeros for the
// fp32 dQ accumulator.  16 threads per row, 4 consecutive elements each
// (16-byte O loads when O is fp32, 8-byte dO loads), 2 rows per warp.
// kOB / kDB: O / dO rows stored [B,T,H,D] (act_row); compile-time, so the usual
// [B,H,T,D] case carries no index arithmetic.
template <typename TO, typename T, bool kOB, bool kDB>
__global__ void prep64_kernel(const TO* __restrict__ o, const T* __restrict__ dout, float* __restrict__ rowdot,
                              float* __restrict__ dq_acc, size_t rows, unsigned* __restrict__ counter,
                              unsigned* __restrict__ ready, int n_ready, int Tn, int H) {
  pdl_wait();
  pdl_launch_dependents();
  const size_t gid = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (gid == 0 && counter) *counter = 0u;   // work-item counter of the persistent backward
  if (ready && gid < (size_t)n_ready) ready[gid] = 0u;   // ordered-dQ turn counters
  const size_t row = gid >> 4;
  const int part = (int)(gid & 15);
  float s = 0.f;
  if (row < rows) {
    const size_t base = row * 64 + 4 * part;
    const size_t obase = (kOB ? act_row(row, Tn, H, 1) * 64 + 4 * part : base);
    const size_t dbase = (kDB ? act_row(row, Tn, H, 1) * 64 + 4 * part : base);
    float ov[4], dv[4];
    if (sizeof(TO) == 4) {
      const float4 x = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(o) + obase);
      ov[0] = x.x; ov[1] = x.y; ov[2] = x.z; ov[3] = x.w;
    } else {
#pragma unroll
      for (int u = 0; u < 4; ++u) ov[u] = to_f32(o[obase + u]);
    }
    if (sizeof(T) == 4) {
      const float4 x = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(dout) + dbase);
      dv[0] = x.x; dv[1] = x.y; dv[2] = x.z; dv[3] = x.w;
    } else {
      const uint2 raw = *reinterpret_cast<const uint2*>(dout + dbase);
      const T* dp = reinterpret_cast<const T*>(&raw);
#pragma unroll
      for (int u = 0; u < 4; ++u) dv[u] = to_f32(dp[u]);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) s = fmaf(ov[u], dv[u], s);
    if (dq_acc) *reinterpret_cast<float4*>(dq_acc + base) = make_float4(0.f, 0.f, 0.f, 0.f);
  }
#pragma unroll
  for (int off = 8; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
  if (row < rows && part == 0) rowdot[row] = s;
}

// d log_gain[h] = sum over batch and key-tile partials, fixed order (deterministic);
// one 256-thread block per head.
__device__ __forceinline__ void gain_reduce_block(const float* __restrict__ part, float* __restrict__ out, int B,
                                                  int H, int nparts, int h) {
  float s = 0.f;
  for (int idx = threadIdx.x; idx < B * nparts; idx += blockDim.x) {
    const int b = idx / nparts, t = idx % nparts;
    s += part[((size_t)b * H + h) * nparts + t];
  }
  __shared__ float red[32];
  for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < (int)(blockDim.x / 32); ++w) t += red[w];
    out[h] = t;
  }
}

// The backward's last launch: fp32 dQ accumulator -> dtype in blocks
// [0, cast_blocks) and, when part != nullptr, the d log_gain reduction of head
// h in block cast_blocks + h.  kVec: 4 elements per thread (n a multiple of 4,
// 16-byte aligned source, dst aligned to 4 elements); otherwise one per thread.
template <typename T, bool kVec>
__global__ void cast_gain_kernel(const float* __restrict__ src, T* __restrict__ dst, size_t n, int cast_blocks,
                                 const float* __restrict__ part, float* __restrict__ gout, int B, int H,
                                 int nparts) {
  pdl_wait();
  pdl_launch_dependents();
  if ((int)blockIdx.x >= cast_blocks) {
    gain_reduce_block(part, gout, B, H, nparts, (int)blockIdx.x - cast_blocks);
    return;
  }
  const size_t stride = (size_t)cast_blocks * blockDim.x;
  if (kVec) {
    const size_t n4 = n / 4;
    for (size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x; idx < n4; idx += stride) {
      const float4 x = reinterpret_cast<const float4*>(src)[idx];
      T out[4] = {from_f32<T>(x.x), from_f32<T>(x.y), from_f32<T>(x.z), from_f32<T>(x.w)};
      if (sizeof(T) == 2)
        reinterpret_cast<uint2*>(dst)[idx] = *reinterpret_cast<const uint2*>(out);
      else
        reinterpret_cast<float4*>(dst)[idx] = *reinterpret_cast<const float4*>(out);
    }
  } else {
    for (size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x; idx < n; idx += stride)
      dst[idx] = from_f32<T>(src[idx]);
  }
}

// ---------------------------------------------------------------------------
// launchers

// 4-element chunks of T at p are aligned for the vector loads and stores (null passes)
template <typename T>
static bool vec_ok(const void* p) {
  return (reinterpret_cast<uintptr_t>(p) & (4 * sizeof(T) - 1)) == 0;
}

template <typename T, int DP>
static cudaError_t launch_fwd(const FwdArgs& a) {
  auto kern = fwd_kernel<T, DP>;
  const size_t smem = FwdSmem<DP>::bytes;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const long long BH = a.B * a.H;
  const long long nqt = (a.T + BQ - 1) / BQ;
  const int vec = a.D == DP && vec_ok<T>(a.q) && vec_ok<T>(a.k) && vec_ok<T>(a.v) && vec_ok<T>(a.o) &&
                  vec_ok<float>(a.o_f32);
  return launch_pdl(kern, dim3((unsigned)(BH * nqt)), dim3(NT), smem, a.stream, (const T*)a.q, (const T*)a.k,
                    (const T*)a.v, a.log_gain, (T*)a.o, a.o_f32, a.row_stats, (int)BH, (int)a.H, (int)a.T,
                    (int)a.D, a.inv_sqrt_d, a.o_bthd, vec);
}

template <typename T>
static cudaError_t fwd_dtype(const FwdArgs& a) {
  if (a.D <= 32) return launch_fwd<T, 32>(a);
  if (a.D <= 64) return launch_fwd<T, 64>(a);
  return launch_fwd<T, 128>(a);
}

cudaError_t forward(const FwdArgs& a) {
  switch (a.dtype) {
    case 0: return fwd_dtype<float>(a);
    case 1: return fwd_dtype<__nv_bfloat16>(a);
    default: return fwd_dtype<__half>(a);
  }
}

template <typename T, int DP>
static cudaError_t launch_bwd(const BwdArgs& a, const BwdWorkspace& w) {
  auto kern = bwd_kernel<T, DP>;
  const size_t smem = BwdSmem<DP>::bytes;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const long long BH = a.B * a.H;
  const long long nkt = (a.T + BK - 1) / BK;
  const int vec = a.D == DP && vec_ok<T>(a.q) && vec_ok<T>(a.k) && vec_ok<T>(a.v) && vec_ok<T>(a.d_o) &&
                  vec_ok<T>(a.dk) && vec_ok<T>(a.dv) && vec_ok<float>(w.dq_acc);
  return launch_pdl(kern, dim3((unsigned)(BH * nkt)), dim3(NT), smem, a.stream, (const T*)a.q, (const T*)a.k,
                    (const T*)a.v, (const T*)a.d_o, a.log_gain, a.row_stats, (const float*)w.rowdot, w.dq_acc,
                    (T*)a.dk, (T*)a.dv, a.dlog_gain ? w.gain_part : nullptr, (int)BH, (int)a.H, (int)a.T,
                    (int)a.D, a.inv_sqrt_d, a.act_bthd, vec);
}

template <typename T>
static cudaError_t rowdot_dtype(const BwdArgs& a, float* rowdot) {
  const size_t rows = (size_t)a.B * a.H * a.T;
  const dim3 grid((unsigned)((rows + 7) / 8));
  if (a.o_f32)
    return launch_pdl(rowdot_kernel<float, T>, grid, dim3(256), 0, a.stream, (const float*)a.o_f32,
                      (const T*)a.d_o, rowdot, rows, (int)a.D, (int)a.T, (int)a.H, 0, a.act_bthd);
  return launch_pdl(rowdot_kernel<T, T>, grid, dim3(256), 0, a.stream, (const T*)a.o, (const T*)a.d_o, rowdot,
                    rows, (int)a.D, (int)a.T, (int)a.H, a.act_bthd, a.act_bthd);
}

template <typename T>
static cudaError_t prep_dtype(const BwdArgs& a, float* rowdot, float* dq_acc, unsigned* counter, unsigned* ready,
                              int n_ready) {
  const size_t rows = (size_t)a.B * a.H * a.T;
  const uintptr_t oal = reinterpret_cast<uintptr_t>(a.o_f32 ? (const void*)a.o_f32 : a.o);
  const bool vec = a.D == 64 && (reinterpret_cast<uintptr_t>(a.d_o) & (4 * sizeof(T) - 1)) == 0 &&
                   (a.o_f32 || sizeof(T) == 4 ? (oal & 15) == 0 : true);
  if (!counter) ready = nullptr;
  if (!vec) {
    cudaError_t e = rowdot_dtype<T>(a, rowdot);
    if (e != cudaSuccess) return e;
    if (counter) {
      e = cudaMemsetAsync(counter, 0, sizeof(unsigned), a.stream);
      if (e != cudaSuccess) return e;
    }
    if (ready && n_ready > 0) {
      e = cudaMemsetAsync(ready, 0, (size_t)n_ready * sizeof(unsigned), a.stream);
      if (e != cudaSuccess) return e;
    }
    return dq_acc ? cudaMemsetAsync(dq_acc, 0, rows * a.D * sizeof(float), a.stream) : cudaSuccess;
  }
  const size_t threads = std::max<size_t>(rows * 16, ready ? (size_t)n_ready : 0);
  const unsigned blocks = (unsigned)((threads + 255) / 256);
  const dim3 g(blocks), b(256);
  if (a.o_f32) {
    auto k = a.act_bthd ? prep64_kernel<float, T, false, true> : prep64_kernel<float, T, false, false>;
    return launch_pdl(k, g, b, 0, a.stream, (const float*)a.o_f32, (const T*)a.d_o, rowdot, dq_acc, rows, counter,
                      ready, n_ready, (int)a.T, (int)a.H);
  }
  auto k = a.act_bthd ? prep64_kernel<T, T, true, true> : prep64_kernel<T, T, false, false>;
  return launch_pdl(k, g, b, 0, a.stream, (const T*)a.o, (const T*)a.d_o, rowdot, dq_acc, rows, counter, ready,
                    n_ready, (int)a.T, (int)a.H);
}

cudaError_t launch_prep(const BwdArgs& a, float* rowdot, float* dq_acc, unsigned* counter, unsigned* ready,
                        int n_ready) {
  switch (a.dtype) {
    case 0: return prep_dtype<float>(a, rowdot, dq_acc, counter, ready, n_ready);
    case 1: return prep_dtype<__nv_bfloat16>(a, rowdot, dq_acc, counter, ready, n_ready);
    default: return prep_dtype<__half>(a, rowdot, dq_acc, counter, ready, n_ready);
  }
}

template <typename T>
static cudaError_t cast_dtype(const BwdArgs& a, const float* dq_acc, const float* part, int nparts) {
  const size_t n = (size_t)a.B * a.H * a.T * a.D;
  const bool vec = n % 4 == 0 && (reinterpret_cast<uintptr_t>(a.dq) & (4 * sizeof(T) - 1)) == 0;
  const size_t items = vec ? n / 4 : n;
  const int cast_blocks = (int)std::min<size_t>(std::max<size_t>((items + 255) / 256, 1), 148 * 16);
  const unsigned blocks = (unsigned)(cast_blocks + (a.dlog_gain ? a.H : 0));
  if (vec)
    return launch_pdl(cast_gain_kernel<T, true>, dim3(blocks), dim3(256), 0, a.stream, dq_acc, (T*)a.dq, n,
                      cast_blocks, part, a.dlog_gain, (int)a.B, (int)a.H, nparts);
  return launch_pdl(cast_gain_kernel<T, false>, dim3(blocks), dim3(256), 0, a.stream, dq_acc, (T*)a.dq, n,
                    cast_blocks, part, a.dlog_gain, (int)a.B, (int)a.H, nparts);
}

cudaError_t launch_cast_dq(const BwdArgs& a, const float* dq_acc, const float* gain_part, int nparts) {
  switch (a.dtype) {
    case 0: return cast_dtype<float>(a, dq_acc, gain_part, nparts);
    case 1: return cast_dtype<__nv_bfloat16>(a, dq_acc, gain_part, nparts);
    default: return cast_dtype<__half>(a, dq_acc, gain_part, nparts);
  }
}

template <typename T>
static cudaError_t bwd_dtype(const BwdArgs& a, const BwdWorkspace& w) {
  cudaError_t e = launch_prep(a, w.rowdot, w.dq_acc, nullptr);
  if (e != cudaSuccess) return e;
  if (a.D <= 32) e = launch_bwd<T, 32>(a, w);
  else if (a.D <= 64) e = launch_bwd<T, 64>(a, w);
  else e = launch_bwd<T, 128>(a, w);
  if (e != cudaSuccess) return e;
  return launch_cast_dq(a, w.dq_acc, w.gain_part, (int)((a.T + BK - 1) / BK));
}

cudaError_t backward(const BwdArgs& a, const BwdWorkspace& w) {
  switch (a.dtype) {
    case 0: return bwd_dtype<float>(a, w);
    case 1: return bwd_dtype<__nv_bfloat16>(a, w);
    default: return bwd_dtype<__half>(a, w);
  }
}

}  // namespace simt
}  // namespace ca
