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

template <int DP>
struct FwdSmem {
  static constexpr int LD = DP + 1;      // padded Q/K row
  static constexpr int SLD = BK + 2;     // score row (keys j0..j0+63, padded)
  static constexpr int PLD = BK + 1;     // P row
  static constexpr int kQ = 0;
  static constexpr int kK = kQ + BQ * LD;
  static constexpr int kV = kK + BK * LD;
  static constexpr int kS = kV + BK * DP;
  static constexpr int kP = kS + BQ * SLD;
  static constexpr int kFirst = kP + BQ * PLD;
  static constexpr int kDiag = kFirst + BQ;
  static constexpr int kFloats = kDiag + BQ;
  static constexpr size_t bytes = sizeof(float) * kFloats;
};

template <typename T, int DP>
__global__ void __launch_bounds__(NT)
fwd_kernel(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
           const float* __restrict__ log_gain, T* __restrict__ o, float* __restrict__ o32,
           float* __restrict__ stats, int BH, int H, int Tn, int D, float inv_sqrt_d, int o_bthd) {
  pdl_wait();
  pdl_launch_dependents();
  using L = FwdSmem<DP>;
  constexpr int DQ = DP / 4;             // O columns per thread
  extern __shared__ float smem[];
  float* Qs = smem + L::kQ;
  float* Ks = smem + L::kK;
  float* Vs = smem + L::kV;
  float* Ss = smem + L::kS;
  float* Ps = smem + L::kP;
  float* sFirst = smem + L::kFirst;
  float* sDiag = smem + L::kDiag;

  const int tid = threadIdx.x;
  const int nqt = (Tn + BQ - 1) / BQ;
  const int bh = blockIdx.x % BH;
  const int qt = nqt - 1 - blockIdx.x / BH;   // heaviest query tiles launch first
  const int h = bh % H;
  const int q0 = qt * BQ;
  const size_t base = (size_t)bh * Tn * D;
  const float scale = expf(log_gain[h]) * inv_sqrt_d;

  for (int idx = tid; idx < BQ * DP; idx += NT) {
    const int r = idx / DP, d = idx % DP, row = q0 + r;
    Qs[r * L::LD + d] = (row < Tn && d < D) ? to_f32(q[base + (size_t)row * D + d]) : 0.f;
  }

  // row-phase identity: 4 consecutive lanes share one query row
  const int r = tid >> 2, quad = tid & 3;
  const int lane = tid & 31;
  const int i = q0 + r;
  const bool row_ok = i < Tn;
  float m_run = -INFINITY, z_part = 0.f, bpend = 0.f, sprev = 0.f;
  float acc[DQ];
#pragma unroll
  for (int x = 0; x < DQ; ++x) acc[x] = 0.f;

  const int last_row = min(q0 + BQ, Tn) - 1;
  const int nkt = last_row / BK + 1;
  const int ty = tid >> 4, tx = tid & 15;

  for (int kt = 0; kt < nkt; ++kt) {
    const int j0 = kt * BK;
    __syncthreads();
    for (int idx = tid; idx < BK * DP; idx += NT) {
      const int c = idx / DP, d = idx % DP;
      const int key = j0 + c, vkey = j0 - 1 + c;
      Ks[c * L::LD + d] = (key < Tn && d < D) ? to_f32(k[base + (size_t)key * D + d]) : 0.f;
      Vs[c * DP + d] = (vkey >= 0 && vkey < Tn && d < D) ? to_f32(v[base + (size_t)vkey * D + d]) : 0.f;
    }
    __syncthreads();
    {
      float sacc[4][4];
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int b = 0; b < 4; ++b) sacc[a][b] = 0.f;
#pragma unroll 4
      for (int d = 0; d < DP; ++d) {
        float qa[4], kb[4];
#pragma unroll
        for (int a = 0; a < 4; ++a) qa[a] = Qs[(ty + 16 * a) * L::LD + d];
#pragma unroll
        for (int b = 0; b < 4; ++b) kb[b] = Ks[(tx + 16 * b) * L::LD + d];
#pragma unroll
        for (int a = 0; a < 4; ++a)
#pragma unroll
          for (int b = 0; b < 4; ++b) sacc[a][b] = fmaf(qa[a], kb[b], sacc[a][b]);
      }
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int b = 0; b < 4; ++b) Ss[(ty + 16 * a) * L::SLD + tx + 16 * b] = sacc[a][b] * scale;
    }
    __syncthreads();
    {
      const float* srow = Ss + r * L::SLD;   // srow[c] = score of key j0 + c
      const int nvis = row_ok ? min(max(i - j0 + 1, 0), BK) : 0;
      const int c0 = 16 * quad;
      float tmax = -INFINITY;
#pragma unroll
      for (int x = 0; x < 16; ++x)
        if (c0 + x < nvis) tmax = fmaxf(tmax, srow[c0 + x]);
      tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 1));
      tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 2));
      const float m_new = fmaxf(m_run, tmax);
      const float alpha = (m_new == -INFINITY) ? 1.f : exp_rel(m_run - m_new);
      m_run = m_new;
#pragma unroll
      for (int x = 0; x < DQ; ++x) acc[x] *= alpha;
      z_part *= alpha;
      bpend *= alpha;

      // left endpoint of segment j0+c0: key j0+c0-1
      float sa, ea, bprev;
      if (quad == 0) {
        sa = sprev;
        ea = (j0 >= 1 && nvis > 0) ? exp_rel(sprev - m_new) : 0.f;
        bprev = bpend;
      } else {
        // recompute segment j0+c0-1 (owned by the previous quad) for its right share
        const float s2 = srow[c0 - 2], s1 = srow[c0 - 1];
        const bool ok = (c0 - 1) < nvis;
        const float e2 = ok ? exp_rel(s2 - m_new) : 0.f;
        const float e1 = ok ? exp_rel(s1 - m_new) : 0.f;
        float M0, M1;
        seg_moments01(e2, e1, s1 - s2, M0, M1);
        bprev = ok ? M1 : 0.f;
        sa = s1;
        ea = e1;
      }
#pragma unroll 4
      for (int x = 0; x < 16; ++x) {
        const int c = c0 + x;
        const bool vis = c < nvis;
        const bool seg_ok = vis && (j0 + c) >= 1;
        const float sb = srow[c];
        const float eb = vis ? exp_rel(sb - m_new) : 0.f;
        float A = 0.f, Bv = 0.f;
        if (seg_ok) {
          float M0, M1;
          seg_moments01(ea, eb, sb - sa, M0, M1);
          A = M0 - M1;
          Bv = M1;
          z_part += M0;
        }
        Ps[r * L::PLD + c] = bprev + A;
        bprev = Bv;
        sa = sb;
        ea = eb;
      }
      if (j0 == 0 && quad == 0) sFirst[r] = srow[0];
      if (row_ok && i >= j0 + c0 && i < j0 + c0 + 16) sDiag[r] = srow[i - j0];
      bpend = __shfl_sync(0xffffffffu, bprev, (lane & ~3) | 3);
      sprev = srow[BK - 1];
    }
    __syncthreads();
    // O += P V  (thread: row r, columns d = quad + 4x)
    for (int c = 0; c < BK; ++c) {
      const float p = Ps[r * L::PLD + c];
      const float* vrow = Vs + c * DP + quad;
#pragma unroll
      for (int x = 0; x < DQ; ++x) acc[x] = fmaf(p, vrow[4 * x], acc[x]);
    }
  }

  // epilogue: caps, last pending weight, normalisation
  z_part += __shfl_xor_sync(0xffffffffu, z_part, 1);
  z_part += __shfl_xor_sync(0xffffffffu, z_part, 2);
  if (!row_ok) return;
  const float e0 = exp_rel(sFirst[r] - m_run);
  const float ei = exp_rel(sDiag[r] - m_run);
  const float Z = z_part + 0.5f * e0 + 0.5f * ei;
  const float w0 = 0.5f * e0, wi = bpend + 0.5f * ei;
  const float inv = 1.f / Z;
  const T* v0 = v + base;
  const T* vi = v + base + (size_t)i * D;
  T* orow = o + act_row((size_t)bh * Tn + i, Tn, H, o_bthd) * D;
#pragma unroll
  for (int x = 0; x < DQ; ++x) {
    const int d = quad + 4 * x;
    if (d < D) {
      const float y = (acc[x] + w0 * to_f32(v0[d]) + wi * to_f32(vi[d])) * inv;
      orow[d] = from_f32<T>(y);
      if (o32) o32[base + (size_t)i * D + d] = y;
    }
  }
  if (quad == 0 && stats) {   // stats == nullptr: inference, no backward follows
    stats[2 * ((size_t)bh * Tn + i)] = m_run;
    stats[2 * ((size_t)bh * Tn + i) + 1] = Z;
  }
}

// ---------------------------------------------------------------------------
// backward

template <int DP>
struct BwdSmem {
  static constexpr int LD = DP + 1;
  static constexpr int HK = BK + 2;      // keys j0-1 .. j0+64
  static constexpr int SLD = BK + 3;     // score / dP row over the HK keys (padded)
  static constexpr int PLD = BK + 1;
  static constexpr int kK = 0;
  static constexpr int kV = kK + HK * LD;
  static constexpr int kQ = kV + HK * LD;
  static constexpr int kO = kQ + BQ * LD;
  static constexpr int kS = kO + BQ * LD;
  static constexpr int kDP = kS + BQ * SLD;
  static constexpr int kP = kDP + BQ * SLD;
  static constexpr int kDS = kP + BQ * PLD;
  static constexpr int kM = kDS + BQ * PLD;
  static constexpr int kIZ = kM + BQ;
  static constexpr int kDD = kIZ + BQ;
  static constexpr int kRed = kDD + BQ;
  static constexpr int kFloats = kRed + NT / 32;
  static constexpr size_t bytes = sizeof(float) * kFloats;
};

template <typename T, int DP>
__global__ void __launch_bounds__(NT)
bwd_kernel(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
           const T* __restrict__ dout, const float* __restrict__ log_gain,
           const float* __restrict__ stats, const float* __restrict__ rowdot,
           float* __restrict__ dq_acc, T* __restrict__ dk, T* __restrict__ dv,
           float* __restrict__ gain_part, int BH, int H, int Tn, int D, float inv_sqrt_d, int do_bthd) {
  pdl_wait();
  pdl_launch_dependents();
  using L = BwdSmem<DP>;
  constexpr int DQ = DP / 4;
  extern __shared__ float smem[];
  float* Ks = smem + L::kK;
  float* Vs = smem + L::kV;
  float* Qs = smem + L::kQ;
  float* Os = smem + L::kO;    // dO tile
  float* Ss = smem + L::kS;
  float* DPs = smem + L::kDP;
  float* Ps = smem + L::kP;
  float* DSs = smem + L::kDS;
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
  const float scale = expf(log_gain[h]) * inv_sqrt_d;

  // stationary K and V with one halo key on each side (keys j0-1 .. j0+64)
  for (int idx = tid; idx < L::HK * DP; idx += NT) {
    const int c = idx / DP, d = idx % DP, key = j0 - 1 + c;
    const bool ok = key >= 0 && key < Tn && d < D;
    Ks[c * L::LD + d] = ok ? to_f32(k[base + (size_t)key * D + d]) : 0.f;
    Vs[c * L::LD + d] = ok ? to_f32(v[base + (size_t)key * D + d]) : 0.f;
  }

  const int r = tid >> 2, quad = tid & 3;      // row phase: query row r, keys 16*quad..+15
  const int kc = tid >> 2;                      // dK/dV phase: key kc, columns quad + 4x
  float dk_acc[DQ], dv_acc[DQ];
#pragma unroll
  for (int x = 0; x < DQ; ++x) dk_acc[x] = dv_acc[x] = 0.f;
  float gsum = 0.f;
  const int ty = tid >> 4, tx = tid & 15;

  for (int q0 = j0 - (j0 % BQ); q0 < Tn; q0 += BQ) {
    __syncthreads();
    for (int idx = tid; idx < BQ * DP; idx += NT) {
      const int rr = idx / DP, d = idx % DP, row = q0 + rr;
      const bool ok = row < Tn && d < D;
      Qs[rr * L::LD + d] = ok ? to_f32(q[base + (size_t)row * D + d]) : 0.f;
      Os[rr * L::LD + d] = ok ? to_f32(dout[act_row((size_t)bh * Tn + row, Tn, H, do_bthd) * D + d]) : 0.f;
    }
    if (tid < BQ) {
      const int row = q0 + tid;
      if (row < Tn) {
        const size_t ri = (size_t)bh * Tn + row;
        sM[tid] = stats[2 * ri];
        sIZ[tid] = 1.f / stats[2 * ri + 1];
        sDD[tid] = rowdot[ri];
      } else {
        sM[tid] = 0.f;
        sIZ[tid] = 0.f;
        sDD[tid] = 0.f;
      }
    }
    __syncthreads();
    // S and dP over the 66 keys of the tile + halo: rows ty+16a, halo-key columns tx+16b (b<5)
    {
      float sacc[4][5], pacc[4][5];
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int b = 0; b < 5; ++b) sacc[a][b] = pacc[a][b] = 0.f;
#pragma unroll 2
      for (int d = 0; d < DP; ++d) {
        float qa[4], oa[4], kb[5], vb[5];
#pragma unroll
        for (int a = 0; a < 4; ++a) {
          qa[a] = Qs[(ty + 16 * a) * L::LD + d];
          oa[a] = Os[(ty + 16 * a) * L::LD + d];
        }
#pragma unroll
        for (int b = 0; b < 5; ++b) {
          const int c = min(tx + 16 * b, L::HK - 1);
          kb[b] = Ks[c * L::LD + d];
          vb[b] = Vs[c * L::LD + d];
        }
#pragma unroll
        for (int a = 0; a < 4; ++a)
#pragma unroll
          for (int b = 0; b < 5; ++b) {
            sacc[a][b] = fmaf(qa[a], kb[b], sacc[a][b]);
            pacc[a][b] = fmaf(oa[a], vb[b], pacc[a][b]);
          }
      }
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int b = 0; b < 5; ++b) {
          const int c = tx + 16 * b;
          if (c < L::HK) {
            Ss[(ty + 16 * a) * L::SLD + c] = sacc[a][b] * scale;
            DPs[(ty + 16 * a) * L::SLD + c] = pacc[a][b];
          }
        }
    }
    __syncthreads();
    {
      // srow[x] / prow[x] hold key j0-1+x
      const float* srow = Ss + r * L::SLD;
      const float* prow = DPs + r * L::SLD;
      const int i = q0 + r;
      const bool row_ok = i < Tn;
      const float m = sM[r], iz = sIZ[r], dd = sDD[r];
      const int c0 = 16 * quad;
      // key j visible iff j <= i; x = j - (j0-1)
      auto vis = [&](int x) { return row_ok && (j0 - 1 + x) >= 0 && (j0 - 1 + x) <= i; };
      // segment into key x (left key x-1) is valid iff key x visible and key x >= 1
      float sa = srow[c0];                    // key j0+c0-1
      float ea = vis(c0) ? exp_rel(sa - m) : 0.f;
      float ga = prow[c0] - dd;
      float Rprev = 0.f, Bprev = 0.f;          // right shares of the segment into the current key
      {
        const int x = c0 + 1;                  // key j0+c0
        const float sb = srow[x];
        const bool ok = vis(x) && (j0 - 1 + x) >= 1;
        const float eb = vis(x) ? exp_rel(sb - m) : 0.f;
        const float gb = prow[x] - dd;
        if (ok) {
          float M0, M1, M2;
          seg_moments012(ea, eb, sb - sa, M0, M1, M2);
          const float G = gb - ga;
          Rprev = fmaf(ga, M1, G * M2);
          Bprev = M1;
        }
        sa = sb; ea = eb; ga = gb;
      }
#pragma unroll 2
      for (int xx = 0; xx < 16; ++xx) {
        const int x = c0 + 1 + xx;             // current key (halo index)
        const int key = j0 - 1 + x;
        // segment from key x to key x+1
        const float sb = srow[x + 1];
        const bool okn = vis(x + 1);           // right key visible (and >= 1 automatically)
        const float eb = okn ? exp_rel(sb - m) : 0.f;
        const float gb = prow[x + 1] - dd;
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
        DSs[r * L::PLD + x - 1] = ds * scale;
        Ps[r * L::PLD + x - 1] = p;
        Rprev = Rn; Bprev = Bn;
        sa = sb; ea = eb; ga = gb;
      }
    }
    __syncthreads();
    // dV += P^T dO, dK += (scale dS)^T Q  (thread: key kc, columns quad + 4x)
    for (int rr = 0; rr < BQ; ++rr) {
      const float p = Ps[rr * L::PLD + kc];
      const float g = DSs[rr * L::PLD + kc];
      const float* orow = Os + rr * L::LD + quad;
      const float* qrow = Qs + rr * L::LD + quad;
#pragma unroll
      for (int x = 0; x < DQ; ++x) {
        dv_acc[x] = fmaf(p, orow[4 * x], dv_acc[x]);
        dk_acc[x] = fmaf(g, qrow[4 * x], dk_acc[x]);
      }
    }
    // dQ += (scale dS) K  (thread: row r, columns quad + 4x), fp32 atomics
    {
      float dqa[DQ];
#pragma unroll
      for (int x = 0; x < DQ; ++x) dqa[x] = 0.f;
      for (int c = 0; c < BK; ++c) {
        const float g = DSs[r * L::PLD + c];
        const float* krow = Ks + (c + 1) * L::LD + quad;
#pragma unroll
        for (int x = 0; x < DQ; ++x) dqa[x] = fmaf(g, krow[4 * x], dqa[x]);
      }
      const int row = q0 + r;
      if (row < Tn) {
        float* dst = dq_acc + base + (size_t)row * D;
#pragma unroll
        for (int x = 0; x < DQ; ++x) {
          const int d = quad + 4 * x;
          if (d < D) atomicAdd(dst + d, dqa[x]);
        }
      }
    }
  }

  const int key = j0 + kc;
  if (key < Tn) {
#pragma unroll
    for (int x = 0; x < DQ; ++x) {
      const int d = quad + 4 * x;
      if (d < D) {
        dk[base + (size_t)key * D + d] = from_f32<T>(dk_acc[x]);
        dv[base + (size_t)key * D + d] = from_f32<T>(dv_acc[x]);
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
                              float* __restrict__ dq_acc, size_t rows, unsigned* __restrict__ counter, int Tn,
                              int H) {
  pdl_wait();
  pdl_launch_dependents();
  const size_t gid = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (gid == 0 && counter) *counter = 0u;   // work-item counter of the persistent backward
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
    *reinterpret_cast<float4*>(dq_acc + base) = make_float4(0.f, 0.f, 0.f, 0.f);
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

template <typename T, int DP>
static cudaError_t launch_fwd(const FwdArgs& a) {
  auto kern = fwd_kernel<T, DP>;
  const size_t smem = FwdSmem<DP>::bytes;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const long long BH = a.B * a.H;
  const long long nqt = (a.T + BQ - 1) / BQ;
  return launch_pdl(kern, dim3((unsigned)(BH * nqt)), dim3(NT), smem, a.stream, (const T*)a.q, (const T*)a.k,
                    (const T*)a.v, a.log_gain, (T*)a.o, a.o_f32, a.row_stats, (int)BH, (int)a.H, (int)a.T,
                    (int)a.D, a.inv_sqrt_d, a.o_bthd);
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
  return launch_pdl(kern, dim3((unsigned)(BH * nkt)), dim3(NT), smem, a.stream, (const T*)a.q, (const T*)a.k,
                    (const T*)a.v, (const T*)a.d_o, a.log_gain, a.row_stats, (const float*)w.rowdot, w.dq_acc,
                    (T*)a.dk, (T*)a.dv, a.dlog_gain ? w.gain_part : nullptr, (int)BH, (int)a.H, (int)a.T,
                    (int)a.D, a.inv_sqrt_d, a.act_bthd);
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
static cudaError_t prep_dtype(const BwdArgs& a, float* rowdot, float* dq_acc, unsigned* counter) {
  const size_t rows = (size_t)a.B * a.H * a.T;
  const uintptr_t oal = reinterpret_cast<uintptr_t>(a.o_f32 ? (const void*)a.o_f32 : a.o);
  const bool vec = a.D == 64 && (reinterpret_cast<uintptr_t>(a.d_o) & (4 * sizeof(T) - 1)) == 0 &&
                   (a.o_f32 || sizeof(T) == 4 ? (oal & 15) == 0 : true);
  if (!vec) {
    cudaError_t e = rowdot_dtype<T>(a, rowdot);
    if (e != cudaSuccess) return e;
    if (counter) {
      e = cudaMemsetAsync(counter, 0, sizeof(unsigned), a.stream);
      if (e != cudaSuccess) return e;
    }
    return cudaMemsetAsync(dq_acc, 0, rows * a.D * sizeof(float), a.stream);
  }
  const unsigned blocks = (unsigned)((rows * 16 + 255) / 256);
  const dim3 g(blocks), b(256);
  if (a.o_f32) {
    auto k = a.act_bthd ? prep64_kernel<float, T, false, true> : prep64_kernel<float, T, false, false>;
    return launch_pdl(k, g, b, 0, a.stream, (const float*)a.o_f32, (const T*)a.d_o, rowdot, dq_acc, rows, counter,
                      (int)a.T, (int)a.H);
  }
  auto k = a.act_bthd ? prep64_kernel<T, T, true, true> : prep64_kernel<T, T, false, false>;
  return launch_pdl(k, g, b, 0, a.stream, (const T*)a.o, (const T*)a.d_o, rowdot, dq_acc, rows, counter, (int)a.T,
                    (int)a.H);
}

cudaError_t launch_prep(const BwdArgs& a, float* rowdot, float* dq_acc, unsigned* counter) {
  switch (a.dtype) {
    case 0: return prep_dtype<float>(a, rowdot, dq_acc, counter);
    case 1: return prep_dtype<__nv_bfloat16>(a, rowdot, dq_acc, counter);
    default: return prep_dtype<__half>(a, rowdot, dq_acc, counter);
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
