// ca_sm100.cu -- sm_100a tensor-core Continuum Attention kernels (bf16 / f16,
// head dim 64): TMA-staged Q/K/V tiles, tcgen05.mma with TMEM accumulators.
//
// Forward, one CTA per 128-row query tile (two CTAs per SM), keys in half-tiles
// of 64 that rotate through three 64-column S/P regions of TMEM:
//   warp 4 is the producer (the whole warp runs converged; lane 0 issues): TMA
//     loads of Q (once) and of K / V' half-tiles into a 4-stage ring, and the
//     tcgen05.mma issue:
//       S_h  = Q K_h^T              128x64 fp32 in region h % 3
//       O   += P_hi,h V'_h + P_lo,h V'_h   128x64 fp32 in TMEM columns [192,256)
//     where V'_h is the V half-tile staged one row early (keys 64h-1 .. 64h+62)
//     and P_h is written by the math warps over the same columns as S_h (each
//     16-key chunk's 16 columns become 8 columns of bf16 hi pairs and 8 of lo
//     pairs).  S_{h+3} is issued right after P V'_h, into the region P_h leaves,
//     so S of the next two half-tiles is ready while the math warps work.
//   warps 0-3 (thread = query row = TMEM lane) load their S row, keep an online
//     row max per half-tile (rescaling O only when the max grows by more than 8
//     nats, after the previous P V' has landed), form the segment moments, and
//     store P split into bf16 hi + lo parts, so the P V product keeps ~16
//     significant bits of every weight.
// P column c of the half-tile starting at key kb holds the weight of key kb-1+c:
//   P[c] = B_{kb+c-1} + A_{kb+c} (+ half caps on key 0 and key i),
// with A_k = M0-M1 and B_k = M1 of segment k (key k-1 -> key k); B of the last
// key of a half-tile is carried to the next one, and a weight still pending
// after the last half-tile (query i on its last key) is added in the epilogue,
// which writes O and the fp32 O through shared-memory staging and TMA stores.
// Replaces the reference's per-query-tile chain bmm(QK^T) -> scale ->
// ca_forward_half_kernel -> bmm(W V) (cuda/continuum_attention.py:670-690).
//
// Every mbarrier wait is bounded (2 s); on expiry the kernel records
// CA_ERR_DEVICE_TIMEOUT in g_device_status, stops issuing work, waits (bounded)
// for its own in-flight copies and MMAs, frees its TMEM and returns.
#include <cuda.h>

#include <algorithm>
#include <cstdio>
#include <cstdlib>

#include "ca_common.cuh"
#include "ca_internal.h"
#include "ca_sm100_ptx.cuh"

namespace ca {
namespace sm100 {

namespace fwd {

constexpr int BM = 128;            // query rows per CTA (= TMEM lanes)
constexpr int HB = 64;             // keys per half-tile, the pipeline unit
constexpr int HD = 64;             // head dim
constexpr int NREG = 3;            // rotating S/P regions of 64 TMEM columns
constexpr int KSTAGES = 4;         // K / V' half-tile ring
constexpr int NUM_THREADS = 160;   // 4 math warps + 1 producer warp
constexpr uint32_t Q_BYTES = BM * HD * 2;      // 16 KB
constexpr uint32_t HALF_BYTES = HB * HD * 2;   // 8 KB
constexpr uint32_t TMEM_COLS = 256;
constexpr uint32_t TMEM_O = 192;   // O accumulator: columns [192,256); region r: [64r, 64r+64)
constexpr float kRescaleNats = 8.0f;

struct __align__(1024) Smem {
  uint8_t q[Q_BYTES];
  uint8_t k[KSTAGES][HALF_BYTES];
  uint8_t v[KSTAGES][HALF_BYTES];
  uint64_t bar_q;
  uint64_t bar_k[KSTAGES];
  uint64_t bar_v[KSTAGES];
  uint64_t bar_kv_free[KSTAGES];   // the half-tile's P V' has completed (its S long before)
  uint64_t bar_s_full[NREG];       // S of a half-tile is in region r
  uint64_t bar_p_ready[NREG];      // P of the half-tile in region r is in TMEM
  uint64_t bar_pv_done[2];         // half-tile h's P V' (and every MMA before it) has
                                   // completed: barrier h & 1, phase h >> 1
  uint64_t bar_o_done;
  uint32_t tmem_base;
  int abort_flag;
};

constexpr size_t kSmemBytes = sizeof(Smem) + 1024;  // + alignment slack

// S = Q K_h^T for one half-tile: M = 128 queries, N = 64 keys, K = 64 (4 MMAs)
// (descriptors: the base one plus byte offset >> 4 in the start-address field, which
// never carries since shared addresses stay below 256 KB)
__device__ __forceinline__ void issue_s(uint32_t q_saddr, uint32_t k_saddr, uint32_t d_tmem, uint32_t idesc) {
  const uint64_t a = sdesc_sw128(q_saddr, 16, 1024), b = sdesc_sw128(k_saddr, 16, 1024);
#pragma unroll
  for (int kk = 0; kk < HD / 16; ++kk) mma_ss(d_tmem, a + 2 * kk, b + 2 * kk, idesc, kk > 0 ? 1u : 0u);
}

// O += P V'_h over the half-tile's 64 keys: hi and lo parts of P, 16 keys per MMA,
// A from TMEM (16 columns per 16 keys: 8 of hi pairs, then 8 of lo pairs)
__device__ __forceinline__ void issue_pv(uint32_t o_tmem, uint32_t p_tmem, uint32_t v_saddr, uint32_t idesc,
                                         bool accumulate) {
  const uint64_t b = sdesc_sw128(v_saddr, 16384, 1024);   // V': MN-major, 2048 bytes per 16 keys
#pragma unroll
  for (int part = 0; part < 2; ++part) {
#pragma unroll
    for (int kk = 0; kk < HB / 16; ++kk) {
      const uint32_t acc = (accumulate || part > 0 || kk > 0) ? 1u : 0u;
      mma_ts(o_tmem, p_tmem + 16 * kk + 8 * part, b + 128 * kk, idesc, acc);
    }
  }
}

// Producer schedule over half-tiles h = 0 .. nh-1 (region h % 3, ring stage h % 4):
//   S_0, S_1, S_2 up front; then per h: wait P_h -> P V'_h (commit pv_done and
//   kv_free) -> S_{h+3} into the region P_h just left (tcgen05 MMAs run in issue
//   order, so it overwrites P_h only after P V'_h has read it) -> refill the ring
//   stage of h with half-tile h+4 once P V'_h has completed.  The math warps thus
//   find S of their next half-tile already computed.
// K half-tile h into ring stage st: rows h*64 .. h*64+63 of head-sequence bh, through
// the permuted 5-D view (kPerm: (D, s, j, chunk, bh), see fwd_chunk_perm) or the 3-D one.
template <bool kPerm>
__device__ __forceinline__ void load_k_half(void* dst, const CUtensorMap* tk, uint64_t* bar, int h, int bh) {
  if (kPerm) tma_load_5d(dst, tk, bar, 0, 0, 0, h * (HB / 16), bh);
  else tma_load_3d(dst, tk, bar, 0, h * HB, bh);
}

template <bool kBF16, bool kPerm>
__device__ void producer(Smem& sm, const CUtensorMap* tq, const CUtensorMap* tk, const CUtensorMap* tv, int bh,
                         int q0, int nh, uint32_t tmem) {
  volatile int* ab = &sm.abort_flag;
  const uint32_t id_s = make_idesc(BM, HB, kBF16, false);
  const uint32_t id_o = make_idesc(BM, HD, kBF16, true);
  bool k_pending[KSTAGES], v_pending[KSTAGES];
  uint32_t k_phase[KSTAGES], v_phase[KSTAGES];
  for (int s2 = 0; s2 < KSTAGES; ++s2) {
    k_pending[s2] = v_pending[s2] = false;
    k_phase[s2] = v_phase[s2] = 0;
  }
  bool q_pending = true;

  mbar_arrive_expect_tx(&sm.bar_q, Q_BYTES);
  tma_load_3d(sm.q, tq, &sm.bar_q, 0, q0, bh);
  for (int t = 0; t < KSTAGES && t < nh; ++t) {
    mbar_arrive_expect_tx(&sm.bar_k[t], HALF_BYTES);
    load_k_half<kPerm>(sm.k[t], tk, &sm.bar_k[t], t, bh);
    mbar_arrive_expect_tx(&sm.bar_v[t], HALF_BYTES);
    tma_load_3d(sm.v[t], tv, &sm.bar_v[t], 0, t * HB - 1, bh);
    k_pending[t] = v_pending[t] = true;
  }
  const uint32_t q_sa = smem_u32(sm.q), o_tmem = tmem + TMEM_O;
  bool good = mbar_wait_warp(&sm.bar_q, 0, ab);
  if (good) q_pending = false;
  for (int h = 0; good && h < NREG && h < nh; ++h) {
    good = mbar_wait_warp(&sm.bar_k[h], 0, ab);
    if (!good) break;
    k_pending[h] = false;
    k_phase[h] ^= 1;
    tc_fence_after();
    issue_s(q_sa, smem_u32(sm.k[h]), tmem + HB * h, id_s);
    mma_commit(&sm.bar_s_full[h]);
  }
  for (int h = 0; good && h < nh; ++h) {
    const int r = h % NREG, st = h % KSTAGES;
    if (!mbar_wait_warp(&sm.bar_p_ready[r], (h / NREG) & 1, ab)) break;
    if (!mbar_wait_warp(&sm.bar_v[st], v_phase[st], ab)) break;
    v_pending[st] = false;
    v_phase[st] ^= 1;
    tc_fence_after();
    issue_pv(o_tmem, tmem + HB * r, smem_u32(sm.v[st]), id_o, h > 0);
    mma_commit(&sm.bar_pv_done[h & 1]);
    mma_commit(&sm.bar_kv_free[st]);
    const int hn = h + NREG;
    if (hn < nh) {
      const int sn = hn % KSTAGES;
      if (!mbar_wait_warp(&sm.bar_k[sn], k_phase[sn], ab)) break;
      k_pending[sn] = false;
      k_phase[sn] ^= 1;
      tc_fence_after();
      issue_s(q_sa, smem_u32(sm.k[sn]), tmem + HB * r, id_s);
      mma_commit(&sm.bar_s_full[r]);
    }
    const int hr = h + KSTAGES;
    if (hr < nh) {
      if (!mbar_wait_warp(&sm.bar_kv_free[st], (h / KSTAGES) & 1, ab)) break;
      mbar_arrive_expect_tx(&sm.bar_k[st], HALF_BYTES);
      load_k_half<kPerm>(sm.k[st], tk, &sm.bar_k[st], hr, bh);
      mbar_arrive_expect_tx(&sm.bar_v[st], HALF_BYTES);
      tma_load_3d(sm.v[st], tv, &sm.bar_v[st], 0, hr * HB - 1, bh);
      k_pending[st] = v_pending[st] = true;
    }
  }
  // completion of every MMA issued so far (also the epilogue's "O ready" signal)
  mma_commit(&sm.bar_o_done);
  // drain: in-flight TMA copies must land before the CTA's shared memory goes away
  int dummy_abort = 0;
  volatile int* nab = &dummy_abort;
  if (q_pending) mbar_wait_warp(&sm.bar_q, 0, nab);
  for (int s2 = 0; s2 < KSTAGES; ++s2) {
    if (k_pending[s2]) mbar_wait_warp(&sm.bar_k[s2], k_phase[s2], nab);
    if (v_pending[s2]) mbar_wait_warp(&sm.bar_v[s2], v_phase[s2], nab);
  }
  mbar_wait_warp(&sm.bar_o_done, 0, nab);
}

// P for 16 keys of one row: keys j0-1+c for c = 16*ch .. 16*ch+15 (P column c of
// the half-tile starting at key j0); nvis = number of visible S columns of the row.
// kEdge: masking and caps (first half-tile, diagonal); interior chunks use fwd_chunk_fast.
template <bool kBF16, bool kEdge>
__device__ __forceinline__ void fwd_chunk(const uint32_t (&cur)[16], int ch, float scale, float m2, int nvis, int j0,
                                          int i, float& sa, float& ea, float& bprev, float& z, uint32_t t_p) {
  uint32_t hi[8], lo[8];
#pragma unroll
  for (int x = 0; x < 16; x += 2) {
    float pv[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int c = 16 * ch + x + u;
      const float sb = __uint_as_float(cur[x + u]) * scale;
      float M0, M1, eb;
      if (kEdge) {
        const bool vis = c < nvis;
        eb = vis ? ex2_approx(fmaf(sb, kLog2e, -m2)) : 0.f;
        seg_moments01_sel(ea, eb, sb - sa, M0, M1);
        const bool seg_ok = vis && (j0 + c) >= 1;
        M0 = seg_ok ? M0 : 0.f;
        M1 = seg_ok ? M1 : 0.f;
      } else {
        eb = ex2_approx(fmaf(sb, kLog2e, -m2));
        seg_moments01_sel(ea, eb, sb - sa, M0, M1);
      }
      float p = bprev + (M0 - M1);
      z += M0;
      if (kEdge) {
        // column 0 holds key j0-1: with 64-key half-tiles that is row i's own key
        // for i = q0+63 (for j0 = 0 it is key -1, and ea = 0 there)
        const int key = j0 - 1 + c;
        // a select, not a product: ea of a key beyond row i may have overflowed
        const float nc = (key == 0 ? 1.f : 0.f) + (key == i ? 1.f : 0.f);
        const float cap = nc > 0.f ? 0.5f * nc * ea : 0.f;
        p += cap;
        z += cap;
      }
      pv[u] = p;
      bprev = M1;
      sa = sb;
      ea = eb;
    }
    const uint32_t h2 = kBF16 ? pack_bf16x2(pv[0], pv[1]) : pack_f16x2(pv[0], pv[1]);
    float h0, h1;
    if (kBF16) {
      h0 = __uint_as_float(h2 << 16);
      h1 = __uint_as_float(h2 & 0xffff0000u);
    } else {
      const __half2 hh = *reinterpret_cast<const __half2*>(&h2);
      h0 = __low2float(hh);
      h1 = __high2float(hh);
    }
    hi[x / 2] = h2;
    lo[x / 2] = kBF16 ? pack_bf16x2(pv[0] - h0, pv[1] - h1) : pack_f16x2(pv[0] - h0, pv[1] - h1);
  }
  tmem_st8(t_p + 16 * ch, hi);       // P hi and lo of these 16 keys replace their own S columns
  tmem_st8(t_p + 16 * ch + 8, lo);
}

// Interior chunk (every key visible, no caps) in packed fp32 pairs: lanes x/y
// are the adjacent keys c = 16*ch + 2x, 2x+1.  Quantities that pair a key with
// its left neighbour (score difference, Ea - Eb, Ea * series) use scalar ops, so
// no register shuffling is needed.  Working with nd = -(b - a) keeps every
// result bit-identical to seg_moments01_sel: rcp(nd) = -1/d exactly, and the
// series constants carry the alternating signs.
template <bool kBF16>
__device__ __forceinline__ void fwd_chunk_fast(const uint32_t (&cur)[16], int ch, float2 scale2, float2 nm2,
                                               float& sa, float& ea, float& bprev, float2& z2, uint32_t t_p) {
  const float2 l2e = splat2(kLog2e), neg1 = splat2(-1.f);
  uint32_t hi[8], lo[8];
#pragma unroll
  for (int x = 0; x < 8; ++x) {
    const float2 raw = make_float2(__uint_as_float(cur[2 * x]), __uint_as_float(cur[2 * x + 1]));
    const float2 sb = mul2(raw, scale2);
    const float2 arg = fma2(sb, l2e, nm2);
    const float2 eb = make_float2(ex2_approx(arg.x), ex2_approx(arg.y));
    const float2 nd = make_float2(sa - sb.x, sb.x - sb.y);
    const float2 rn = make_float2(rcp_approx(nd.x), rcp_approx(nd.y));
    const float2 m0c = mul2(make_float2(ea - eb.x, eb.x - eb.y), rn);
    const float2 m1c = mul2(fma2(eb, neg1, m0c), rn);
    float2 ps = fma2(splat2(-1.f / 30.f), nd, splat2(1.f / 8.f));
    ps = fma2(ps, nd, splat2(-1.f / 3.f));
    ps = fma2(ps, nd, splat2(1.f / 2.f));
    float2 M1;
    M1.x = fabsf(nd.x) < kSeriesMaxFwd ? ea * ps.x : m1c.x;
    M1.y = fabsf(nd.y) < kSeriesMaxFwd ? eb.x * ps.y : m1c.y;
    const float2 M0 = fma2(nd, M1, eb);
    const float2 A = fma2(M1, neg1, M0);
    const float pv0 = bprev + A.x, pv1 = M1.x + A.y;
    z2 = add2(z2, M0);
    bprev = M1.y;
    sa = sb.y;
    ea = eb.y;
    if (kBF16) {
      // hi = the upper 16 bits of each fp32 weight (a bf16 by truncation, one byte
      // permute for the pair), lo = the exact fp32 remainder rounded to bf16: the
      // pair still carries ~16 significant bits
      const uint32_t u0 = __float_as_uint(pv0), u1 = __float_as_uint(pv1);
      hi[x] = __byte_perm(u0, u1, 0x7632);
      const float2 r = fma2(make_float2(__uint_as_float(u0 & 0xffff0000u), __uint_as_float(u1 & 0xffff0000u)),
                            neg1, make_float2(pv0, pv1));
      lo[x] = pack_bf16x2(r.x, r.y);
    } else {
      const uint32_t h2 = pack_f16x2(pv0, pv1);
      const __half2 hh = *reinterpret_cast<const __half2*>(&h2);
      hi[x] = h2;
      lo[x] = pack_f16x2(pv0 - __low2float(hh), pv1 - __high2float(hh));
    }
  }
  tmem_st8(t_p + 16 * ch, hi);       // P hi and lo of these 16 keys replace their own S columns
  tmem_st8(t_p + 16 * ch + 8, lo);
}

// A chunk past every row's diagonal: all weights are zero.
__device__ __forceinline__ void fwd_chunk_zero(int ch, float& ea, float& bprev, uint32_t t_p) {
  uint32_t zz[8];
#pragma unroll
  for (int x = 0; x < 8; ++x) zz[x] = 0u;
  tmem_st8(t_p + 16 * ch, zz);
  tmem_st8(t_p + 16 * ch + 8, zz);
  ea = 0.f;
  bprev = 0.f;
}

// Which path chunk ch (keys kb-1+16ch .. kb+14+16ch) of half-tile kb takes for
// this warp's rows i = q0+32w .. q0+32w+31: 0 = all zero, 1 = interior, 2 = edge
// (masking and caps).  Outside the two diagonal half-tiles every key is visible.
// On them, every segment of the chunk is visible to all the warp's rows, with no
// cap, when kb+16ch+15 <= q0+32w; a row's last nonzero P column holds its own key
// (half cap), so the chunk is zero for every row when kb+16ch-1 > q0+32w+31.
// Chunk 0 of half-tile 0 holds key 0 (cap) and the empty segment before it.
__device__ __forceinline__ int fwd_chunk_kind(int ch, int kb, int q0, int warp, bool diag) {
  if (kb == 0 && ch == 0) return 2;
  if (!diag) return 1;
  if (kb + 16 * ch + 15 <= q0 + 32 * warp) return 1;
  if (kb + 16 * ch - 1 > q0 + 32 * warp + 31) return 0;
  return 2;
}

// ---- permuted-key form (T a multiple of 16) ----
// K half-tiles are staged through a 5-D view of K that puts key kc+j+8s of every
// 16-key chunk (kc = first key of the chunk) in shared-memory row 2j+s.  S column
// 2j+s of the chunk then holds key kc+j+8s, so the register pair (2j, 2j+1) of the
// chunk's sixteen TMEM columns is the key pair (j, j+8), and the left neighbours
// (j-1, j+7) of pair j are pair j-1 (pair 0's are the previous chunk's last key and
// key 7).  Every quantity that pairs a key with its left neighbour -- the score
// difference, Ea - Eb, Ea * series, B_{k-1} + A_k -- is then one packed f32x2
// operation for two keys.  P goes back to TMEM in natural key order (hi/lo bf16
// pairs), so V' is staged unpermuted as before.
//
// 16 keys of one row, keys kc..kc+15 in permuted order in raw[0..15]; output
// slot t = weight of key kc-1+t (pair j: slots j and j+8).  On entry (sa, ea,
// bprev) are the scaled score, exponential and right share B of key kc-1.
// kEdge: keys beyond row i are masked (their moments and caps select to zero, so
// an exponential that overflowed never reaches a result), segment k counts only
// when 1 <= k <= i, and key 0 and key i get half caps.
template <bool kBF16, bool kEdge>
__device__ __forceinline__ void fwd_chunk_perm(const uint32_t* raw, float2 scale2, float2 nm2, int kc, int i,
                                               float& sa, float& ea, float& bprev, float2& z2, uint32_t t_p) {
  const float2 l2e = splat2(kLog2e);
  float2 sv[8], ev[8], nd[8], rn[8], ps[8];
#pragma unroll
  for (int j = 0; j < 8; ++j)
    sv[j] = mul2(make_float2(__uint_as_float(raw[2 * j]), __uint_as_float(raw[2 * j + 1])), scale2);
  // the special-function work (two exponentials, two reciprocals per pair) interleaved
  // with the series polynomial, which needs only the score differences
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float2 arg = fma2(sv[j], l2e, nm2);
    nd[j] = sub2(j ? sv[j - 1] : make_float2(sa, sv[7].x), sv[j]);        // a - b = -d
    ev[j] = make_float2(ex2_approx(arg.x), ex2_approx(arg.y));
    rn[j] = make_float2(rcp_approx(nd[j].x), rcp_approx(nd[j].y));        // -1/d
    float2 p = fma2(splat2(-1.f / 30.f), nd[j], splat2(1.f / 8.f));      // J1 series in -nd
    p = fma2(p, nd[j], splat2(-1.f / 3.f));
    ps[j] = fma2(p, nd[j], splat2(1.f / 2.f));
  }
  float2 M1[8], W[8], za = splat2(0.f), zb = splat2(0.f);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float2 eL = j ? ev[j - 1] : make_float2(ea, ev[7].x);
    const float2 m0c = mul2(sub2(eL, ev[j]), rn[j]);                     // (Eb - Ea) / d
    const float2 m1c = mul2(sub2(m0c, ev[j]), rn[j]);                    // (Eb - M0) / d
    float2 m1 = make_float2(sel_series(m1c.x, nd[j].x, eL.x, ps[j].x, kSeriesMaxFwd),
                            sel_series(m1c.y, nd[j].y, eL.y, ps[j].y, kSeriesMaxFwd));
    float2 m0 = fma2(nd[j], m1, ev[j]);                                   // Eb - d M1
    if (kEdge) {
      const int kx = kc + j, ky = kc + j + 8;                            // right keys of the two segments
      const bool okx = kx >= 1 && kx <= i, oky = ky <= i;
      m1 = make_float2(okx ? m1.x : 0.f, oky ? m1.y : 0.f);
      m0 = make_float2(okx ? m0.x : 0.f, oky ? m0.y : 0.f);
    }
    M1[j] = m1;
    float2 w = sub2(m0, m1);                                             // A of the segment
    if (j & 1) zb = add2(zb, m0);
    else za = add2(za, m0);
    if (kEdge) {
      // slots j, j+8 hold keys kc-1+j, kc+7+j: half caps on key 0 and key i
      const int wx = kc - 1 + j, wy = kc + 7 + j;
      const float nx = (wx == 0 ? 1.f : 0.f) + (wx == i ? 1.f : 0.f);
      const float ny = (wy == i ? 1.f : 0.f);
      const float2 cap = make_float2(nx > 0.f ? 0.5f * nx * eL.x : 0.f, ny > 0.f ? 0.5f * eL.y : 0.f);
      w = add2(w, cap);
      za = add2(za, cap);
    }
    W[j] = w;
  }
  z2 = add2(z2, add2(za, zb));
#pragma unroll
  for (int j = 0; j < 8; ++j) W[j] = add2(W[j], j ? M1[j - 1] : make_float2(bprev, M1[7].x));
  bprev = M1[7].y;
  sa = sv[7].y;
  ea = ev[7].y;
  // natural order: TMEM column m of each half holds slots (2m, 2m+1)
  uint32_t hi[8], lo[8];
  if (kBF16) {
    // hi = the upper 16 bits of each weight (bf16 by truncation), lo = the exact fp32
    // remainder rounded to bf16: ~16 significant bits per weight
    float2 rz[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float2 tr = make_float2(__uint_as_float(__float_as_uint(W[j].x) & 0xffff0000u),
                                    __uint_as_float(__float_as_uint(W[j].y) & 0xffff0000u));
      rz[j] = sub2(W[j], tr);
    }
#pragma unroll
    for (int m = 0; m < 8; ++m) {
      const float a = m < 4 ? W[2 * m].x : W[2 * m - 8].y, b = m < 4 ? W[2 * m + 1].x : W[2 * m - 7].y;
      const float ra = m < 4 ? rz[2 * m].x : rz[2 * m - 8].y, rb = m < 4 ? rz[2 * m + 1].x : rz[2 * m - 7].y;
      hi[m] = __byte_perm(__float_as_uint(a), __float_as_uint(b), 0x7632);
      lo[m] = pack_bf16x2(ra, rb);
    }
  } else {
#pragma unroll
    for (int m = 0; m < 8; ++m) {
      const float a = m < 4 ? W[2 * m].x : W[2 * m - 8].y, b = m < 4 ? W[2 * m + 1].x : W[2 * m - 7].y;
      const uint32_t h2 = pack_f16x2(a, b);
      const __half2 hh = *reinterpret_cast<const __half2*>(&h2);
      hi[m] = h2;
      lo[m] = pack_f16x2(a - __low2float(hh), b - __high2float(hh));
    }
  }
  tmem_st8(t_p, hi);
  tmem_st8(t_p + 8, lo);
}

// Half-tile row max over the visible keys of 64 raw scores in permuted order
// (column 16c+2j+s = key kb+16c+j+8s): a tree of three-input maxima.
template <bool kDiag>
__device__ __forceinline__ float perm_max64(const uint32_t (&a)[32], const uint32_t (&b)[32], int kb, int i) {
  float v[64];
#pragma unroll
  for (int x = 0; x < 64; ++x) {
    const float f = __uint_as_float(x < 32 ? a[x] : b[x - 32]);
    if (kDiag) {
      const int key = kb + 16 * (x >> 4) + ((x & 15) >> 1) + 8 * (x & 1);
      v[x] = key <= i ? f : -INFINITY;
    } else {
      v[x] = f;
    }
  }
  float m[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    m[k] = max3f(v[8 * k], v[8 * k + 1], v[8 * k + 2]);
    m[k] = max3f(m[k], v[8 * k + 3], v[8 * k + 4]);
    m[k] = max3f(m[k], v[8 * k + 5], v[8 * k + 6]);
    m[k] = fmaxf(m[k], v[8 * k + 7]);
  }
  return max3f(max3f(m[0], m[1], m[2]), max3f(m[3], m[4], m[5]), fmaxf(m[6], m[7]));
}

// The epilogue's output rows leave through shared memory and TMA stores: each math
// thread writes its row of O (dtype) and of the fp32 O into the K/V' ring (free once
// the last P V' has completed), 128-byte rows with the 128-byte swizzle (16-byte chunk
// c of row r at chunk c ^ (r & 7), so the 32 rows of a warp hit distinct banks); after
// the math warps sync, thread 0 stores the tiles with whole-row writes (rows past T are
// not written) and waits for them.  O goes to v[0..1] (128 rows x 128 bytes), the fp32
// O to k[0..3] as two 32-column halves.  Scattered per-thread 16-byte stores of the same
// rows cost one L1 tag lookup per row per instruction.
template <bool kBF16>
__device__ __forceinline__ void store_out_rows(Smem& sm, const float (&acc)[HD], float inv, int r, bool has32,
                                               const CUtensorMap* tm_o, const CUtensorMap* tm_o32, int bh, int H,
                                               int q0, int o_bthd) {
  uint8_t* const orow = &sm.v[0][0] + (uint32_t)r * 128;
#pragma unroll
  for (int c = 0; c < HD / 8; ++c) {
    uint32_t w[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const float a0 = acc[8 * c + 2 * u] * inv, a1 = acc[8 * c + 2 * u + 1] * inv;
      w[u] = kBF16 ? pack_bf16x2(a0, a1) : pack_f16x2(a0, a1);
    }
    *reinterpret_cast<uint4*>(orow + ((c ^ (r & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
  }
  if (has32) {
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      uint8_t* const row32 = &sm.k[0][0] + hf * (BM * 128) + (uint32_t)r * 128;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const int d = 32 * hf + 4 * c;
        *reinterpret_cast<float4*>(row32 + ((c ^ (r & 7)) << 4)) =
            make_float4(acc[d] * inv, acc[d + 1] * inv, acc[d + 2] * inv, acc[d + 3] * inv);
      }
    }
  }
  fence_proxy_async_smem();
  named_bar_sync(1, BM);
  if (threadIdx.x == 0 && !sm.abort_flag) {
    if (o_bthd) tma_store_4d(tm_o, &sm.v[0][0], 0, bh % H, q0, bh / H);
    else tma_store_3d(tm_o, &sm.v[0][0], 0, q0, bh);
    if (has32) {
      tma_store_3d(tm_o32, &sm.k[0][0], 0, q0, bh);
      tma_store_3d(tm_o32, &sm.k[0][0] + BM * 128, 32, q0, bh);
    }
    bulk_commit_group();
    bulk_wait_group0();
  }
}

template <bool kBF16>
__device__ void math_warps_perm(Smem& sm, const void* vptr, const float* log_gain, const CUtensorMap* tm_o,
                                const CUtensorMap* tm_o32, float* o32, float* stats, int bh, int h, int Tn, int q0, int nh, uint32_t tmem, float inv_sqrt_d,
                                int H, int o_bthd) {
  volatile int* ab = &sm.abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = warp * 32 + lane;
  const int i = q0 + r;
  const bool row_ok = i < Tn;
  const float scale = expf(log_gain[h]) * inv_sqrt_d;
  const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
  const uint32_t tO = tmem + TMEM_O + lane_base;

  float m_used = -INFINITY, bpend = 0.f, sprev = 0.f;
  float2 z2 = splat2(0.f);
  const float2 scale2 = splat2(scale);
  bool ok = true;
  for (int hh = 0; hh < nh; ++hh) {
    const int reg = hh % NREG;
    const bool got = mbar_wait(&sm.bar_s_full[reg], (hh / NREG) & 1, ab);
    if (!__all_sync(0xffffffffu, got)) { ok = false; break; }
    tc_fence_after();
    const uint32_t tS = tmem + HB * reg + lane_base;
    const int kb = hh * HB;
    const bool diag = hh >= nh - 2;
    float tmax;
    {
      uint32_t sa_[32], sb_[32];
      tmem_ld32(tS, sa_);
      tmem_ld32(tS + 32, sb_);
      tmem_ld_wait();
      tmem_reg_fence(sa_);
      tmem_reg_fence(sb_);
      tmax = diag ? perm_max64<true>(sa_, sb_, kb, i) : perm_max64<false>(sa_, sb_, kb, i);
    }
    tmax *= scale;
    const bool need = tmax > m_used + kRescaleNats;
    if (hh == 0) {
      m_used = tmax;
    } else if (__any_sync(0xffffffffu, need)) {
      // as in math_warps: wait for the last P V' before touching O
      const bool got2 = mbar_wait(&sm.bar_pv_done[(hh - 1) & 1], ((hh - 1) >> 1) & 1, ab);
      if (!__all_sync(0xffffffffu, got2)) { ok = false; break; }
      tc_fence_after();
      const float m_new = need ? tmax : m_used;
      const float alpha = exp_rel(m_used - m_new);
      z2 = mul2(z2, splat2(alpha));
      bpend *= alpha;
      m_used = m_new;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t ov[32];
        tmem_ld32(tO + 32 * half, ov);
        tmem_ld_wait();
        tmem_reg_fence(ov);
#pragma unroll
        for (int x = 0; x < 32; ++x) ov[x] = __float_as_uint(__uint_as_float(ov[x]) * alpha);
        tmem_st32(tO + 32 * half, ov);
      }
      tmem_st_wait();
    }
    const float m2 = m_used * kLog2e;
    const float2 nm2 = splat2(-m2);
    float sa = sprev;
    float ea = (kb > 0) ? ex2_approx(fmaf(sprev, kLog2e, -m2)) : 0.f;
    float bprev = bpend;
    // P, 16 keys at a time; the next chunk's TMEM load overlaps this chunk's math
    uint32_t bufA[16], bufB[16];
    tmem_ld16(tS, bufA);
    tmem_ld_wait();
    tmem_reg_fence(bufA);
    if (!diag && kb > 0) {
      // every key of the half-tile is visible to every row of the CTA, no caps
#pragma unroll 1
      for (int ch = 0; ch < HB / 16; ch += 2) {
        tmem_ld16(tS + 16 * (ch + 1), bufB);
        fwd_chunk_perm<kBF16, false>(bufA, scale2, nm2, kb + 16 * ch, i, sa, ea, bprev, z2, tS + 16 * ch);
        tmem_ld_wait();
        tmem_reg_fence(bufB);
        if (ch + 2 < HB / 16) tmem_ld16(tS + 16 * (ch + 2), bufA);
        fwd_chunk_perm<kBF16, false>(bufB, scale2, nm2, kb + 16 * (ch + 1), i, sa, ea, bprev, z2,
                                     tS + 16 * (ch + 1));
        tmem_ld_wait();
        tmem_reg_fence(bufA);
      }
    } else {
#define CA_FWD_PCHUNK(BUF, CH)                                                                                \
  {                                                                                                         \
    const int kind = fwd_chunk_kind(CH, kb, q0, warp, diag);                                                \
    if (kind == 1) fwd_chunk_perm<kBF16, false>(BUF, scale2, nm2, kb + 16 * (CH), i, sa, ea, bprev, z2,      \
                                                tS + 16 * (CH));                                            \
    else if (kind == 2) fwd_chunk_perm<kBF16, true>(BUF, scale2, nm2, kb + 16 * (CH), i, sa, ea, bprev, z2,  \
                                                    tS + 16 * (CH));                                        \
    else fwd_chunk_zero(CH, ea, bprev, tS);                                                                 \
  }
#pragma unroll 1
      for (int ch = 0; ch < HB / 16; ch += 2) {
        tmem_ld16(tS + 16 * (ch + 1), bufB);
        CA_FWD_PCHUNK(bufA, ch);
        tmem_ld_wait();
        tmem_reg_fence(bufB);
        if (ch + 2 < HB / 16) tmem_ld16(tS + 16 * (ch + 2), bufA);
        CA_FWD_PCHUNK(bufB, ch + 1);
        tmem_ld_wait();
        tmem_reg_fence(bufA);
      }
#undef CA_FWD_PCHUNK
    }
    if (hh == nh - 1 && i == kb + HB - 1) {   // key i is the last key: its cap stays pending
      bprev += 0.5f * ea;
      z2.x += 0.5f * ea;
    }
    bpend = bprev;
    sprev = sa;
    tmem_st_wait();
    tc_fence_before();
    mbar_arrive_warp(&sm.bar_p_ready[reg]);
  }

  if (ok) ok = mbar_wait(&sm.bar_o_done, 0, ab);
  tc_fence_after();
  uint32_t oa[2][32];
  tmem_ld32(tO, oa[0]);
  tmem_ld32(tO + 32, oa[1]);
  tmem_ld_wait();
  tmem_reg_fence(oa[0]);
  tmem_reg_fence(oa[1]);
  float acc[HD];
#pragma unroll
  for (int d = 0; d < HD; ++d) acc[d] = __uint_as_float(oa[d / 32][d % 32]);
  const size_t row = (size_t)bh * Tn + i;
  if (ok && row_ok && bpend != 0.f) {
    // v of key i, eight 16-byte loads
    const uint4* vr = reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(vptr) + row * HD);
    uint4 vq[HD / 8];
#pragma unroll
    for (int c = 0; c < HD / 8; ++c) vq[c] = __ldg(vr + c);
#pragma unroll
    for (int c = 0; c < HD / 8; ++c) {
      const uint32_t wv[4] = {vq[c].x, vq[c].y, vq[c].z, vq[c].w};
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        float v0, v1;
        if (kBF16) {
          v0 = __uint_as_float(wv[u] << 16);
          v1 = __uint_as_float(wv[u] & 0xffff0000u);
        } else {
          v0 = __half2float(__ushort_as_half((unsigned short)(wv[u] & 0xffffu)));
          v1 = __half2float(__ushort_as_half((unsigned short)(wv[u] >> 16)));
        }
        acc[8 * c + 2 * u] = fmaf(bpend, v0, acc[8 * c + 2 * u]);
        acc[8 * c + 2 * u + 1] = fmaf(bpend, v1, acc[8 * c + 2 * u + 1]);
      }
    }
  }
  const float z = z2.x + z2.y;
  const float inv = 1.f / z;
  store_out_rows<kBF16>(sm, acc, inv, r, o32 != nullptr, tm_o, tm_o32, bh, H, q0, o_bthd);
  if (stats && ok && row_ok) {
    stats[2 * row] = m_used;
    stats[2 * row + 1] = z;
  }
}

template <bool kBF16>
__device__ void math_warps(Smem& sm, const void* vptr, const float* log_gain, const CUtensorMap* tm_o,
                           const CUtensorMap* tm_o32, float* o32, float* stats, int bh, int h, int Tn, int q0, int nh, uint32_t tmem, float inv_sqrt_d, int H,
                           int o_bthd) {
  volatile int* ab = &sm.abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = warp * 32 + lane;
  const int i = q0 + r;
  const bool row_ok = i < Tn;
  const float scale = expf(log_gain[h]) * inv_sqrt_d;
  const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
  const uint32_t tO = tmem + TMEM_O + lane_base;

  float m_used = -INFINITY, z = 0.f, bpend = 0.f, sprev = 0.f;
  float2 z2 = splat2(0.f);   // packed partial of z from interior chunks
  const float2 scale2 = splat2(scale);
  bool ok = true;
  for (int hh = 0; hh < nh; ++hh) {
    const int reg = hh % NREG;
    const bool got = mbar_wait(&sm.bar_s_full[reg], (hh / NREG) & 1, ab);
    if (!__all_sync(0xffffffffu, got)) { ok = false; break; }
    tc_fence_after();
    const uint32_t tS = tmem + HB * reg + lane_base;
    const int kb = hh * HB;                     // first key of this half-tile
    const bool diag = hh >= nh - 2;             // the two half-tiles the diagonal crosses
    const int nvis = diag ? min(i - kb + 1, HB) : HB;
    // pass 1: half-tile max over the visible keys
    uint32_t sr[2][32];
    float tmax = -INFINITY;
    tmem_ld32(tS, sr[0]);
    tmem_ld32(tS + 32, sr[1]);
    tmem_ld_wait();
    tmem_reg_fence(sr[0]);
    tmem_reg_fence(sr[1]);
#pragma unroll
    for (int c2 = 0; c2 < 2; ++c2) {
      if (diag) {
#pragma unroll
        for (int x = 0; x < 32; ++x)
          if (32 * c2 + x < nvis) tmax = fmaxf(tmax, __uint_as_float(sr[c2][x]));
      } else {
#pragma unroll
        for (int x = 0; x < 32; ++x) tmax = fmaxf(tmax, __uint_as_float(sr[c2][x]));
      }
    }
    tmax *= scale;
    const bool need = tmax > m_used + kRescaleNats;
    if (hh == 0) {
      m_used = tmax;
    } else if (__any_sync(0xffffffffu, need)) {
      // O holds P V' of every earlier half-tile: wait until the last of them has
      // landed (its commit covers every MMA issued before it).  The barrier of
      // half-tile hh-1 cannot be a phase further on (that needs P_{hh+1}) nor a
      // phase behind (P V'_{hh-3} completed before S_hh), so its parity is exact.
      const bool got2 = mbar_wait(&sm.bar_pv_done[(hh - 1) & 1], ((hh - 1) >> 1) & 1, ab);
      if (!__all_sync(0xffffffffu, got2)) { ok = false; break; }
      tc_fence_after();
      const float m_new = need ? tmax : m_used;
      const float alpha = exp_rel(m_used - m_new);
      z *= alpha;
      z2 = mul2(z2, splat2(alpha));
      bpend *= alpha;
      m_used = m_new;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        tmem_ld32(tO + 32 * half, sr[1]);
        tmem_ld_wait();
        tmem_reg_fence(sr[1]);
#pragma unroll
        for (int x = 0; x < 32; ++x) sr[1][x] = __float_as_uint(__uint_as_float(sr[1][x]) * alpha);
        tmem_st32(tO + 32 * half, sr[1]);
      }
      tmem_st_wait();
    }
    const float m2 = m_used * kLog2e;
    float sa = sprev;
    float ea = (kb > 0) ? ex2_approx(fmaf(sprev, kLog2e, -m2)) : 0.f;
    float bprev = bpend;
    // pass 2: P for 16 keys at a time; the next chunk's load overlaps this chunk's math
    const float2 nm2 = splat2(-m2);
    uint32_t bufA[16], bufB[16];
    tmem_ld16(tS, bufA);
    tmem_ld_wait();
    tmem_reg_fence(bufA);
#define CA_FWD_CHUNK(BUF, CH)                                                                    \
  {                                                                                              \
    const int kind = fwd_chunk_kind(CH, kb, q0, warp, diag);                                     \
    if (kind == 1) fwd_chunk_fast<kBF16>(BUF, CH, scale2, nm2, sa, ea, bprev, z2, tS);           \
    else if (kind == 2) fwd_chunk<kBF16, true>(BUF, CH, scale, m2, nvis, kb, i, sa, ea, bprev, z, tS); \
    else fwd_chunk_zero(CH, ea, bprev, tS);                                                      \
  }
#pragma unroll 1
    for (int ch = 0; ch < HB / 16; ch += 2) {
      tmem_ld16(tS + 16 * (ch + 1), bufB);
      CA_FWD_CHUNK(bufA, ch);
      tmem_ld_wait();
      tmem_reg_fence(bufB);
      if (ch + 2 < HB / 16) tmem_ld16(tS + 16 * (ch + 2), bufA);
      CA_FWD_CHUNK(bufB, ch + 1);
      tmem_ld_wait();
      tmem_reg_fence(bufA);
    }
#undef CA_FWD_CHUNK
    if (hh == nh - 1 && i == kb + HB - 1) {   // key i is the last key: its cap stays pending
      bprev += 0.5f * ea;
      z += 0.5f * ea;
    }
    bpend = bprev;
    sprev = sa;
    tmem_st_wait();
    tc_fence_before();
    mbar_arrive_warp(&sm.bar_p_ready[reg]);
  }

  if (ok) ok = mbar_wait(&sm.bar_o_done, 0, ab);
  tc_fence_after();
  uint32_t oa[2][32];
  tmem_ld32(tO, oa[0]);
  tmem_ld32(tO + 32, oa[1]);
  tmem_ld_wait();
  tmem_reg_fence(oa[0]);
  tmem_reg_fence(oa[1]);
  float acc[HD];
#pragma unroll
  for (int d = 0; d < HD; ++d) acc[d] = __uint_as_float(oa[d / 32][d % 32]);
  const size_t row = (size_t)bh * Tn + i;
  if (ok && row_ok && bpend != 0.f) {
    // v of key i, eight 16-byte loads
    const uint4* vr = reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(vptr) + row * HD);
    uint4 vq[HD / 8];
#pragma unroll
    for (int c = 0; c < HD / 8; ++c) vq[c] = __ldg(vr + c);
#pragma unroll
    for (int c = 0; c < HD / 8; ++c) {
      const uint32_t wv[4] = {vq[c].x, vq[c].y, vq[c].z, vq[c].w};
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        float v0, v1;
        if (kBF16) {
          v0 = __uint_as_float(wv[u] << 16);
          v1 = __uint_as_float(wv[u] & 0xffff0000u);
        } else {
          v0 = __half2float(__ushort_as_half((unsigned short)(wv[u] & 0xffffu)));
          v1 = __half2float(__ushort_as_half((unsigned short)(wv[u] >> 16)));
        }
        acc[8 * c + 2 * u] = fmaf(bpend, v0, acc[8 * c + 2 * u]);
        acc[8 * c + 2 * u + 1] = fmaf(bpend, v1, acc[8 * c + 2 * u + 1]);
      }
    }
  }
  z += z2.x + z2.y;
  const float inv = 1.f / z;
  store_out_rows<kBF16>(sm, acc, inv, r, o32 != nullptr, tm_o, tm_o32, bh, H, q0, o_bthd);
  if (stats && ok && row_ok) {   // nullptr: inference, no backward follows
    stats[2 * row] = m_used;
    stats[2 * row + 1] = z;
  }
}

template <bool kBF16, bool kPerm>
__global__ void __launch_bounds__(NUM_THREADS, 2)
fwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
           const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_o,
           const __grid_constant__ CUtensorMap tm_o32, const void* __restrict__ vptr,
           const float* __restrict__ log_gain, float* __restrict__ o32,
           float* __restrict__ stats, int BH, int H, int Tn, float inv_sqrt_d, int o_bthd, int grp) {
  extern __shared__ uint8_t smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nqt = (Tn + BM - 1) / BM;
  // head-sequences in groups of grp, one group after another; inside a group the
  // heaviest query tiles first (see head_group())
  const int gi = blockIdx.x / (grp * nqt);
  const int gr = blockIdx.x - gi * grp * nqt;
  const int gs = min(grp, BH - gi * grp);
  const int bh = gi * grp + gr % gs;
  const int qt = nqt - 1 - gr / gs;
  const int q0 = qt * BM;
  const int nh = 2 * (qt + 1);                // key half-tiles 0 .. 2qt+1 (keys 0 .. q0+127)

  if (warp == 4) {
    if (lane == 0) {
      mbar_init(&sm.bar_q, 1);
      for (int s = 0; s < KSTAGES; ++s) {
        mbar_init(&sm.bar_k[s], 1);
        mbar_init(&sm.bar_v[s], 1);
        mbar_init(&sm.bar_kv_free[s], 1);
      }
      for (int g = 0; g < NREG; ++g) {
        mbar_init(&sm.bar_s_full[g], 1);
        mbar_init(&sm.bar_p_ready[g], 4);   // one arrival per math warp
      }
      mbar_init(&sm.bar_pv_done[0], 1);
      mbar_init(&sm.bar_pv_done[1], 1);
      mbar_init(&sm.bar_o_done, 1);
      sm.abort_flag = 0;
      fence_mbar_init();
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      tma_prefetch_desc(&tm_o);
      if (o32) tma_prefetch_desc(&tm_o32);
    }
    __syncwarp();
    tmem_alloc(&sm.tmem_base, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  // the set-up above touches no global data; everything below may read or write
  // what the previous kernel in the stream produced or consumed
  pdl_wait();
  pdl_launch_dependents();

  if (warp == 4) {
    producer<kBF16, kPerm>(sm, &tm_q, &tm_k, &tm_v, bh, q0, nh, tmem);   // whole warp, converged
    __syncwarp();
  } else if (kPerm) {
    math_warps_perm<kBF16>(sm, vptr, log_gain, &tm_o, &tm_o32, o32, stats, bh, bh % H, Tn, q0, nh, tmem, inv_sqrt_d, H,
                           o_bthd);
  } else {
    math_warps<kBF16>(sm, vptr, log_gain, &tm_o, &tm_o32, o32, stats, bh, bh % H, Tn, q0, nh, tmem, inv_sqrt_d, H,
                      o_bthd);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 4) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

}  // namespace fwd

// ---------------------------------------------------------------------------
// Backward, persistent (one CTA per SM): a work item is one 128-key tile
// [j0, j0+128) of one head-sequence, looping over its query tiles from the last
// one down to the diagonal; a CTA takes items heaviest first from a counter (see
// producer and decode_item):
//   warp 16 is the producer (the whole warp runs converged; lane 0 issues):
//     TMA: K' and V' (keys j0-16 .. j0+143, stationary), Q and dO tiles (2 stages)
//     S  = Q K'^T   128x160 fp32, TMEM columns [0,160)    (key j0+x at column 16+x)
//     dP = dO V'^T  128x160 fp32, TMEM columns [160,320)
//     dQ  = dS K        128x64 fp32, TMEM [320,384)  (fresh per query tile)
//     dV += P^T dO      128x64 fp32, TMEM [384,448)  (lane = key)
//     dK += dS^T Q      128x64 fp32, TMEM [448,512)
//   warps 0-15: thread = (query row 32*(w%4)+lane, key quarter w/4 of 32 keys).
//     It loads its 34 S and dP values (one halo key each side), forms the 33
//     segment moments M0..M2, the analytic VJP in the form (see bwd_keys8)
//       p_j = (B_j + A_{j+1} + cap_j) / Z,   dS_j = g_j p_j + H_{j+1} - H_j,
//     with g = dP - D_i (D_i = dO_i . O_i) and H_k = (g_k - g_{k-1}) (M1 - M2)_k,
//     and writes p and scale*dS as bf16 into a 128-byte-swizzled shared buffer
//     [2 key halves][128 queries][64 keys].
//     The same bytes are the MN-major A operand of dV / dK (M = keys) and the
//     K-major A operand of dQ (M = queries).  dQ of the previous query tile is
//     read from TMEM into a swizzled f32 staging tile; the producer adds it to
//     the global fp32 dQ accumulator with two TMA reduce-adds (32 columns each),
//     so the adds travel as whole 128-byte rows instead of per-thread atomics.
//     At an item's end dK and dV leave TMEM through a swizzled staging tile in the
//     P buffer and two TMA stores.
// Replaces cuda/continuum_attention.py:713-764 (recompute, dW = dY V^T, the
// analytic score VJP kernels :192-293/:337-405, and the dV/dQ/dK GEMMs).
namespace bwd {

constexpr int BM = 128;              // query rows per tile
constexpr int BN = 128;              // keys per CTA
constexpr int HD = 64;
constexpr int KH = 160;              // staged key rows: j0-16 .. j0+143
constexpr int KOFF = 16;             // TMEM / SMEM row of key j0
constexpr int NUM_MATH_WARPS = 16;
constexpr int NUM_THREADS = (NUM_MATH_WARPS + 1) * 32;
constexpr int QSTAGES = 2;
constexpr uint32_t KV_BYTES = KH * HD * 2;      // 20 KB
constexpr uint32_t QT_BYTES = BM * HD * 2;      // 16 KB
constexpr uint32_t HALF_BYTES = BM * 128;       // 16 KB: 128 query rows x 64 keys bf16
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t T_S = 0, T_DP = 160, T_DQ = 320, T_DV = 384, T_DK = 448;

struct __align__(1024) Smem {
  uint8_t k[KV_BYTES];
  uint8_t v[KV_BYTES];
  uint8_t q[QSTAGES][QT_BYTES];
  uint8_t dout[QSTAGES][QT_BYTES];
  uint8_t p[2][HALF_BYTES];          // P   (bf16), [key half][query row][64 keys], swizzled
  uint8_t ds[2][HALF_BYTES];         // scale * dS (bf16), same layout
  uint8_t dqs[2][HALF_BYTES];        // dQ of one query tile (f32): [32-column half][row][128 B], swizzled
  uint64_t bar_kv;
  uint64_t bar_qdo[QSTAGES];
  uint64_t bar_s_full;
  uint64_t bar_s_consumed;
  uint64_t bar_p_ready;
  uint64_t bar_mma_done;
  uint64_t bar_drain;
  uint64_t bar_dq_free;              // the staged dQ tile has been read by its reduce
  uint64_t bar_item;                 // the producer has published the next work item
  uint32_t tmem_base;
  int abort_flag;
  int item;                          // published work item (n_items: none left)
  int decision;                      // the item every math warp takes next
  float red[NUM_MATH_WARPS];
};

constexpr size_t kSmemBytes = sizeof(Smem) + 1024;

// The shared-memory descriptors of one operand differ only in the start-address
// field ([0,14), address >> 4), which never carries (shared addresses stay below
// 256 KB): each is its base descriptor plus the byte offset >> 4, one add per MMA.
template <bool kBF16>
__device__ __forceinline__ void issue_s_dp(const Smem& sm, int st, uint32_t tmem, uint32_t idesc) {
  const uint64_t dq = sdesc_sw128(smem_u32(sm.q[st]), 16, 1024), dk = sdesc_sw128(smem_u32(sm.k), 16, 1024);
  const uint64_t ddo = sdesc_sw128(smem_u32(sm.dout[st]), 16, 1024), dv = sdesc_sw128(smem_u32(sm.v), 16, 1024);
#pragma unroll
  for (int kk = 0; kk < HD / 16; ++kk)   // 32 bytes of K per step
    mma_ss(tmem + T_S, dq + 2 * kk, dk + 2 * kk, idesc, kk > 0 ? 1u : 0u);
#pragma unroll
  for (int kk = 0; kk < HD / 16; ++kk)
    mma_ss(tmem + T_DP, ddo + 2 * kk, dv + 2 * kk, idesc, kk > 0 ? 1u : 0u);
}

template <bool kBF16>
__device__ __forceinline__ void issue_grads(const Smem& sm, int st, uint32_t tmem, bool first, uint32_t id_mn,
                                            uint32_t id_dq) {
  const uint64_t dp = sdesc_sw128(smem_u32(sm.p[0]), HALF_BYTES, 1024);
  const uint64_t dds = sdesc_sw128(smem_u32(sm.ds[0]), HALF_BYTES, 1024);
  const uint64_t dq = sdesc_sw128(smem_u32(sm.q[st]), 16384, 1024);
  const uint64_t ddo = sdesc_sw128(smem_u32(sm.dout[st]), 16384, 1024);
  const uint64_t dsk = sdesc_sw128(smem_u32(sm.ds[0]), 16, 1024);
  const uint64_t dk = sdesc_sw128(smem_u32(sm.k) + KOFF * 128, 16384, 1024);
#pragma unroll
  for (int kk = 0; kk < BM / 16; ++kk) {   // K = query rows, 16 per step (2048 bytes)
    const uint32_t acc = (!first || kk > 0) ? 1u : 0u;
    // dV += P^T dO : A = P (MN-major, M = keys), B = dO (MN-major, N = d)
    mma_ss(tmem + T_DV, dp + 128 * kk, ddo + 128 * kk, id_mn, acc);
    // dK += dS^T Q
    mma_ss(tmem + T_DK, dds + 128 * kk, dq + 128 * kk, id_mn, acc);
  }
#pragma unroll
  for (int kk = 0; kk < BN / 16; ++kk) {   // K = keys, 16 per step
    // dQ = dS K : A = dS (K-major, M = queries; key half kk / 4, 32 bytes per step),
    // B = K rows j0.. (MN-major, N = d, 2048 bytes per step)
    mma_ss(tmem + T_DQ, dsk + (HALF_BYTES >> 4) * (kk / 4) + 2 * (kk % 4), dk + 128 * kk, id_dq,
           kk > 0 ? 1u : 0u);
  }
}

// Work item w: head-sequences go in groups of grp (see head_group()), one group
// after another; inside a group the heaviest items first: key tile kt = r / gs of
// head-sequence bh = g * grp + r % gs (group g, r = w - g * grp * nkt, gs the
// group's size), with n = nkt - kt query tiles.  Tile t of an item is query tile kt + n - 1 - t:
// the last query tile first and the diagonal tile last, so that every item reaches
// a given query tile at the same offset from its start, and the items of a head,
// started in key-tile order (heaviest first), reach it in key-tile order too.
struct Item {
  int bh, kt, j0, n;
  __device__ __forceinline__ int row0(int t) const { return j0 + (n - 1 - t) * BM; }
};
__device__ __forceinline__ Item decode_item(int w, int BH, int nkt, int grp) {
  Item it;
  const int g = w / (grp * nkt);
  const int r = w - g * grp * nkt;
  const int gs = min(grp, BH - g * grp);
  it.bh = g * grp + r % gs;
  it.kt = r / gs;
  it.j0 = it.kt * BN;
  it.n = nkt - it.kt;
  return it;
}

// Persistent producer: items come from a global counter (the first is blockIdx.x,
// then gridDim.x + atomicAdd(counter)).  Barrier phases are counted in global
// tiles g (all items of this CTA in order): s_full, s_consumed, mma_done and the
// dQ reduces advance once per tile, p_ready once per tile plus once per item (the
// last dQ is staged after the item's tile loop), the Q/dO ring by stage.  The next
// item's first Q/dO tiles go into the ring as soon as this item's last tiles free
// their stages, its K'/V' boxes are prefetched into L2 when it is claimed and
// copied in once this item's last gradient MMAs complete, it is published to the
// math warps at this item's last tile, and this item's final dQ reduce waits until
// the next item's first S/dP is issued: the next item's start overlaps this
// item's epilogue.
// kDet: each dQ tile receives its key tiles' contributions in ascending key-tile
// order -- key tile 0 stores, key tile k adds once ready[bh, query tile] == k, then
// raises it -- so dQ is the same fp32 sum on every run (and the accumulator needs
// no zeroing).  Otherwise the contributions are reduce-adds in arrival order.
template <bool kBF16, bool kDOB, bool kDet>
__device__ void producer(Smem& sm, const CUtensorMap* tq, const CUtensorMap* tk, const CUtensorMap* tv,
                         const CUtensorMap* tdo, const CUtensorMap* tdq, int BH, int nkt, int grp, int n_items,
                         unsigned* counter, unsigned* ready, uint32_t tmem, int H) {
  volatile int* ab = &sm.abort_flag;
  const int lane = threadIdx.x & 31;
  const uint32_t id_s = make_idesc(BM, KH, kBF16, false, false);
  const uint32_t id_mn = make_idesc(BN, HD, kBF16, true, true);
  const uint32_t id_dq = make_idesc(BM, HD, kBF16, true, false);
  bool kv_pending = false;
  uint32_t kv_phase = 0;
  bool q_pending[QSTAGES];
  uint32_t q_phase[QSTAGES];
  for (int s2 = 0; s2 < QSTAGES; ++s2) {
    q_pending[s2] = false;
    q_phase[s2] = 0;
  }
  auto fetch = [&]() -> int {
    unsigned k = 0;
    if (lane == 0) k = atomicAdd(counter, 1u);
    k = __shfl_sync(0xffffffffu, k, 0);
    return (int)(gridDim.x + k);
  };
  auto load_kv = [&](const Item& it) {
    mbar_arrive_expect_tx(&sm.bar_kv, 2 * KV_BYTES);
    tma_load_3d(sm.k, tk, &sm.bar_kv, 0, it.j0 - KOFF, it.bh);
    tma_load_3d(sm.v, tv, &sm.bar_kv, 0, it.j0 - KOFF, it.bh);
    kv_pending = true;
  };
  auto load_qdo = [&](int st, const Item& it, int t) {
    mbar_arrive_expect_tx(&sm.bar_qdo[st], 2 * QT_BYTES);
    tma_load_3d(sm.q[st], tq, &sm.bar_qdo[st], 0, it.row0(t), it.bh);
    if (kDOB)   // dO stored [B][T][H][D]: map (D, H, T, B)
      tma_load_4d(sm.dout[st], tdo, &sm.bar_qdo[st], 0, it.bh % H, it.row0(t), it.bh / H);
    else
      tma_load_3d(sm.dout[st], tdo, &sm.bar_qdo[st], 0, it.row0(t), it.bh);
    q_pending[st] = true;
  };
  unsigned* ready_pending = nullptr;
  // Deterministic: once the last dQ tile has reached global memory, hand its query
  // tile to the next key tile (a release increment of its turn counter).
  auto release_ready = [&]() {
    if (kDet && ready_pending) {
      bulk_wait_group0();
      fence_proxy_async_global();
      if (lane == 0) red_release_add_gpu(ready_pending, 1u);
      __syncwarp();
      ready_pending = nullptr;
    }
  };
  // the staged dQ tile of tile t of item it (two 32-column halves) into the accumulator
  auto issue_dq = [&](const Item& it, int t) -> bool {
    const int row0 = it.row0(t);
    if (kDet) {
      release_ready();
      unsigned* rdy = ready + (size_t)it.bh * nkt + row0 / BM;
      if (it.kt == 0) {
        tma_store_3d(tdq, sm.dqs[0], 0, row0, it.bh);
        tma_store_3d(tdq, sm.dqs[1], 32, row0, it.bh);
      } else {
        if (!wait_count(rdy, (unsigned)it.kt, ab)) return false;
        fence_proxy_async_global();
        tma_reduce_add_3d(tdq, sm.dqs[0], 0, row0, it.bh);
        tma_reduce_add_3d(tdq, sm.dqs[1], 32, row0, it.bh);
      }
      ready_pending = rdy;
    } else {
      tma_reduce_add_3d(tdq, sm.dqs[0], 0, row0, it.bh);
      tma_reduce_add_3d(tdq, sm.dqs[1], 32, row0, it.bh);
    }
    bulk_commit_group();
    return true;
  };
  // the staging tile has been read (and, deterministic, the tile written to global
  // memory, which the next key tile's turn then follows): free it for the math warps
  auto dq_done = [&]() {
    bulk_wait_group_read0();
    if (lane == 0) mbar_arrive(&sm.bar_dq_free);
    __syncwarp();
    release_ready();
  };
  auto publish = [&](int w) {
    if (lane == 0) {
      sm.item = w;
      mbar_arrive(&sm.bar_item);
    }
    __syncwarp();
  };

  int item = blockIdx.x;
  int next = -1;         // claimed next item (-1: not claimed yet; claims happen late, see below)
  uint32_t g0 = 0;       // global index of the current item's first tile
  uint32_t pr = 0;       // p_ready phases consumed
  uint32_t issued = 0;   // global tiles whose Q/dO load has been issued
  int committed = -1;    // last global tile whose gradient MMAs were committed
  int completed = -1;    // last global tile whose gradient MMAs are known complete
  // Issue Q/dO loads for global tiles issued .. upto-1 that belong to the current
  // or the next item.  Global tile x uses stage x % QSTAGES, last read by the
  // gradient MMAs of tile x - QSTAGES; those are waited for through the most
  // recent commit (its phase is the only open one, so the parity is exact).
  auto ensure_loaded = [&](const Item& it, bool has_next, const Item& nx, uint32_t upto) -> bool {
    while (issued < upto) {
      const uint32_t x = issued;
      const bool mine = x < g0 + it.n;
      if (!mine && !(has_next && x < g0 + it.n + nx.n)) break;
      if ((int)x - QSTAGES > completed) {
        if (!mbar_wait_warp(&sm.bar_mma_done, (uint32_t)committed & 1, ab)) return false;
        completed = committed;
      }
      if (mine) load_qdo((int)(x % QSTAGES), it, (int)(x - g0));
      else load_qdo((int)(x % QSTAGES), nx, (int)(x - g0 - it.n));
      ++issued;
    }
    return true;
  };
  // the last dQ tile of an item is staged by the math warps after their tile loop
  // (one more p_ready phase); its reduce is issued after the next item's first
  // S/dP, so that the next item starts as early as its K'/V' allow
  auto final_reduce = [&](const Item& pi) -> bool {
    if (!mbar_wait_warp(&sm.bar_p_ready, pr & 1, ab)) return false;
    ++pr;
    if (!issue_dq(pi, pi.n - 1)) return false;
    dq_done();
    return true;
  };
  bool good = item < n_items;
  if (good) {
    const Item it = decode_item(item, BH, nkt, grp);
    load_kv(it);
  }
  publish(good ? item : n_items);
  bool pending = false;   // the previous item's last dQ tile still has to be reduced
  Item prev = decode_item(0, BH, nkt, grp);
  while (good) {
    const Item it = decode_item(item, BH, nkt, grp);
    // The next item is claimed as late as its first Q/dO prefetch allows (the
    // item's second-to-last tile, or its start when it has one tile), so that the
    // counter hands the heaviest remaining items to the CTAs that free up first.
    // Its K'/V' boxes are prefetched into L2 at once; the shared-memory copy
    // follows when this item's last gradient MMAs have read K'.
    bool has_next = false;
    Item nx = decode_item(0, BH, nkt, grp);
    auto claim = [&]() {
      next = fetch();
      has_next = next < n_items;
      if (has_next) {
        nx = decode_item(next, BH, nkt, grp);
        tma_prefetch_l2_3d(tk, 0, max(nx.j0 - KOFF, 0), nx.bh);
        tma_prefetch_l2_3d(tv, 0, max(nx.j0 - KOFF, 0), nx.bh);
      }
    };
    next = -1;
    if (it.n == 1) claim();
    if (!ensure_loaded(it, has_next, nx, g0 + (uint32_t)min(QSTAGES, it.n))) { good = false; break; }
    const int st0 = (int)(g0 % QSTAGES);
    if (!mbar_wait_warp(&sm.bar_kv, kv_phase, ab) || !mbar_wait_warp(&sm.bar_qdo[st0], q_phase[st0], ab)) {
      good = false;
      break;
    }
    kv_pending = false;
    kv_phase ^= 1;
    q_pending[st0] = false;
    q_phase[st0] ^= 1;
    tc_fence_after();
    issue_s_dp<kBF16>(sm, st0, tmem, id_s);
    mma_commit(&sm.bar_s_full);
    if (pending) {
      if (!final_reduce(prev)) { good = false; break; }
      pending = false;
    }
    for (int t = 0; t < it.n && good; ++t) {
      const uint32_t g = g0 + t;
      const int st = (int)(g % QSTAGES);
      const bool last = t == it.n - 1;
      if (t == it.n - 2) claim();
      if (!mbar_wait_warp(&sm.bar_s_consumed, g & 1, ab)) { good = false; break; }
      if (t + 1 < it.n) {
        const int st1 = (int)((g + 1) % QSTAGES);
        if (!mbar_wait_warp(&sm.bar_qdo[st1], q_phase[st1], ab)) { good = false; break; }
        q_pending[st1] = false;
        q_phase[st1] ^= 1;
        tc_fence_after();
        issue_s_dp<kBF16>(sm, st1, tmem, id_s);
        mma_commit(&sm.bar_s_full);
      }
      if (!mbar_wait_warp(&sm.bar_p_ready, pr & 1, ab)) { good = false; break; }
      ++pr;
      tc_fence_after();
      issue_grads<kBF16>(sm, st, tmem, t == 0, id_mn, id_dq);
      mma_commit(&sm.bar_mma_done);
      committed = (int)g;
      // the math warps staged dQ of tile t-1 before arriving on p_ready (in the
      // deterministic order its turn may still be ahead: that reduce goes out below,
      // after the ring refill, so that the wait for the turn overlaps it)
      if (!kDet && t > 0 && !issue_dq(it, t - 1)) { good = false; break; }
      // every math warp is inside this item (it arrived on this tile's p_ready), so
      // the published slot is free: the next item goes out now, and the math warps
      // find it when they finish this one
      if (last) publish(has_next ? next : n_items);
      // stage st takes global tile g + QSTAGES (this item's or the next item's)
      if (!ensure_loaded(it, has_next, nx, g + QSTAGES + 1)) { good = false; break; }
      if (last && has_next) {
        // K' is read by this tile's dQ MMAs: the next item's K'/V' go in once those
        // have completed
        if (completed < (int)g) {
          if (!mbar_wait_warp(&sm.bar_mma_done, g & 1, ab)) { good = false; break; }
          completed = (int)g;
        }
        load_kv(nx);
      }
      if (kDet && t > 0 && !issue_dq(it, t - 1)) { good = false; break; }
      if (t > 0) dq_done();
    }
    if (!good) break;
    pending = true;
    prev = it;
    g0 += it.n;
    item = next;
    good = item < n_items;
  }
  if (pending && !*ab) final_reduce(prev);   // the loop ended normally: the last item's last dQ tile
  if (!*ab) release_ready();
  // drain: every copy lands and every MMA completes before shared memory / TMEM go away
  mma_commit(&sm.bar_drain);
  int dummy = 0;
  volatile int* nab = &dummy;
  if (kv_pending) mbar_wait_warp(&sm.bar_kv, kv_phase, nab);
  for (int s2 = 0; s2 < QSTAGES; ++s2)
    if (q_pending[s2]) mbar_wait_warp(&sm.bar_qdo[s2], q_phase[s2], nab);
  mbar_wait_warp(&sm.bar_drain, 0, nab);
  bulk_wait_group0();   // dQ reduces complete (shared source read, global adds done)
}

// scale*dS and P for 8 consecutive keys of one query row, packed as 16-bit pairs.
// The exponentials are taken against m + ln Z (E = e^{s-m}/Z), so every moment,
// and with it P and dS, comes out normalised; g = (dP - D) * scale, so the
// result is the scale*dS the dK/dQ products need.
// The analytic VJP (analytic_reference.py:52-75) gives key c, between segments
// c (key c-1 -> c) and c+1, the score gradient
//   dS_c = g_{c-1} (M1-M2)_c + g_c M2_c + g_c (M0-M1)_{c+1} + g_{c+1} (M1-M2)_{c+1} + cap_c g_c,
// and with P_c = M1_c + (M0-M1)_{c+1} + cap_c and H_k = (g_k - g_{k-1}) (M1-M2)_k
// that is  dS_c = g_c P_c + H_{c+1} - H_c:  per segment one product H, per key one
// fused multiply-add, the caps included through P.
// On entry (sc, ec, gc) belong to the current key (kfirst) and (Hprev, Bprev) are
// H and M1 of the segment into it; sv/pv[off .. off+7] hold the raw scores / dP of
// keys kfirst .. kfirst+7 (entry off is the current key) and the next key's come
// from sv/pv[off+8] or, past the end, from s_next / p_next.  gsum collects
// scale * sum dS*s.  kEdge handles masking and caps.
template <bool kBF16, bool kEdge>
__device__ __forceinline__ void bwd_keys8(const uint32_t (&sv)[16], const uint32_t (&pv)[16], int off,
                                          uint32_t s_next, uint32_t p_next, int kfirst, int i, bool row_ok,
                                          float scale, float m2, float dds, float& sc, float& ec, float& gc,
                                          float& Hprev, float& Bprev, float& gsum, uint32_t (&pk)[4],
                                          uint32_t (&dk)[4]) {
#pragma unroll
  for (int x = 0; x < 8; x += 2) {
    float po[2], dso[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int c = x + u;
      const int key = kfirst + c;
      const int nxt = off + c + 1;
      const uint32_t sn_bits = (nxt < 16) ? sv[nxt & 15] : s_next;
      const uint32_t pn_bits = (nxt < 16) ? pv[nxt & 15] : p_next;
      const float sn = __uint_as_float(sn_bits) * scale;
      const float gn = fmaf(__uint_as_float(pn_bits), scale, -dds);
      float en, M0, M1, M2;
      bool vn = true;
      if (kEdge) {
        vn = row_ok && (key + 1) <= i;
        en = vn ? ex2_approx(fmaf(sn, kLog2e, -m2)) : 0.f;
      } else {
        en = ex2_approx(fmaf(sn, kLog2e, -m2));
      }
      seg_moments012_sel(ec, en, sn - sc, M0, M1, M2);
      if (kEdge) {
        M0 = vn ? M0 : 0.f;
        M1 = vn ? M1 : 0.f;
        M2 = vn ? M2 : 0.f;
      }
      const float Anext = M0 - M1;
      const float Hn = (gn - gc) * (M1 - M2);
      float ds, p;
      if (kEdge) {
        const bool vc = row_ok && key >= 0 && key <= i;
        const float nc = (key == 0 ? 1.f : 0.f) + (key == i ? 1.f : 0.f);
        p = Bprev + Anext + (nc > 0.f ? 0.5f * nc * ec : 0.f);
        ds = fmaf(gc, p, Hn - Hprev);
        ds = vc ? ds : 0.f;
        p = vc ? p : 0.f;
      } else {
        p = Bprev + Anext;
        ds = fmaf(gc, p, Hn - Hprev);
      }
      gsum = fmaf(ds, sc, gsum);
      po[u] = p;
      dso[u] = ds;
      Hprev = Hn;
      Bprev = M1;
      sc = sn;
      ec = en;
      gc = gn;
    }
    pk[x / 2] = kBF16 ? pack_bf16x2(po[0], po[1]) : pack_f16x2(po[0], po[1]);
    dk[x / 2] = kBF16 ? pack_bf16x2(dso[0], dso[1]) : pack_f16x2(dso[0], dso[1]);
  }
}

// Interior version of bwd_keys8 (every key visible, no caps) in packed fp32
// pairs.  Segment pairs (2x -> 2x+1, 2x+1 -> 2x+2) are the lanes: their left
// keys (2x, 2x+1) form the natural register pairs of the raw TMEM rows, so s,
// g and the exponent argument are computed packed there; each exponential goes
// straight into the right-key pair (2x+1, 2x+2) where the moment recurrences use
// it.  Products that mix the two layouts (differences, the final sums with the
// previous segment's H and M1) are scalar.  The moments match seg_moments012_sel
// bit for bit; dS = g P + H_next - H as in bwd_keys8.  ec carries e of key 0
// between calls (sc, gc are recomputed from the raw row); gsum2 collects
// scale * dS * s.
template <bool kBF16>
__device__ __forceinline__ void bwd_keys8_fast(const uint32_t (&sv)[16], const uint32_t (&pv)[16], int off,
                                               uint32_t s_next, uint32_t p_next, float scale, float m2, float dds,
                                               float& ec, float& Hprev, float& Bprev, float2& gsum2,
                                               uint32_t (&pk)[4], uint32_t (&dk)[4]) {
  const float2 scale2 = splat2(scale), l2e = splat2(kLog2e), nm2 = splat2(-m2), ndds = splat2(-dds);
  const float2 neg1 = splat2(-1.f), neg2 = splat2(-2.f), half = splat2(0.5f);
  float2 sA[4], gA[4];
  float e[9];
  e[0] = ec;
#pragma unroll
  for (int x = 0; x < 4; ++x) {
    const float2 raw = make_float2(__uint_as_float(sv[(off + 2 * x) & 15]), __uint_as_float(sv[(off + 2 * x + 1) & 15]));
    const float2 praw = make_float2(__uint_as_float(pv[(off + 2 * x) & 15]), __uint_as_float(pv[(off + 2 * x + 1) & 15]));
    sA[x] = mul2(raw, scale2);
    gA[x] = fma2(praw, scale2, ndds);
    const float2 arg = fma2(sA[x], l2e, nm2);
    if (x > 0) e[2 * x] = ex2_approx(arg.x);
    e[2 * x + 1] = ex2_approx(arg.y);
  }
  const uint32_t s8_bits = (off + 8 < 16) ? sv[(off + 8) & 15] : s_next;
  const uint32_t p8_bits = (off + 8 < 16) ? pv[(off + 8) & 15] : p_next;
  const float s8 = __uint_as_float(s8_bits) * scale;
  const float g8 = fmaf(__uint_as_float(p8_bits), scale, -dds);
  e[8] = ex2_approx(fmaf(s8, kLog2e, -m2));
#pragma unroll
  for (int x = 0; x < 4; ++x) {
    const float sBy = (x < 3) ? sA[x + 1].x : s8;
    const float gBy = (x < 3) ? gA[x + 1].x : g8;
    const float2 EB = make_float2(e[2 * x + 1], e[2 * x + 2]);
    // nd = -(b - a) straight from the two subtractions; 1/d takes the negation as
    // the reciprocal's operand, and the series below runs in nd with alternating
    // signs (every value bit-identical to working with d)
    const float2 nd = make_float2(sA[x].x - sA[x].y, sA[x].y - sBy);
    const float2 r = make_float2(rcp_approx(-nd.x), rcp_approx(-nd.y));
    const float2 m0c = mul2(make_float2(EB.x - e[2 * x], EB.y - e[2 * x + 1]), r);
    const float2 m1c = mul2(fma2(m0c, neg1, EB), r);
    const float2 m2c = mul2(fma2(m1c, neg2, EB), r);
    float2 ser = fma2(splat2(-1.f / 36.f), nd, splat2(1.f / 10.f));
    ser = fma2(ser, nd, splat2(-1.f / 4.f));
    ser = fma2(ser, nd, splat2(1.f / 3.f));
    const float2 M2 = make_float2(sel_series(m2c.x, nd.x, e[2 * x], ser.x, kSeriesMaxBwd),
                                  sel_series(m2c.y, nd.y, e[2 * x + 1], ser.y, kSeriesMaxBwd));
    const float2 M1 = mul2(fma2(nd, M2, EB), half);
    const float2 M0 = fma2(nd, M1, EB);
    const float2 A = sub2(M0, M1);
    const float2 H = mul2(make_float2(gA[x].y - gA[x].x, gBy - gA[x].y), sub2(M1, M2));
    const float p0 = Bprev + A.x, p1 = M1.x + A.y;
    const float2 DS = fma2(gA[x], make_float2(p0, p1), make_float2(H.x - Hprev, H.y - H.x));
    const float ds0 = DS.x, ds1 = DS.y;
    gsum2 = fma2(DS, sA[x], gsum2);
    Hprev = H.y;
    Bprev = M1.y;
    pk[x] = kBF16 ? pack_bf16x2(p0, p1) : pack_f16x2(p0, p1);
    dk[x] = kBF16 ? pack_bf16x2(ds0, ds1) : pack_f16x2(ds0, ds1);
  }
  ec = e[8];
}

// one 16-byte chunk (8 keys) of a query row; 128-byte swizzle: chunk ^ (row & 7)
__device__ __forceinline__ void store_chunk(uint8_t* prow, uint8_t* drow, int chunk, int swz,
                                            const uint32_t (&pk)[4], const uint32_t (&dk)[4]) {
  const uint32_t off = (uint32_t)((chunk ^ swz) * 16);
  *reinterpret_cast<uint4*>(prow + off) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
  *reinterpret_cast<uint4*>(drow + off) = make_uint4(dk[0], dk[1], dk[2], dk[3]);
}

// One thread's 16 dQ columns (16qk .. 16qk+15) of query row r into the staging
// tile: half qk/2 holds columns 32(qk/2) .. +31 as 128-byte rows with the TMA
// 128-byte swizzle (16-byte chunk c of row r at chunk c ^ (r & 7)).
__device__ __forceinline__ void stage_dq(Smem& sm, int r, int qk, const uint32_t (&qv)[16]) {
  uint8_t* const row = sm.dqs[qk >> 1] + (uint32_t)r * 128;
#pragma unroll
  for (int x = 0; x < 4; ++x) {
    const int chunk = 4 * (qk & 1) + x;
    *reinterpret_cast<uint4*>(row + ((chunk ^ (r & 7)) << 4)) =
        make_uint4(qv[4 * x], qv[4 * x + 1], qv[4 * x + 2], qv[4 * x + 3]);
  }
}

// One work item of the math warps: key tile kt of head-sequence bh, its n_tiles
// query tiles being global tiles g0 .. g0+n_tiles-1 of this CTA.
template <bool kBF16>
__device__ void math_item(Smem& sm, const float* log_gain, const float* stats, const float* rowdot,
                          const CUtensorMap* tm_dk, const CUtensorMap* tm_dv, float* gain_part, int bh, int h, int Tn, int j0,
                          int kt, int nkt, int n_tiles, uint32_t g0, uint32_t tmem, float inv_sqrt_d, bool& ok) {
  volatile int* ab = &sm.abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rq = warp & 3;                 // TMEM lane quarter
  const int qk = warp >> 2;                // key quarter: keys j0+32qk .. +31
  const int r = rq * 32 + lane;            // query row in tile / key row in epilogue
  const uint32_t lane_base = (uint32_t)(rq * 32) << 16;
  const float scale = expf(log_gain[h]) * inv_sqrt_d;
  const uint32_t colS = tmem + lane_base + T_S + KOFF + 32 * qk;    // key j0+32qk
  const uint32_t colP = tmem + lane_base + T_DP + KOFF + 32 * qk;
  uint8_t* const pbuf = sm.p[qk >> 1];
  uint8_t* const dbuf = sm.ds[qk >> 1];
  const int chunk0 = 4 * (qk & 1);         // first 16-byte chunk of this quarter in a 128-byte row
  float gsum = 0.f;
  float2 gsum2 = splat2(0.f);   // packed partial of gsum from interior key groups

  // row statistics of the next query tile are loaded one iteration ahead; tile t is
  // query tile kt + n_tiles - 1 - t (the last query tile first, the diagonal last)
  float nm = 0.f, nz = 1.f, nd = 0.f;
  if (j0 + (n_tiles - 1) * BM + r < Tn) {
    const size_t ri = (size_t)bh * Tn + j0 + (n_tiles - 1) * BM + r;
    nm = stats[2 * ri];
    nz = stats[2 * ri + 1];
    nd = rowdot[ri];
  }
  for (int t = 0; t < n_tiles; ++t) {
    const int i0 = j0 + (n_tiles - 1 - t) * BM;
    const int i = i0 + r;
    const bool row_ok = i < Tn;
    const float m = nm, zrow = nz, dd = nd;
    if (t + 1 < n_tiles) {   // rows i - BM of the next tile are all inside [0, T)
      const size_t ri = (size_t)bh * Tn + i - BM;
      nm = stats[2 * ri];
      nz = stats[2 * ri + 1];
      nd = rowdot[ri];
    }
    const bool got = mbar_wait(&sm.bar_s_full, (g0 + t) & 1, ab);
    if (!__all_sync(0xffffffffu, got)) { ok = false; break; }
    tc_fence_after();
    const float m2 = row_ok ? fmaf(m, kLog2e, lg2_approx(zrow)) : 0.f;   // E = e^{s-m} / Z
    const float dds = dd * scale;
    // interior: every key this warp touches (kbase-1 .. kbase+32) is visible to all of
    // its rows (i0+32rq .. i0+32rq+31), inside [0, T) and capless: no masking needed
    const int kbase = j0 + 32 * qk;              // key of local column 0
    const bool interior = kbase >= 1 && kbase + 32 <= i0 + 32 * rq && i0 + 32 * rq + 32 <= Tn;
    uint8_t* const prow = pbuf + (uint32_t)r * 128;
    uint8_t* const drow = dbuf + (uint32_t)r * 128;
    const int swz = r & 7;
    // only on the diagonal tile: every key of this quarter lies beyond every row of
    // the warp, so its P and dS are zero (its left neighbour quarter reads the
    // halo key from TMEM itself)
    const bool dead = kbase > i0 + 32 * rq + 31;
    if (dead) {
      tc_fence_before();
      mbar_arrive_warp(&sm.bar_s_consumed);
      if (t > 0) {
        const bool got2 = mbar_wait(&sm.bar_mma_done, (g0 + t - 1) & 1, ab);
        if (!__all_sync(0xffffffffu, got2)) { ok = false; break; }
      }
      const uint32_t zz[4] = {0u, 0u, 0u, 0u};
#pragma unroll
      for (int c = 0; c < 4; ++c) store_chunk(prow, drow, chunk0 + c, swz, zz, zz);
    } else {
      // chunk 0: left halo, keys 0..15, key 16
      uint32_t s_lo, p_lo, s16, p16, sv[16], pv[16];
      tmem_ld1(colS - 1, s_lo);
      tmem_ld16(colS, sv);
      tmem_ld1(colS + 16, s16);
      tmem_ld1(colP - 1, p_lo);
      tmem_ld16(colP, pv);
      tmem_ld1(colP + 16, p16);
      tmem_ld_wait();
      tmem_reg_fence(s_lo);
      tmem_reg_fence(sv);
      tmem_reg_fence(s16);
      tmem_reg_fence(p_lo);
      tmem_reg_fence(pv);
      tmem_reg_fence(p16);
      // the segment from the left halo key into key kbase
      float sa = __uint_as_float(s_lo) * scale;
      float ga = fmaf(__uint_as_float(p_lo), scale, -dds);
      float sc = __uint_as_float(sv[0]) * scale;
      float gc = fmaf(__uint_as_float(pv[0]), scale, -dds);
      float ea, ec, Hprev, Bprev;
      {
        const bool va = interior || (row_ok && kbase - 1 >= 0 && kbase - 1 <= i);
        const bool vc = interior || (row_ok && kbase <= i);
        ea = va ? ex2_approx(fmaf(sa, kLog2e, -m2)) : 0.f;
        ec = vc ? ex2_approx(fmaf(sc, kLog2e, -m2)) : 0.f;
        float M0, M1, M2;
        seg_moments012_sel(ea, ec, sc - sa, M0, M1, M2);
        const bool ok0 = vc && kbase >= 1;
        Hprev = ok0 ? (gc - ga) * (M1 - M2) : 0.f;
        Bprev = ok0 ? M1 : 0.f;
      }
      uint32_t pk[4], dk[4], pk1[4], dk1[4];
#define CA_KEYS8(EDGE, OFF, SN, PN, KF, PK, DK)                                                           \
    bwd_keys8<kBF16, EDGE>(sv, pv, OFF, SN, PN, KF, i, row_ok, scale, m2, dds, sc, ec, gc, Hprev, Bprev, gsum, PK, DK)
#define CA_KEYS8_ANY_TO(OFF, SN, PN, KF, PK, DK)                                                          \
    if (interior) bwd_keys8_fast<kBF16>(sv, pv, OFF, SN, PN, scale, m2, dds, ec, Hprev, Bprev, gsum2, PK, DK); \
    else CA_KEYS8(true, OFF, SN, PN, KF, PK, DK);
#define CA_KEYS8_ANY(OFF, SN, PN, KF) CA_KEYS8_ANY_TO(OFF, SN, PN, KF, pk, dk)
      // keys 0..15 are computed before waiting for the previous tile's dV/dK/dQ products,
      // which still read the shared P/dS buffer: the 24 gradient MMAs (about 1.2k
      // tensor-pipe cycles) finish behind this work
      CA_KEYS8_ANY_TO(0, s16, p16, kbase, pk, dk);
      CA_KEYS8_ANY_TO(8, s16, p16, kbase + 8, pk1, dk1);
      if (t > 0) {
        const bool got2 = mbar_wait(&sm.bar_mma_done, (g0 + t - 1) & 1, ab);
        if (!__all_sync(0xffffffffu, got2)) { ok = false; break; }
      }
      store_chunk(prow, drow, chunk0, swz, pk, dk);
      store_chunk(prow, drow, chunk0 + 1, swz, pk1, dk1);
      // chunk 1: keys 16..31 and the right halo; S/dP in TMEM are free after this load
      uint32_t s_hi, p_hi;
      tmem_ld16(colS + 16, sv);
      tmem_ld1(colS + 32, s_hi);
      tmem_ld16(colP + 16, pv);
      tmem_ld1(colP + 32, p_hi);
      tmem_ld_wait();
      tmem_reg_fence(sv);
      tmem_reg_fence(s_hi);
      tmem_reg_fence(pv);
      tmem_reg_fence(p_hi);
      tc_fence_before();
      mbar_arrive_warp(&sm.bar_s_consumed);
      CA_KEYS8_ANY(0, s_hi, p_hi, kbase + 16);
      store_chunk(prow, drow, chunk0 + 2, swz, pk, dk);
      CA_KEYS8_ANY(8, s_hi, p_hi, kbase + 24);
      store_chunk(prow, drow, chunk0 + 3, swz, pk, dk);
#undef CA_KEYS8_ANY
#undef CA_KEYS8_ANY_TO
#undef CA_KEYS8
    }
    // dQ of the previous query tile: TMEM -> swizzled f32 staging tile, which the
    // producer adds into the global accumulator with two TMA reduces once every
    // warp has arrived on p_ready.  The staging tile is free once the reduce of
    // global tile g0+t-2 has read it.
    if (t > 0) {
      if (g0 + t > 1) {
        const bool got3 = mbar_wait(&sm.bar_dq_free, (g0 + t) & 1, ab);
        if (!__all_sync(0xffffffffu, got3)) { ok = false; break; }
      }
      uint32_t qv[16];
      tmem_ld16(tmem + lane_base + T_DQ + 16 * qk, qv);
      tmem_ld_wait();
      tmem_reg_fence(qv);
      stage_dq(sm, r, qk, qv);
    }
    fence_proxy_async_smem();
    tc_fence_before();
    mbar_arrive_warp(&sm.bar_p_ready);
  }

  // last dQ tile (staged for the producer's final reduce) and the dK / dV accumulators
  if (ok) ok = mbar_wait(&sm.bar_mma_done, (g0 + n_tiles - 1) & 1, ab);
  ok = __all_sync(0xffffffffu, ok);
  tc_fence_after();
  if (ok) {
    if (g0 + n_tiles > 1) ok = mbar_wait(&sm.bar_dq_free, (g0 + n_tiles) & 1, ab);
    ok = __all_sync(0xffffffffu, ok);
    uint32_t qv[16];
    tmem_ld16(tmem + lane_base + T_DQ + 16 * qk, qv);
    tmem_ld_wait();
    tmem_reg_fence(qv);
    if (ok) {
      stage_dq(sm, r, qk, qv);
      fence_proxy_async_smem();
      mbar_arrive_warp(&sm.bar_p_ready);
    }
  }
  {
    // warps with qk 0/1 store dV columns 32qk..32qk+31, qk 2/3 store dK columns 32(qk-2)..
    const bool is_k = qk >= 2;
    const int c0 = 32 * (qk & 1);
    uint32_t av[32];
    tmem_ld32(tmem + lane_base + (is_k ? T_DK : T_DV) + c0, av);
    tmem_ld_wait();
    tmem_reg_fence(av);
    // staged in the P buffer (free once the item's last gradient MMAs have completed)
    // as the TMA store box: dV in p[0], dK in p[1], row r = key j0 + r, 128-byte rows
    // with the 128-byte swizzle (16-byte chunk c of row r at chunk c ^ (r & 7)), so
    // that the 32 rows of a warp hit distinct banks
    uint8_t* const srow = sm.p[is_k ? 1 : 0] + (uint32_t)r * 128;
#pragma unroll
    for (int x = 0; x < 4; ++x) {
      uint32_t w[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float a0 = __uint_as_float(av[8 * x + 2 * u]), a1 = __uint_as_float(av[8 * x + 2 * u + 1]);
        w[u] = kBF16 ? pack_bf16x2(a0, a1) : pack_f16x2(a0, a1);
      }
      const int chunk = 4 * (qk & 1) + x;
      *reinterpret_cast<uint4*>(srow + ((chunk ^ (r & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
    }
    fence_proxy_async_smem();
  }
  // d log_gain partial of this key tile: sum over the CTA of dS * s (gsum holds scale * that)
  gsum = (gsum + (gsum2.x + gsum2.y)) / scale;
  for (int off = 16; off > 0; off >>= 1) gsum += __shfl_xor_sync(0xffffffffu, gsum, off);
  if (lane == 0) sm.red[warp] = gsum;
  named_bar_sync(1, NUM_MATH_WARPS * 32);
  // dK, dV out with two TMA stores (whole 128-byte rows; rows past T are not
  // written); the P buffer is reused only after they have read it (math_warps waits
  // for that at the item boundary)
  if (threadIdx.x == 0 && ok) {
    tma_store_3d(tm_dv, sm.p[0], 0, j0, bh);
    tma_store_3d(tm_dk, sm.p[1], 0, j0, bh);
    bulk_commit_group();
  }
  if (gain_part && threadIdx.x == 0) {
    float tsum = 0.f;
    for (int w = 0; w < NUM_MATH_WARPS; ++w) tsum += sm.red[w];
    gain_part[(size_t)bh * nkt + kt] = tsum;
  }
}

// The math warps' item loop.  At each item boundary thread 0 alone waits for the
// producer's published item (or gives up on an abort) and every math warp then
// takes its decision, so all of them run the same items and the same named
// barriers.
template <bool kBF16>
__device__ void math_warps(Smem& sm, const float* log_gain, const float* stats, const float* rowdot,
                           const CUtensorMap* tm_dk, const CUtensorMap* tm_dv, float* gain_part, int BH, int H, int Tn,
                           int nkt, int grp, int n_items, uint32_t tmem, float inv_sqrt_d) {
  volatile int* ab = &sm.abort_flag;
  uint32_t g0 = 0;
  uint32_t published = 0;
  bool ok = true;
  while (true) {
    named_bar_sync(2, NUM_MATH_WARPS * 32);
    if (threadIdx.x == 0) {
      // the previous item's dK/dV stores have read the P buffer, which the next
      // item's first P/dS overwrites (no bulk group: returns at once)
      bulk_wait_group_read0();
      const bool got = ok && mbar_wait(&sm.bar_item, published & 1, ab);
      sm.decision = got ? sm.item : n_items;
    }
    ++published;
    named_bar_sync(2, NUM_MATH_WARPS * 32);
    const int item = sm.decision;
    if (item >= n_items) break;
    const Item it = decode_item(item, BH, nkt, grp);
    math_item<kBF16>(sm, log_gain, stats, rowdot, tm_dk, tm_dv, gain_part, it.bh, it.bh % H, Tn, it.j0, it.kt,
                     nkt, it.n, g0, tmem, inv_sqrt_d, ok);
    ok = ok && !*ab;
    g0 += it.n;
  }
  if (threadIdx.x == 0) bulk_wait_group0();   // the last dK/dV stores have landed
}

template <bool kBF16, bool kDOB, bool kDet>
__global__ void __launch_bounds__(NUM_THREADS, 1)
bwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
           const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
           const __grid_constant__ CUtensorMap tm_dq, const __grid_constant__ CUtensorMap tm_dk,
           const __grid_constant__ CUtensorMap tm_dv, const float* __restrict__ log_gain,
           const float* __restrict__ stats, const float* __restrict__ rowdot,
           float* __restrict__ gain_part, unsigned* __restrict__ counter, unsigned* __restrict__ ready, int BH,
           int H, int Tn, float inv_sqrt_d, int grp) {
  extern __shared__ uint8_t smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nkt = (Tn + BN - 1) / BN;
  const int n_items = BH * nkt;             // (bh, key tile) pairs, heaviest (kt = 0) first

  if (warp == NUM_MATH_WARPS) {
    if (lane == 0) {
      mbar_init(&sm.bar_kv, 1);
      for (int s = 0; s < QSTAGES; ++s) mbar_init(&sm.bar_qdo[s], 1);
      mbar_init(&sm.bar_s_full, 1);
      mbar_init(&sm.bar_s_consumed, NUM_MATH_WARPS);   // one arrival per math warp
      mbar_init(&sm.bar_p_ready, NUM_MATH_WARPS);
      mbar_init(&sm.bar_mma_done, 1);
      mbar_init(&sm.bar_drain, 1);
      mbar_init(&sm.bar_dq_free, 1);
      mbar_init(&sm.bar_item, 1);
      sm.abort_flag = 0;
      fence_mbar_init();
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      tma_prefetch_desc(&tm_do);
      tma_prefetch_desc(&tm_dq);
      tma_prefetch_desc(&tm_dk);
      tma_prefetch_desc(&tm_dv);
    }
    __syncwarp();
    tmem_alloc(&sm.tmem_base, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  // the set-up above touches no global data; everything below may read or write
  // what the previous kernel in the stream produced or consumed
  pdl_wait();
  pdl_launch_dependents();

  if (warp == NUM_MATH_WARPS) {
    producer<kBF16, kDOB, kDet>(sm, &tm_q, &tm_k, &tm_v, &tm_do, &tm_dq, BH, nkt, grp, n_items, counter, ready, tmem,
                                H);   // converged
    __syncwarp();
  } else {
    math_warps<kBF16>(sm, log_gain, stats, rowdot, &tm_dk, &tm_dv, gain_part, BH, H, Tn, nkt, grp, n_items, tmem,
                      inv_sqrt_d);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == NUM_MATH_WARPS) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

}  // namespace bwd

// ------------------------------------------------------------------ host side

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

thread_local char g_map_error[160] = "";

// [BH, T, D] 16-bit tensor, box = {64 (D), box_rows, 1}, 128-byte swizzle, OOB -> 0
static bool make_map(CUtensorMap* m, const void* base, long long BH, long long T, long long D, bool bf16,
                     unsigned box_rows = 128) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) {
    snprintf(g_map_error, sizeof(g_map_error), "cuTensorMapEncodeTiled unavailable");
    return false;
  }
  cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)T, (cuuint64_t)BH};
  cuuint64_t strides[2] = {(cuuint64_t)(D * 2), (cuuint64_t)(T * D * 2)};
  cuuint32_t box[3] = {64, box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
                   const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    snprintf(g_map_error, sizeof(g_map_error), "encode %d: base %p dims %lld,%lld,%lld box %u", (int)r, base,
             (long long)D, (long long)T, (long long)BH, box_rows);
  return r == CUDA_SUCCESS;
}
const char* map_error() { return g_map_error; }

// [BH, T, D] 16-bit tensor (D = 64, T a multiple of 16) viewed as (D, s, j, chunk, BH) with
// row = 16 chunk + j + 8 s, box = {64, 2, 8, box_rows/16, 1}: a box lands in shared memory
// with key 16c+j+8s of its c-th 16-row chunk in row 16c+2j+s (128-byte swizzle, OOB -> 0)
static bool make_map_perm(CUtensorMap* m, const void* base, long long BH, long long T, bool bf16,
                          unsigned box_rows) {
  EncodeTiledFn enc = encode_fn();
  if (!enc || T % 16 != 0 || box_rows % 16 != 0) return false;
  cuuint64_t dims[5] = {64, 2, 8, (cuuint64_t)(T / 16), (cuuint64_t)BH};
  cuuint64_t strides[4] = {8 * 128, 128, 16 * 128, (cuuint64_t)(T * 128)};
  cuuint32_t box[5] = {64, 2, 8, box_rows / 16, 1};
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  CUresult r = enc(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 5,
                   const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// [B, T, H, D] 16-bit tensor viewed as (D, H, T, B), box = {64 (D), 1, box_rows, 1}: for
// one (b, h) the same box_rows rows of 128 bytes as make_map's box, 128-byte swizzle, OOB -> 0
static bool make_map_bthd(CUtensorMap* m, const void* base, long long B, long long H, long long T, long long D,
                          bool bf16, unsigned box_rows = 128) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)H, (cuuint64_t)T, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)(D * 2), (cuuint64_t)(H * D * 2), (cuuint64_t)(T * H * D * 2)};
  cuuint32_t box[4] = {64, 1, box_rows, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4,
                   const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// [BH, T, 64] f32 accumulator, box = {32, 128, 1} (128-byte rows), 128-byte swizzle
static bool make_map_f32(CUtensorMap* m, void* base, long long BH, long long T) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  cuuint64_t dims[3] = {64, (cuuint64_t)T, (cuuint64_t)BH};
  cuuint64_t strides[2] = {64 * 4, (cuuint64_t)(T * 64 * 4)};
  cuuint32_t box[3] = {32, 128, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, base, dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// The tensor-map encoder is a driver call and needs the device's context current
// on the calling thread.  A thread that has made no runtime call yet -- torch's
// autograd thread running a backward whose buffers all come from the caching
// allocator, for instance -- has none, and the encoder then fails with
// CUDA_ERROR_INVALID_CONTEXT.  cudaSetDevice on the current device binds its
// primary context to the thread.
static cudaError_t bind_context() {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  return cudaSetDevice(dev);
}

static int num_sms() { return num_sms_cached(); }

// CA_B200_NO_PERM=1 in the environment selects the unpermuted kernels for every T
// (a comparison switch for tests; read once).
static bool perm_disabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("CA_B200_NO_PERM");
    v = (e && e[0] == '1') ? 1 : 0;
  }
  return v == 1;
}

bool forward_supported(const FwdArgs& a) {
  return (a.dtype == 1 || a.dtype == 2) && a.D == 64 && aligned16(a.q) && aligned16(a.k) && aligned16(a.v) &&
         aligned16(a.o) && (!a.o_f32 || aligned16(a.o_f32)) && encode_fn() != nullptr;
}
bool backward_supported(const BwdArgs& a) {
  return (a.dtype == 1 || a.dtype == 2) && a.D == 64 && aligned16(a.q) && aligned16(a.k) && aligned16(a.v) &&
         aligned16(a.d_o) && aligned16(a.dk) && aligned16(a.dv) && encode_fn() != nullptr;
}
int forward_launches(const FwdArgs&) { return 1; }
int backward_launches(const BwdArgs&) { return 3; }   // prep, kernel, dQ cast (+ d log_gain)

// Work order over head-sequences.  Both kernels hand out their work heaviest first
// (longest query rows in the forward, key tiles with the most query tiles in the
// backward), so the CTAs running at one moment work on the same few key / query
// tile positions of every head-sequence.  At long T with many head-sequences the
// tiles they read then come from HBM once each: a [8,16,16384,64] backward runs
// at 1.15x the cost per head-sequence of a 16-head-sequence one, whose concurrent
// CTAs share each head-sequence's Q/dO tiles in L2 (forward: 1.05x, K/V tiles).
// So at T >= 4096 the head-sequences go in groups of 16, one group after another,
// each group heaviest first; shorter sequences keep one group (their whole
// working set stays in L2, and smaller groups would lengthen the tail of the
// heaviest-first order).  CA_B200_HEAD_GROUP=<n> overrides the group size
// (a tuning switch; read once).
static int head_group(long long BH, long long ntiles) {
  static int env = -1;
  if (env < 0) {
    const char* e = getenv("CA_B200_HEAD_GROUP");
    env = e ? std::max(0, atoi(e)) : 0;
  }
  long long g = env > 0 ? env : (ntiles >= 32 ? 16 : BH);
  return (int)std::max<long long>(1, std::min<long long>(g, BH));
}

// The permuted-key kernels need T a multiple of 16 (whole 16-key chunks in the 5-D view).
static bool perm_layout(long long T) { return T % 16 == 0 && !perm_disabled(); }

template <bool kBF16>
static cudaError_t launch_fwd(const FwdArgs& a) {
  cudaError_t ce = bind_context();
  if (ce != cudaSuccess) return ce;
  const long long BH = a.B * a.H;
  const bool perm = perm_layout(a.T);
  CUtensorMap mq, mk, mv;
  const bool k_ok = perm ? make_map_perm(&mk, a.k, BH, a.T, kBF16, fwd::HB) : make_map(&mk, a.k, BH, a.T, a.D, kBF16, fwd::HB);
  if (!make_map(&mq, a.q, BH, a.T, a.D, kBF16, fwd::BM) || !k_ok || !make_map(&mv, a.v, BH, a.T, a.D, kBF16, fwd::HB))
    return cudaErrorInvalidValue;
  // outputs: O ([B,H,T,D], or [B,T,H,D] through the 4-D view) and the fp32 O, stored by TMA
  CUtensorMap mo, mo32;
  const bool o_ok = a.o_bthd ? make_map_bthd(&mo, a.o, a.B, a.H, a.T, a.D, kBF16, fwd::BM)
                             : make_map(&mo, a.o, BH, a.T, a.D, kBF16, fwd::BM);
  if (!o_ok) return cudaErrorInvalidValue;
  if (a.o_f32) {
    if (!make_map_f32(&mo32, a.o_f32, BH, a.T)) return cudaErrorInvalidValue;
  } else {
    mo32 = mo;   // not read: the kernel stores no fp32 O without o_f32
  }
  auto kern = perm ? fwd::fwd_kernel<kBF16, true> : fwd::fwd_kernel<kBF16, false>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)fwd::kSmemBytes);
  if (e != cudaSuccess) return e;
  const long long nqt = (a.T + fwd::BM - 1) / fwd::BM;
  return launch_pdl(kern, dim3((unsigned)(BH * nqt)), dim3(fwd::NUM_THREADS), fwd::kSmemBytes, a.stream, mq, mk, mv,
                    mo, mo32, a.v, a.log_gain, a.o_f32, a.row_stats, (int)BH, (int)a.H, (int)a.T, a.inv_sqrt_d,
                    a.o_bthd, head_group(BH, nqt));
}

cudaError_t forward(const FwdArgs& a) { return a.dtype == 1 ? launch_fwd<true>(a) : launch_fwd<false>(a); }

thread_local const char* g_bwd_stage = "";
thread_local char g_bwd_stage_buf[256];
const char* backward_stage() {
  snprintf(g_bwd_stage_buf, sizeof(g_bwd_stage_buf), "%s%s%s", g_bwd_stage, g_map_error[0] ? "; " : "", g_map_error);
  return g_bwd_stage_buf;
}

template <bool kBF16>
static cudaError_t launch_bwd(const BwdArgs& a, const BwdWorkspace& w) {
  g_bwd_stage = "context";
  g_map_error[0] = 0;
  cudaError_t ce = bind_context();
  if (ce != cudaSuccess) return ce;
  const long long BH = a.B * a.H;
  CUtensorMap mq, mk, mv, mdo, mdq, mdk, mdv;
  g_bwd_stage = "tensor map of dO";
  const bool do_ok = a.act_bthd ? make_map_bthd(&mdo, a.d_o, a.B, a.H, a.T, a.D, kBF16, bwd::BM)
                                : make_map(&mdo, a.d_o, BH, a.T, a.D, kBF16, bwd::BM);
  if (!do_ok) return cudaErrorInvalidValue;
  g_bwd_stage = "tensor map of q";
  if (!make_map(&mq, a.q, BH, a.T, a.D, kBF16, bwd::BM)) return cudaErrorInvalidValue;
  g_bwd_stage = "tensor map of k";
  if (!make_map(&mk, a.k, BH, a.T, a.D, kBF16, bwd::KH)) return cudaErrorInvalidValue;
  g_bwd_stage = "tensor map of v";
  if (!make_map(&mv, a.v, BH, a.T, a.D, kBF16, bwd::KH)) return cudaErrorInvalidValue;
  g_bwd_stage = "tensor maps of dk, dv";
  if (!make_map(&mdk, a.dk, BH, a.T, a.D, kBF16, bwd::BN) || !make_map(&mdv, a.dv, BH, a.T, a.D, kBF16, bwd::BN))
    return cudaErrorInvalidValue;
  g_bwd_stage = "tensor map of the dQ accumulator";
  if (!make_map_f32(&mdq, w.dq_acc, BH, a.T)) return cudaErrorInvalidValue;
  g_bwd_stage = "prep";
  // deterministic: the dQ accumulator is written by stores (key tile 0 first), not zeroed
  cudaError_t e = simt::launch_prep(a, w.rowdot, a.deterministic ? nullptr : w.dq_acc, w.counter, w.ready,
                                    w.n_ready);
  if (e != cudaSuccess) return e;
  g_bwd_stage = "kernel";
  auto kern = a.deterministic ? (a.act_bthd ? bwd::bwd_kernel<kBF16, true, true> : bwd::bwd_kernel<kBF16, false, true>)
                              : (a.act_bthd ? bwd::bwd_kernel<kBF16, true, false> : bwd::bwd_kernel<kBF16, false, false>);
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bwd::kSmemBytes);
  if (e != cudaSuccess) return e;
  const long long nkt = (a.T + bwd::BN - 1) / bwd::BN;
  const long long n_items = BH * nkt;
  // persistent: one CTA per SM (at most one per work item); items beyond the first
  // gridDim.x come from the counter, which the prep kernel has zeroed
  const unsigned grid = (unsigned)std::min<long long>(n_items, num_sms());
  e = launch_pdl(kern, dim3(grid), dim3(bwd::NUM_THREADS), bwd::kSmemBytes, a.stream, mq, mk, mv, mdo, mdq, mdk,
                 mdv, a.log_gain, a.row_stats, (const float*)w.rowdot, a.dlog_gain ? w.gain_part : nullptr,
                 w.counter, w.ready, (int)BH, (int)a.H, (int)a.T, a.inv_sqrt_d, head_group(BH, nkt));
  if (e != cudaSuccess) return e;
  g_bwd_stage = "cast";
  return simt::launch_cast_dq(a, w.dq_acc, w.gain_part, (int)nkt);
}

cudaError_t backward(const BwdArgs& a, const BwdWorkspace& w) {
  return a.dtype == 1 ? launch_bwd<true>(a, w) : launch_bwd<false>(a, w);
}

// Self-test of the bounded waits: one CTA waits on an mbarrier that nothing
// arrives on.  The wait gives up after limit_ns, records CA_ERR_DEVICE_TIMEOUT in
// the status word and the kernel returns -- no fault, trap or hang -- so a test
// can check that a timed-out device wait is reported and leaves the context usable.
__global__ void wait_timeout_selftest_kernel(unsigned long long limit_ns) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x < 32) mbar_wait(&bar, 0, &abort_flag, limit_ns);
}

cudaError_t launch_wait_timeout_selftest(unsigned long long limit_ns, cudaStream_t s) {
  wait_timeout_selftest_kernel<<<1, 32, 0, s>>>(limit_ns);
  return cudaGetLastError();
}

}  // namespace sm100

cudaError_t read_device_status(int* out, bool reset) {
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return e;
  e = cudaMemcpyFromSymbol(out, sm100::g_device_status, sizeof(int));
  if (e != cudaSuccess || !reset) return e;
  const int zero = 0;
  return cudaMemcpyToSymbol(sm100::g_device_status, &zero, sizeof(int));
}

}  // namespace ca
