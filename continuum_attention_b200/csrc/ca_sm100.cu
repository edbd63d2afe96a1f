// ca_sm100.cu -- sm_100a tensor-core Continuum Attention kernels (bf16 / f16,
// head dim 64): TMA-staged Q/K/V tiles, tcgen05.mma with TMEM accumulators.
//
// Forward, one CTA per 128-row query tile (two CTAs per SM):
//   warp 4 (one elected lane) is the producer: TMA loads of Q (once) and of
//     K/V tiles into a 2-stage ring, and the tcgen05.mma issue:
//       S(j)  = Q K_j^T              128x128 fp32 in TMEM columns [0,128)
//       O    += P_hi(j) V'_j + P_lo(j) V'_j   128x64 fp32 in TMEM columns [128,192)
//     where V'_j is the V tile staged one row early (keys j0-1 .. j0+126) and
//     P(j) is written by the math warps over the same TMEM columns as S(j).
//   warps 0-3 (thread = query row = TMEM lane) load their S row, keep an online
//     row max (rescaling O only when the max grows by more than 8 nats), form
//     the segment moments, and store P split into bf16 hi + lo parts, so the
//     P V product keeps ~16 significant bits of every weight.
// P column c of key tile j0 holds the weight of key j0-1+c:
//   P[c] = B_{j0+c-1} + A_{j0+c} (+ half caps on key 0 and key i),
// with A_k = M0-M1 and B_k = M1 of segment k (key k-1 -> key k); B of the last
// key of a tile is carried to the next tile, and a weight still pending after
// the diagonal tile (query i on the last column) is added in the epilogue.
// Replaces the reference's per-query-tile chain bmm(QK^T) -> scale ->
// ca_forward_half_kernel -> bmm(W V) (cuda/continuum_attention.py:670-690).
//
// Every mbarrier wait is bounded (2 s); on expiry the kernel records
// CA_ERR_DEVICE_TIMEOUT in g_device_status, stops issuing work, waits (bounded)
// for its own in-flight copies and MMAs, frees its TMEM and returns.
#include <cuda.h>

#include "ca_common.cuh"
#include "ca_internal.h"
#include "ca_sm100_ptx.cuh"

namespace ca {
namespace sm100 {

namespace fwd {

constexpr int BM = 128;            // query rows per CTA (= TMEM lanes)
constexpr int BN = 128;            // keys per tile
constexpr int HD = 64;             // head dim
constexpr int STAGES = 2;
constexpr int NUM_THREADS = 160;   // 4 math warps + 1 producer warp
constexpr uint32_t TILE_BYTES = BN * HD * 2;
constexpr uint32_t TMEM_COLS = 256;
constexpr uint32_t TMEM_S = 0;     // S(j): columns [0,128); P_hi(j) overwrites [0,64)
constexpr uint32_t TMEM_O = 128;   // O accumulator: columns [128,192)
constexpr uint32_t TMEM_PLO = 192; // P_lo(j): columns [192,256)
constexpr float kRescaleNats = 8.0f;

struct __align__(1024) Smem {
  uint8_t q[TILE_BYTES];
  uint8_t k[STAGES][TILE_BYTES];
  uint8_t v[STAGES][TILE_BYTES];
  uint64_t bar_q;
  uint64_t bar_k[STAGES];
  uint64_t bar_v[STAGES];
  uint64_t bar_kv_free[STAGES];
  uint64_t bar_s_full;
  uint64_t bar_p_ready;
  uint64_t bar_o_done;
  uint32_t tmem_base;
  int abort_flag;
};

constexpr size_t kSmemBytes = sizeof(Smem) + 1024;  // + alignment slack

__device__ __forceinline__ void issue_s(uint32_t q_saddr, uint32_t k_saddr, uint32_t d_tmem, uint32_t idesc) {
#pragma unroll
  for (int kk = 0; kk < HD / 16; ++kk) {
    const uint64_t a = sdesc_sw128(q_saddr + kk * 32, 16, 1024);
    const uint64_t b = sdesc_sw128(k_saddr + kk * 32, 16, 1024);
    mma_ss(d_tmem, a, b, idesc, kk > 0 ? 1u : 0u);
  }
}

__device__ __forceinline__ void issue_pv(uint32_t o_tmem, uint32_t p_tmem, uint32_t v_saddr, uint32_t idesc,
                                         bool accumulate) {
#pragma unroll
  for (int part = 0; part < 2; ++part) {
#pragma unroll
    for (int kk = 0; kk < BN / 16; ++kk) {
      const uint64_t b = sdesc_sw128(v_saddr + kk * 2048, 16384, 1024);   // V: MN-major
      const uint32_t acc = (accumulate || part > 0 || kk > 0) ? 1u : 0u;
      mma_ts(o_tmem, p_tmem + (part ? TMEM_PLO : TMEM_S) + kk * 8, b, idesc, acc);
    }
  }
}

template <bool kBF16>
__device__ void producer(Smem& sm, const CUtensorMap* tq, const CUtensorMap* tk, const CUtensorMap* tv, int bh,
                         int q0, int n_tiles, uint32_t tmem) {
  volatile int* ab = &sm.abort_flag;
  const uint32_t id_s = make_idesc(BM, BN, kBF16, false);
  const uint32_t id_o = make_idesc(BM, HD, kBF16, true);
  bool k_pending[STAGES] = {false, false}, v_pending[STAGES] = {false, false};
  uint32_t k_phase[STAGES] = {0, 0}, v_phase[STAGES] = {0, 0};
  bool q_pending = true;
  bool mma_issued = false;

  mbar_arrive_expect_tx(&sm.bar_q, TILE_BYTES);
  tma_load_3d(sm.q, tq, &sm.bar_q, 0, q0, bh);
  for (int t = 0; t < STAGES && t < n_tiles; ++t) {
    mbar_arrive_expect_tx(&sm.bar_k[t], TILE_BYTES);
    tma_load_3d(sm.k[t], tk, &sm.bar_k[t], 0, t * BN, bh);
    mbar_arrive_expect_tx(&sm.bar_v[t], TILE_BYTES);
    tma_load_3d(sm.v[t], tv, &sm.bar_v[t], 0, t * BN - 1, bh);
    k_pending[t] = v_pending[t] = true;
  }
  const uint32_t q_sa = smem_u32(sm.q);
  const uint32_t s_tmem = tmem + TMEM_S, o_tmem = tmem + TMEM_O;

  if (mbar_wait(&sm.bar_q, 0, ab) && mbar_wait(&sm.bar_k[0], 0, ab)) {
    q_pending = false;
    k_pending[0] = false;
    k_phase[0] ^= 1;
    tc_fence_after();
    issue_s(q_sa, smem_u32(sm.k[0]), s_tmem, id_s);
    mma_commit(&sm.bar_s_full);
    mma_issued = true;
    for (int j = 0; j < n_tiles; ++j) {
      const int st = j % STAGES;
      if (!mbar_wait(&sm.bar_p_ready, j & 1, ab)) break;
      if (!mbar_wait(&sm.bar_v[st], v_phase[st], ab)) break;
      v_pending[st] = false;
      v_phase[st] ^= 1;
      tc_fence_after();
      issue_pv(o_tmem, tmem, smem_u32(sm.v[st]), id_o, j > 0);
      mma_commit(&sm.bar_kv_free[st]);
      if (j + 1 < n_tiles) {
        const int st1 = (j + 1) % STAGES;
        if (!mbar_wait(&sm.bar_k[st1], k_phase[st1], ab)) break;
        k_pending[st1] = false;
        k_phase[st1] ^= 1;
        tc_fence_after();
        issue_s(q_sa, smem_u32(sm.k[st1]), s_tmem, id_s);
        mma_commit(&sm.bar_s_full);
      }
      if (j + STAGES < n_tiles) {
        // stage st is free once S(j) and PV(j) have consumed it
        if (!mbar_wait(&sm.bar_kv_free[st], (j / STAGES) & 1, ab)) break;
        const int t = j + STAGES;
        mbar_arrive_expect_tx(&sm.bar_k[st], TILE_BYTES);
        tma_load_3d(sm.k[st], tk, &sm.bar_k[st], 0, t * BN, bh);
        mbar_arrive_expect_tx(&sm.bar_v[st], TILE_BYTES);
        tma_load_3d(sm.v[st], tv, &sm.bar_v[st], 0, t * BN - 1, bh);
        k_pending[st] = v_pending[st] = true;
      }
    }
  }
  // completion of every MMA issued so far (also the epilogue's "O ready" signal)
  mma_commit(&sm.bar_o_done);
  // drain: in-flight TMA copies must land before the CTA's shared memory goes away
  int dummy_abort = 0;
  volatile int* nab = &dummy_abort;
  if (q_pending) mbar_wait(&sm.bar_q, 0, nab);
  for (int s = 0; s < STAGES; ++s) {
    if (k_pending[s]) mbar_wait(&sm.bar_k[s], k_phase[s], nab);
    if (v_pending[s]) mbar_wait(&sm.bar_v[s], v_phase[s], nab);
  }
  (void)mma_issued;
  mbar_wait(&sm.bar_o_done, 0, nab);
}

template <bool kBF16>
__device__ void math_warps(Smem& sm, const void* vptr, const float* log_gain, void* optr, float* o32, float* stats,
                           int bh, int h, int Tn, int q0, int n_tiles, uint32_t tmem, float inv_sqrt_d) {
  volatile int* ab = &sm.abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = warp * 32 + lane;
  const int i = q0 + r;
  const bool row_ok = i < Tn;
  const float scale = expf(log_gain[h]) * inv_sqrt_d;
  const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
  const uint32_t tS = tmem + TMEM_S + lane_base;
  const uint32_t tO = tmem + TMEM_O + lane_base;

  float m_used = -INFINITY, z = 0.f, bpend = 0.f, sprev = 0.f;
  bool ok = true;
  for (int j = 0; j < n_tiles; ++j) {
    const bool got = mbar_wait(&sm.bar_s_full, j & 1, ab);
    if (!__all_sync(0xffffffffu, got)) { ok = false; break; }
    tc_fence_after();
    const int j0 = j * BN;
    const bool diag = (j == n_tiles - 1);
    const int nvis = diag ? min(i - j0 + 1, BN) : BN;
    // pass 1: tile max over the visible keys
    uint32_t sr[2][32];
    float tmax = -INFINITY;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      tmem_ld32(tS + 32 * c, sr[0]);
      tmem_ld_wait();
#pragma unroll
      for (int x = 0; x < 32; ++x)
        if (32 * c + x < nvis) tmax = fmaxf(tmax, __uint_as_float(sr[0][x]));
    }
    tmax *= scale;
    const bool need = tmax > m_used + kRescaleNats;
    if (j == 0) {
      m_used = tmax;
    } else if (__any_sync(0xffffffffu, need)) {
      const float m_new = need ? tmax : m_used;
      const float alpha = exp_rel(m_used - m_new);
      z *= alpha;
      bpend *= alpha;
      m_used = m_new;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        tmem_ld32(tO + 32 * half, sr[1]);
        tmem_ld_wait();
#pragma unroll
        for (int x = 0; x < 32; ++x) sr[1][x] = __float_as_uint(__uint_as_float(sr[1][x]) * alpha);
        tmem_st32(tO + 32 * half, sr[1]);
      }
    }
    const float m2 = m_used * kLog2e;
    float sa = sprev;
    float ea = (j0 > 0) ? ex2_approx(fmaf(sprev, kLog2e, -m2)) : 0.f;
    float bprev = bpend;
    // pass 2: P for 16 keys at a time; the next chunk's load overlaps this chunk's math
    auto chunk = [&](const uint32_t (&cur)[16], int ch) {
      uint32_t hi[8], lo[8];
#pragma unroll
      for (int x = 0; x < 16; x += 2) {
        float pv[2];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int c = 16 * ch + x + u;
          const float sb = __uint_as_float(cur[x + u]) * scale;
          const bool vis = c < nvis;
          const float eb = vis ? ex2_approx(fmaf(sb, kLog2e, -m2)) : 0.f;
          float M0, M1;
          seg_moments01(ea, eb, sb - sa, M0, M1);
          const bool seg_ok = vis && (j0 + c) >= 1;
          float p = bprev + (seg_ok ? M0 - M1 : 0.f);
          z += seg_ok ? M0 : 0.f;
          if (c >= 1) {
            const int key = j0 - 1 + c;
            const float cap = 0.5f * ea * ((key == 0 ? 1.f : 0.f) + (key == i ? 1.f : 0.f));
            p += cap;
            z += cap;
          }
          pv[u] = p;
          bprev = seg_ok ? M1 : 0.f;
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
      tmem_st8(tS + 8 * ch, hi);
      tmem_st8(tmem + TMEM_PLO + lane_base + 8 * ch, lo);
    };
    uint32_t bufA[16], bufB[16];
    tmem_ld16(tS, bufA);
    tmem_ld_wait();
#pragma unroll 1
    for (int ch = 0; ch < 8; ch += 2) {
      tmem_ld16(tS + 16 * (ch + 1), bufB);
      chunk(bufA, ch);
      tmem_ld_wait();
      if (ch + 2 < 8) tmem_ld16(tS + 16 * (ch + 2), bufA);
      chunk(bufB, ch + 1);
      tmem_ld_wait();
    }
    if (diag && i == j0 + BN - 1) {   // cap of key i sits in the last column: keep it pending
      bprev += 0.5f * ea;
      z += 0.5f * ea;
    }
    bpend = bprev;
    sprev = sa;
    tmem_st_wait();
    tc_fence_before();
    mbar_arrive(&sm.bar_p_ready);
  }

  if (ok) ok = mbar_wait(&sm.bar_o_done, 0, ab);
  tc_fence_after();
  uint32_t oa[2][32];
  tmem_ld32(tO, oa[0]);
  tmem_ld32(tO + 32, oa[1]);
  tmem_ld_wait();
  if (!ok || !row_ok) return;
  float acc[HD];
#pragma unroll
  for (int d = 0; d < HD; ++d) acc[d] = __uint_as_float(oa[d / 32][d % 32]);
  const size_t row = (size_t)bh * Tn + i;
  if (bpend != 0.f) {
    const uint16_t* vr = reinterpret_cast<const uint16_t*>(vptr) + row * HD;
#pragma unroll
    for (int d = 0; d < HD; ++d) {
      const uint32_t bits = (uint32_t)vr[d];
      float vv;
      if (kBF16) vv = __uint_as_float(bits << 16);
      else vv = __half2float(__ushort_as_half((unsigned short)bits));
      acc[d] = fmaf(bpend, vv, acc[d]);
    }
  }
  const float inv = 1.f / z;
  uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(optr) + row * HD);
#pragma unroll
  for (int c = 0; c < HD / 8; ++c) {
    uint32_t w[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const float a0 = acc[8 * c + 2 * u] * inv, a1 = acc[8 * c + 2 * u + 1] * inv;
      w[u] = kBF16 ? pack_bf16x2(a0, a1) : pack_f16x2(a0, a1);
    }
    dst[c] = make_uint4(w[0], w[1], w[2], w[3]);
  }
  if (o32) {
    float4* d32 = reinterpret_cast<float4*>(o32 + row * HD);
#pragma unroll
    for (int c = 0; c < HD / 4; ++c)
      d32[c] = make_float4(acc[4 * c] * inv, acc[4 * c + 1] * inv, acc[4 * c + 2] * inv, acc[4 * c + 3] * inv);
  }
  stats[2 * row] = m_used;
  stats[2 * row + 1] = z;
}

template <bool kBF16>
__global__ void __launch_bounds__(NUM_THREADS, 2)
fwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
           const __grid_constant__ CUtensorMap tm_v, const void* __restrict__ vptr,
           const float* __restrict__ log_gain, void* __restrict__ optr, float* __restrict__ o32,
           float* __restrict__ stats, int BH, int H, int Tn, float inv_sqrt_d) {
  extern __shared__ uint8_t smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nqt = (Tn + BM - 1) / BM;
  const int bh = blockIdx.x % BH;
  const int qt = nqt - 1 - blockIdx.x / BH;   // heaviest query tiles first
  const int q0 = qt * BM;
  const int n_tiles = qt + 1;                 // key tiles 0..qt (BN == BM)

  if (warp == 4) {
    if (lane == 0) {
      mbar_init(&sm.bar_q, 1);
      for (int s = 0; s < STAGES; ++s) {
        mbar_init(&sm.bar_k[s], 1);
        mbar_init(&sm.bar_v[s], 1);
        mbar_init(&sm.bar_kv_free[s], 1);
      }
      mbar_init(&sm.bar_s_full, 1);
      mbar_init(&sm.bar_p_ready, 128);
      mbar_init(&sm.bar_o_done, 1);
      sm.abort_flag = 0;
      fence_mbar_init();
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
    }
    __syncwarp();
    tmem_alloc(&sm.tmem_base, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;

  if (warp == 4) {
    if (lane == 0) producer<kBF16>(sm, &tm_q, &tm_k, &tm_v, bh, q0, n_tiles, tmem);
    __syncwarp();
  } else {
    math_warps<kBF16>(sm, vptr, log_gain, optr, o32, stats, bh, bh % H, Tn, q0, n_tiles, tmem, inv_sqrt_d);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 4) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

}  // namespace fwd

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

// [BH, T, D] 16-bit tensor, box = {64 (D), 128 (rows), 1}, 128-byte swizzle, OOB -> 0
static bool make_map(CUtensorMap* m, const void* base, long long BH, long long T, long long D, bool bf16) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)T, (cuuint64_t)BH};
  cuuint64_t strides[2] = {(cuuint64_t)(D * 2), (cuuint64_t)(T * D * 2)};
  cuuint32_t box[3] = {64, 128, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
                   const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

bool forward_supported(const FwdArgs& a) {
  return (a.dtype == 1 || a.dtype == 2) && a.D == 64 && aligned16(a.q) && aligned16(a.k) && aligned16(a.v) &&
         aligned16(a.o) && (!a.o_f32 || aligned16(a.o_f32)) && encode_fn() != nullptr;
}
bool backward_supported(const BwdArgs&) { return false; }
int forward_launches(const FwdArgs&) { return 1; }
int backward_launches(const BwdArgs&) { return 0; }

template <bool kBF16>
static cudaError_t launch_fwd(const FwdArgs& a) {
  const long long BH = a.B * a.H;
  CUtensorMap mq, mk, mv;
  if (!make_map(&mq, a.q, BH, a.T, a.D, kBF16) || !make_map(&mk, a.k, BH, a.T, a.D, kBF16) ||
      !make_map(&mv, a.v, BH, a.T, a.D, kBF16))
    return cudaErrorInvalidValue;
  auto kern = fwd::fwd_kernel<kBF16>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)fwd::kSmemBytes);
  if (e != cudaSuccess) return e;
  const long long nqt = (a.T + fwd::BM - 1) / fwd::BM;
  kern<<<dim3((unsigned)(BH * nqt)), fwd::NUM_THREADS, fwd::kSmemBytes, a.stream>>>(
      mq, mk, mv, a.v, a.log_gain, a.o, a.o_f32, a.row_stats, (int)BH, (int)a.H, (int)a.T, a.inv_sqrt_d);
  return cudaGetLastError();
}

cudaError_t forward(const FwdArgs& a) { return a.dtype == 1 ? launch_fwd<true>(a) : launch_fwd<false>(a); }
cudaError_t backward(const BwdArgs&, const BwdWorkspace&) { return cudaErrorNotSupported; }

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
