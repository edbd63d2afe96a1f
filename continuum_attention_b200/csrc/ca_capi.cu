// ca_capi.cu -- the extern "C" entry points declared in
// include/continuum_attention_b200.h: argument validation, workspace layout
// and dispatch between the SIMT and tcgen05 kernel families.
//
// Error behaviour mirrors the reference binding (TORCH_CHECK on dtype, shape
// and contiguity, then C10_CUDA_KERNEL_LAUNCH_CHECK after each launch,
// cuda/continuum_attention.py:460-605): every check failure returns a status
// code and leaves a message for ca_last_error(); nothing is launched after a
// failed check.
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <initializer_list>
#include <string>

#include "ca_internal.h"
#include "continuum_attention_b200.h"

namespace {

thread_local std::string g_last_error;
thread_local int g_last_launches = 0;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int ok() {
  g_last_error.clear();
  return CA_OK;
}

int cuda_fail(cudaError_t e, const char* where) {
  return fail(CA_ERR_CUDA, "%s: %s (%s)", where, cudaGetErrorString(e), cudaGetErrorName(e));
}

constexpr size_t kAlign = 256;
constexpr long long kMinKeyTile = 64;  // smallest key tile of any backward kernel

size_t align_up(size_t x) { return (x + kAlign - 1) / kAlign * kAlign; }

struct Layout {
  size_t rowdot, dq_acc, gain_part, counter, ready, total;
  int nparts;
};

Layout workspace_layout(long long B, long long H, long long T, long long D) {
  Layout l;
  const size_t rows = (size_t)B * H * T;
  l.nparts = (int)((T + kMinKeyTile - 1) / kMinKeyTile);
  l.rowdot = 0;
  l.dq_acc = align_up(l.rowdot + rows * sizeof(float));
  l.gain_part = align_up(l.dq_acc + rows * (size_t)D * sizeof(float));
  l.counter = align_up(l.gain_part + (size_t)B * H * l.nparts * sizeof(float));
  l.ready = align_up(l.counter + sizeof(unsigned));
  l.total = align_up(l.ready + (size_t)B * H * l.nparts * sizeof(unsigned));
  return l;
}

int check_shape(long long B, long long H, long long T, long long D, int dtype, int impl) {
  if (B < 0 || H < 0 || T < 0 || D < 0)
    return fail(CA_ERR_INVALID_ARGUMENT, "negative shape [B,H,T,D]=[%lld,%lld,%lld,%lld]", B, H, T, D);
  if (D == 0 && B * H * T > 0) return fail(CA_ERR_INVALID_ARGUMENT, "head dim D must be >= 1");
  if (dtype < CA_DTYPE_F32 || dtype > CA_DTYPE_F16)
    return fail(CA_ERR_INVALID_ARGUMENT, "unknown dtype code %d", dtype);
  if (impl < CA_IMPL_AUTO || impl > CA_IMPL_TCGEN05)
    return fail(CA_ERR_INVALID_ARGUMENT, "unknown impl code %d", impl);
  if (D > 128) return fail(CA_ERR_UNSUPPORTED, "head dim D=%lld > 128 is not supported", D);
  if (T > (1LL << 30)) return fail(CA_ERR_UNSUPPORTED, "sequence length T=%lld too large", T);
  const long long BH = B * H;
  const long long tiles = BH * ((T + 63) / 64);
  if (tiles > 0x7fffffffLL) return fail(CA_ERR_UNSUPPORTED, "B*H*ceil(T/64)=%lld exceeds the grid", tiles);
  return CA_OK;
}

}  // namespace

extern "C" {

int ca_abi_version(void) { return CA_ABI_VERSION; }

const char* ca_last_error(void) { return g_last_error.c_str(); }

int ca_row_stats_floats(void) { return 2; }

int ca_last_launch_count(void) { return g_last_launches; }

static int check_layout(const char* fn, int layout) {
  if (layout != CA_LAYOUT_BHTD && layout != CA_LAYOUT_BTHD)
    return fail(CA_ERR_INVALID_ARGUMENT, "%s: unknown activation layout code %d", fn, layout);
  return CA_OK;
}

static int forward_impl(const void* q, const void* k, const void* v, const float* log_gain, void* o,
                        float* o_f32, float* row_stats, int64_t B, int64_t H, int64_t T, int64_t D,
                        int dtype, int impl, void* stream, int layout) {
  int st = check_shape(B, H, T, D, dtype, impl);
  if (st != CA_OK) return st;
  st = check_layout("ca_forward", layout);
  if (st != CA_OK) return st;
  if (B * H * T == 0) return ok();
  if (!q || !k || !v || !log_gain || !o)
    return fail(CA_ERR_INVALID_ARGUMENT, "ca_forward: null q/k/v/log_gain/o pointer");
  ca::FwdArgs a{q, k, v, log_gain, o, o_f32, row_stats, B, H, T, D, dtype,
                (float)(1.0 / std::sqrt((double)D)), (cudaStream_t)stream, layout};
  cudaError_t e;
  g_last_launches = 0;
  if (impl == CA_IMPL_SIMT) {
    e = ca::simt::forward(a);
    g_last_launches = ca::simt::kForwardLaunches;
  } else if (ca::sm100::forward_supported(a)) {
    e = ca::sm100::forward(a);
    g_last_launches = ca::sm100::forward_launches(a);
  } else if (impl == CA_IMPL_TCGEN05) {
    return fail(CA_ERR_UNSUPPORTED,
                "ca_forward: tcgen05 kernels need bf16/f16, D in {64}, 16-byte aligned buffers "
                "(got dtype=%d D=%lld)", dtype, (long long)D);
  } else {
    e = ca::simt::forward(a);
    g_last_launches = ca::simt::kForwardLaunches;
  }
  if (e != cudaSuccess) return cuda_fail(e, "ca_forward launch");
  return ok();
}

int ca_forward(const void* q, const void* k, const void* v, const float* log_gain, void* o,
               float* o_f32, float* row_stats, int64_t B, int64_t H, int64_t T, int64_t D,
               int dtype, int impl, void* stream) {
  return forward_impl(q, k, v, log_gain, o, o_f32, row_stats, B, H, T, D, dtype, impl, stream, CA_LAYOUT_BHTD);
}

int ca_forward_ex(const void* q, const void* k, const void* v, const float* log_gain, void* o,
                  float* o_f32, float* row_stats, int64_t B, int64_t H, int64_t T, int64_t D,
                  int dtype, int impl, int layout, void* stream) {
  return forward_impl(q, k, v, log_gain, o, o_f32, row_stats, B, H, T, D, dtype, impl, stream, layout);
}

size_t ca_backward_workspace_size(int64_t B, int64_t H, int64_t T, int64_t D, int dtype) {
  (void)dtype;
  if (B <= 0 || H <= 0 || T <= 0 || D <= 0) return 0;
  return workspace_layout(B, H, T, D).total;
}

static int backward_impl(const void* q, const void* k, const void* v, const void* o, const float* o_f32,
                         const void* d_o, const float* log_gain, const float* row_stats, void* dq, void* dk,
                         void* dv, float* dlog_gain, void* workspace, size_t workspace_bytes, int64_t B,
                         int64_t H, int64_t T, int64_t D, int dtype, int impl, void* stream, int layout,
                         int flags = 0) {
  int st = check_shape(B, H, T, D, dtype, impl);
  if (st != CA_OK) return st;
  st = check_layout("ca_backward", layout);
  if (st != CA_OK) return st;
  if (flags & ~CA_BWD_DETERMINISTIC) return fail(CA_ERR_INVALID_ARGUMENT, "ca_backward: unknown flags 0x%x", flags);
  const bool det = (flags & CA_BWD_DETERMINISTIC) != 0;
  cudaStream_t s = (cudaStream_t)stream;
  if (B * H * T == 0) {
    if (dlog_gain && H > 0) {
      cudaError_t e = cudaMemsetAsync(dlog_gain, 0, (size_t)H * sizeof(float), s);
      if (e != cudaSuccess) return cuda_fail(e, "ca_backward memset");
    }
    return ok();
  }
  if (!q || !k || !v || (!o && !o_f32) || !d_o || !log_gain || !row_stats || !dq || !dk || !dv)
    return fail(CA_ERR_INVALID_ARGUMENT, "ca_backward: null tensor pointer");
  const Layout l = workspace_layout(B, H, T, D);
  if (!workspace || workspace_bytes < l.total)
    return fail(CA_ERR_WORKSPACE, "ca_backward: workspace of %zu bytes < required %zu", workspace_bytes,
                l.total);
  if (((uintptr_t)workspace) % kAlign != 0)
    return fail(CA_ERR_INVALID_ARGUMENT, "ca_backward: workspace must be %zu-byte aligned", kAlign);
  char* ws = (char*)workspace;
  ca::BwdWorkspace w{(float*)(ws + l.rowdot), (float*)(ws + l.dq_acc), (float*)(ws + l.gain_part),
                     l.nparts, (unsigned*)(ws + l.counter), (unsigned*)(ws + l.ready), (int)(B * H * l.nparts)};
  ca::BwdArgs a{q, k, v, o, o_f32, d_o, log_gain, row_stats, dq, dk, dv, dlog_gain, B, H, T, D, dtype,
                (float)(1.0 / std::sqrt((double)D)), s, layout, det ? 1 : 0};
  cudaError_t e;
  g_last_launches = 0;
  const bool tc = impl != CA_IMPL_SIMT && ca::sm100::backward_supported(a);
  if (det && !tc)
    return fail(CA_ERR_UNSUPPORTED,
                "ca_backward: a deterministic backward needs the tcgen05 kernels (bf16/f16, D = 64, 16-byte "
                "aligned buffers); the CUDA-core kernels add dQ with atomics (dtype=%d D=%lld impl=%d)",
                dtype, (long long)D, impl);
  if (impl == CA_IMPL_SIMT) {
    e = ca::simt::backward(a, w);
    g_last_launches = ca::simt::backward_launches(a);
  } else if (tc) {
    e = ca::sm100::backward(a, w);
    g_last_launches = ca::sm100::backward_launches(a);
    if (e != cudaSuccess) {
      char where[320];
      snprintf(where, sizeof(where), "ca_backward launch (tcgen05 %s)", ca::sm100::backward_stage());
      return cuda_fail(e, where);
    }
  } else if (impl == CA_IMPL_TCGEN05) {
    return fail(CA_ERR_UNSUPPORTED, "ca_backward: tcgen05 kernels do not cover dtype=%d D=%lld", dtype,
                (long long)D);
  } else {
    e = ca::simt::backward(a, w);
    g_last_launches = ca::simt::backward_launches(a);
  }
  if (e != cudaSuccess) return cuda_fail(e, "ca_backward launch");
  return ok();
}

int ca_backward(const void* q, const void* k, const void* v, const void* o, const float* o_f32,
                const void* d_o, const float* log_gain, const float* row_stats, void* dq, void* dk, void* dv,
                float* dlog_gain, void* workspace, size_t workspace_bytes, int64_t B, int64_t H,
                int64_t T, int64_t D, int dtype, int impl, void* stream) {
  return backward_impl(q, k, v, o, o_f32, d_o, log_gain, row_stats, dq, dk, dv, dlog_gain, workspace,
                       workspace_bytes, B, H, T, D, dtype, impl, stream, CA_LAYOUT_BHTD);
}

int ca_backward_ex(const void* q, const void* k, const void* v, const void* o, const float* o_f32,
                   const void* d_o, const float* log_gain, const float* row_stats, void* dq, void* dk, void* dv,
                   float* dlog_gain, void* workspace, size_t workspace_bytes, int64_t B, int64_t H,
                   int64_t T, int64_t D, int dtype, int impl, int layout, void* stream) {
  return backward_impl(q, k, v, o, o_f32, d_o, log_gain, row_stats, dq, dk, dv, dlog_gain, workspace,
                       workspace_bytes, B, H, T, D, dtype, impl, stream, layout);
}

int ca_backward_ex2(const void* q, const void* k, const void* v, const void* o, const float* o_f32,
                    const void* d_o, const float* log_gain, const float* row_stats, void* dq, void* dk, void* dv,
                    float* dlog_gain, void* workspace, size_t workspace_bytes, int64_t B, int64_t H,
                    int64_t T, int64_t D, int dtype, int impl, int layout, int flags, void* stream) {
  return backward_impl(q, k, v, o, o_f32, d_o, log_gain, row_stats, dq, dk, dv, dlog_gain, workspace,
                       workspace_bytes, B, H, T, D, dtype, impl, stream, layout, flags);
}

static int check_rope(const char* fn, const void* a, const void* b, const void* c, const void* d,
                      const float* cs, int64_t B, int64_t T, int64_t H, int64_t D, int dtype) {
  if (B < 0 || T < 0 || H < 0 || D < 0)
    return fail(CA_ERR_INVALID_ARGUMENT, "%s: negative shape [B,T,H,D]=[%lld,%lld,%lld,%lld]", fn, (long long)B,
                (long long)T, (long long)H, (long long)D);
  if (dtype < CA_DTYPE_F32 || dtype > CA_DTYPE_F16)
    return fail(CA_ERR_INVALID_ARGUMENT, "%s: unknown dtype code %d", fn, dtype);
  if (D % 8 != 0 || D > 256)
    return fail(CA_ERR_UNSUPPORTED, "%s: head dim D=%lld must be a multiple of 8 and <= 256", fn, (long long)D);
  // the kernels index tokens (b*T + t) and per-token work items (3*H*D/8) in 32 bits
  if (T > 0x7fffffffLL || (T > 0 && B > 0x7fffffffLL / T))
    return fail(CA_ERR_UNSUPPORTED, "%s: B*T=%lld*%lld tokens exceed 2^31-1", fn, (long long)B, (long long)T);
  if (H > (1LL << 20))
    return fail(CA_ERR_UNSUPPORTED, "%s: H=%lld heads exceed 2^20", fn, (long long)H);
  if (B * T * H * D == 0) return CA_OK;
  if (!a || !b || !c || !d || !cs) return fail(CA_ERR_INVALID_ARGUMENT, "%s: null pointer", fn);
  const uintptr_t m = (uintptr_t)a | (uintptr_t)b | (uintptr_t)c | (uintptr_t)d | (uintptr_t)cs;
  if (m & 15) return fail(CA_ERR_INVALID_ARGUMENT, "%s: buffers must be 16-byte aligned", fn);
  return CA_OK;
}

int ca_rope_qkv_forward(const void* qkv, const float* cos_sin, void* q, void* k, void* v, int64_t B, int64_t T,
                        int64_t H, int64_t D, int dtype, void* stream) {
  int st = check_rope("ca_rope_qkv_forward", qkv, q, k, v, cos_sin, B, T, H, D, dtype);
  if (st != CA_OK) return st;
  g_last_launches = 0;
  if (B * T * H * D == 0) return ok();
  cudaError_t e = ca::rope::forward(qkv, cos_sin, q, k, v, B, T, H, D, dtype, (cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_fail(e, "ca_rope_qkv_forward launch");
  g_last_launches = 1;
  return ok();
}

int ca_rope_qkv_backward(const void* dq, const void* dk, const void* dv, const float* cos_sin, void* dqkv,
                         int64_t B, int64_t T, int64_t H, int64_t D, int dtype, void* stream) {
  int st = check_rope("ca_rope_qkv_backward", dq, dk, dv, dqkv, cos_sin, B, T, H, D, dtype);
  if (st != CA_OK) return st;
  g_last_launches = 0;
  if (B * T * H * D == 0) return ok();
  cudaError_t e = ca::rope::backward(dq, dk, dv, cos_sin, dqkv, B, T, H, D, dtype, (cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_fail(e, "ca_rope_qkv_backward launch");
  g_last_launches = 1;
  return ok();
}

static int check_norm(const char* fn, int64_t rows, int64_t D, int x_dtype, int y_dtype) {
  if (rows < 0 || D < 0)
    return fail(CA_ERR_INVALID_ARGUMENT, "%s: negative shape [rows,D]=[%lld,%lld]", fn, (long long)rows,
                (long long)D);
  if ((x_dtype != CA_DTYPE_F32 && x_dtype != CA_DTYPE_BF16) || (y_dtype != CA_DTYPE_F32 && y_dtype != CA_DTYPE_BF16))
    return fail(CA_ERR_UNSUPPORTED, "%s: dtypes must be float32 or bfloat16 (codes %d, %d)", fn, x_dtype, y_dtype);
  if (!ca::norm::supported_dim(D))
    return fail(CA_ERR_UNSUPPORTED, "%s: D=%lld must be 128, 256, 512 or 1024", fn, (long long)D);
  return CA_OK;
}

static bool all_aligned16(std::initializer_list<const void*> ps) {
  uintptr_t m = 0;
  for (const void* p : ps) m |= (uintptr_t)p;
  return (m & 15) == 0;
}

size_t ca_rmsnorm_workspace_size(int64_t rows, int64_t D) {
  if (rows <= 0 || D <= 0) return 0;
  return align_up(ca::norm::workspace_floats(rows, D) * sizeof(float));
}

int ca_rmsnorm_forward(const void* x, const float* w, void* y, float* rstd, int64_t rows, int64_t D, float eps,
                       int x_dtype, int y_dtype, void* stream) {
  int st = check_norm("ca_rmsnorm_forward", rows, D, x_dtype, y_dtype);
  if (st != CA_OK) return st;
  if (!(eps >= 0.f)) return fail(CA_ERR_INVALID_ARGUMENT, "ca_rmsnorm_forward: eps must be >= 0");
  g_last_launches = 0;
  if (rows == 0) return ok();
  if (!x || !w || !y || !rstd) return fail(CA_ERR_INVALID_ARGUMENT, "ca_rmsnorm_forward: null pointer");
  if (!all_aligned16({x, w, y, rstd}))
    return fail(CA_ERR_INVALID_ARGUMENT, "ca_rmsnorm_forward: buffers must be 16-byte aligned");
  cudaError_t e = ca::norm::forward(x, w, y, rstd, rows, D, eps, x_dtype, y_dtype, (cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_fail(e, "ca_rmsnorm_forward launch");
  g_last_launches = 1;
  return ok();
}

int ca_rmsnorm_backward(const void* x, const float* w, const void* dy, const float* rstd, void* dx, float* dw,
                        void* workspace, size_t workspace_bytes, int64_t rows, int64_t D, int x_dtype, int y_dtype,
                        void* stream) {
  int st = check_norm("ca_rmsnorm_backward", rows, D, x_dtype, y_dtype);
  if (st != CA_OK) return st;
  g_last_launches = 0;
  if (rows == 0) {
    if (dw && D > 0) {
      cudaError_t e = cudaMemsetAsync(dw, 0, (size_t)D * sizeof(float), (cudaStream_t)stream);
      if (e != cudaSuccess) return cuda_fail(e, "ca_rmsnorm_backward memset");
    }
    return ok();
  }
  if (!x || !w || !dy || !rstd || !dx || !dw || !workspace)
    return fail(CA_ERR_INVALID_ARGUMENT, "ca_rmsnorm_backward: null pointer");
  if (!all_aligned16({x, w, dy, rstd, dx, dw, workspace}))
    return fail(CA_ERR_INVALID_ARGUMENT, "ca_rmsnorm_backward: buffers must be 16-byte aligned");
  const size_t need = ca_rmsnorm_workspace_size(rows, D);
  if (workspace_bytes < need)
    return fail(CA_ERR_WORKSPACE, "ca_rmsnorm_backward: workspace of %zu bytes, %zu needed", workspace_bytes, need);
  cudaError_t e = ca::norm::backward(x, w, dy, rstd, dx, dw, (float*)workspace, rows, D, x_dtype, y_dtype,
                                     (cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_fail(e, "ca_rmsnorm_backward launch");
  g_last_launches = 2;
  return ok();
}

int ca_add_rmsnorm_forward(const float* x, const void* r, const float* w, float* x_new, void* y, float* rstd,
                           int64_t rows, int64_t D, float eps, void* stream) {
  int st = check_norm("ca_add_rmsnorm_forward", rows, D, CA_DTYPE_F32, CA_DTYPE_BF16);
  if (st != CA_OK) return st;
  if (!(eps >= 0.f)) return fail(CA_ERR_INVALID_ARGUMENT, "ca_add_rmsnorm_forward: eps must be >= 0");
  g_last_launches = 0;
  if (rows == 0) return ok();
  if (!x || !r || !w || !x_new || !y || !rstd)
    return fail(CA_ERR_INVALID_ARGUMENT, "ca_add_rmsnorm_forward: null pointer");
  if (!all_aligned16({x, r, w, x_new, y, rstd}))
    return fail(CA_ERR_INVALID_ARGUMENT, "ca_add_rmsnorm_forward: buffers must be 16-byte aligned");
  cudaError_t e = ca::norm::add_forward(x, r, w, x_new, y, rstd, rows, D, eps, (cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_fail(e, "ca_add_rmsnorm_forward launch");
  g_last_launches = 1;
  return ok();
}

int ca_add_rmsnorm_backward(const float* x_new, const float* w, const void* dy, const float* rstd,
                            const float* dx_new, float* dx, void* dr, float* dw, void* workspace,
                            size_t workspace_bytes, int64_t rows, int64_t D, void* stream) {
  int st = check_norm("ca_add_rmsnorm_backward", rows, D, CA_DTYPE_F32, CA_DTYPE_BF16);
  if (st != CA_OK) return st;
  g_last_launches = 0;
  if (rows == 0) {
    if (dw && D > 0) {
      cudaError_t e = cudaMemsetAsync(dw, 0, (size_t)D * sizeof(float), (cudaStream_t)stream);
      if (e != cudaSuccess) return cuda_fail(e, "ca_add_rmsnorm_backward memset");
    }
    return ok();
  }
  if (!x_new || !w || !dy || !rstd || !dx || !dr || !dw || !workspace)
    return fail(CA_ERR_INVALID_ARGUMENT, "ca_add_rmsnorm_backward: null pointer");
  if (!all_aligned16({x_new, w, dy, rstd, dx_new, dx, dr, dw, workspace}))
    return fail(CA_ERR_INVALID_ARGUMENT, "ca_add_rmsnorm_backward: buffers must be 16-byte aligned");
  const size_t need = ca_rmsnorm_workspace_size(rows, D);
  if (workspace_bytes < need)
    return fail(CA_ERR_WORKSPACE, "ca_add_rmsnorm_backward: workspace of %zu bytes, %zu needed", workspace_bytes,
                need);
  cudaError_t e = ca::norm::add_backward(x_new, w, dy, rstd, dx_new, dx, dr, dw, (float*)workspace, rows, D,
                                         (cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_fail(e, "ca_add_rmsnorm_backward launch");
  g_last_launches = 2;
  return ok();
}

int ca_selftest_wait_timeout(int64_t limit_us, void* stream) {
  if (limit_us < 1 || limit_us > 10000000)
    return fail(CA_ERR_INVALID_ARGUMENT, "ca_selftest_wait_timeout: limit_us=%lld outside [1, 1e7]",
                (long long)limit_us);
  g_last_launches = 0;
  cudaError_t e = ca::sm100::launch_wait_timeout_selftest((unsigned long long)limit_us * 1000ull,
                                                          (cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_fail(e, "ca_selftest_wait_timeout launch");
  g_last_launches = 1;
  return ok();
}

static int check_gelu(const char* fn, int64_t n, int dtype, std::initializer_list<const void*> ptrs) {
  if (dtype < CA_DTYPE_F32 || dtype > CA_DTYPE_F16) return fail(CA_ERR_INVALID_ARGUMENT, "%s: unknown dtype %d", fn, dtype);
  if (n < 0) return fail(CA_ERR_INVALID_ARGUMENT, "%s: n must be >= 0", fn);
  const int vec = ca::gelu::vector_elems(dtype);
  if (n % vec) return fail(CA_ERR_UNSUPPORTED, "%s: n must be a multiple of %d for this dtype", fn, vec);
  if (n == 0) return CA_OK;
  for (const void* p : ptrs)
    if (!p) return fail(CA_ERR_INVALID_ARGUMENT, "%s: null pointer", fn);
  if (!all_aligned16(ptrs)) return fail(CA_ERR_INVALID_ARGUMENT, "%s: buffers must be 16-byte aligned", fn);
  return CA_OK;
}

int ca_gelu_tanh_forward(const void* x, void* y, int64_t n, int dtype, void* stream) {
  g_last_launches = 0;
  int st = check_gelu("ca_gelu_tanh_forward", n, dtype, {x, y});
  if (st != CA_OK) return st;
  if (n == 0) return ok();
  cudaError_t e = ca::gelu::forward(x, y, (size_t)n, dtype, (cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_fail(e, "ca_gelu_tanh_forward launch");
  g_last_launches = 1;
  return ok();
}

int ca_gelu_tanh_backward(const void* x, const void* dy, void* dx, int64_t n, int dtype, void* stream) {
  g_last_launches = 0;
  int st = check_gelu("ca_gelu_tanh_backward", n, dtype, {x, dy, dx});
  if (st != CA_OK) return st;
  if (n == 0) return ok();
  cudaError_t e = ca::gelu::backward(x, dy, dx, (size_t)n, dtype, (cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_fail(e, "ca_gelu_tanh_backward launch");
  g_last_launches = 1;
  return ok();
}

int ca_device_status(int reset) {
  int value = 0;
  cudaError_t e = ca::read_device_status(&value, reset != 0);
  if (e != cudaSuccess) return cuda_fail(e, "ca_device_status");
  return value;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// ca_backward_noalloc: the backward pass for callers that cannot allocate
// device memory.
//
// ca_backward needs scratch space (the per-row terms D_i, the fp32 dQ
// accumulator and the per-tile gain partial sums) and expects the caller to
// pass it in.  Some callers have no way to provide it: host code that reaches
// this library only through the C interface while another component owns every
// device allocation (for example a framework's caching allocator the caller
// cannot call), or a service that fixes its device memory when it starts and
// must not call cudaMalloc later (cudaMalloc can synchronise the device and
// fails once the budget is spent).  For them the scratch lives in one fixed
// array inside this library instead.
//
// Limits and behaviour:
//   - the array holds kNoAllocScratchBytes (32 MiB); every GPU that loads this
//     library keeps it until the process exits;
//   - a problem whose scratch need (ca_backward_workspace_size) exceeds it is
//     rejected with CA_ERR_UNSUPPORTED and a message naming both sizes;
//   - the first call in a device's context looks up the array's device address
//     there (cudaGetSymbolAddress) and caches it under that context's id, so
//     make that first call before any stream capture on that device; a context
//     torn down and rebuilt (cudaDeviceReset, or a framework that recreates its
//     context) has a new id, and the next call looks the address up again -- that
//     call, too, belongs before any stream capture;
//   - all calls on a device share the one array and leave their contents in
//     it; the backward clears what must start at zero (the dQ accumulator)
//     itself, but two calls whose work overlaps on the GPU (different streams
//     with no ordering between them) race on the array and give wrong results;
//   - nothing here calls cudaMalloc, cudaFree or an allocating library routine.
#include <cuda.h>

#include <mutex>

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(32) << 20;
constexpr int kNoAllocMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

struct NoAllocSlot {
  bool valid;
  unsigned long long ctx_id;   // id of the context the address belongs to
  void* ptr;
};

std::mutex g_noalloc_mutex;
NoAllocSlot g_noalloc_slot[kNoAllocMaxDevices] = {};

typedef CUresult (*CtxGetCurrentFn)(CUcontext*);
typedef CUresult (*CtxGetIdFn)(CUcontext, unsigned long long*);

// Unique id of the calling thread's current context (cuCtxGetId, through the
// runtime's driver entry points); false when there is none or the driver lacks the call.
bool current_context_id(unsigned long long* id) {
  static CtxGetCurrentFn get_current = nullptr;
  static CtxGetIdFn get_id = nullptr;
  static bool looked_up = false;
  if (!looked_up) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<CtxGetCurrentFn>(p);
    p = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<CtxGetIdFn>(p);
    looked_up = true;
  }
  if (!get_current || !get_id) return false;
  CUcontext ctx = nullptr;
  if (get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr) return false;
  return get_id(ctx, id) == CUDA_SUCCESS;
}

// Device address of g_noalloc_scratch in the current device's context.  Looked
// up once per context and cached under the context's id; without a context id
// (a driver that lacks cuCtxGetId) it is looked up on every call.
int noalloc_scratch_here(void** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "ca_backward_noalloc: cudaGetDevice");
  if (dev < 0 || dev >= kNoAllocMaxDevices)
    return fail(CA_ERR_UNSUPPORTED, "ca_backward_noalloc: device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  NoAllocSlot& slot = g_noalloc_slot[dev];
  unsigned long long id = 0;
  if (slot.valid && current_context_id(&id) && id == slot.ctx_id) {
    *out = slot.ptr;
    return CA_OK;
  }
  void* p = nullptr;
  e = cudaGetSymbolAddress(&p, g_noalloc_scratch);   // makes the device's context current if it is not
  if (e != cudaSuccess) return cuda_fail(e, "ca_backward_noalloc: cudaGetSymbolAddress of the scratch array");
  if (!p) return fail(CA_ERR_CUDA, "ca_backward_noalloc: scratch array has no device address");
  slot.ptr = p;
  slot.valid = current_context_id(&slot.ctx_id);
  *out = p;
  return CA_OK;
}

}  // namespace

extern "C" int ca_backward_noalloc(const void* q, const void* k, const void* v, const void* o,
                                   const float* o_f32, const void* d_o, const float* log_gain,
                                   const float* row_stats, void* dq, void* dk, void* dv, float* dlog_gain,
                                   int64_t B, int64_t H, int64_t T, int64_t D, int dtype, int impl,
                                   void* stream) {
  int st = check_shape(B, H, T, D, dtype, impl);
  if (st != CA_OK) return st;
  const size_t need = ca_backward_workspace_size(B, H, T, D, dtype);
  if (need > kNoAllocScratchBytes)
    return fail(CA_ERR_UNSUPPORTED,
                "ca_backward_noalloc: [B,H,T,D]=[%lld,%lld,%lld,%lld] needs %zu bytes of scratch, more than "
                "the library's fixed %zu-byte array; call ca_backward with a workspace instead",
                (long long)B, (long long)H, (long long)T, (long long)D, need, kNoAllocScratchBytes);
  void* scratch = nullptr;
  if (need > 0) {
    st = noalloc_scratch_here(&scratch);
    if (st != CA_OK) return st;
  }
  return ca_backward(q, k, v, o, o_f32, d_o, log_gain, row_stats, dq, dk, dv, dlog_gain, scratch,
                     kNoAllocScratchBytes, B, H, T, D, dtype, impl, stream);
}
