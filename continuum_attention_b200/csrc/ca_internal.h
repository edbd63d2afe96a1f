// ca_internal.h -- argument bundles passed from the C ABI (ca_capi.cu) to the
// kernel families (ca_simt.cu, ca_sm100.cu).  Not part of the public ABI.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace ca {

struct FwdArgs {
  const void* q;
  const void* k;
  const void* v;
  const float* log_gain;
  void* o;
  float* o_f32;
  float* row_stats;  // [B*H*T][2] = (row max m, normaliser Z relative to m)
  long long B, H, T, D;
  int dtype;         // enum ca_dtype
  float inv_sqrt_d;  // float32(1/sqrt(D)), as the reference's D**-0.5 scalar
  cudaStream_t stream;
  int o_bthd;        // o stored [B,T,H,D] instead of [B,H,T,D] (o_f32 stays [B,H,T,D])
};

struct BwdArgs {
  const void* q;
  const void* k;
  const void* v;
  const void* o;
  const float* o_f32;  // may be null: then D_i uses o
  const void* d_o;
  const float* log_gain;
  const float* row_stats;
  void* dq;
  void* dk;
  void* dv;
  float* dlog_gain;  // may be null
  long long B, H, T, D;
  int dtype;
  float inv_sqrt_d;
  cudaStream_t stream;
  int act_bthd;        // o and d_o stored [B,T,H,D] instead of [B,H,T,D] (o_f32 stays [B,H,T,D])
  int deterministic;   // dQ summed in a fixed order (tcgen05 kernels; bitwise reproducible)
};

// Carved out of the caller's workspace (ca_capi.cu: workspace_layout).
struct BwdWorkspace {
  float* rowdot;     // [B*H*T]      D_i = dO_i . O_i
  float* dq_acc;     // [B*H*T*D]    fp32 dQ accumulator
  float* gain_part;  // [B*H*nparts] per-(head, key tile) partial sums of dS*s
  int nparts;
  unsigned* counter; // work-item counter of the persistent tcgen05 backward (zeroed by prep)
  unsigned* ready;   // [B*H*nparts] per (head, query tile): dQ contributions added so far (zeroed by prep)
  int n_ready;
};

// Launch with programmatic stream serialisation (the kernel calls pdl_wait()
// before its first global-memory access).
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                              Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

namespace simt {
constexpr int kForwardLaunches = 1;
inline int backward_launches(const BwdArgs&) { return 3; }   // prep, kernel, dQ cast (+ d log_gain)
cudaError_t forward(const FwdArgs& a);
cudaError_t backward(const BwdArgs& a, const BwdWorkspace& w);
// backward helpers shared with the tcgen05 path
// D_i = dO_i . O_i; dq_acc = 0 (when dq_acc != nullptr); *counter = 0 and ready[0 .. n_ready) = 0
// (when counter != nullptr)
cudaError_t launch_prep(const BwdArgs& a, float* rowdot, float* dq_acc, unsigned* counter, unsigned* ready = nullptr,
                        int n_ready = 0);
// fp32 dQ -> dtype, and (when a.dlog_gain) d log_gain from the per-key-tile partials, one launch
cudaError_t launch_cast_dq(const BwdArgs& a, const float* dq_acc, const float* gain_part, int nparts);
}  // namespace simt

namespace sm100 {
// true when the tcgen05 kernels cover this problem (dtype, D, alignment)
bool forward_supported(const FwdArgs& a);
bool backward_supported(const BwdArgs& a);
int forward_launches(const FwdArgs& a);
int backward_launches(const BwdArgs& a);
cudaError_t forward(const FwdArgs& a);
cudaError_t backward(const BwdArgs& a, const BwdWorkspace& w);
// which step of the calling thread's last backward() ran last (for error messages)
const char* backward_stage();
// one CTA whose bounded mbarrier wait runs out after limit_ns (nothing completes the barrier)
cudaError_t launch_wait_timeout_selftest(unsigned long long limit_ns, cudaStream_t s);
}  // namespace sm100

// SM count of the calling thread's current device (cached per device)
inline int num_sms_cached() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cached[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cached[dev] = n;
  }
  return cached[dev];
}

namespace rope {
// qkv [B][T][3][H][D] -> q, k (rotary embedding applied), v [B][H][T][D]; cos_sin float32 [T][D/2][2]
cudaError_t forward(const void* qkv, const float* cos_sin, void* q, void* k, void* v, long long B, long long T,
                    long long H, long long D, int dtype, cudaStream_t s);
// dq, dk, dv [B][H][T][D] -> dqkv [B][T][3][H][D] (transposed rotation on dq, dk)
cudaError_t backward(const void* dq, const void* dk, const void* dv, const float* cos_sin, void* dqkv,
                     long long B, long long T, long long H, long long D, int dtype, cudaStream_t s);
}  // namespace rope

namespace norm {
// RMSNorm over the last axis (D in {128, 256, 512, 1024}); dtype codes as the ABI's
// (0 f32, 1 bf16): x in x_dtype, y / dy in y_dtype, w / dw / rstd float32.
bool supported_dim(long long D);
cudaError_t forward(const void* x, const float* w, void* y, float* rstd, long long rows, long long D, float eps,
                    int x_dtype, int y_dtype, cudaStream_t s);
cudaError_t backward(const void* x, const float* w, const void* dy, const float* rstd, void* dx, float* dw,
                     float* dw_part, long long rows, long long D, int x_dtype, int y_dtype, cudaStream_t s);
// floats of scratch backward needs (per-block partials of dw)
size_t workspace_floats(long long rows, long long D);
// residual add fused with the norm: x_new = x + r (x, x_new float32, r bfloat16),
// y = norm(x_new) in bfloat16; backward gives dx = g_xnew + dnorm (float32) and
// dr = the same in bfloat16 (g_xnew may be null: zero); same workspace as backward.
cudaError_t add_forward(const float* x, const void* r, const float* w, float* xn, void* y, float* rstd,
                        long long rows, long long D, float eps, cudaStream_t s);
cudaError_t add_backward(const float* xn, const float* w, const void* dy, const float* rstd, const float* gxn,
                         float* dx, void* dr, float* dw, float* dw_part, long long rows, long long D, cudaStream_t s);
}  // namespace norm

namespace gelu {
// tanh-approximate GELU over n contiguous elements (dtype codes as the ABI's);
// n a multiple of vector_elems(dtype), buffers 16-byte aligned
int vector_elems(int dtype);
cudaError_t forward(const void* x, void* y, size_t n, int dtype, cudaStream_t s);
cudaError_t backward(const void* x, const void* dy, void* dx, size_t n, int dtype, cudaStream_t s);
}  // namespace gelu

cudaError_t read_device_status(int* out, bool reset);

}  // namespace ca
