/*
 * continuum_attention_b200.h -- C ABI of the B200 (sm_100a) Continuum
 * Attention operator.
 *
 * The operator computes causal Continuum Attention over [B,H,T,D] tensors:
 * scores s_ij = exp(log_gain[h]) * q_i.k_j / sqrt(D), keys and values
 * linearly interpolated between adjacent positions, exact per-segment
 * exponential moments, half-token caps on the first and the last visible key,
 * row normalisation, y = W V.  Backward is the analytic VJP.
 *
 * This ABI replaces the reference's pybind torch extension and the per-tile
 * autograd loop around it:
 *   - ca_forward  replaces _CAExactTiled.forward (cuda/continuum_attention.py:651-694)
 *                 together with the kernels it drives: ca_scale_scores_half_kernel
 *                 (:81-90), ca_weights_kernel (:136-163), ca_forward_half_kernel
 *                 (:300-328), ca_direct_output_kernel (:412-457) and the torch.bmm
 *                 GEMMs QK^T and W V (:677-690).
 *   - ca_backward replaces _CAExactTiled.backward (:696-766) with
 *                 ca_backward_fused_kernel (:230-293), ca_backward_half_kernel
 *                 (:337-405), ca_scores_backward_kernel (:192-223) and the five
 *                 torch.bmm GEMMs plus prefix add_ accumulations (:720-764).
 *   - the Python binding that the reference loads with load_inline (:608-620,
 *     pybind module :35-63) becomes a ctypes binding of this library.
 *
 * Conventions
 *   - All tensor arguments are device pointers owned by the caller, contiguous
 *     row-major [B,H,T,D] for q/k/v/o/do/dq/dk/dv.  The library never
 *     allocates device memory; scratch space is passed in by the caller.
 *   - dtype selects the element type of q/k/v/o/do/dq/dk/dv (all the same).
 *   - log_gain is float32 [H] on the device: scale_h = exp(log_gain[h])/sqrt(D).
 *     The fixed-tau variant passes log(1/tau) for every head.
 *   - stream is a cudaStream_t (NULL = legacy default stream).  All work is
 *     enqueued on it; the calls return without synchronising.
 *   - Return value 0 = success; otherwise a CA_ERR_* code and a message that
 *     ca_last_error() returns (thread-local, valid until the next call on the
 *     same thread).
 *   - Stateless and reentrant: calls on different streams from different host
 *     threads are safe, given disjoint output and workspace buffers.
 */
#ifndef CONTINUUM_ATTENTION_B200_H
#define CONTINUUM_ATTENTION_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define CA_ABI_VERSION 1

/* element types of q/k/v/o/do/dq/dk/dv */
enum ca_dtype { CA_DTYPE_F32 = 0, CA_DTYPE_BF16 = 1, CA_DTYPE_F16 = 2 };

/* status codes */
enum ca_status {
  CA_OK = 0,
  CA_ERR_INVALID_ARGUMENT = 1, /* null pointer, bad shape, misaligned buffer */
  CA_ERR_UNSUPPORTED = 2,      /* shape/dtype outside what the kernels cover */
  CA_ERR_CUDA = 3,             /* a CUDA runtime call or a launch failed */
  CA_ERR_WORKSPACE = 4,        /* workspace smaller than ca_backward_workspace_size() */
  CA_ERR_DEVICE_TIMEOUT = 5    /* a bounded device-side wait gave up (see ca_device_status) */
};

/* Kernel family used by a call (ca_forward / ca_backward 'impl' argument). */
enum ca_impl {
  CA_IMPL_AUTO = 0,   /* tcgen05 tensor-core kernels where they apply, else SIMT */
  CA_IMPL_SIMT = 1,   /* CUDA-core kernels: every dtype, D <= 128, fp32 arithmetic */
  CA_IMPL_TCGEN05 = 2 /* sm_100a tcgen05/TMEM/TMA kernels: bf16/f16, D = 64 */
};

/* Storage order of the activations o (forward output, backward input) and d_o
 * (ca_forward_ex / ca_backward_ex): [B,H,T,D] like q, k, v, or [B,T,H,D], the
 * order in which a decoder's output projection reads the attention output.
 * o_f32, q, k, v and the gradients dq, dk, dv are always [B,H,T,D]. */
enum ca_layout { CA_LAYOUT_BHTD = 0, CA_LAYOUT_BTHD = 1 };

/* Version of this ABI (CA_ABI_VERSION of the built library). */
int ca_abi_version(void);

/* Message of the last failed call on this thread ("" if none). */
const char* ca_last_error(void);

/* Number of float32 per query row in the row-statistics buffer that
 * ca_forward writes and ca_backward reads ([B*H*T * ca_row_stats_floats()]). */
int ca_row_stats_floats(void);

/*
 * Forward.  o = CA(q, k, v) [B,H,T,D] in dtype; row_stats receives the
 * per-row statistics the backward needs (row max and normaliser).  For
 * inference row_stats may be NULL: nothing but o (and o_f32) is written.
 * o_f32 (optional, may be NULL) additionally receives the float32
 * accumulator before the final rounding to dtype (o is exactly the
 * round-to-nearest-even of o_f32 when both are written).
 * Replaces _CAExactTiled.forward, cuda/continuum_attention.py:651-694.
 */
int ca_forward(const void* q, const void* k, const void* v, const float* log_gain,
               void* o, float* o_f32, float* row_stats,
               int64_t B, int64_t H, int64_t T, int64_t D,
               int dtype, int impl, void* stream);

/* ca_forward with o written in the given ca_layout.  CA_LAYOUT_BTHD replaces the
 * copy the reference decoder makes of the attention output before its output
 * projection (y.transpose(1, 2).contiguous(), cuda/continuum_attention.py:854):
 * o [B][T][H][D] is that projection's input as it stands. */
int ca_forward_ex(const void* q, const void* k, const void* v, const float* log_gain,
                  void* o, float* o_f32, float* row_stats,
                  int64_t B, int64_t H, int64_t T, int64_t D,
                  int dtype, int impl, int layout, void* stream);

/* Bytes of scratch space ca_backward needs for this shape (>= 0). */
size_t ca_backward_workspace_size(int64_t B, int64_t H, int64_t T, int64_t D, int dtype);

/*
 * Backward.  Given the forward's o and row_stats and the upstream gradient
 * do, writes dq, dk, dv ([B,H,T,D], dtype) and, if dlog_gain is not NULL,
 * d loss / d log_gain [H] in float32 (summed over the batch).
 * o_f32 (optional, may be NULL) is the forward's float32 accumulator; when
 * given, the row terms D_i = do_i . o_i use it instead of the dtype-rounded o
 * (which may then be NULL), keeping bf16/f16 score gradients free of the
 * output rounding.
 * workspace must hold ca_backward_workspace_size() bytes (256-byte aligned);
 * its contents on entry are ignored, and it belongs to this call until the
 * call's GPU work has finished (calls whose work may overlap on the GPU need
 * separate workspaces: the backward's work counter lives there too).
 * Replaces _CAExactTiled.backward, cuda/continuum_attention.py:696-766.
 */
int ca_backward(const void* q, const void* k, const void* v, const void* o, const float* o_f32,
                const void* d_o, const float* log_gain, const float* row_stats,
                void* dq, void* dk, void* dv, float* dlog_gain,
                void* workspace, size_t workspace_bytes,
                int64_t B, int64_t H, int64_t T, int64_t D,
                int dtype, int impl, void* stream);

/* ca_backward with o and d_o read in the given ca_layout (the layout ca_forward_ex
 * wrote o in; with CA_LAYOUT_BTHD d_o is the output projection's input gradient as
 * it stands, [B][T][H][D], instead of its transposed copy). */
int ca_backward_ex(const void* q, const void* k, const void* v, const void* o, const float* o_f32,
                   const void* d_o, const float* log_gain, const float* row_stats,
                   void* dq, void* dk, void* dv, float* dlog_gain,
                   void* workspace, size_t workspace_bytes,
                   int64_t B, int64_t H, int64_t T, int64_t D,
                   int dtype, int impl, int layout, void* stream);

/* Flags of ca_backward_ex2. */
enum ca_backward_flags {
  /* dQ summed in one fixed order, so every output is bitwise reproducible run to
   * run (dK, dV and d log_gain always are): each dQ tile takes its key tiles'
   * contributions in ascending key-tile order.  Needs the tcgen05 kernels
   * (bf16/f16, D = 64); with the CUDA-core kernels the call returns
   * CA_ERR_UNSUPPORTED. */
  CA_BWD_DETERMINISTIC = 1
};

/* ca_backward_ex with flags (ca_backward_flags).  Replaces the same reference code
 * as ca_backward; CA_BWD_DETERMINISTIC is the counterpart of the fixed per-tile
 * accumulation order of the reference backward (gq add_ per query tile,
 * cuda/continuum_attention.py:754-764). */
int ca_backward_ex2(const void* q, const void* k, const void* v, const void* o, const float* o_f32,
                    const void* d_o, const float* log_gain, const float* row_stats,
                    void* dq, void* dk, void* dv, float* dlog_gain,
                    void* workspace, size_t workspace_bytes,
                    int64_t B, int64_t H, int64_t T, int64_t D,
                    int dtype, int impl, int layout, int flags, void* stream);

/*
 * Backward without caller-provided scratch.  No counterpart in the reference
 * (its backward allocates through torch inside the extension).
 * Same arguments and results as ca_backward minus the workspace.  It is meant
 * for callers that cannot allocate device memory: code that reaches this
 * library only through the C interface while something else owns all device
 * allocations, or a service whose device memory is fixed at start-up and must
 * not call cudaMalloc afterwards.  The scratch is a fixed 32 MiB array inside
 * the library (held on every GPU that loads it until the process exits);
 * problems whose ca_backward_workspace_size() exceeds it return
 * CA_ERR_UNSUPPORTED.  The first call in a device's context looks up the
 * array's device address and caches it under the context's id, so make it
 * before any stream capture on that device; after the context is torn down and
 * rebuilt (cudaDeviceReset) the next call looks it up again and belongs before
 * any capture as well.  All calls on
 * a device share the array: calls whose GPU work overlaps (unordered streams)
 * race and produce wrong results.  It allocates nothing.
 */
int ca_backward_noalloc(const void* q, const void* k, const void* v, const void* o, const float* o_f32,
                        const void* d_o, const float* log_gain, const float* row_stats,
                        void* dq, void* dk, void* dv, float* dlog_gain,
                        int64_t B, int64_t H, int64_t T, int64_t D,
                        int dtype, int impl, void* stream);

/*
 * CA-S decoder attention block, input side: rotary position embedding fused
 * with the unpacking of the QKV projection.  Replaces apply_rope
 * (cuda/continuum_attention.py:825-835) together with the reshape / permute /
 * unbind of ContinuumSelfAttention.forward (:850-852) and the contiguity
 * copies continuum_attention makes of its operands (:783).
 *   qkv      [B][T][3][H][D]  the projection output (q, k, v along axis 2)
 *   cos_sin  float32 [T][D/2][2]: (cos, sin)(t * theta^(-2p/D)) for pair p
 *   q, k, v  [B][H][T][D] outputs; q and k rotated pairwise
 *            (x_{2p}, x_{2p+1}) -> (x_{2p} c - x_{2p+1} s, x_{2p+1} c + x_{2p} s)
 * dtype as for the operator; D a multiple of 8, at most 256; every buffer
 * 16-byte aligned.  One launch, no allocation.
 */
int ca_rope_qkv_forward(const void* qkv, const float* cos_sin, void* q, void* k, void* v,
                        int64_t B, int64_t T, int64_t H, int64_t D, int dtype, void* stream);

/* Gradient of ca_rope_qkv_forward: dq, dk, dv [B][H][T][D] -> dqkv
 * [B][T][3][H][D] with the transposed rotation on dq and dk. */
int ca_rope_qkv_backward(const void* dq, const void* dk, const void* dv, const float* cos_sin, void* dqkv,
                         int64_t B, int64_t T, int64_t H, int64_t D, int dtype, void* stream);

/*
 * CA-S decoder block RMSNorm (cuda/continuum_attention.py:815-821, the module
 * RMSNorm: y = w * x * rsqrt(mean(x^2) + eps) over the last axis).  No
 * reference counterpart in native code: the reference runs it as separate torch
 * kernels.  x [rows][D] in x_dtype, y [rows][D] in y_dtype (float32 or
 * bfloat16 each: the block writes the bfloat16 input of the next projection
 * directly), w float32 [D], rstd float32 [rows] (written by the forward, read by
 * the backward).  D in {128, 256, 512, 1024}; buffers 16-byte aligned.
 * The backward writes dx [rows][D] (x_dtype) and dw float32 [D] (summed over
 * rows in a fixed order) and needs ca_rmsnorm_workspace_size() bytes of
 * scratch.  One launch forward, two backward, no allocation.
 */
size_t ca_rmsnorm_workspace_size(int64_t rows, int64_t D);
int ca_rmsnorm_forward(const void* x, const float* w, void* y, float* rstd, int64_t rows, int64_t D, float eps,
                       int x_dtype, int y_dtype, void* stream);
int ca_rmsnorm_backward(const void* x, const float* w, const void* dy, const float* rstd, void* dx, float* dw,
                        void* workspace, size_t workspace_bytes, int64_t rows, int64_t D, int x_dtype, int y_dtype,
                        void* stream);

/*
 * The residual add before a pre-norm block's norm, fused with it: x_new = x + r,
 * y = w * x_new * rsqrt(mean(x_new^2) + eps) (the reference block's
 * `x = x + self.attn(...)` / `x + self.mlp(...)` followed by the next RMSNorm,
 * cuda/continuum_attention.py:815-821 and the block's forward).  x, x_new float32
 * (the residual stream), r and y bfloat16 (a branch output and the next
 * projection's input under bf16 autocast), w float32 [D], rstd float32 [rows];
 * D in {128, 256, 512, 1024}.  The backward takes the gradient of y (dy,
 * bfloat16) and of x_new where it is used further on (dx_new, float32, NULL for
 * none), and writes dx (float32) and dr (bfloat16), both equal to dx_new plus the
 * norm's input gradient, and dw; scratch as ca_rmsnorm_workspace_size().
 */
int ca_add_rmsnorm_forward(const float* x, const void* r, const float* w, float* x_new, void* y, float* rstd,
                           int64_t rows, int64_t D, float eps, void* stream);
int ca_add_rmsnorm_backward(const float* x_new, const float* w, const void* dy, const float* rstd,
                            const float* dx_new, float* dx, void* dr, float* dw, void* workspace,
                            size_t workspace_bytes, int64_t rows, int64_t D, void* stream);

/*
 * Tanh-approximate GELU, the CA-S decoder MLP's activation
 * (cuda/continuum_attention.py:866-867, F.gelu(fc1(x), approximate='tanh')):
 * y = 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))) elementwise over n
 * contiguous elements, fp32 arithmetic; the backward gives dx = dy * gelu'(x).
 * dtype CA_DTYPE_*; n a multiple of 16 bytes' worth of elements (4 fp32, 8
 * bf16/fp16) and every buffer 16-byte aligned.  One launch each.
 */
int ca_gelu_tanh_forward(const void* x, void* y, int64_t n, int dtype, void* stream);
int ca_gelu_tanh_backward(const void* x, const void* dy, void* dx, int64_t n, int dtype, void* stream);

/* Number of kernels the last successful ca_forward / ca_backward /
 * ca_rope_qkv_* / ca_rmsnorm_* / ca_add_rmsnorm_* / ca_gelu_tanh_* call on this
 * thread enqueued (memsets excluded).  Diagnostic for launch accounting. */
int ca_last_launch_count(void);

/*
 * Device status word of the calling thread's current device: 0 if every
 * bounded device-side wait since the last reset completed, else a CA_ERR_*
 * code recorded by a kernel that gave up waiting.  Synchronises the device.
 * reset != 0 clears the word after reading it.
 */
int ca_device_status(int reset);

/*
 * Diagnostics (no reference counterpart): enqueue one CTA that waits, with the
 * kernels' bounded-wait routine, on an mbarrier nothing ever completes.  The
 * wait gives up after limit_us microseconds (1 .. 1e7), records
 * CA_ERR_DEVICE_TIMEOUT in the device status word and the kernel returns, so a
 * caller can check that device-side timeouts are reported by
 * ca_device_status() and that the context stays usable.  No fault, trap or
 * hang is involved.
 */
int ca_selftest_wait_timeout(int64_t limit_us, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* CONTINUUM_ATTENTION_B200_H */
