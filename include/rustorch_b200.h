/*
 * rustorch_b200 — C ABI of the B200 (sm_100a) dense-contraction backend for
 * RusTorch.  Plain pointers and sizes only; every function returns an int
 * status (RTB_OK = 0).  Device pointers are CUDA device addresses on the
 * context's device; `stream` is a cudaStream_t (NULL = the legacy default
 * stream, as in the CUDA runtime; rtb_context_stream gives the context's own
 * non-blocking stream).  All compute entry points are asynchronous and stream-ordered like
 * cuBLAS: errors detected on the host (bad shapes, launch failures) are
 * returned immediately; a device-side bounded wait that expired is reported by
 * the next rtb_stream_synchronize / rtb_device_error on that context.
 *
 * Reference interfaces replaced (paths relative to the RusTorch project root):
 *   ops::matmul                 rustorch-core/src/ops.rs:1888      -> rtb_sgemm
 *   ops::matmul_fused           rustorch-core/src/ops.rs:1543      -> rtb_sgemm (bias, act)
 *   nn::Linear::forward         rustorch-nn/src/linear.rs:75-95    -> rtb_sgemm (transB=1)
 *   ops::conv2d                 rustorch-core/src/ops/conv.rs:738  -> rtb_conv2d_fwd
 *   nn::Conv2d::forward         rustorch-nn/src/conv.rs:52-63      -> rtb_conv2d_fwd (bias)
 *   jit Conv2dRelu lowering     rustorch-core/src/jit.rs:254-262   -> rtb_conv2d_fwd (act=ReLU)
 *   ops::max_pool2d             rustorch-core/src/ops/pool.rs:115  -> rtb_max_pool2d
 *   ops::add (same shape)       rustorch-core/src/ops.rs:223       -> rtb_add
 *   ops::relu                   rustorch-core/src/ops.rs:449       -> rtb_relu
 *   Storage / Device::Cuda      rustorch-core/src/storage.rs:13-43,201-216 -> rtb_malloc/memcpy
 *   rustorch-cuda extern "C"    rustorch-cuda/src/lib.rs:1-8       -> this header
 */
#ifndef RUSTORCH_B200_H
#define RUSTORCH_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct rtb_ctx rtb_ctx;

/* Status codes.  The reference panics on these conditions (e.g.
 * "Matmul dimension mismatch", rustorch-core/src/ops.rs:1898); the Rust shim
 * turns a non-zero status into the same panic. */
enum {
  RTB_OK = 0,
  RTB_E_INVALID = 1,     /* bad argument or shape */
  RTB_E_OOM = 2,         /* device or host allocation failed */
  RTB_E_CUDA = 3,        /* CUDA runtime / driver error */
  RTB_E_TIMEOUT = 4,     /* a device-side bounded wait expired */
  RTB_E_UNSUPPORTED = 5, /* valid request the library does not implement */
  RTB_E_NCCL = 6         /* NCCL error */
};

/* backend::Activation (rustorch-core/src/backend/mod.rs:1-7).  Every entry
 * point that takes `act` applies all four in its epilogue, after the bias and
 * residual: RELU = max(x, 0) (NaN -> 0), SIGMOID = 1/(1+exp(-x)), TANH
 * (matmul_fused's staged activation, rustorch-core/src/ops.rs:1703-1708). */
enum { RTB_ACT_NONE = 0, RTB_ACT_RELU = 1, RTB_ACT_SIGMOID = 2, RTB_ACT_TANH = 3 };

/* Contraction precision.  3xTF32 (default) splits every fp32 operand into a
 * TF32 high part and an fp32 remainder and accumulates hi*hi + hi*lo + lo*hi
 * on the tensor cores (relative Frobenius error vs f64 <= 1e-5); TF32 is the
 * opt-in fast mode (<= 5e-3).  RTB_PREC_DEFAULT reads RUSTORCH_B200_PRECISION
 * ("3xtf32" | "tf32") once per context. */
enum { RTB_PREC_3XTF32 = 0, RTB_PREC_TF32 = 1, RTB_PREC_DEFAULT = -1 };

/* Activation tensor layouts for conv / pooling. */
enum { RTB_LAYOUT_NCHW = 0, RTB_LAYOUT_NHWC = 1 };

/* ---------------------------------------------------------------- context */
/* Create a context on `device` (owns a stream, an error word and the
 * stream-ordered workspace pool).  Thread-safe to use from many threads. */
int rtb_init(int device, rtb_ctx** out);
int rtb_destroy(rtb_ctx* ctx);
int rtb_device_count(int* count);
int rtb_get_device_info(rtb_ctx* ctx, int* sm_count, int* cc_major, int* cc_minor,
                        size_t* total_mem);
const char* rtb_status_string(int status);
/* Last error message recorded on this thread (empty if none). */
int rtb_last_error(char* buf, size_t len);
/* Wall-clock limit for every device-side wait (default 2 s). */
int rtb_set_timeout_ns(rtb_ctx* ctx, uint64_t ns);
/* Diagnostics: record a per-CTA timeline of the contraction kernels
 * (%globaltimer ns stamps; 20 per CTA: start, end, and for each of the CTA's
 * first 3 tiles the producer's first issue, the MMA's first ready k-block,
 * the MMA's last commit, the epilogue seeing the first and the last
 * accumulation unit, and the epilogue's completion) into `buf`, a device
 * buffer of `capacity` 64-bit words; a launch whose grid needs more is not
 * traced.  capacity = 0 turns tracing off. */
int rtb_set_kernel_trace(rtb_ctx* ctx, uint64_t* buf, int64_t capacity);
/* Failure-detection probe: launches a kernel whose single bounded wait can
 * never be satisfied; after timeout_ns (1 us .. 1 s) the wait gives up,
 * records device error code 8 and the kernel returns.  The next
 * rtb_stream_synchronize / rtb_device_error then reports RTB_E_TIMEOUT, and
 * the context stays usable.  Exercises the timeout path every kernel's waits
 * use, without faulting or hanging the GPU. */
int rtb_debug_wait_probe(rtb_ctx* ctx, uint64_t timeout_ns, void* stream);
/* Read and clear the device error word (synchronises the context's device).
 * *code receives 0 or the device error code; returns RTB_E_TIMEOUT if set. */
int rtb_device_error(rtb_ctx* ctx, int* code);

/* ---------------------------------------------------------------- memory */
int rtb_malloc(rtb_ctx* ctx, void** ptr, size_t bytes, void* stream);
int rtb_free(rtb_ctx* ctx, void* ptr, void* stream);
int rtb_host_alloc(rtb_ctx* ctx, void** ptr, size_t bytes); /* pinned */
int rtb_host_free(rtb_ctx* ctx, void* ptr);
int rtb_memcpy_h2d(rtb_ctx* ctx, void* dst, const void* src, size_t bytes, void* stream);
int rtb_memcpy_d2h(rtb_ctx* ctx, void* dst, const void* src, size_t bytes, void* stream);
int rtb_memcpy_d2d(rtb_ctx* ctx, void* dst, const void* src, size_t bytes, void* stream);
int rtb_memset_zero(rtb_ctx* ctx, void* dst, size_t bytes, void* stream);

/* ---------------------------------------------------------------- streams */
/* The context's own non-blocking stream (created by rtb_init). */
int rtb_context_stream(rtb_ctx* ctx, void** stream);
/* Streams for the calls below.  The library keeps a small block of
 * split-tile arrival counters per stream it launches on (the launches of one
 * stream run in order and share it; cudaStreamPerThread and captured launches
 * get counters of their own).  rtb_stream_destroy releases the block in the
 * stream's order.  A stream made elsewhere keeps its block until rtb_destroy:
 * synchronise such a stream before destroying it if its handle may be reused
 * for a new stream. */
int rtb_stream_create(rtb_ctx* ctx, void** stream);
int rtb_stream_destroy(rtb_ctx* ctx, void* stream);
/* Synchronise `stream`, then report a device-side timeout if one occurred. */
int rtb_stream_synchronize(rtb_ctx* ctx, void* stream);

/* ---------------------------------------------------------------- GEMM */
/* C[M,N] = act(op(A) . op(B) + bias), fp32 in/out, row-major C with ldc.
 *   transA = 0: A is [M,K] row-major (lda >= K); 1: A is [K,M] row-major.
 *   transB = 0: B is [K,N] row-major (Tensor::matmul's rhs, ldb >= N);
 *            1: B is [N,K] row-major (nn::Linear's weight, ldb >= K).
 *   bias: [N] or NULL.  act: any RTB_ACT_*.
 * Replaces ops::matmul (rustorch-core/src/ops.rs:1888-2066) and
 * ops::matmul_fused (ops.rs:1543-1710); M=N=K=0 edge cases follow the
 * reference (K=0 gives bias or zeros). */
int rtb_sgemm(rtb_ctx* ctx, int64_t M, int64_t N, int64_t K, const float* A, int64_t lda,
              int transA, const float* B, int64_t ldb, int transB, const float* bias, int act,
              float* C, int64_t ldc, int precision, void* stream);

/* Strided batch of independent GEMMs (extension: the reference's matmul is
 * 2-D only, rustorch-core/src/ops.rs:1892-1894; its oracle is a loop of 2-D
 * matmuls).  strideA/B/C in elements; bias shared by all batches. */
int rtb_sgemm_batched(rtb_ctx* ctx, int64_t batch, int64_t M, int64_t N, int64_t K,
                      const float* A, int64_t lda, int64_t strideA, int transA, const float* B,
                      int64_t ldb, int64_t strideB, int transB, const float* bias, int act,
                      float* C, int64_t ldc, int64_t strideC, int precision, void* stream);

/* C[M,N] = act(layer_norm_N(op(A) . op(B) + bias) * norm_weight + norm_bias):
 * ops::matmul_bias_norm_activation (rustorch-core/src/ops.rs:1815-1886, with
 * layer_norm over the last dimension, ops/norm.rs:613-700, and
 * apply_activation, ops.rs:1773-1780).  Arguments as rtb_sgemm; norm_weight,
 * norm_bias: [N] or NULL (1 and 0); eps as the reference's (LayerNorm's
 * default is 1e-5); act: any RTB_ACT_* (sigmoid = 1/(1+exp(-x)), tanh).  The
 * mean and variance are taken in two passes (the reference uses
 * E[x^2] - E[x]^2 in f32); results agree with the exact values to the
 * contraction's precision. */
int rtb_matmul_bias_norm_act(rtb_ctx* ctx, int64_t M, int64_t N, int64_t K, const float* A,
                             int64_t lda, int transA, const float* B, int64_t ldb, int transB,
                             const float* bias, const float* norm_weight, const float* norm_bias,
                             float eps, int act, float* C, int64_t ldc, int precision,
                             void* stream);

/* y[r, :] = act(layer_norm(x[r, :]) * norm_weight + norm_bias) for r < rows:
 * ops::layer_norm over the last dimension (rustorch-core/src/ops/norm.rs:
 * 613-700, normalized_shape = [d]) with an optional activation.  x and y are
 * row-major with leading dimensions ldx, ldy >= d; x == y (in place) is
 * allowed.  Mean and variance in two passes, as rtb_matmul_bias_norm_act. */
int rtb_layer_norm(rtb_ctx* ctx, int64_t rows, int64_t d, const float* x, int64_t ldx,
                   const float* norm_weight, const float* norm_bias, float eps, int act, float* y,
                   int64_t ldy, void* stream);

/* ---------------------------------------------------------------- conv */
/* y = act(conv2d(x, w, stride, padding) + bias + residual).
 *   x: [N,Ci,H,W] (NCHW) or [N,H,W,Ci] (NHWC) per x_layout.
 *   w: [Co,Ci,kh,kw] (the reference's weight layout, rustorch-nn/src/conv.rs:27-32).
 *   bias: [Co] or NULL; residual: same shape/layout as y, or NULL.
 *   y: [N,Co,Ho,Wo] or [N,Ho,Wo,Co] per y_layout; Ho = (H+2ph-kh)/sh+1.
 * Implicit GEMM (M = N*Ho*Wo, N = Co, K = kh*kw*Ci) on the tensor cores with
 * the bias/residual/activation epilogue fused.  Replaces ops::conv2d
 * (rustorch-core/src/ops/conv.rs:738-919) + nn::Conv2d's bias add
 * (rustorch-nn/src/conv.rs:52-63) + the JIT's Conv2dRelu lowering
 * (rustorch-core/src/jit.rs:254-262). */
int rtb_conv2d_fwd(rtb_ctx* ctx, int64_t N, int64_t Ci, int64_t H, int64_t W, int64_t Co,
                   int64_t kh, int64_t kw, int64_t sh, int64_t sw, int64_t ph, int64_t pw,
                   const float* x, int x_layout, const float* w, const float* bias,
                   const float* residual, int act, float* y, int y_layout, int precision,
                   void* stream);

/* Weight prepacking for repeated convs (nn::Conv2d / JIT graphs): packed
 * layout [Co, kh*kw*Cp] with Cp = roundup(Ci, 4), zero padded.  Size in
 * floats from rtb_conv2d_packed_weight_size. */
int64_t rtb_conv2d_packed_weight_size(int64_t Co, int64_t Ci, int64_t kh, int64_t kw);
int rtb_conv2d_prepack_weight(rtb_ctx* ctx, int64_t Co, int64_t Ci, int64_t kh, int64_t kw,
                              const float* w, float* w_packed, void* stream);
/* As rtb_conv2d_fwd with a prepacked weight and NHWC input whose channel
 * stride is Cp = roundup(Ci, 4) (x_cp_stride must equal Cp). */
int rtb_conv2d_fwd_packed(rtb_ctx* ctx, int64_t N, int64_t Ci, int64_t H, int64_t W, int64_t Co,
                          int64_t kh, int64_t kw, int64_t sh, int64_t sw, int64_t ph, int64_t pw,
                          const float* x_nhwc_padded, const float* w_packed, const float* bias,
                          const float* residual, int act, float* y, int y_layout, int precision,
                          void* stream);
/* Extension (no counterpart in the reference, whose f32 conv has no 3xTF32
 * split): the packed weight as rtb_conv2d_prepack_weight writes it, plus its
 * 3xTF32 low part w_lo[i] = w_packed[i] - trunc_tf32(w_packed[i]) (same size
 * and layout, 16-byte aligned).  A weight reused across calls keeps both, and
 * rtb_conv2d_fwd_packed_lo then reads w_lo instead of computing it per call. */
int rtb_conv2d_prepack_weight_lo(rtb_ctx* ctx, int64_t Co, int64_t Ci, int64_t kh, int64_t kw,
                                 const float* w, float* w_packed, float* w_lo, void* stream);
/* rtb_conv2d_fwd_packed with the weight's low part from
 * rtb_conv2d_prepack_weight_lo (null: as rtb_conv2d_fwd_packed); the same
 * results, one pass over the weight fewer per 3xTF32 call. */
int rtb_conv2d_fwd_packed_lo(rtb_ctx* ctx, int64_t N, int64_t Ci, int64_t H, int64_t W, int64_t Co,
                             int64_t kh, int64_t kw, int64_t sh, int64_t sw, int64_t ph, int64_t pw,
                             const float* x_nhwc_padded, const float* w_packed, const float* w_lo,
                             const float* bias, const float* residual, int act, float* y,
                             int y_layout, int precision, void* stream);
/* rtb_conv2d_fwd for callers that cannot allocate device memory (no
 * counterpart in the reference: RusTorch's CPU conv allocates freely).  Same
 * arguments and results as rtb_conv2d_fwd, but the scratch it needs (the
 * channel-padded NHWC input copy and the repacked weight) lives in a 16 MiB
 * array compiled into the library, so the call allocates nothing; a request
 * whose scratch would exceed 16 MiB returns RTB_E_INVALID.  Every GPU that
 * loads the library holds the 16 MiB until process exit.  All calls on a
 * device share the array: calls that overlap on the GPU race and must be
 * ordered by the caller.  The first call on each device looks up the array's
 * address (once per device) and should come before any stream capture. */
int rtb_conv2d_fwd_noalloc(rtb_ctx* ctx, int64_t N, int64_t Ci, int64_t H, int64_t W, int64_t Co,
                           int64_t kh, int64_t kw, int64_t sh, int64_t sw, int64_t ph, int64_t pw,
                           const float* x, int x_layout, const float* w, const float* bias,
                           const float* residual, int act, float* y, int y_layout, int precision,
                           void* stream);

/* NCHW [N,C,H,W] -> NHWC with channel stride Cp = roundup(C,4), zero padded. */
int rtb_nchw_to_nhwc_padded(rtb_ctx* ctx, int64_t N, int64_t C, int64_t H, int64_t W,
                            const float* x, float* y, void* stream);

/* ---------------------------------------------------------------- backward */
/* MatmulBackward (rustorch-core/src/ops.rs:529-570) for C = A . B with A
 * [M,K], B [K,N], dC [M,N], all row-major contiguous:
 *   dA = dC . B^T  (grad_lhs = matmul(grad, rhs.t()))   when dA != NULL
 *   dB = A^T . dC  (grad_rhs = matmul(lhs.t(), grad))   when dB != NULL
 * accumulate != 0 adds into dA / dB (the reference's accumulate_grad) instead
 * of overwriting.  Both products run on the same tensor-core engine. */
int rtb_matmul_backward(rtb_ctx* ctx, int64_t M, int64_t N, int64_t K, const float* A,
                        const float* B, const float* dC, float* dA, float* dB, int accumulate,
                        int precision, void* stream);
/* Conv2dBackward (rustorch-core/src/ops/conv.rs:336-736) for the NCHW conv of
 * x [N,Ci,H,W] with w [Co,Ci,kh,kw] (stride, padding as in rtb_conv2d_fwd) and
 * incoming gradient dy [N,Co,Ho,Wo]:
 *   dx [N,Ci,H,W]     (conv2d_grad_input_*_core)   when dx != NULL
 *   dw [Co,Ci,kh,kw]  (conv2d_grad_weight_*_core)  when dw != NULL
 * accumulate != 0 adds into dx / dw.  grad_input needs padding <= kernel - 1
 * (RTB_E_UNSUPPORTED otherwise). */
int rtb_conv2d_backward(rtb_ctx* ctx, int64_t N, int64_t Ci, int64_t H, int64_t W, int64_t Co,
                        int64_t kh, int64_t kw, int64_t sh, int64_t sw, int64_t ph, int64_t pw,
                        const float* x, const float* w, const float* dy, float* dx, float* dw,
                        int accumulate, int precision, void* stream);

/* ---------------------------------------------------------------- small ops */
/* ops::max_pool2d (rustorch-core/src/ops/pool.rs:115-191): -inf init, padding skipped. */
int rtb_max_pool2d(rtb_ctx* ctx, int64_t N, int64_t C, int64_t H, int64_t W, int64_t kh,
                   int64_t kw, int64_t sh, int64_t sw, int64_t ph, int64_t pw, const float* x,
                   float* y, int layout, void* stream);
/* Global average pool -> [N, C] (absent from the reference; needed by ResNet-18). */
int rtb_global_avg_pool(rtb_ctx* ctx, int64_t N, int64_t C, int64_t H, int64_t W, const float* x,
                        float* y, int layout, void* stream);
/* Elementwise: y = a + b (ops::add same shape), y = max(x, 0) (ops::relu). */
int rtb_add(rtb_ctx* ctx, int64_t n, const float* a, const float* b, float* y, void* stream);
int rtb_relu(rtb_ctx* ctx, int64_t n, const float* x, float* y, void* stream);
/* y = a op b (op 0 = add, 1 = mul) over an n-d output `shape` (1..8 dims,
 * row-major y) with per-operand element strides, 0 for broadcast dimensions:
 * ops::add / ops::mul with broadcasting (rustorch-core/src/ops.rs:223-291,
 * rustorch-core/src/broadcast.rs:23-136). */
int rtb_elementwise_broadcast(rtb_ctx* ctx, int op, int ndim, const int64_t* shape,
                              const float* a, const int64_t* a_strides, const float* b,
                              const int64_t* b_strides, float* y, void* stream);

/* ---------------------------------------------------------------- data */
/* The documented synthetic-input generator: SplitMix64 stream keyed by
 * (seed, tensor_id); N(mean, std) by Box-Muller on draw pairs; U(lo, hi) from
 * the top 24 bits of each draw.  Host version (multi-threaded). */
int rtb_fill_normal_host(float* out, int64_t n, uint64_t seed, uint64_t tensor_id, float mean,
                         float std_dev);
int rtb_fill_uniform_host(float* out, int64_t n, uint64_t seed, uint64_t tensor_id, float lo,
                          float hi);

/* ---------------------------------------------------------------- multi-GPU */
/* One process per GPU.  Rank 0 creates an id (128 opaque bytes), the caller
 * broadcasts it (e.g. over torch.distributed), every rank joins. */
int rtb_nccl_unique_id(void* id_out_128b);
int rtb_nccl_comm_init(rtb_ctx* ctx, const void* id_128b, int nranks, int rank, void** comm);
int rtb_nccl_comm_destroy(void* comm);
/* N-split GEMM: rank r holds A [M,K] (replicated) and B_r = B[:, r*N/P:(r+1)*N/P]
 * as a [K, N/P] row-major block; computes C_r = A . B_r into its slice and
 * all-gathers so every rank ends with C [M,N] row-major.  `c_parts` is a
 * [P, M, N/P] scratch the caller provides (device memory, P*M*(N/P) floats).
 * Requires N % P == 0. */
int rtb_sgemm_nsplit_allgather(rtb_ctx* ctx, void* comm, int64_t M, int64_t N, int64_t K,
                               const float* A, const float* B_local, float* c_parts, float* C,
                               int precision, void* stream);

/* N-split GEMM fused with its exchange: C [M,N] = A [M,K] . B [K,N] with B's
 * columns split over the communicator's ranks (B_local = B[:, cols(rank)],
 * [K, N/P] row-major).  The GEMM epilogue stores each finished tile of the
 * rank's block into every rank's C over NVLink (P2P stores into CUDA IPC
 * mappings), overlapping the exchange with the remaining tiles; a one-int
 * all-reduce before and after the GEMM orders it against the previous
 * reader and the peers' stores.  C lives in a peer buffer made once per
 * communicator (collective calls, every rank with the same size):
 * rtb_peer_buffer_local gives this rank's copy (valid until the next call on
 * any rank).  Needs K and N/P multiples of 4 and 16-byte aligned A, B_local
 * (RTB_E_UNSUPPORTED otherwise; rtb_sgemm_nsplit_allgather has no such
 * limits).  No counterpart in the reference (multi-GPU extension). */
int rtb_peer_buffer_create(rtb_ctx* ctx, void* comm, size_t bytes, void** peer_buffer);
int rtb_peer_buffer_local(void* peer_buffer, float** local);
int rtb_peer_buffer_destroy(void* peer_buffer, void* comm);
int rtb_sgemm_nsplit_p2p(rtb_ctx* ctx, void* comm, void* peer_buffer, int64_t M, int64_t N,
                         int64_t K, const float* A, const float* B_local, int precision,
                         void* stream);

#ifdef __cplusplus
}
#endif
#endif /* RUSTORCH_B200_H */
