// C-ABI implementation: contexts, memory, streams, argument validation and
// dispatch of GEMM / conv / pooling onto the sm_100a kernels.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "rtb_internal.h"

namespace rtb {

static thread_local std::string g_last_error;

int set_error(int status, const std::string& msg) {
  g_last_error = msg;
  return status;
}

int cuda_status(cudaError_t e, const char* what) {
  const int st = (e == cudaErrorMemoryAllocation) ? RTB_E_OOM : RTB_E_CUDA;
  (void)cudaGetLastError();  // consume it so a later launch check does not see it again
  return set_error(st, std::string(what) + ": " + cudaGetErrorString(e));
}

// ---------------------------------------------------------------- tensor maps
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_tiled() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

int make_tmap_2d(CUtensorMap* map, const void* base, uint64_t dim0, uint64_t dim1,
                 uint64_t row_stride_elems, uint32_t box0, uint32_t box1, bool atom32) {
  return make_tmap_2d_swz(map, base, dim0, dim1, row_stride_elems, box0, box1,
                          atom32 ? kTmapSwizzle128Atom32 : kTmapSwizzle128);
}

int make_tmap_2d_swz(CUtensorMap* map, const void* base, uint64_t dim0, uint64_t dim1,
                     uint64_t row_stride_elems, uint32_t box0, uint32_t box1, int swizzle) {
  EncodeTiledFn enc = get_encode_tiled();
  if (!enc) return set_error(RTB_E_CUDA, "cuTensorMapEncodeTiled unavailable");
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0 || (row_stride_elems * 4) % 16 != 0)
    return set_error(RTB_E_INVALID, "tensor map: base must be 16-byte aligned, row stride % 4 == 0");
  const cuuint64_t dims[2] = {dim0, dim1};
  const cuuint64_t strides[1] = {row_stride_elems * 4};
  const cuuint32_t box[2] = {box0, box1};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(base), dims, strides,
                   box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   swizzle == kTmapSwizzle128Atom32 ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B
                   : swizzle == kTmapSwizzle128     ? CU_TENSOR_MAP_SWIZZLE_128B
                                                    : CU_TENSOR_MAP_SWIZZLE_NONE,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    char buf[160];
    snprintf(buf, sizeof buf, "cuTensorMapEncodeTiled failed (%d): dims %llu x %llu stride %llu",
             (int)r, (unsigned long long)dim0, (unsigned long long)dim1,
             (unsigned long long)row_stride_elems);
    return set_error(RTB_E_CUDA, buf);
  }
  return RTB_OK;
}

typedef CUresult (*EncodeIm2colFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const int*, const int*,
                                   cuuint32_t, cuuint32_t, const cuuint32_t*,
                                   CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeIm2colFn get_encode_im2col() {
  static EncodeIm2colFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeIm2col", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeIm2colFn>(p);
  });
  return fn;
}

int make_tmap_im2col(CUtensorMap* map, const void* x, int N, int H, int W, int Cp, int R, int S,
                     int sh, int sw, int ph, int pw, uint32_t channels_per_pixel,
                     uint32_t pixels_per_column, int swizzle_bytes) {
  EncodeIm2colFn enc = get_encode_im2col();
  if (!enc) return set_error(RTB_E_CUDA, "cuTensorMapEncodeIm2col unavailable");
  if ((reinterpret_cast<uintptr_t>(x) & 15u) != 0 || (Cp * 4) % 16 != 0)
    return set_error(RTB_E_INVALID, "im2col map: base must be 16-byte aligned, Cp % 4 == 0");
  const cuuint64_t dims[4] = {(cuuint64_t)Cp, (cuuint64_t)W, (cuuint64_t)H, (cuuint64_t)N};
  const cuuint64_t strides[3] = {(cuuint64_t)Cp * 4, (cuuint64_t)W * Cp * 4,
                                 (cuuint64_t)H * W * Cp * 4};
  // Bounding box of the traversal in (W, H): from -pad to (size-1 + pad - (filter-1)),
  // so the traversal visits exactly the Wo x Ho top-left tap positions.
  const int lower[2] = {-pw, -ph};
  const int upper[2] = {pw - (S - 1), ph - (R - 1)};
  const cuuint32_t estr[4] = {1, (cuuint32_t)sw, (cuuint32_t)sh, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<void*>(x), dims, strides,
                   lower, upper, channels_per_pixel, pixels_per_column, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE,
                   swizzle_bytes == 128  ? CU_TENSOR_MAP_SWIZZLE_128B
                   : swizzle_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                   : swizzle_bytes == 32 ? CU_TENSOR_MAP_SWIZZLE_32B
                                         : CU_TENSOR_MAP_SWIZZLE_NONE,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    char buf[160];
    snprintf(buf, sizeof buf, "cuTensorMapEncodeIm2col failed (%d)", (int)r);
    return set_error(RTB_E_CUDA, buf);
  }
  return RTB_OK;
}

// ---------------------------------------------------------------- workspace
int ws_alloc(rtb_ctx* ctx, void** p, size_t bytes, cudaStream_t s) {
  (void)ctx;
  cudaError_t e = cudaMallocAsync(p, bytes ? bytes : 16, s);
  if (e != cudaSuccess) return cuda_status(e, "workspace cudaMallocAsync");
  return RTB_OK;
}

void ws_free(void* p, cudaStream_t s) {
  if (p) cudaFreeAsync(p, s);
}

int split_counters(rtb_ctx* ctx, cudaStream_t s, unsigned long long** d, unsigned long long* gen) {
  // A captured launch replays with the generation baked into its parameters,
  // so under stream capture the caller zeroes per-launch counters instead.
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(s, &cap) != cudaSuccess || cap != cudaStreamCaptureStatusNone) {
    clear_stale_cuda_error();
    return RTB_E_UNSUPPORTED;
  }
  // cudaStreamPerThread is one handle for a different stream in every host
  // thread: launches under it from two threads may run at the same time, so
  // they cannot share a block either; they get per-launch counters too.
  if (s == cudaStreamPerThread) return RTB_E_UNSUPPORTED;
  std::lock_guard<std::mutex> lk(ctx->cnt_mu);
  auto& c = ctx->split_cnt[s];
  if (!c.d) {
    // zeroed once (generation 0 is never issued); later launches on this
    // stream tag their arrivals with increasing generations.  Stream-ordered,
    // so rtb_stream_destroy can release it behind the stream's last launch.
    cudaError_t e = cudaMallocAsync(&c.d, kSplitCounters * sizeof(unsigned long long), s);
    if (e == cudaSuccess)
      e = cudaMemsetAsync(c.d, 0, kSplitCounters * sizeof(unsigned long long), s);
    if (e != cudaSuccess) {
      if (c.d) cudaFreeAsync(c.d, s);
      ctx->split_cnt.erase(s);
      return cuda_status(e, "split counters");
    }
  }
  *d = c.d;
  *gen = ++c.gen;
  return RTB_OK;
}

// Drops the counter block of a stream that is about to be destroyed: freed in
// the stream's order (after its last launch), so a later stream that reuses
// the handle starts with a fresh block.
static void release_split_counters(rtb_ctx* ctx, cudaStream_t s) {
  std::lock_guard<std::mutex> lk(ctx->cnt_mu);
  auto it = ctx->split_cnt.find(s);
  if (it == ctx->split_cnt.end()) return;
  if (it->second.d) cudaFreeAsync(it->second.d, s);
  ctx->split_cnt.erase(it);
}

}  // namespace rtb

using namespace rtb;

#define RTB_CHECK_CTX(ctx)                                              \
  do {                                                                  \
    if (!(ctx)) return set_error(RTB_E_INVALID, "null rtb_ctx");        \
  } while (0)

static inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
static inline int64_t round_up(int64_t v, int64_t m) { return (v + m - 1) / m * m; }

extern "C" {

// ---------------------------------------------------------------- context
int rtb_device_count(int* count) {
  if (!count) return set_error(RTB_E_INVALID, "null count");
  cudaError_t e = cudaGetDeviceCount(count);
  if (e != cudaSuccess) {
    *count = 0;
    return cuda_status(e, "cudaGetDeviceCount");
  }
  return RTB_OK;
}

int rtb_init(int device, rtb_ctx** out) {
  if (!out) return set_error(RTB_E_INVALID, "null output pointer");
  *out = nullptr;
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess) return cuda_status(e, "cudaGetDeviceCount");
  if (device < 0 || device >= n) return set_error(RTB_E_INVALID, "device index out of range");
  DeviceGuard g(device);
  cudaDeviceProp prop;
  e = cudaGetDeviceProperties(&prop, device);
  if (e != cudaSuccess) return cuda_status(e, "cudaGetDeviceProperties");
  if (prop.major != 10)
    return set_error(RTB_E_UNSUPPORTED, "this library is built for sm_100a (B200) only");
  rtb_ctx* c = new (std::nothrow) rtb_ctx();
  if (!c) return set_error(RTB_E_OOM, "context allocation");
  c->device = device;
  c->sm_count = prop.multiProcessorCount;
  c->cc_major = prop.major;
  c->cc_minor = prop.minor;
  c->total_mem = prop.totalGlobalMem;
  e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking);
  if (e != cudaSuccess) {
    delete c;
    return cuda_status(e, "cudaStreamCreate");
  }
  e = cudaMalloc(&c->d_err, sizeof(int));
  if (e == cudaSuccess) e = cudaMemset(c->d_err, 0, sizeof(int));
  if (e != cudaSuccess) {
    cudaStreamDestroy(c->stream);
    delete c;
    return cuda_status(e, "error-word allocation");
  }
  // Keep freed workspace in the pool (no release back to the OS between calls).
  cudaMemPool_t pool;
  if (cudaDeviceGetDefaultMemPool(&pool, device) == cudaSuccess) {
    uint64_t thr = UINT64_MAX;
    cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &thr);
  }
  const char* prec = std::getenv("RUSTORCH_B200_PRECISION");
  if (prec && (std::strcmp(prec, "tf32") == 0 || std::strcmp(prec, "TF32") == 0))
    c->default_precision = RTB_PREC_TF32;
  *out = c;
  return RTB_OK;
}

int rtb_destroy(rtb_ctx* ctx) {
  RTB_CHECK_CTX(ctx);
  DeviceGuard g(ctx->device);
  cudaStreamSynchronize(ctx->stream);
  cudaDeviceSynchronize();  // launches on other streams may still use the counter blocks
  for (auto& kv : ctx->split_cnt)  // stream-ordered blocks: freed on the context's stream
    if (kv.second.d) cudaFreeAsync(kv.second.d, ctx->stream);
  ctx->split_cnt.clear();
  cudaStreamSynchronize(ctx->stream);
  cudaFree(ctx->d_err);
  cudaStreamDestroy(ctx->stream);
  delete ctx;
  return RTB_OK;
}

int rtb_get_device_info(rtb_ctx* ctx, int* sm_count, int* cc_major, int* cc_minor,
                        size_t* total_mem) {
  RTB_CHECK_CTX(ctx);
  if (sm_count) *sm_count = ctx->sm_count;
  if (cc_major) *cc_major = ctx->cc_major;
  if (cc_minor) *cc_minor = ctx->cc_minor;
  if (total_mem) *total_mem = ctx->total_mem;
  return RTB_OK;
}

const char* rtb_status_string(int status) {
  switch (status) {
    case RTB_OK: return "ok";
    case RTB_E_INVALID: return "invalid argument";
    case RTB_E_OOM: return "out of memory";
    case RTB_E_CUDA: return "CUDA error";
    case RTB_E_TIMEOUT: return "device wait timed out";
    case RTB_E_UNSUPPORTED: return "unsupported";
    case RTB_E_NCCL: return "NCCL error";
    default: return "unknown status";
  }
}

int rtb_last_error(char* buf, size_t len) {
  if (!buf || len == 0) return RTB_E_INVALID;
  std::snprintf(buf, len, "%s", g_last_error.c_str());
  return RTB_OK;
}

int rtb_set_timeout_ns(rtb_ctx* ctx, uint64_t ns) {
  RTB_CHECK_CTX(ctx);
  if (ns < 1000000ull) return set_error(RTB_E_INVALID, "timeout below 1 ms");
  ctx->timeout_ns = ns;
  return RTB_OK;
}

int rtb_set_kernel_trace(rtb_ctx* ctx, uint64_t* buf, int64_t capacity) {
  RTB_CHECK_CTX(ctx);
  if (capacity < 0 || (capacity > 0 && !buf)) return set_error(RTB_E_INVALID, "bad trace buffer");
  ctx->trace = reinterpret_cast<unsigned long long*>(capacity ? buf : nullptr);
  ctx->trace_capacity = capacity;
  return RTB_OK;
}

int rtb_debug_wait_probe(rtb_ctx* ctx, uint64_t timeout_ns, void* stream) {
  RTB_CHECK_CTX(ctx);
  if (timeout_ns < 1000ull || timeout_ns > 1000000000ull)
    return set_error(RTB_E_INVALID, "wait probe: timeout must be in [1 us, 1 s]");
  DeviceGuard g(ctx->device);
  return launch_wait_probe(ctx->d_err, timeout_ns, pick_stream(ctx, stream));
}

int rtb_device_error(rtb_ctx* ctx, int* code) {
  RTB_CHECK_CTX(ctx);
  DeviceGuard g(ctx->device);
  int h = 0;
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_status(e, "cudaDeviceSynchronize");
  e = cudaMemcpy(&h, ctx->d_err, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_status(e, "read error word");
  if (h) cudaMemset(ctx->d_err, 0, sizeof(int));
  if (code) *code = h;
  if (h) {
    char buf[96];
    std::snprintf(buf, sizeof buf, "device-side bounded wait expired (code %d)", h);
    return set_error(RTB_E_TIMEOUT, buf);
  }
  return RTB_OK;
}

// ---------------------------------------------------------------- memory
int rtb_malloc(rtb_ctx* ctx, void** ptr, size_t bytes, void* stream) {
  RTB_CHECK_CTX(ctx);
  if (!ptr) return set_error(RTB_E_INVALID, "null ptr");
  DeviceGuard g(ctx->device);
  cudaError_t e = cudaMallocAsync(ptr, bytes ? bytes : 16, pick_stream(ctx, stream));
  if (e != cudaSuccess) return cuda_status(e, "rtb_malloc");
  return RTB_OK;
}

int rtb_free(rtb_ctx* ctx, void* ptr, void* stream) {
  RTB_CHECK_CTX(ctx);
  if (!ptr) return RTB_OK;
  DeviceGuard g(ctx->device);
  cudaError_t e = cudaFreeAsync(ptr, pick_stream(ctx, stream));
  if (e != cudaSuccess) return cuda_status(e, "rtb_free");
  return RTB_OK;
}

int rtb_host_alloc(rtb_ctx* ctx, void** ptr, size_t bytes) {
  RTB_CHECK_CTX(ctx);
  if (!ptr) return set_error(RTB_E_INVALID, "null ptr");
  DeviceGuard g(ctx->device);
  cudaError_t e = cudaMallocHost(ptr, bytes ? bytes : 16);
  if (e != cudaSuccess) return cuda_status(e, "rtb_host_alloc");
  return RTB_OK;
}

int rtb_host_free(rtb_ctx* ctx, void* ptr) {
  RTB_CHECK_CTX(ctx);
  if (!ptr) return RTB_OK;
  cudaError_t e = cudaFreeHost(ptr);
  if (e != cudaSuccess) return cuda_status(e, "rtb_host_free");
  return RTB_OK;
}

static int copy_impl(rtb_ctx* ctx, void* dst, const void* src, size_t bytes, void* stream,
                     cudaMemcpyKind kind, const char* what) {
  RTB_CHECK_CTX(ctx);
  if (bytes == 0) return RTB_OK;
  if (!dst || !src) return set_error(RTB_E_INVALID, std::string(what) + ": null pointer");
  DeviceGuard g(ctx->device);
  cudaError_t e = cudaMemcpyAsync(dst, src, bytes, kind, pick_stream(ctx, stream));
  if (e != cudaSuccess) return cuda_status(e, what);
  return RTB_OK;
}

int rtb_memcpy_h2d(rtb_ctx* ctx, void* dst, const void* src, size_t bytes, void* stream) {
  return copy_impl(ctx, dst, src, bytes, stream, cudaMemcpyHostToDevice, "rtb_memcpy_h2d");
}
int rtb_memcpy_d2h(rtb_ctx* ctx, void* dst, const void* src, size_t bytes, void* stream) {
  return copy_impl(ctx, dst, src, bytes, stream, cudaMemcpyDeviceToHost, "rtb_memcpy_d2h");
}
int rtb_memcpy_d2d(rtb_ctx* ctx, void* dst, const void* src, size_t bytes, void* stream) {
  return copy_impl(ctx, dst, src, bytes, stream, cudaMemcpyDeviceToDevice, "rtb_memcpy_d2d");
}

int rtb_memset_zero(rtb_ctx* ctx, void* dst, size_t bytes, void* stream) {
  RTB_CHECK_CTX(ctx);
  if (bytes == 0) return RTB_OK;
  if (!dst) return set_error(RTB_E_INVALID, "rtb_memset_zero: null pointer");
  DeviceGuard g(ctx->device);
  cudaError_t e = cudaMemsetAsync(dst, 0, bytes, pick_stream(ctx, stream));
  if (e != cudaSuccess) return cuda_status(e, "rtb_memset_zero");
  return RTB_OK;
}

// ---------------------------------------------------------------- streams
int rtb_context_stream(rtb_ctx* ctx, void** stream) {
  RTB_CHECK_CTX(ctx);
  if (!stream) return set_error(RTB_E_INVALID, "null stream out");
  *stream = ctx->stream;
  return RTB_OK;
}

int rtb_stream_create(rtb_ctx* ctx, void** stream) {
  RTB_CHECK_CTX(ctx);
  if (!stream) return set_error(RTB_E_INVALID, "null stream out");
  DeviceGuard g(ctx->device);
  cudaStream_t s;
  cudaError_t e = cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking);
  if (e != cudaSuccess) return cuda_status(e, "rtb_stream_create");
  *stream = s;
  return RTB_OK;
}

int rtb_stream_destroy(rtb_ctx* ctx, void* stream) {
  RTB_CHECK_CTX(ctx);
  if (!stream) return RTB_OK;
  DeviceGuard g(ctx->device);
  release_split_counters(ctx, static_cast<cudaStream_t>(stream));
  cudaError_t e = cudaStreamDestroy(static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_status(e, "rtb_stream_destroy");
  return RTB_OK;
}

int rtb_stream_synchronize(rtb_ctx* ctx, void* stream) {
  RTB_CHECK_CTX(ctx);
  DeviceGuard g(ctx->device);
  cudaError_t e = cudaStreamSynchronize(pick_stream(ctx, stream));
  if (e != cudaSuccess) return cuda_status(e, "rtb_stream_synchronize");
  int h = 0;
  e = cudaMemcpy(&h, ctx->d_err, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_status(e, "read error word");
  if (h) {
    cudaMemset(ctx->d_err, 0, sizeof(int));
    char buf[96];
    std::snprintf(buf, sizeof buf, "device-side bounded wait expired (code %d)", h);
    return set_error(RTB_E_TIMEOUT, buf);
  }
  return RTB_OK;
}

// ---------------------------------------------------------------- GEMM
static int resolve_precision(rtb_ctx* ctx, int precision, int* split3) {
  if (precision == RTB_PREC_DEFAULT) precision = ctx->default_precision;
  if (precision != RTB_PREC_3XTF32 && precision != RTB_PREC_TF32)
    return set_error(RTB_E_INVALID, "precision must be RTB_PREC_3XTF32, RTB_PREC_TF32 or DEFAULT");
  *split3 = precision == RTB_PREC_3XTF32 ? 1 : 0;
  return RTB_OK;
}

// The reference's Activation enum (rustorch-core/src/backend/mod.rs:1-7):
// None, ReLU, Sigmoid and Tanh are all applied in the contraction's epilogue.
static int check_act(int act) {
  if (act < RTB_ACT_NONE || act > RTB_ACT_TANH)
    return set_error(RTB_E_INVALID, "unknown activation");
  return RTB_OK;
}

// Skinny products in 3xTF32 (up to 128 rows against many columns: a small
// batch through a large weight) run as C^T = B^T . A^T.  The 128-row tiles
// then walk B, the large operand, 16 KB of it per k-block split once per
// element by the converter warps (a 64-column tile of the direct form reads
// 8 KB of B in the same k-block time, and leaves most of its 128 rows empty),
// while A becomes the narrow B operand that stays in L2.  The transposed tile
// leaves through the channel-major (NCHW) epilogue with the channel stride
// set to ldc, and the caller's bias becomes a per-row bias there.
// RTB_SKINNY_T=0 turns this off, 2 takes it wherever it is legal.
static bool skinny_transposed(const GemmDesc& d, int64_t M, int64_t N, int64_t K, int64_t ldc) {
  static const int env = [] {
    const char* v = std::getenv("RTB_SKINNY_T");
    return v ? std::atoi(v) : 1;
  }();
  if (env == 0 || !d.split3 || d.residual || M > 128 || ldc > INT32_MAX) return false;
  return env == 2 || (N >= 2048 && K >= 256);
}

static GemmDesc transposed_desc(const GemmDesc& d) {
  GemmDesc t;
  t.M = d.N;
  t.N = d.M;
  t.K = d.K;
  t.A = d.B;  // [K,N] row-major (MN-major A) or [N,K] (K-major A)
  t.lda = d.ldb;
  t.a_mn_major = d.b_mn_major;
  t.B = d.A;  // A's K-major [M,K] storage is B^T's K-major [N', K] form
  t.ldb = d.lda;
  t.b_mn_major = 0;
  t.C = d.C;
  t.ldc = d.ldc;
  t.out_mode = 1;  // element (row n', channel m) at m * hw + n' with one "image"
  t.hw = (int)d.ldc;
  t.row_bias = d.bias;
  t.act = d.act;
  t.split3 = d.split3;
  return t;
}

// One 2-D GEMM on the current device/stream (helper for single and batched).
// residual (optional, same indexing as C): C = act(A.B + bias + residual);
// residual == C accumulates into C.
static int sgemm_one(rtb_ctx* ctx, int64_t M, int64_t N, int64_t K, const float* A, int64_t lda,
                     int transA, const float* B, int64_t ldb, int transB, const float* bias,
                     int act, float* C, int64_t ldc, int split3, cudaStream_t s,
                     const float* residual = nullptr) {
  if (M == 0 || N == 0) return RTB_OK;
  if (K == 0) {
    if (residual == C && !bias && act == RTB_ACT_NONE) return RTB_OK;  // C += 0
    if (residual) return set_error(RTB_E_UNSUPPORTED, "K == 0 with a residual");
    return launch_fill_rows(C, M, N, ldc, bias, act, s);
  }

  GemmDesc d;
  d.M = M; d.N = N; d.K = K;
  d.C = C; d.ldc = ldc; d.bias = bias; d.act = act; d.split3 = split3;
  d.residual = residual; d.ldr = ldc;
  float* wsA = nullptr;
  float* wsB = nullptr;
  int st = RTB_OK;

  // A must be K-major, 16-byte aligned, row stride a multiple of 4 floats.
  if (!transA && aligned16(A) && lda % 4 == 0) {
    d.A = A; d.lda = lda;
  } else {
    const int64_t Kp = round_up(K, 4);
    st = ws_alloc(ctx, (void**)&wsA, (size_t)(M * Kp) * 4, s);
    if (st) return st;
    st = transA ? launch_pack_kmajor(A, M, K, 1, lda, wsA, Kp, s)
                : launch_pack_kmajor(A, M, K, lda, 1, wsA, Kp, s);
    d.A = wsA; d.lda = Kp;
  }
  if (st == RTB_OK) {
    if (!transB && aligned16(B) && ldb % 4 == 0) {
      d.B = B; d.ldb = ldb; d.b_mn_major = 1;           // [K,N] row-major
    } else if (transB && aligned16(B) && ldb % 4 == 0) {
      d.B = B; d.ldb = ldb; d.b_mn_major = 0;           // [N,K] row-major
    } else {
      const int64_t Kp = round_up(K, 4);
      st = ws_alloc(ctx, (void**)&wsB, (size_t)(N * Kp) * 4, s);
      if (st == RTB_OK)
        st = transB ? launch_pack_kmajor(B, N, K, ldb, 1, wsB, Kp, s)
                    : launch_pack_kmajor(B, N, K, 1, ldb, wsB, Kp, s);
      d.B = wsB; d.ldb = Kp; d.b_mn_major = 0;
    }
  }
  if (st == RTB_OK) {
    // Few rows: a stream over B on the CUDA cores beats a padded 128-row
    // tensor-core tile (RTB_SMALLM=0 turns the small-M path off).
    static const bool smallm_on = [] {
      const char* v = std::getenv("RTB_SMALLM");
      return !(v && v[0] == '0');
    }();
    if (smallm_on && M <= kSmallMMax && !residual)
      st = smallm_run(ctx, d, s);
    else if (skinny_transposed(d, M, N, K, ldc))
      st = gemm_run(ctx, transposed_desc(d), s);
    else
      st = gemm_run(ctx, d, s);
  }
  ws_free(wsA, s);
  ws_free(wsB, s);
  return st;
}

static int check_gemm_args(int64_t M, int64_t N, int64_t K, const float* A, int64_t lda,
                           int transA, const float* B, int64_t ldb, int transB, float* C,
                           int64_t ldc) {
  if (M < 0 || N < 0 || K < 0) return set_error(RTB_E_INVALID, "negative dimension");
  if (transA != 0 && transA != 1) return set_error(RTB_E_INVALID, "transA must be 0 or 1");
  if (transB != 0 && transB != 1) return set_error(RTB_E_INVALID, "transB must be 0 or 1");
  if (M == 0 || N == 0) return RTB_OK;
  if (!C) return set_error(RTB_E_INVALID, "null C");
  if (ldc < N) return set_error(RTB_E_INVALID, "ldc < N");
  if (K == 0) return RTB_OK;
  if (!A || !B) return set_error(RTB_E_INVALID, "null A or B");
  if (lda < (transA ? M : K)) return set_error(RTB_E_INVALID, "lda too small");
  if (ldb < (transB ? K : N)) return set_error(RTB_E_INVALID, "ldb too small");
  return RTB_OK;
}

int rtb_sgemm(rtb_ctx* ctx, int64_t M, int64_t N, int64_t K, const float* A, int64_t lda,
              int transA, const float* B, int64_t ldb, int transB, const float* bias, int act,
              float* C, int64_t ldc, int precision, void* stream) {
  RTB_CHECK_CTX(ctx);
  int st = check_gemm_args(M, N, K, A, lda, transA, B, ldb, transB, C, ldc);
  if (st) return st;
  int split3 = 1;
  if ((st = check_act(act))) return st;
  if ((st = resolve_precision(ctx, precision, &split3))) return st;
  DeviceGuard g(ctx->device);
  return sgemm_one(ctx, M, N, K, A, lda, transA, B, ldb, transB, bias, act, C, ldc, split3,
                   pick_stream(ctx, stream));
}

int rtb_sgemm_batched(rtb_ctx* ctx, int64_t batch, int64_t M, int64_t N, int64_t K,
                      const float* A, int64_t lda, int64_t strideA, int transA, const float* B,
                      int64_t ldb, int64_t strideB, int transB, const float* bias, int act,
                      float* C, int64_t ldc, int64_t strideC, int precision, void* stream) {
  RTB_CHECK_CTX(ctx);
  if (batch < 0) return set_error(RTB_E_INVALID, "negative batch");
  int st = check_gemm_args(M, N, K, A, lda, transA, B, ldb, transB, C, ldc);
  if (st) return st;
  int split3 = 1;
  if ((st = check_act(act))) return st;
  if ((st = resolve_precision(ctx, precision, &split3))) return st;
  DeviceGuard g(ctx->device);
  cudaStream_t s = pick_stream(ctx, stream);
  for (int64_t b = 0; b < batch; ++b) {
    st = sgemm_one(ctx, M, N, K, A ? A + b * strideA : nullptr, lda, transA,
                   B ? B + b * strideB : nullptr, ldb, transB, bias, act, C + b * strideC, ldc,
                   split3, s);
    if (st) return st;
  }
  return RTB_OK;
}

// ops::matmul_bias_norm_activation (rustorch-core/src/ops.rs:1815-1886): the
// engine's GEMM with the bias in its epilogue, then one row-wise LayerNorm +
// activation pass over C (the reference's pipeline_fused order).
int rtb_matmul_bias_norm_act(rtb_ctx* ctx, int64_t M, int64_t N, int64_t K, const float* A,
                             int64_t lda, int transA, const float* B, int64_t ldb, int transB,
                             const float* bias, const float* norm_weight, const float* norm_bias,
                             float eps, int act, float* C, int64_t ldc, int precision,
                             void* stream) {
  RTB_CHECK_CTX(ctx);
  int st = check_gemm_args(M, N, K, A, lda, transA, B, ldb, transB, C, ldc);
  if (st) return st;
  if (act < RTB_ACT_NONE || act > RTB_ACT_TANH) return set_error(RTB_E_INVALID, "unknown activation");
  int split3 = 1;
  if ((st = resolve_precision(ctx, precision, &split3))) return st;
  DeviceGuard g(ctx->device);
  cudaStream_t s = pick_stream(ctx, stream);
  if ((st = sgemm_one(ctx, M, N, K, A, lda, transA, B, ldb, transB, bias, 0, C, ldc, split3, s)))
    return st;
  if (M == 0 || N == 0) return RTB_OK;
  return launch_layernorm_act(ctx, C, ldc, C, ldc, M, N, norm_weight, norm_bias, eps, act, s);
}

// ops::layer_norm over the last dimension (rustorch-core/src/ops/norm.rs:613-700)
// followed by an activation, rows of X into rows of Y.
int rtb_layer_norm(rtb_ctx* ctx, int64_t rows, int64_t d, const float* x, int64_t ldx,
                   const float* norm_weight, const float* norm_bias, float eps, int act, float* y,
                   int64_t ldy, void* stream) {
  RTB_CHECK_CTX(ctx);
  if (rows < 0 || d < 0) return set_error(RTB_E_INVALID, "negative size");
  if (rows == 0 || d == 0) return RTB_OK;
  if (!x || !y) return set_error(RTB_E_INVALID, "null tensor");
  if (ldx < d || ldy < d) return set_error(RTB_E_INVALID, "leading dimension below d");
  if (act < RTB_ACT_NONE || act > RTB_ACT_TANH) return set_error(RTB_E_INVALID, "unknown activation");
  DeviceGuard g(ctx->device);
  return launch_layernorm_act(ctx, x, ldx, y, ldy, rows, d, norm_weight, norm_bias, eps, act,
                              pick_stream(ctx, stream));
}

// ---------------------------------------------------------------- conv
int64_t rtb_conv2d_packed_weight_size(int64_t Co, int64_t Ci, int64_t kh, int64_t kw) {
  return Co * kh * kw * round_up(Ci, 4);
}

int rtb_conv2d_prepack_weight(rtb_ctx* ctx, int64_t Co, int64_t Ci, int64_t kh, int64_t kw,
                              const float* w, float* w_packed, void* stream) {
  RTB_CHECK_CTX(ctx);
  if (Co <= 0 || Ci <= 0 || kh <= 0 || kw <= 0 || !w || !w_packed)
    return set_error(RTB_E_INVALID, "prepack: bad arguments");
  DeviceGuard g(ctx->device);
  return launch_prepack_weight(w, Co, Ci, kh, kw, round_up(Ci, 4), w_packed, nullptr,
                               pick_stream(ctx, stream));
}

int rtb_conv2d_prepack_weight_lo(rtb_ctx* ctx, int64_t Co, int64_t Ci, int64_t kh, int64_t kw,
                                 const float* w, float* w_packed, float* w_lo, void* stream) {
  RTB_CHECK_CTX(ctx);
  if (Co <= 0 || Ci <= 0 || kh <= 0 || kw <= 0 || !w || !w_packed || !w_lo)
    return set_error(RTB_E_INVALID, "prepack: bad arguments");
  DeviceGuard g(ctx->device);
  return launch_prepack_weight(w, Co, Ci, kh, kw, round_up(Ci, 4), w_packed, w_lo,
                               pick_stream(ctx, stream));
}

int rtb_nchw_to_nhwc_padded(rtb_ctx* ctx, int64_t N, int64_t C, int64_t H, int64_t W,
                            const float* x, float* y, void* stream) {
  RTB_CHECK_CTX(ctx);
  if (N < 0 || C <= 0 || H < 0 || W < 0 || !x || !y)
    return set_error(RTB_E_INVALID, "nchw_to_nhwc: bad arguments");
  if (N == 0 || H == 0 || W == 0) return RTB_OK;
  DeviceGuard g(ctx->device);
  return launch_nchw_to_nhwc_padded(x, N, C, H, W, round_up(C, 4), y, pick_stream(ctx, stream));
}

static int conv_check(int64_t N, int64_t Ci, int64_t H, int64_t W, int64_t Co, int64_t kh,
                      int64_t kw, int64_t sh, int64_t sw, int64_t ph, int64_t pw, int64_t* Ho,
                      int64_t* Wo) {
  // ops::conv2d panics (rustorch-core/src/ops/conv.rs:747-764) on these.
  if (N < 0 || Ci <= 0 || H <= 0 || W <= 0 || Co <= 0 || kh <= 0 || kw <= 0)
    return set_error(RTB_E_INVALID, "Conv2d requires 4D tensors with positive sizes");
  if (sh <= 0 || sw <= 0 || ph < 0 || pw < 0) return set_error(RTB_E_INVALID, "bad stride/padding");
  if (H + 2 * ph < kh || W + 2 * pw < kw)
    return set_error(RTB_E_INVALID, "kernel larger than padded input");
  *Ho = (H + 2 * ph - kh) / sh + 1;
  *Wo = (W + 2 * pw - kw) / sw + 1;
  return RTB_OK;
}

static int conv_core(rtb_ctx* ctx, int64_t N, int64_t Ci, int64_t H, int64_t W, int64_t Co,
                     int64_t kh, int64_t kw, int64_t sh, int64_t sw, int64_t ph, int64_t pw,
                     int64_t Ho, int64_t Wo, const float* x_nhwc, const float* wp,
                     const float* bias, const float* residual, int act, float* y, int y_layout,
                     int split3, cudaStream_t s, bool allow_workspace = true,
                     const float* wlo = nullptr) {
  const int64_t Cp = round_up(Ci, 4);
  const int64_t M = N * Ho * Wo;
  if (M == 0) return RTB_OK;
  if (M > INT32_MAX || N * H * W * Cp > ((int64_t)1 << 40))
    return set_error(RTB_E_UNSUPPORTED, "conv: problem too large for one launch");
  GemmDesc d;
  d.M = M; d.N = Co; d.K = kh * kw * Cp;
  d.B = wp; d.ldb = d.K; d.b_mn_major = 0;
  d.B_lo = wlo;
  d.C = y; d.bias = bias; d.residual = residual; d.act = act;
  if (y_layout == RTB_LAYOUT_NHWC) {
    d.out_mode = 0; d.ldc = Co; d.ldr = Co;
  } else {
    d.out_mode = 1; d.ldc = Co; d.hw = (int)(Ho * Wo);
  }
  // TMA im2col when every k-block is a single filter tap (Cp % 32 == 0), the
  // corners fit the map's signed 8-bit range, and the tensor is not tiny;
  // otherwise the cp.async gather producer.
  const bool tma_ok = pw <= 127 && ph <= 127 && (kw - 1 - pw) <= 128 && (kh - 1 - ph) <= 128 &&
                      N * H * W * Cp * 4 >= (int64_t)(256 << 10) &&
                      std::getenv("RTB_CONV_GATHER") == nullptr;
  // Cp in {8, 16}: several taps per k-block, each one TMA im2col box of Cp
  // channels, read by the 3xTF32 converters.  Measured faster than the gather
  // at Cp = 16 (52.6 vs 68.9 us) and 8 (39.9 vs 48.2 us, [64,Cp,56,56] 3x3);
  // at Cp = 4 (the 3-channel stem) eight 2 KB boxes per k-block are slower
  // than the gather (1492 vs 1214 us), so Cp = 4 keeps the gather.
  const bool multitap_ok = split3 && (Cp == 8 || Cp == 16);
  d.gather = (tma_ok && Cp % 32 == 0) ? 2 : ((tma_ok && multitap_ok) ? 3 : 1);
  d.x = x_nhwc;
  d.Nimg = (int)N;
  d.H = (int)H; d.W = (int)W; d.Cp = (int)Cp; d.Ho = (int)Ho; d.Wo = (int)Wo;
  d.R = (int)kh; d.S = (int)kw; d.sh = (int)sh; d.sw = (int)sw; d.ph = (int)ph; d.pw = (int)pw;
  d.split3 = split3;
  d.allow_workspace = allow_workspace ? 1 : 0;
  return gemm_run(ctx, d, s);
}

static int conv_packed_impl(rtb_ctx* ctx, int64_t N, int64_t Ci, int64_t H, int64_t W,
                            int64_t Co, int64_t kh, int64_t kw, int64_t sh, int64_t sw,
                            int64_t ph, int64_t pw, const float* x_nhwc_padded,
                            const float* w_packed, const float* bias, const float* residual,
                            int act, float* y, int y_layout, int precision, void* stream,
                            bool allow_workspace, const float* w_lo = nullptr) {
  RTB_CHECK_CTX(ctx);
  int64_t Ho, Wo;
  int st = conv_check(N, Ci, H, W, Co, kh, kw, sh, sw, ph, pw, &Ho, &Wo);
  if (st) return st;
  if (N == 0) return RTB_OK;
  if (!x_nhwc_padded || !w_packed || !y) return set_error(RTB_E_INVALID, "conv: null pointer");
  if (!aligned16(x_nhwc_padded) || !aligned16(w_packed) || (w_lo && !aligned16(w_lo)))
    return set_error(RTB_E_INVALID, "conv: packed input/weight must be 16-byte aligned");
  if (y_layout != RTB_LAYOUT_NCHW && y_layout != RTB_LAYOUT_NHWC)
    return set_error(RTB_E_INVALID, "conv: bad y_layout");
  int split3 = 1;
  if ((st = check_act(act))) return st;
  if ((st = resolve_precision(ctx, precision, &split3))) return st;
  DeviceGuard g(ctx->device);
  return conv_core(ctx, N, Ci, H, W, Co, kh, kw, sh, sw, ph, pw, Ho, Wo, x_nhwc_padded, w_packed,
                   bias, residual, act, y, y_layout, split3, pick_stream(ctx, stream),
                   allow_workspace, split3 ? w_lo : nullptr);
}

}  // extern "C"

namespace rtb {
int conv2d_fwd_packed_noalloc(rtb_ctx* ctx, int64_t N, int64_t Ci, int64_t H, int64_t W,
                              int64_t Co, int64_t kh, int64_t kw, int64_t sh, int64_t sw,
                              int64_t ph, int64_t pw, const float* x_nhwc_padded,
                              const float* w_packed, const float* bias, const float* residual,
                              int act, float* y, int y_layout, int precision, void* stream) {
  return conv_packed_impl(ctx, N, Ci, H, W, Co, kh, kw, sh, sw, ph, pw, x_nhwc_padded, w_packed,
                          bias, residual, act, y, y_layout, precision, stream, false);
}
}  // namespace rtb

extern "C" {

int rtb_conv2d_fwd_packed(rtb_ctx* ctx, int64_t N, int64_t Ci, int64_t H, int64_t W, int64_t Co,
                          int64_t kh, int64_t kw, int64_t sh, int64_t sw, int64_t ph, int64_t pw,
                          const float* x_nhwc_padded, const float* w_packed, const float* bias,
                          const float* residual, int act, float* y, int y_layout, int precision,
                          void* stream) {
  return conv_packed_impl(ctx, N, Ci, H, W, Co, kh, kw, sh, sw, ph, pw, x_nhwc_padded, w_packed,
                          bias, residual, act, y, y_layout, precision, stream, true);
}

int rtb_conv2d_fwd_packed_lo(rtb_ctx* ctx, int64_t N, int64_t Ci, int64_t H, int64_t W, int64_t Co,
                             int64_t kh, int64_t kw, int64_t sh, int64_t sw, int64_t ph, int64_t pw,
                             const float* x_nhwc_padded, const float* w_packed, const float* w_lo,
                             const float* bias, const float* residual, int act, float* y,
                             int y_layout, int precision, void* stream) {
  return conv_packed_impl(ctx, N, Ci, H, W, Co, kh, kw, sh, sw, ph, pw, x_nhwc_padded, w_packed,
                          bias, residual, act, y, y_layout, precision, stream, true, w_lo);
}

int rtb_conv2d_fwd(rtb_ctx* ctx, int64_t N, int64_t Ci, int64_t H, int64_t W, int64_t Co,
                   int64_t kh, int64_t kw, int64_t sh, int64_t sw, int64_t ph, int64_t pw,
                   const float* x, int x_layout, const float* w, const float* bias,
                   const float* residual, int act, float* y, int y_layout, int precision,
                   void* stream) {
  RTB_CHECK_CTX(ctx);
  int64_t Ho, Wo;
  int st = conv_check(N, Ci, H, W, Co, kh, kw, sh, sw, ph, pw, &Ho, &Wo);
  if (st) return st;
  if (N == 0) return RTB_OK;
  if (!x || !w || !y) return set_error(RTB_E_INVALID, "conv: null pointer");
  if (x_layout != RTB_LAYOUT_NCHW && x_layout != RTB_LAYOUT_NHWC)
    return set_error(RTB_E_INVALID, "conv: bad x_layout");
  if (y_layout != RTB_LAYOUT_NCHW && y_layout != RTB_LAYOUT_NHWC)
    return set_error(RTB_E_INVALID, "conv: bad y_layout");
  int split3 = 1;
  if ((st = check_act(act))) return st;
  if ((st = resolve_precision(ctx, precision, &split3))) return st;
  DeviceGuard g(ctx->device);
  cudaStream_t s = pick_stream(ctx, stream);
  const int64_t Cp = round_up(Ci, 4);
  float* xs = nullptr;
  float* ws = nullptr;
  const float* xin = x;
  // Stride-2 convs over <= 4 channels (the ResNet stem: 7x7 s2 over RGB): as
  // a stride-1 conv of the 16-channel space-to-depth input, whose k-blocks
  // are two 16-channel filter taps fetched by TMA im2col, instead of the
  // 4-channel cp.async gather.  3xTF32 only (the multi-tap producer feeds the
  // split converters).
  static const bool s2d_env = std::getenv("RTB_CONV_S2D") == nullptr ||
                              std::string(std::getenv("RTB_CONV_S2D")) != "0";
  if (x_layout == RTB_LAYOUT_NCHW && split3 && Ci <= 4 && sh == 2 && sw == 2 && kh >= 2 &&
      kw >= 2 && s2d_env && std::getenv("RTB_CONV_GATHER") == nullptr) {
    const int64_t kh2 = (kh + 1) / 2, kw2 = (kw + 1) / 2;
    const int64_t Hs = Ho + kh2 - 1, Ws = Wo + kw2 - 1;
    // the packed weight and its 3xTF32 low part, written by the prologue
    const int64_t wsz = Co * kh2 * kw2 * 16;
    st = ws_alloc(ctx, (void**)&ws, (size_t)(2 * wsz) * 4, s);
    if (st) return st;
    st = ws_alloc(ctx, (void**)&xs, (size_t)(N * Hs * Ws * 16) * 4, s);
    if (st == RTB_OK)
      st = launch_conv_prologue_s2d(x, N, Ci, H, W, ph, pw, Hs, Ws, xs, w, Co, kh, kw, ws,
                                    ws + wsz, s);
    if (st == RTB_OK)
      st = conv_core(ctx, N, 16, Hs, Ws, Co, kh2, kw2, 1, 1, 0, 0, Ho, Wo, xs, ws, bias, residual,
                     act, y, y_layout, split3, s, true, ws + wsz);
    ws_free(xs, s);
    ws_free(ws, s);
    return st;
  }
  // the packed weight, and (3xTF32) its low part: the prologue writes both, so
  // the GEMM needs no separate low-part pass
  const int64_t wsz = rtb_conv2d_packed_weight_size(Co, Ci, kh, kw);
  st = ws_alloc(ctx, (void**)&ws, (size_t)((split3 ? 2 : 1) * wsz) * 4, s);
  if (st) return st;
  float* wlo = split3 ? ws + wsz : nullptr;
  if (x_layout == RTB_LAYOUT_NCHW || Cp != Ci || !aligned16(x)) {
    st = ws_alloc(ctx, (void**)&xs, (size_t)(N * H * W * Cp) * 4, s);
    if (st == RTB_OK) {
      if (x_layout == RTB_LAYOUT_NCHW) {
        // layout change and weight repack in one launch
        st = launch_conv_prologue(x, N, Ci, H, W, Cp, xs, w, Co, kh, kw, ws, wlo, s);
      } else {
        // NHWC with Ci % 4 != 0 or unaligned: repack rows of Ci into rows of Cp.
        st = launch_pack_kmajor(x, N * H * W, Ci, Ci, 1, xs, Cp, s);
        if (st == RTB_OK) st = launch_prepack_weight(w, Co, Ci, kh, kw, Cp, ws, wlo, s);
      }
    }
    xin = xs;
  } else {
    st = launch_prepack_weight(w, Co, Ci, kh, kw, Cp, ws, wlo, s);
  }
  if (st == RTB_OK)
    st = conv_core(ctx, N, Ci, H, W, Co, kh, kw, sh, sw, ph, pw, Ho, Wo, xin, ws, bias, residual,
                   act, y, y_layout, split3, s, true, wlo);
  ws_free(xs, s);
  ws_free(ws, s);
  return st;
}

// ---------------------------------------------------------------- backward
int rtb_matmul_backward(rtb_ctx* ctx, int64_t M, int64_t N, int64_t K, const float* A,
                        const float* B, const float* dC, float* dA, float* dB, int accumulate,
                        int precision, void* stream) {
  RTB_CHECK_CTX(ctx);
  if (M < 0 || N < 0 || K < 0) return set_error(RTB_E_INVALID, "negative dimension");
  if ((dA && (!dC || !B)) || (dB && (!dC || !A)))
    return set_error(RTB_E_INVALID, "matmul_backward: null operand");
  int split3 = 1, st;
  if ((st = resolve_precision(ctx, precision, &split3))) return st;
  DeviceGuard g(ctx->device);
  cudaStream_t s = pick_stream(ctx, stream);
  // grad_lhs = grad . rhs^T: [M,N] . [N,K]; rhs [K,N] row-major is the [N',K'] view
  if (dA && M > 0 && K > 0) {
    if (N == 0) {
      if (!accumulate) {
        cudaError_t e = cudaMemsetAsync(dA, 0, (size_t)(M * K) * 4, s);
        if (e != cudaSuccess) return cuda_status(e, "matmul_backward memset");
      }
    } else if ((st = sgemm_one(ctx, M, K, N, dC, N, 0, B, N, 1, nullptr, 0, dA, K, split3, s,
                               accumulate ? dA : nullptr))) {
      return st;
    }
  }
  // grad_rhs = lhs^T . grad: [K,M] . [M,N]
  if (dB && K > 0 && N > 0) {
    if (M == 0) {
      if (!accumulate) {
        cudaError_t e = cudaMemsetAsync(dB, 0, (size_t)(K * N) * 4, s);
        if (e != cudaSuccess) return cuda_status(e, "matmul_backward memset");
      }
    } else if ((st = sgemm_one(ctx, K, N, M, A, K, 1, dC, N, 0, nullptr, 0, dB, N, split3, s,
                               accumulate ? dB : nullptr))) {
      return st;
    }
  }
  return RTB_OK;
}

int rtb_conv2d_backward(rtb_ctx* ctx, int64_t N, int64_t Ci, int64_t H, int64_t W, int64_t Co,
                        int64_t kh, int64_t kw, int64_t sh, int64_t sw, int64_t ph, int64_t pw,
                        const float* x, const float* w, const float* dy, float* dx, float* dw,
                        int accumulate, int precision, void* stream) {
  RTB_CHECK_CTX(ctx);
  int64_t Ho, Wo;
  int st = conv_check(N, Ci, H, W, Co, kh, kw, sh, sw, ph, pw, &Ho, &Wo);
  if (st) return st;
  if (!dy || (dx && !w) || (dw && !x)) return set_error(RTB_E_INVALID, "conv_backward: null pointer");
  int split3 = 1;
  if ((st = resolve_precision(ctx, precision, &split3))) return st;
  if (dx && (ph > kh - 1 || pw > kw - 1))
    return set_error(RTB_E_UNSUPPORTED, "conv_backward: padding larger than kernel-1");
  DeviceGuard g(ctx->device);
  cudaStream_t s = pick_stream(ctx, stream);
  if (N == 0) return RTB_OK;

  if (dx) {
    // grad_input: conv (stride 1, padding k-1-p) of dy dilated by the stride
    // (plus the rows/columns of x no window reaches) with the flipped filter.
    const int64_t Cop = round_up(Co, 4);
    const int64_t Hd = (Ho - 1) * sh + 1 + (H + 2 * ph - kh) % sh;
    const int64_t Wd = (Wo - 1) * sw + 1 + (W + 2 * pw - kw) % sw;
    const int64_t qh = kh - 1 - ph, qw = kw - 1 - pw;
    if (Hd + 2 * qh - kh + 1 != H || Wd + 2 * qw - kw + 1 != W)
      return set_error(RTB_E_INVALID, "conv_backward: inconsistent geometry");
    float* dyd = nullptr;
    float* wt = nullptr;
    const size_t dyd_bytes = (size_t)(N * Hd * Wd * Cop) * 4;
    st = ws_alloc(ctx, (void**)&dyd, dyd_bytes, s);
    if (st == RTB_OK && Hd == Ho && Wd == Wo) {
      // nothing to dilate (stride 1): the plain channel-padded NHWC copy
      st = launch_nchw_to_nhwc_padded(dy, N, Co, Ho, Wo, Cop, dyd, s);
    } else if (st == RTB_OK) {
      cudaError_t e = cudaMemsetAsync(dyd, 0, dyd_bytes, s);
      st = e == cudaSuccess ? RTB_OK : cuda_status(e, "conv_backward memset");
      if (st == RTB_OK)
        st = launch_dilate_nchw_to_nhwc(dy, N, Co, Ho, Wo, sh, sw, Hd, Wd, Cop, dyd, s);
    }
    if (st == RTB_OK) st = ws_alloc(ctx, (void**)&wt, (size_t)(Ci * kh * kw * Cop) * 4, s);
    if (st == RTB_OK) st = launch_prepack_flip(w, Co, Ci, kh, kw, Cop, wt, s);
    if (st == RTB_OK)
      st = conv_core(ctx, N, Co, Hd, Wd, Ci, kh, kw, 1, 1, qh, qw, H, W, dyd, wt, nullptr,
                     accumulate ? dx : nullptr, 0, dx, RTB_LAYOUT_NCHW, split3, s);
    ws_free(dyd, s);
    ws_free(wt, s);
    if (st) return st;
  }
  if (dw) {
    // grad_weight = dy^T [Co, P] . im2col(x) [P, kh*kw*Cp], P = N*Ho*Wo
    const int64_t Cp = round_up(Ci, 4);
    const int64_t P = N * Ho * Wo;
    const int64_t Pp = round_up(P, 4);
    const int64_t Kp = kh * kw * Cp;
    float *xh = nullptr, *col = nullptr, *dyt = nullptr, *dwp = nullptr;
    st = ws_alloc(ctx, (void**)&xh, (size_t)(N * H * W * Cp) * 4, s);
    if (st == RTB_OK) st = launch_nchw_to_nhwc_padded(x, N, Ci, H, W, Cp, xh, s);
    if (st == RTB_OK) st = ws_alloc(ctx, (void**)&col, (size_t)(P * Kp) * 4, s);
    if (st == RTB_OK) st = launch_im2col_nhwc(xh, N, H, W, Cp, Ho, Wo, kh, kw, sh, sw, ph, pw, col, s);
    if (st == RTB_OK) st = ws_alloc(ctx, (void**)&dyt, (size_t)(Co * Pp) * 4, s);
    if (st == RTB_OK) st = launch_nchw_to_cmajor(dy, N, Co, Ho * Wo, Pp, dyt, s);
    if (st == RTB_OK) st = ws_alloc(ctx, (void**)&dwp, (size_t)(Co * Kp) * 4, s);
    if (st == RTB_OK)
      st = sgemm_one(ctx, Co, Kp, P, dyt, Pp, 0, col, Kp, 0, nullptr, 0, dwp, Kp, split3, s);
    if (st == RTB_OK) st = launch_unpack_weight_grad(dwp, Co, Ci, kh, kw, Cp, accumulate, dw, s);
    ws_free(xh, s);
    ws_free(col, s);
    ws_free(dyt, s);
    ws_free(dwp, s);
    if (st) return st;
  }
  return RTB_OK;
}

// ---------------------------------------------------------------- small ops
int rtb_max_pool2d(rtb_ctx* ctx, int64_t N, int64_t C, int64_t H, int64_t W, int64_t kh,
                   int64_t kw, int64_t sh, int64_t sw, int64_t ph, int64_t pw, const float* x,
                   float* y, int layout, void* stream) {
  RTB_CHECK_CTX(ctx);
  if (N < 0 || C <= 0 || H <= 0 || W <= 0 || kh <= 0 || kw <= 0 || sh <= 0 || sw <= 0 || ph < 0 ||
      pw < 0 || H + 2 * ph < kh || W + 2 * pw < kw)
    return set_error(RTB_E_INVALID, "MaxPool2d requires 4D tensor (N, C, H, W)");
  if (layout != RTB_LAYOUT_NCHW && layout != RTB_LAYOUT_NHWC)
    return set_error(RTB_E_INVALID, "max_pool2d: bad layout");
  if (N == 0) return RTB_OK;
  if (!x || !y) return set_error(RTB_E_INVALID, "max_pool2d: null pointer");
  DeviceGuard g(ctx->device);
  return launch_max_pool2d(x, y, N, C, H, W, kh, kw, sh, sw, ph, pw, layout,
                           pick_stream(ctx, stream));
}

int rtb_global_avg_pool(rtb_ctx* ctx, int64_t N, int64_t C, int64_t H, int64_t W, const float* x,
                        float* y, int layout, void* stream) {
  RTB_CHECK_CTX(ctx);
  if (N < 0 || C <= 0 || H <= 0 || W <= 0) return set_error(RTB_E_INVALID, "avg_pool: bad shape");
  if (layout != RTB_LAYOUT_NCHW && layout != RTB_LAYOUT_NHWC)
    return set_error(RTB_E_INVALID, "avg_pool: bad layout");
  if (N == 0) return RTB_OK;
  if (!x || !y) return set_error(RTB_E_INVALID, "avg_pool: null pointer");
  DeviceGuard g(ctx->device);
  return launch_global_avg_pool(x, y, N, C, H * W, layout, pick_stream(ctx, stream));
}

int rtb_add(rtb_ctx* ctx, int64_t n, const float* a, const float* b, float* y, void* stream) {
  RTB_CHECK_CTX(ctx);
  if (n < 0) return set_error(RTB_E_INVALID, "add: negative size");
  if (n == 0) return RTB_OK;
  if (!a || !b || !y) return set_error(RTB_E_INVALID, "add: null pointer");
  DeviceGuard g(ctx->device);
  return launch_add(a, b, y, n, pick_stream(ctx, stream));
}

int rtb_elementwise_broadcast(rtb_ctx* ctx, int op, int ndim, const int64_t* shape,
                              const float* a, const int64_t* a_strides, const float* b,
                              const int64_t* b_strides, float* y, void* stream) {
  RTB_CHECK_CTX(ctx);
  if (op != 0 && op != 1) return set_error(RTB_E_INVALID, "elementwise: op must be 0 (add) or 1 (mul)");
  if (!shape || !a_strides || !b_strides) return set_error(RTB_E_INVALID, "elementwise: null shape");
  for (int k = 0; k < ndim; ++k)
    if (shape[k] < 0) return set_error(RTB_E_INVALID, "elementwise: negative extent");
  int64_t n = 1;
  for (int k = 0; k < ndim; ++k) n *= shape[k];
  if (n == 0) return RTB_OK;
  if (!a || !b || !y) return set_error(RTB_E_INVALID, "elementwise: null pointer");
  DeviceGuard g(ctx->device);
  return launch_broadcast(op, ndim, shape, a, a_strides, b, b_strides, y, pick_stream(ctx, stream));
}

int rtb_relu(rtb_ctx* ctx, int64_t n, const float* x, float* y, void* stream) {
  RTB_CHECK_CTX(ctx);
  if (n < 0) return set_error(RTB_E_INVALID, "relu: negative size");
  if (n == 0) return RTB_OK;
  if (!x || !y) return set_error(RTB_E_INVALID, "relu: null pointer");
  DeviceGuard g(ctx->device);
  return launch_relu(x, y, n, pick_stream(ctx, stream));
}

}  // extern "C"

// ---------------------------------------------------------------- data
// SplitMix64-based generator (documented in the header).  Same arithmetic as
// the published spec: finaliser constants of SplitMix64, Box-Muller in double.
static inline uint64_t sm_fin(uint64_t x) {
  x ^= x >> 30;
  x *= 0xBF58476D1CE4E5B9ULL;
  x ^= x >> 27;
  x *= 0x94D049BB133111EBULL;
  x ^= x >> 31;
  return x;
}
static inline uint64_t sm_key(uint64_t seed, uint64_t tid) {
  return sm_fin(seed * 0x9E3779B97F4A7C15ULL + tid * 0xD1B54A32D192ED03ULL + 1ULL);
}
static inline uint64_t sm_draw(uint64_t key, uint64_t i) {
  return sm_fin(i + key * 0x9E3779B97F4A7C15ULL);
}

template <class F>
static void parallel_ranges(int64_t n, F f) {
  unsigned nt = std::thread::hardware_concurrency();
  if (nt == 0) nt = 1;
  if (nt > 64) nt = 64;
  if (n < (int64_t)1 << 16) nt = 1;
  std::vector<std::thread> th;
  const int64_t chunk = (n + nt - 1) / nt;
  for (unsigned t = 0; t < nt; ++t) {
    const int64_t a = (int64_t)t * chunk, b = a + chunk < n ? a + chunk : n;
    if (a >= b) break;
    th.emplace_back([=] { f(a, b); });
  }
  for (auto& x : th) x.join();
}

extern "C" {

int rtb_fill_normal_host(float* out, int64_t n, uint64_t seed, uint64_t tensor_id, float mean,
                         float std_dev) {
  if (n < 0 || (n > 0 && !out)) return set_error(RTB_E_INVALID, "fill_normal: bad arguments");
  const uint64_t key = sm_key(seed, tensor_id);
  const int64_t npairs = (n + 1) / 2;
  parallel_ranges(npairs, [=](int64_t a, int64_t b) {
    for (int64_t j = a; j < b; ++j) {
      const uint64_t d1 = sm_draw(key, (uint64_t)(2 * j)), d2 = sm_draw(key, (uint64_t)(2 * j + 1));
      const double u1 = ((double)(d1 >> 11) + 0.5) * (1.0 / 9007199254740992.0);
      const double u2 = ((double)(d2 >> 11) + 0.5) * (1.0 / 9007199254740992.0);
      const double r = std::sqrt(-2.0 * std::log(u1));
      const double t = 6.283185307179586476925286766559 * u2;
      out[2 * j] = (float)((double)mean + (double)std_dev * r * std::cos(t));
      if (2 * j + 1 < n) out[2 * j + 1] = (float)((double)mean + (double)std_dev * r * std::sin(t));
    }
  });
  return RTB_OK;
}

int rtb_fill_uniform_host(float* out, int64_t n, uint64_t seed, uint64_t tensor_id, float lo,
                          float hi) {
  if (n < 0 || (n > 0 && !out)) return set_error(RTB_E_INVALID, "fill_uniform: bad arguments");
  const uint64_t key = sm_key(seed, tensor_id);
  parallel_ranges(n, [=](int64_t a, int64_t b) {
    for (int64_t i = a; i < b; ++i) {
      const uint64_t d = sm_draw(key, (uint64_t)i);
      const double u = ((double)(d >> 40) + 0.5) * (1.0 / 16777216.0);
      out[i] = (float)((double)lo + ((double)hi - (double)lo) * u);
    }
  });
  return RTB_OK;
}

}  // extern "C"
