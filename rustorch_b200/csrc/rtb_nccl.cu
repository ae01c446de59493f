// Multi-GPU: NCCL communicator bootstrap and the N-split GEMM, either as a
// GEMM followed by an NCCL all-gather of C, or fused: the GEMM epilogue
// stores every finished tile straight into all ranks' C over NVLink (CUDA IPC
// mappings of the peers' buffers), so the exchange overlaps the remaining
// tiles' math, and a one-element NCCL all-reduce closes it as a barrier.  One
// process per GPU.
#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "rtb_internal.h"

using namespace rtb;

// NCCL is resolved at first use with dlopen("libnccl.so.2") instead of being
// linked: a process that already loaded an NCCL (e.g. torch's bundled one,
// same soname) then shares that instance, and loading this library never
// changes which NCCL other libraries bind to.
namespace {
struct NcclApi {
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*CommCount)(const ncclComm_t, int*) = nullptr;
  ncclResult_t (*CommUserRank)(const ncclComm_t, int*) = nullptr;
  ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
  bool ok = false;
};

const NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return;
    api.GetUniqueId = (decltype(api.GetUniqueId))dlsym(h, "ncclGetUniqueId");
    api.CommInitRank = (decltype(api.CommInitRank))dlsym(h, "ncclCommInitRank");
    api.CommDestroy = (decltype(api.CommDestroy))dlsym(h, "ncclCommDestroy");
    api.CommCount = (decltype(api.CommCount))dlsym(h, "ncclCommCount");
    api.CommUserRank = (decltype(api.CommUserRank))dlsym(h, "ncclCommUserRank");
    api.AllGather = (decltype(api.AllGather))dlsym(h, "ncclAllGather");
    api.AllReduce = (decltype(api.AllReduce))dlsym(h, "ncclAllReduce");
    api.GetErrorString = (decltype(api.GetErrorString))dlsym(h, "ncclGetErrorString");
    api.ok = api.GetUniqueId && api.CommInitRank && api.CommDestroy && api.CommCount &&
             api.CommUserRank && api.AllGather && api.AllReduce && api.GetErrorString;
  });
  return api;
}

int nccl_missing() { return set_error(RTB_E_NCCL, "libnccl.so.2 could not be loaded"); }
}  // namespace

static int nccl_status(ncclResult_t r, const char* what) {
  return set_error(RTB_E_NCCL, std::string(what) + ": " + nccl().GetErrorString(r));
}

static int comm_rank_count(ncclComm_t cm, int* P, int* rank) {
  ncclResult_t r = nccl().CommCount(cm, P);
  if (r == ncclSuccess) r = nccl().CommUserRank(cm, rank);
  return r == ncclSuccess ? RTB_OK : nccl_status(r, "ncclCommCount/UserRank");
}

// A C buffer of `bytes` on every rank, each rank holding pointers to all of
// them (its own plus the peers' CUDA IPC mappings).
struct rtb_peer_buffer {
  int device = 0;
  int P = 0, rank = 0;
  float* local = nullptr;
  size_t bytes = 0;
  std::vector<float*> ptrs;    // [P]; ptrs[rank] == local
  float** d_ptrs = nullptr;    // device copy for the epilogue
  int* d_flag = nullptr;       // one int for the barrier all-reduce
};

// Every rank reaches this point before the call returns on the stream.
static int stream_barrier(ncclComm_t cm, int* d_flag, cudaStream_t s) {
  ncclResult_t r = nccl().AllReduce(d_flag, d_flag, 1, ncclInt32, ncclSum, cm, s);
  return r == ncclSuccess ? RTB_OK : nccl_status(r, "ncclAllReduce (barrier)");
}

extern "C" {

int rtb_nccl_unique_id(void* id_out_128b) {
  if (!id_out_128b) return set_error(RTB_E_INVALID, "null id buffer");
  static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId is 128 bytes");
  if (!nccl().ok) return nccl_missing();
  ncclUniqueId id;
  ncclResult_t r = nccl().GetUniqueId(&id);
  if (r != ncclSuccess) return nccl_status(r, "ncclGetUniqueId");
  std::memcpy(id_out_128b, &id, sizeof id);
  return RTB_OK;
}

int rtb_nccl_comm_init(rtb_ctx* ctx, const void* id_128b, int nranks, int rank, void** comm) {
  if (!ctx || !id_128b || !comm) return set_error(RTB_E_INVALID, "nccl_comm_init: null argument");
  if (nranks <= 0 || rank < 0 || rank >= nranks)
    return set_error(RTB_E_INVALID, "nccl_comm_init: bad rank/nranks");
  if (!nccl().ok) return nccl_missing();
  DeviceGuard g(ctx->device);
  ncclUniqueId id;
  std::memcpy(&id, id_128b, sizeof id);
  ncclComm_t c = nullptr;
  ncclResult_t r = nccl().CommInitRank(&c, nranks, id, rank);
  if (r != ncclSuccess) return nccl_status(r, "ncclCommInitRank");
  *comm = c;
  return RTB_OK;
}

int rtb_nccl_comm_destroy(void* comm) {
  if (!comm) return RTB_OK;
  if (!nccl().ok) return nccl_missing();
  ncclResult_t r = nccl().CommDestroy(static_cast<ncclComm_t>(comm));
  if (r != ncclSuccess) return nccl_status(r, "ncclCommDestroy");
  return RTB_OK;
}

int rtb_sgemm_nsplit_allgather(rtb_ctx* ctx, void* comm, int64_t M, int64_t N, int64_t K,
                               const float* A, const float* B_local, float* c_parts, float* C,
                               int precision, void* stream) {
  if (!ctx || !comm) return set_error(RTB_E_INVALID, "nsplit: null ctx/comm");
  if (!nccl().ok) return nccl_missing();
  ncclComm_t cm = static_cast<ncclComm_t>(comm);
  int P = 0, rank = 0;
  ncclResult_t r = nccl().CommCount(cm, &P);
  if (r == ncclSuccess) r = nccl().CommUserRank(cm, &rank);
  if (r != ncclSuccess) return nccl_status(r, "ncclCommCount/UserRank");
  if (M <= 0 || N <= 0 || K < 0 || N % P != 0)
    return set_error(RTB_E_INVALID, "nsplit: need M,N > 0 and N divisible by the rank count");
  if (!A || !B_local || !c_parts || !C) return set_error(RTB_E_INVALID, "nsplit: null pointer");
  const int64_t Nl = N / P;
  float* mine = c_parts + (int64_t)rank * M * Nl;
  // Local block C_r = A . B_r  ([M,K] x [K,Nl] row-major).
  int st = rtb_sgemm(ctx, M, Nl, K, A, K, 0, B_local, Nl, 0, nullptr, RTB_ACT_NONE, mine, Nl,
                     precision, stream);
  if (st) return st;
  DeviceGuard g(ctx->device);
  cudaStream_t s = pick_stream(ctx, stream);
  // In-place all-gather: rank r's block already sits at offset r*M*Nl.
  r = nccl().AllGather(mine, c_parts, (size_t)(M * Nl), ncclFloat, cm, s);
  if (r != ncclSuccess) return nccl_status(r, "ncclAllGather");
  return launch_unsplit_cols(c_parts, C, P, M, Nl, s);
}

int rtb_peer_buffer_create(rtb_ctx* ctx, void* comm, size_t bytes, void** out) {
  if (!ctx || !comm || !out || bytes == 0)
    return set_error(RTB_E_INVALID, "peer_buffer_create: bad argument");
  if (!nccl().ok) return nccl_missing();
  *out = nullptr;
  ncclComm_t cm = static_cast<ncclComm_t>(comm);
  int P = 0, rank = 0;
  int st = comm_rank_count(cm, &P, &rank);
  if (st) return st;
  DeviceGuard g(ctx->device);
  auto* pb = new rtb_peer_buffer;
  pb->device = ctx->device;
  pb->P = P;
  pb->rank = rank;
  pb->bytes = bytes;
  pb->ptrs.assign(P, nullptr);
  cudaStream_t s = ctx->stream;
  char* d_handles = nullptr;
  std::vector<cudaIpcMemHandle_t> handles(P);
  cudaError_t e = cudaMalloc(&pb->local, bytes);
  if (e == cudaSuccess) e = cudaMalloc(&pb->d_flag, sizeof(int));
  if (e == cudaSuccess) e = cudaMemset(pb->d_flag, 0, sizeof(int));
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&handles[rank], pb->local);
  if (e == cudaSuccess) e = cudaMalloc(&d_handles, sizeof(cudaIpcMemHandle_t) * P);
  if (e == cudaSuccess)
    e = cudaMemcpy(d_handles + sizeof(cudaIpcMemHandle_t) * rank, &handles[rank],
                   sizeof(cudaIpcMemHandle_t), cudaMemcpyHostToDevice);
  if (e != cudaSuccess) st = cuda_status(e, "peer_buffer_create");
  if (st == RTB_OK) {
    // exchange the handles over the communicator (in place)
    ncclResult_t r = nccl().AllGather(d_handles + sizeof(cudaIpcMemHandle_t) * rank, d_handles,
                                      sizeof(cudaIpcMemHandle_t), ncclChar, cm, s);
    if (r != ncclSuccess) st = nccl_status(r, "ncclAllGather (IPC handles)");
  }
  if (st == RTB_OK) {
    e = cudaStreamSynchronize(s);
    if (e == cudaSuccess)
      e = cudaMemcpy(handles.data(), d_handles, sizeof(cudaIpcMemHandle_t) * P,
                     cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) st = cuda_status(e, "peer_buffer_create (handles)");
  }
  for (int q = 0; st == RTB_OK && q < P; ++q) {
    if (q == rank) {
      pb->ptrs[q] = pb->local;
      continue;
    }
    void* ptr = nullptr;
    e = cudaIpcOpenMemHandle(&ptr, handles[q], cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) st = cuda_status(e, "cudaIpcOpenMemHandle");
    pb->ptrs[q] = static_cast<float*>(ptr);
  }
  if (st == RTB_OK) {
    e = cudaMalloc(&pb->d_ptrs, sizeof(float*) * P);
    if (e == cudaSuccess)
      e = cudaMemcpy(pb->d_ptrs, pb->ptrs.data(), sizeof(float*) * P, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) st = cuda_status(e, "peer_buffer_create (pointer table)");
  }
  if (d_handles) cudaFree(d_handles);
  if (st != RTB_OK) {
    // every rank makes the same collective calls, so a failure on one rank
    // has been reported as an error (not a hang) on the others as well
    for (int q = 0; q < P; ++q)
      if (q != rank && pb->ptrs[q]) cudaIpcCloseMemHandle(pb->ptrs[q]);
    cudaFree(pb->d_ptrs);
    cudaFree(pb->d_flag);
    cudaFree(pb->local);
    delete pb;
    return st;
  }
  *out = pb;
  return RTB_OK;
}

int rtb_peer_buffer_local(void* pb_, float** local) {
  if (!pb_ || !local) return set_error(RTB_E_INVALID, "peer_buffer_local: null argument");
  *local = static_cast<rtb_peer_buffer*>(pb_)->local;
  return RTB_OK;
}

int rtb_peer_buffer_destroy(void* pb_, void* comm) {
  if (!pb_) return RTB_OK;
  if (!comm) return set_error(RTB_E_INVALID, "peer_buffer_destroy: null comm");
  if (!nccl().ok) return nccl_missing();
  auto* pb = static_cast<rtb_peer_buffer*>(pb_);
  DeviceGuard g(pb->device);
  // Unmap the peers' buffers, then wait until every rank has done the same
  // before freeing this rank's buffer.
  cudaDeviceSynchronize();
  for (int q = 0; q < pb->P; ++q)
    if (q != pb->rank && pb->ptrs[q]) cudaIpcCloseMemHandle(pb->ptrs[q]);
  int st = stream_barrier(static_cast<ncclComm_t>(comm), pb->d_flag, nullptr);
  cudaError_t e = cudaDeviceSynchronize();
  if (st == RTB_OK && e != cudaSuccess) st = cuda_status(e, "peer_buffer_destroy");
  cudaFree(pb->d_ptrs);
  cudaFree(pb->d_flag);
  cudaFree(pb->local);
  delete pb;
  return st;
}

int rtb_sgemm_nsplit_p2p(rtb_ctx* ctx, void* comm, void* pbuf, int64_t M, int64_t N, int64_t K,
                         const float* A, const float* B_local, int precision, void* stream) {
  if (!ctx || !comm || !pbuf) return set_error(RTB_E_INVALID, "nsplit_p2p: null ctx/comm/buffer");
  if (!nccl().ok) return nccl_missing();
  auto* pb = static_cast<rtb_peer_buffer*>(pbuf);
  ncclComm_t cm = static_cast<ncclComm_t>(comm);
  const int P = pb->P, rank = pb->rank;
  if (M <= 0 || N <= 0 || K <= 0 || N % P != 0)
    return set_error(RTB_E_INVALID, "nsplit_p2p: need M,N,K > 0 and N divisible by the rank count");
  if ((size_t)(M * N) * sizeof(float) > pb->bytes)
    return set_error(RTB_E_INVALID, "nsplit_p2p: C does not fit the peer buffer");
  if (!A || !B_local) return set_error(RTB_E_INVALID, "nsplit_p2p: null operand");
  const int64_t Nl = N / P;
  auto al16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
  if (K % 4 || Nl % 4 || !al16(A) || !al16(B_local))
    return set_error(RTB_E_UNSUPPORTED,
                     "nsplit_p2p: needs K and N/ranks multiples of 4 and 16-byte aligned operands");
  int split3 = precision == RTB_PREC_TF32 ? 0 : 1;
  if (precision == RTB_PREC_DEFAULT) split3 = ctx->default_precision == RTB_PREC_TF32 ? 0 : 1;
  else if (precision != RTB_PREC_TF32 && precision != RTB_PREC_3XTF32)
    return set_error(RTB_E_INVALID, "bad precision");
  DeviceGuard g(ctx->device);
  cudaStream_t s = pick_stream(ctx, stream);
  GemmDesc d;
  d.M = M; d.N = Nl; d.K = K;
  d.A = A; d.lda = K;
  d.B = B_local; d.ldb = Nl; d.b_mn_major = 1;  // [K, N/P] row-major
  d.C = pb->local; d.ldc = N;
  d.out_mode = 2;
  d.peer_c = pb->d_ptrs;
  d.npeers = P;
  d.col_off = (int64_t)rank * Nl;
  d.split3 = split3;
  // entry barrier: no rank overwrites C while another may still be reading
  // the previous call's result; exit barrier: every rank's tiles have landed
  int st = stream_barrier(cm, pb->d_flag, s);
  if (st) return st;
  st = gemm_run(ctx, d, s);
  if (st) return st;
  return stream_barrier(cm, pb->d_flag, s);
}

}  // extern "C"
