// Multi-GPU: NCCL communicator bootstrap and the N-split GEMM with an
// all-gather of C over NVLink / NVSwitch (one process per GPU).
#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>
#include <string>

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
    api.GetErrorString = (decltype(api.GetErrorString))dlsym(h, "ncclGetErrorString");
    api.ok = api.GetUniqueId && api.CommInitRank && api.CommDestroy && api.CommCount &&
             api.CommUserRank && api.AllGather && api.GetErrorString;
  });
  return api;
}

int nccl_missing() { return set_error(RTB_E_NCCL, "libnccl.so.2 could not be loaded"); }
}  // namespace

static int nccl_status(ncclResult_t r, const char* what) {
  return set_error(RTB_E_NCCL, std::string(what) + ": " + nccl().GetErrorString(r));
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

}  // extern "C"
