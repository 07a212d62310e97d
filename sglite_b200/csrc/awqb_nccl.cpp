// NCCL communicator for the tensor-parallel all-reduce that follows every
// row-parallel projection. Restates the reference's native NCCLWrapper
// (kernels/csrc/src/pynccl.cu:75-189): a communicator built from a unique id
// that rank 0 creates and the other ranks receive out of band, an in-place SUM
// all-reduce of fp16/bf16 buffers, and a symmetric buffer allocated with
// ncclMemAlloc and registered as an NCCL_WIN_COLL_SYMMETRIC window, through
// which messages up to its size are reduced (NCCL can then use its
// low-latency symmetric / NVLS kernels over NVSwitch).
#include <cuda_runtime.h>
#include <nccl.h>

#include <cstring>

#include "awqb200.h"
#include "awqb_common.h"

namespace awqb {
namespace {

struct Comm {
  ncclComm_t comm = nullptr;
  int rank = 0, world = 1, device = 0;
  void* sym = nullptr;  // symmetric staging buffer (ncclMemAlloc)
  size_t sym_bytes = 0;
  ncclWindow_t win = nullptr;
};

}  // namespace
}  // namespace awqb

#define AWQB_NCCL(expr)                                                                     \
  do {                                                                                      \
    ncclResult_t _r = (expr);                                                               \
    if (_r != ncclSuccess) {                                                                \
      char _buf[512];                                                                       \
      snprintf(_buf, sizeof(_buf), "%s failed: %s", #expr, ncclGetErrorString(_r));         \
      ::awqb::set_last_error(_buf);                                                         \
      return ::awqb::kNcclError;                                                            \
    }                                                                                       \
  } while (0)

using namespace awqb;

extern "C" int awqb_nccl_unique_id_bytes(void) { return (int)sizeof(ncclUniqueId); }

extern "C" int awqb_nccl_get_unique_id(uint8_t* out) {
  AWQB_REQUIRE(out != nullptr, kInvalidArgument, "out is null");
  ncclUniqueId id;
  AWQB_NCCL(ncclGetUniqueId(&id));
  std::memcpy(out, &id, sizeof(id));
  return kOk;
}

extern "C" int awqb_nccl_init(const uint8_t* uid, int rank, int world, int64_t sym_bytes,
                              void** comm_out) {
  AWQB_REQUIRE(uid != nullptr && comm_out != nullptr, kInvalidArgument, "null pointer");
  AWQB_REQUIRE(world >= 1 && rank >= 0 && rank < world, kInvalidArgument, "bad rank %d / world %d",
               rank, world);
  AWQB_REQUIRE(sym_bytes >= 0, kInvalidArgument, "negative symmetric buffer size");
  ncclUniqueId id;
  std::memcpy(&id, uid, sizeof(id));
  Comm* c = new Comm();
  c->rank = rank;
  c->world = world;
  cudaGetDevice(&c->device);
  ncclResult_t r = ncclCommInitRank(&c->comm, world, id, rank);
  if (r != ncclSuccess) {
    delete c;
    AWQB_REQUIRE(false, kNcclError, "ncclCommInitRank failed: %s", ncclGetErrorString(r));
  }
  if (sym_bytes > 0) {
    r = ncclMemAlloc(&c->sym, (size_t)sym_bytes);
    if (r == ncclSuccess) r = ncclCommWindowRegister(c->comm, c->sym, (size_t)sym_bytes, &c->win,
                                                     NCCL_WIN_COLL_SYMMETRIC);
    if (r != ncclSuccess) {
      if (c->sym) ncclMemFree(c->sym);
      ncclCommDestroy(c->comm);
      delete c;
      AWQB_REQUIRE(false, kNcclError, "symmetric buffer setup failed: %s", ncclGetErrorString(r));
    }
    c->sym_bytes = (size_t)sym_bytes;
  }
  *comm_out = c;
  return kOk;
}

// Device pointer and size of the communicator's symmetric buffer (0 if none).
// A producer may write its output straight into it and then call
// awqb_nccl_all_reduce on that pointer, which skips the staging copy.
extern "C" int awqb_nccl_symmetric_buffer(void* comm, void** ptr, int64_t* bytes) {
  AWQB_REQUIRE(comm && ptr && bytes, kInvalidArgument, "null pointer");
  Comm* c = static_cast<Comm*>(comm);
  *ptr = c->sym;
  *bytes = (int64_t)c->sym_bytes;
  return kOk;
}

extern "C" int awqb_nccl_all_reduce(void* comm, void* buf, int64_t count, int dtype, void* stream) {
  AWQB_REQUIRE(comm != nullptr, kInvalidArgument, "comm is null");
  AWQB_REQUIRE(dtype == AWQB_DTYPE_F16 || dtype == AWQB_DTYPE_BF16, kInvalidArgument,
               "all-reduce supports fp16/bf16 only (got %d)", dtype);
  AWQB_REQUIRE(count >= 0 && (count == 0 || buf != nullptr), kInvalidArgument, "bad buffer");
  Comm* c = static_cast<Comm*>(comm);
  if (count == 0 || c->world == 1) return kOk;
  const ncclDataType_t t = dtype == AWQB_DTYPE_F16 ? ncclFloat16 : ncclBfloat16;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const size_t bytes = (size_t)count * 2;
  const bool in_sym = c->sym != nullptr && buf >= c->sym &&
                      static_cast<char*>(buf) + bytes <= static_cast<char*>(c->sym) + c->sym_bytes;
  if (in_sym || c->sym == nullptr || bytes > c->sym_bytes) {
    AWQB_NCCL(ncclAllReduce(buf, buf, (size_t)count, t, ncclSum, c->comm, s));
    return kOk;
  }
  AWQB_CUDA(cudaMemcpyAsync(c->sym, buf, bytes, cudaMemcpyDeviceToDevice, s));
  AWQB_NCCL(ncclAllReduce(c->sym, c->sym, (size_t)count, t, ncclSum, c->comm, s));
  AWQB_CUDA(cudaMemcpyAsync(buf, c->sym, bytes, cudaMemcpyDeviceToDevice, s));
  return kOk;
}

extern "C" int awqb_nccl_destroy(void* comm) {
  if (comm == nullptr) return kOk;
  Comm* c = static_cast<Comm*>(comm);
  int st = kOk;
  if (c->win != nullptr && ncclCommWindowDeregister(c->comm, c->win) != ncclSuccess) st = kNcclError;
  if (c->sym != nullptr && ncclMemFree(c->sym) != ncclSuccess) st = kNcclError;
  if (c->comm != nullptr && ncclCommDestroy(c->comm) != ncclSuccess) st = kNcclError;
  delete c;
  if (st != kOk) set_last_error("NCCL teardown reported an error");
  return st;
}
