// Column all-gather of a column-sharded W8A8 linear (multi-GPU inference).
//
// Rank r of G holds output columns [r*n_loc, (r+1)*n_loc) of Y [rows, G*n_loc]
// as a contiguous [rows, n_loc] tile.  qi8_allgather_cols runs one
// ncclAllGather into a caller scratch [G, rows, n_loc] on the caller's
// stream and then re-lays it out into Y (row stride ld_out) with one kernel.
// NCCL is resolved at run time (dlopen of libnccl.so.2, reusing the copy the
// process already loaded, e.g. PyTorch's), so the library itself loads on
// hosts without NCCL; only this entry point then reports QI8_EUNSUPPORTED.
#include <dlfcn.h>
#include <nccl.h>

#include <cstdint>
#include <mutex>

#include "common.cuh"

namespace qi8 {
namespace {

typedef ncclResult_t (*AllGatherFn)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t);
typedef ncclResult_t (*CommCountFn)(const ncclComm_t, int*);
typedef const char* (*ErrStrFn)(ncclResult_t);

struct Nccl {
  AllGatherFn all_gather = nullptr;
  CommCountFn comm_count = nullptr;
  ErrStrFn err_str = nullptr;
};

const Nccl* nccl() {
  static Nccl api;
  static bool ok = false;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
    if (!h) return;
    api.all_gather = reinterpret_cast<AllGatherFn>(dlsym(h, "ncclAllGather"));
    api.comm_count = reinterpret_cast<CommCountFn>(dlsym(h, "ncclCommCount"));
    api.err_str = reinterpret_cast<ErrStrFn>(dlsym(h, "ncclGetErrorString"));
    ok = api.all_gather && api.comm_count && api.err_str;
  });
  return ok ? &api : nullptr;
}

// y[t, r*n_loc + j] = g[(r*rows + t)*n_loc + j], in units of U (16 bytes when
// every row start is 16-byte aligned, else the element itself).
template <typename U>
__global__ void gather_layout_kernel(const U* __restrict__ g, U* __restrict__ y, int64_t rows, int64_t n_loc_u,
                                     int64_t ld_out_u, int world) {
  const int64_t total = (int64_t)world * rows * n_loc_u;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t j = i % n_loc_u;
    const int64_t rt = i / n_loc_u;  // r * rows + t
    const int64_t t = rt % rows, r = rt / rows;
    y[t * ld_out_u + r * n_loc_u + j] = g[i];
  }
}

template <typename U>
int launch_layout(const void* g, void* y, int64_t rows, int64_t n_loc_u, int64_t ld_out_u, int world, cudaStream_t st) {
  const int64_t total = (int64_t)world * rows * n_loc_u;
  int64_t blocks = (total + 255) / 256;
  const int64_t cap = (int64_t)(sm_count() > 0 ? sm_count() : 148) * 8;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  gather_layout_kernel<U><<<(unsigned)blocks, 256, 0, st>>>(static_cast<const U*>(g), static_cast<U*>(y), rows,
                                                            n_loc_u, ld_out_u, world);
  return check_cuda(cudaGetLastError(), "gather_layout_kernel launch");
}

bool nccl_dtype(int dtype, ncclDataType_t* t) {
  switch (dtype) {
    case QI8_BF16: *t = ncclBfloat16; return true;
    case QI8_F16: *t = ncclFloat16; return true;
    case QI8_F32: *t = ncclFloat32; return true;
    case QI8_I32: *t = ncclInt32; return true;
    case QI8_I8: *t = ncclInt8; return true;
    default: return false;
  }
}

}  // namespace
}  // namespace qi8

using namespace qi8;

extern "C" int qi8_gather_layout(const void* gathered, int dtype, int world, int64_t rows, int64_t n_loc,
                                 void* y_out, int64_t ld_out, void* stream) {
  QI8_REQUIRE(device_ok(), QI8_EUNSUPPORTED, "no sm_100 device current");
  QI8_REQUIRE(gathered && y_out, QI8_EINVAL, "null pointer");
  QI8_REQUIRE(world >= 1 && rows >= 0 && n_loc > 0, QI8_ESHAPE, "bad sizes world=%d rows=%lld n_loc=%lld", world,
              (long long)rows, (long long)n_loc);
  QI8_REQUIRE(ld_out >= (int64_t)world * n_loc, QI8_ESHAPE, "ld_out %lld < world * n_loc = %lld", (long long)ld_out,
              (long long)world * n_loc);
  const int es = elem_size(dtype);
  QI8_REQUIRE(es > 0, QI8_EDTYPE, "dtype %d", dtype);
  if (rows == 0) return QI8_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool vec = aligned16(gathered) && aligned16(y_out) && (n_loc * es) % 16 == 0 && (ld_out * es) % 16 == 0;
  if (vec) return launch_layout<uint4>(gathered, y_out, rows, n_loc * es / 16, ld_out * es / 16, world, st);
  switch (es) {
    case 1: return launch_layout<uint8_t>(gathered, y_out, rows, n_loc, ld_out, world, st);
    case 2: return launch_layout<uint16_t>(gathered, y_out, rows, n_loc, ld_out, world, st);
    default: return launch_layout<uint32_t>(gathered, y_out, rows, n_loc, ld_out, world, st);
  }
}

extern "C" int qi8_allgather_cols(const void* y_local, int dtype, int64_t rows, int64_t n_loc, void* y_out,
                                  int64_t ld_out, void* nccl_comm, void* scratch, int64_t scratch_bytes,
                                  void* stream) {
  QI8_REQUIRE(device_ok(), QI8_EUNSUPPORTED, "no sm_100 device current");
  QI8_REQUIRE(y_local && y_out && nccl_comm, QI8_EINVAL, "null pointer");
  QI8_REQUIRE(rows >= 0 && n_loc > 0, QI8_ESHAPE, "bad sizes rows=%lld n_loc=%lld", (long long)rows,
              (long long)n_loc);
  ncclDataType_t nt;
  QI8_REQUIRE(nccl_dtype(dtype, &nt), QI8_EDTYPE, "dtype %d has no NCCL counterpart here", dtype);
  const Nccl* api = nccl();
  QI8_REQUIRE(api, QI8_EUNSUPPORTED, "libnccl.so.2 could not be loaded");
  ncclComm_t comm = static_cast<ncclComm_t>(nccl_comm);
  int world = 0;
  ncclResult_t nr = api->comm_count(comm, &world);
  QI8_REQUIRE(nr == ncclSuccess && world >= 1, QI8_ECUDA, "ncclCommCount: %s", api->err_str(nr));
  QI8_REQUIRE(ld_out >= (int64_t)world * n_loc, QI8_ESHAPE, "ld_out %lld < world * n_loc = %lld", (long long)ld_out,
              (long long)world * n_loc);
  if (rows == 0) return QI8_OK;
  const int es = elem_size(dtype);
  const int64_t need = (int64_t)world * rows * n_loc * es;
  QI8_REQUIRE(scratch && scratch_bytes >= need, QI8_EINVAL, "scratch of %lld bytes needed (got %lld)",
              (long long)need, (long long)scratch_bytes);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  nr = api->all_gather(y_local, scratch, (size_t)(rows * n_loc), nt, comm, st);
  QI8_REQUIRE(nr == ncclSuccess, QI8_ECUDA, "ncclAllGather: %s", api->err_str(nr));
  return qi8_gather_layout(scratch, dtype, world, rows, n_loc, y_out, ld_out, stream);
}
