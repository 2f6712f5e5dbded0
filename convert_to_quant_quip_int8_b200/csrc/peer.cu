// Peer-memory plumbing of the column-parallel W8A8 linear (one process per
// GPU on one NVLink/NVSwitch node).
//
// The fused gather (qi8_gemm_i8_gather) has every rank's GEMM epilogue store
// its column tile straight into every rank's [T, N] output buffer; the
// buffers are exchanged as CUDA IPC handles (qi8_ipc_handle / qi8_ipc_open)
// and a stream-ordered barrier kernel (qi8_peer_barrier) tells each rank when
// all peers' tiles of a step have landed in its buffer.  Only plain loads and
// stores touch peer memory (no TMA, no multicast objects).
#include <cuda.h>

#include <cstdint>
#include <cstring>

#include "common.cuh"

namespace qi8 {
namespace {

typedef CUresult (*GetRangeFn)(CUdeviceptr*, size_t*, CUdeviceptr);

GetRangeFn get_range_fn() {
  static GetRangeFn fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<GetRangeFn>(ptr);
  }
  return fn;
}

constexpr uint64_t BARRIER_LIMIT_NS = 2000000000ull;  // 2 s

struct PeerFlags {
  uint32_t* flags[QI8_MAX_PEERS];  // rank p's flag words, mapped into this process
};

__device__ __forceinline__ uint64_t gtimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Flag words of rank p: [0, QI8_MAX_PEERS) arrival slots written by the
// ranks, [QI8_MAX_PEERS] the number of barriers p has completed (written by p
// only).  Every rank runs the same sequence of barriers, so the counters
// agree; a slot holding a value >= the current epoch means that rank has
// arrived (a peer can be at most one barrier ahead).
__global__ void peer_barrier_kernel(const __grid_constant__ PeerFlags f, int world, int rank, unsigned int* status,
                                    uint64_t limit) {
  __shared__ uint32_t epoch;
  __shared__ int expired;
  const int t = threadIdx.x;
  if (t == 0) {
    epoch = f.flags[rank][QI8_MAX_PEERS] + 1u;
    expired = 0;
  }
  __syncthreads();
  const uint32_t e = epoch;
  // once a barrier has expired (a peer is gone), later ones arrive but do not
  // wait, so a lost rank costs one limit and not one per remaining barrier
  const bool failed = (*reinterpret_cast<volatile unsigned int*>(status) & ST_PEER_BARRIER) != 0;
  if (t < world) {
    // the kernels before this one in the stream (the GEMM's peer stores) are
    // complete; order them before the arrival at system scope
    asm volatile("fence.acq_rel.sys;" ::: "memory");
    st_release_sys(f.flags[t] + rank, e);
    const uint64_t t0 = gtimer();
    while (!failed && (int32_t)(ld_acquire_sys(f.flags[rank] + t) - e) < 0) {
      if (gtimer() - t0 > limit) {
        expired = 1;
        break;
      }
      __nanosleep(100);
    }
  }
  __syncthreads();
  if (t == 0) {
    f.flags[rank][QI8_MAX_PEERS] = e;
    if (expired) atomicOr(status, ST_PEER_BARRIER);
  }
}

}  // namespace
}  // namespace qi8

using namespace qi8;

extern "C" int qi8_ipc_handle(const void* ptr, void* handle_out, int64_t* offset_out) {
  QI8_REQUIRE(ptr && handle_out && offset_out, QI8_EINVAL, "null pointer");
  GetRangeFn range = get_range_fn();
  QI8_REQUIRE(range, QI8_ECUDA, "cuMemGetAddressRange unavailable");
  CUdeviceptr base = 0;
  size_t size = 0;
  CUresult r = range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr));
  QI8_REQUIRE(r == CUDA_SUCCESS, QI8_ECUDA, "cuMemGetAddressRange failed (%d)", (int)r);
  cudaIpcMemHandle_t h;
  QI8_CUDA(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)));
  std::memcpy(handle_out, &h, sizeof(h));
  *offset_out = (int64_t)(reinterpret_cast<CUdeviceptr>(ptr) - base);
  return QI8_OK;
}

extern "C" int qi8_ipc_open(const void* handle, int64_t offset, void** ptr_out) {
  QI8_REQUIRE(handle && ptr_out && offset >= 0, QI8_EINVAL, "bad arguments");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  QI8_CUDA(cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess));
  *ptr_out = static_cast<char*>(base) + offset;
  return QI8_OK;
}

extern "C" int qi8_ipc_close(void* ptr, int64_t offset) {
  QI8_REQUIRE(ptr && offset >= 0, QI8_EINVAL, "bad arguments");
  QI8_CUDA(cudaIpcCloseMemHandle(static_cast<char*>(ptr) - offset));
  return QI8_OK;
}

extern "C" int qi8_peer_barrier(uint32_t* const* flags, int world, int rank, void* stream) {
  QI8_REQUIRE(device_ok(), QI8_EUNSUPPORTED, "no sm_100 device current");
  QI8_REQUIRE(flags, QI8_EINVAL, "null flags");
  QI8_REQUIRE(world >= 1 && world <= QI8_MAX_PEERS && rank >= 0 && rank < world, QI8_EINVAL,
              "world %d / rank %d (at most %d ranks)", world, rank, QI8_MAX_PEERS);
  PeerFlags f{};
  for (int r = 0; r < world; ++r) {
    QI8_REQUIRE(flags[r], QI8_EINVAL, "null flag pointer of rank %d", r);
    QI8_REQUIRE((reinterpret_cast<uintptr_t>(flags[r]) & 3u) == 0, QI8_EALIGN, "flag words must be 4-byte aligned");
    f.flags[r] = flags[r];
  }
  peer_barrier_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(f, world, rank, device_status_ptr(),
                                                                        BARRIER_LIMIT_NS);
  return check_cuda(cudaGetLastError(), "peer_barrier_kernel launch");
}
