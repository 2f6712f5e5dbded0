// Library-wide entry points: version, error strings, device checks and the
// device status word written by kernels whose bounded waits expire.
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>

#include "common.cuh"

namespace {

thread_local char g_err[512] = "";

constexpr int kMaxDevices = 64;

// One word per device.  Kernels receive its address as an argument; a wait
// that runs out of time ORs a role bit into it and the kernel returns early.
__device__ unsigned int g_status_word;

struct DevInfo {
  bool init = false;
  int sms = 0;
  bool ok = false;
  unsigned int* status = nullptr;
};
DevInfo g_dev[kMaxDevices];

DevInfo& dev_info() {
  int d = 0;
  cudaGetDevice(&d);
  DevInfo& di = g_dev[d < kMaxDevices ? d : 0];
  if (!di.init) {
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, d) == cudaSuccess) {
      di.sms = prop.multiProcessorCount;
      di.ok = (prop.major == 10 && prop.minor == 0);
    }
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_status_word) == cudaSuccess) di.status = static_cast<unsigned int*>(p);
    di.init = true;
  }
  return di;
}

}  // namespace

namespace qi8 {

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int check_cuda(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return QI8_OK;
  return fail(QI8_ECUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

bool pdl_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("QI8_PDL");
    return v && *v && std::strcmp(v, "0") != 0;
  }();
  return on;
}

unsigned int* device_status_ptr() { return dev_info().status; }
int sm_count() { return dev_info().sms; }
bool device_ok() { return dev_info().ok && dev_info().status != nullptr; }

}  // namespace qi8

extern "C" {

int qi8_version(void) { return QI8_ABI_VERSION; }

const char* qi8_last_error(void) { return g_err; }

int qi8_device_supported(int device) {
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return prop.major == 10 && prop.minor == 0;
}

int qi8_device_status(int reset) {
  unsigned int* p = qi8::device_status_ptr();
  if (!p) return qi8::fail(QI8_ECUDA, "device status word unavailable");
  QI8_CUDA(cudaDeviceSynchronize());
  unsigned int v = 0;
  QI8_CUDA(cudaMemcpy(&v, p, sizeof(v), cudaMemcpyDeviceToHost));
  if (reset) QI8_CUDA(cudaMemset(p, 0, sizeof(v)));
  if (v) return qi8::fail(QI8_ETIMEOUT, "a kernel wait expired (status bits 0x%x)", v);
  return QI8_OK;
}

}  // extern "C"
