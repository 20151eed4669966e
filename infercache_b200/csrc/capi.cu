// Library-level entry points of the C ABI: status strings, ABI version,
// device check and the last-error string.
#include <stdio.h>
#include <string.h>

#include "common.cuh"

namespace ic {

static thread_local char g_last_error[256] = "";

void set_last_error(const char* msg) {
  strncpy(g_last_error, msg, sizeof(g_last_error) - 1);
  g_last_error[sizeof(g_last_error) - 1] = '\0';
}

int launch_status(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) return IC_OK;
  snprintf(g_last_error, sizeof(g_last_error), "%s: %s", what, cudaGetErrorString(e));
  return IC_ERR_LAUNCH;
}

}  // namespace ic

extern "C" const char* ic_status_str(int status) {
  switch (status) {
    case IC_OK: return "ok";
    case IC_ERR_INVALID_ARG: return "invalid argument";
    case IC_ERR_UNSUPPORTED: return "unsupported shape or dtype";
    case IC_ERR_OUT_OF_PAGES: return "page pool exhausted";
    case IC_ERR_SESSION_CAP: return "session page cap exceeded";
    case IC_ERR_CORRUPT_TABLE: return "slot or page table entry out of range";
    case IC_ERR_LAUNCH: return "kernel launch failed";
    case IC_ERR_DEVICE_TIMEOUT: return "device-side wait timed out";
    case IC_ERR_CUDA: return "CUDA runtime error";
    case IC_ERR_NO_DEVICE: return "no sm_100 device";
    default: return "unknown status";
  }
}

extern "C" int ic_abi_version(void) { return IC_ABI_VERSION; }

extern "C" int ic_host_device_pointer(const void* host, void** device) {
  if (!host || !device) return IC_ERR_INVALID_ARG;
  void* d = nullptr;
  if (cudaHostGetDevicePointer(&d, const_cast<void*>(host), 0) != cudaSuccess) {
    cudaGetLastError();
    ic::set_last_error("ic_host_device_pointer: not page-locked mapped host memory");
    return IC_ERR_INVALID_ARG;
  }
  *device = d;
  return IC_OK;
}

extern "C" int ic_device_check(void) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    ic::set_last_error("no CUDA device");
    return IC_ERR_NO_DEVICE;
  }
  cudaDeviceProp p;
  if (cudaGetDeviceProperties(&p, dev) != cudaSuccess) {
    cudaGetLastError();
    return IC_ERR_NO_DEVICE;
  }
  if (p.major != 10) {
    ic::set_last_error("device is not sm_100 (B200)");
    return IC_ERR_NO_DEVICE;
  }
  return IC_OK;
}

extern "C" const char* ic_last_error(void) { return ic::g_last_error; }

namespace {

// One thread waits for phase 0 of an mbarrier whose single expected arrival
// never comes; the bounded wait reports the timeout in *status and returns.
__global__ void wait_probe_kernel(int32_t* status, uint64_t limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  ic::mbar_init(&bar, 1);
  ic::fence_barrier_init();
  ic::mbar_wait_bounded(&bar, 0, status, limit_ns);
}

}  // namespace

extern "C" int ic_wait_probe(int32_t* dev_status, int64_t limit_ns, void* stream) {
  if (!dev_status || limit_ns <= 0 || limit_ns > 2000000000LL) {
    ic::set_last_error("wait_probe: dev_status required, 0 < limit_ns <= 2e9");
    return IC_ERR_INVALID_ARG;
  }
  wait_probe_kernel<<<1, 1, 0, static_cast<cudaStream_t>(stream)>>>(dev_status, static_cast<uint64_t>(limit_ns));
  return ic::launch_status("wait_probe");
}

extern "C" int ic_graph_replay(void* const* execs, void* const* streams, int32_t n, int32_t rounds) {
  if (!execs || !streams || n < 1 || n > 4096 || rounds < 0) {
    ic::set_last_error("graph_replay: execs and streams required, 1 <= n <= 4096, rounds >= 0");
    return IC_ERR_INVALID_ARG;
  }
  for (int32_t i = 0; i < n; ++i) {
    if (!execs[i]) {
      ic::set_last_error("graph_replay: null graph");
      return IC_ERR_INVALID_ARG;
    }
  }
  for (int32_t r = 0; r < rounds; ++r) {
    for (int32_t i = 0; i < n; ++i) {
      const cudaError_t e = cudaGraphLaunch(static_cast<cudaGraphExec_t>(execs[i]),
                                            static_cast<cudaStream_t>(streams[i]));
      if (e != cudaSuccess) {
        ic::set_last_error(cudaGetErrorString(e));
        return IC_ERR_LAUNCH;
      }
    }
  }
  return IC_OK;
}
