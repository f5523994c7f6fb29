// capi.cu -- library-wide state of the C ABI: per-thread error messages,
// device checks, the device watchdog word and its self-test.
#include <cstdarg>
#include <cstdio>
#include <mutex>

#include "common.cuh"

namespace rb {

static thread_local char t_err[1024] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_err, sizeof(t_err), fmt, ap);
  va_end(ap);
}

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_err, sizeof(t_err), fmt, ap);
  va_end(ap);
  return code;
}

int check_cuda(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return RB_OK;
  return fail(RB_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

static constexpr int kMaxDevices = 64;
static int g_sm_count[kMaxDevices];
static int g_cc_major[kMaxDevices];
static std::once_flag g_dev_once[kMaxDevices];

static void query_device(int dev) {
  int v = 0;
  cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
  g_sm_count[dev] = v;
  v = 0;
  cudaDeviceGetAttribute(&v, cudaDevAttrComputeCapabilityMajor, dev);
  g_cc_major[dev] = v;
}

static int current_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return -1;
  std::call_once(g_dev_once[dev], query_device, dev);
  return dev;
}

int sm_count() {
  int dev = current_device();
  return (dev >= 0 && g_sm_count[dev] > 0) ? g_sm_count[dev] : 148;
}

bool device_is_sm100() {
  int dev = current_device();
  return dev >= 0 && g_cc_major[dev] == 10;
}

__global__ void selftest_wait_kernel(uint64_t budget_ns) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    abort_flag = 0;
    mbar_init(smem_u32(&bar), 1);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    // Nothing arrives on this barrier: the bounded wait must give up, record
    // the watchdog code and return.
    (void)mbar_wait_bounded(smem_u32(&bar), 0, kWaitTimeoutSelftest, &abort_flag, budget_ns);
  }
}

}  // namespace rb

using namespace rb;

extern "C" const char* rb_last_error(void) { return t_err; }

extern "C" int rb_version(void) { return 1; }

extern "C" int rb_device_supported(void) { return device_is_sm100() ? 1 : 0; }

extern "C" int rb_device_error(int reset) {
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int));
  if (e != cudaSuccess) {
    check_cuda(e, "reading the device watchdog word");
    return -1;
  }
  if (reset) {
    int z = 0;
    e = cudaMemcpyToSymbol(g_device_error, &z, sizeof(int));
    if (e != cudaSuccess) {
      check_cuda(e, "resetting the device watchdog word");
      return -1;
    }
  }
  return v;
}

extern "C" int rb_selftest_wait_timeout(uint64_t budget_ns, void* stream) {
  if (budget_ns > 5000000000ull) return fail(RB_ERR_VALUE, "budget above 5 s");
  selftest_wait_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(budget_ns);
  return check_cuda(cudaGetLastError(), "selftest_wait_kernel launch");
}
