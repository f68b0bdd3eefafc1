// libvcb: version, error strings and launch helpers shared by all kernels.
#include <cstdarg>
#include <mutex>
#include <unordered_map>

#include "vcb_common.cuh"
#include "vcb_crown_tc.cuh"

namespace vcb {

static thread_local std::string g_last_error;

void set_error(const std::string& msg) { g_last_error = msg; }

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return VCB_OK;
  int code = (e == cudaErrorMemoryAllocation) ? VCB_ERR_OOM : VCB_ERR_CUDA;
  return fail(code, "%s: %s (%s)", what, cudaGetErrorName(e),
              cudaGetErrorString(e));
}

int check_launch(const char* what) {
  return cuda_fail(cudaGetLastError(), what);
}

int sm_count() {
  static std::mutex mu;
  static std::unordered_map<int, int> cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  std::lock_guard<std::mutex> lk(mu);
  auto it = cache.find(dev);
  if (it != cache.end()) return it->second;
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) !=
          cudaSuccess || n <= 0)
    n = 148;
  cache[dev] = n;
  return n;
}

int ensure_smem(const void* kernel, int bytes) {
  static std::mutex mu;
  static std::unordered_map<const void*, int> done;
  int dev = 0;
  cudaGetDevice(&dev);
  const void* key = reinterpret_cast<const void*>(
      reinterpret_cast<uintptr_t>(kernel) ^ (uintptr_t(dev) << 56));
  std::lock_guard<std::mutex> lk(mu);
  auto it = done.find(key);
  if (it != done.end() && it->second >= bytes) return VCB_OK;
  cudaError_t e = cudaFuncSetAttribute(
      kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(smem)");
  done[key] = bytes;
  return VCB_OK;
}

}  // namespace vcb

extern "C" int vcb_version(void) { return 101; }

extern "C" int vcb_fault_check(void* stream) {
  int set = 0;
  const int rc = vcb::crown_tc_fault_take(static_cast<cudaStream_t>(stream), &set);
  if (rc) return rc;
  if (set)
    return vcb::fail(VCB_ERR_TIMEOUT,
                     "crown_tc_kernel: a bounded device-side wait expired; the bounds of the "
                     "boxes it had not finished are NaN");
  return VCB_OK;
}

extern "C" const char* vcb_last_error(void) {
  return vcb::g_last_error.c_str();
}

// ---------------------------------------------------------------------------
// FP32 FFMA throughput probe: the measured denominator for the roofline of the
// SIMT fp32 kernels (MEASURED_PEAKS.json only holds HBM and bf16 tensor peaks).
// Each thread runs 8 independent FMA chains; FLOPs = blocks*threads*iters*64*2.
// ---------------------------------------------------------------------------
namespace {
__global__ void __launch_bounds__(256) ffma_probe_kernel(float* out, int iters,
                                                         float seed) {
  float a[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) a[j] = seed + 0.001f * (threadIdx.x + j);
  const float m = 0.9999f, c = 1e-7f;
  for (int i = 0; i < iters; ++i) {
#pragma unroll
    for (int u = 0; u < 8; ++u) {
#pragma unroll
      for (int j = 0; j < 8; ++j) a[j] = fmaf(a[j], m, c);
    }
  }
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < 8; ++j) s += a[j];
  if (s == 12345.678f) out[blockIdx.x * blockDim.x + threadIdx.x] = s;
}
}  // namespace

extern "C" int vcb_probe_ffma(float* out, int32_t blocks, int32_t iters,
                              void* stream) {
  if (!out || blocks <= 0 || iters <= 0)
    return vcb::fail(VCB_ERR_INVALID, "vcb_probe_ffma: bad arguments");
  ffma_probe_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      out, iters, 1.0f);
  return vcb::check_launch("vcb_probe_ffma");
}
