// Batch entry points for the correctly rounded exp / tanh of crmath.cuh, on the host (threads) and on the device, so
// that their agreement can be checked over every f32 input. The decoder and the VAD head use the same functions inline.
#include <algorithm>
#include <thread>
#include <vector>

#include "common.h"
#include "crmath.cuh"

namespace vxg {
namespace crm {

__global__ void math_kernel(const float* x, size_t n, float* y, int which) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    y[i] = which == 0 ? expf_cr(x[i]) : tanhf_cr(x[i]);
}

static void host_batch(const float* x, size_t n, float* y, int which) {
  const unsigned nt = std::max(1u, std::min(64u, std::thread::hardware_concurrency()));
  if (n < 65536 || nt == 1) {
    for (size_t i = 0; i < n; i++) y[i] = which == 0 ? expf_cr(x[i]) : tanhf_cr(x[i]);
    return;
  }
  std::vector<std::thread> th;
  for (unsigned t = 0; t < nt; t++)
    th.emplace_back([=] {
      const size_t a = n * t / nt, b = n * (t + 1) / nt;
      for (size_t i = a; i < b; i++) y[i] = which == 0 ? expf_cr(x[i]) : tanhf_cr(x[i]);
    });
  for (auto& t : th) t.join();
}

}  // namespace crm
}  // namespace vxg

using namespace vxg;

extern "C" {

vxg_status vxg_math_host(int fn, const float* x, size_t n, float* y) {
  clear_error();
  VXG_ARG(x && y && (fn == 0 || fn == 1), "bad arguments");
  crm::host_batch(x, n, y, fn);
  return VXG_OK;
}

vxg_status vxg_math_device(int fn, const float* x, size_t n, float* y, void* stream) {
  clear_error();
  VXG_ARG(x && y && (fn == 0 || fn == 1), "bad arguments");
  if (n == 0) return VXG_OK;
  const int grid = (int)std::min<size_t>((n + 255) / 256, (size_t)sm_count() * 16);
  crm::math_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(x, n, y, fn);
  note_launch();
  VXG_CUDA(cudaGetLastError());
  return VXG_OK;
}

}  // extern "C"
