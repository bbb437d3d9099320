#include <atomic>
#include <mutex>
#include <vector>

#include "common.h"

namespace vxg {

static thread_local std::string g_last_error;

void set_error(const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_last_error = buf;
}

void clear_error() { g_last_error.clear(); }

static std::mutex g_status_mu;
static std::vector<int*> g_status;  // per device

int* device_status() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
  std::lock_guard<std::mutex> lk(g_status_mu);
  if ((int)g_status.size() <= dev) g_status.resize(dev + 1, nullptr);
  if (!g_status[dev]) {
    int* p = nullptr;
    if (cudaMalloc(&p, sizeof(int)) != cudaSuccess) return nullptr;
    if (cudaMemset(p, 0, sizeof(int)) != cudaSuccess) return nullptr;
    if (cudaDeviceSynchronize() != cudaSuccess) return nullptr;
    g_status[dev] = p;
  }
  return g_status[dev];
}

// (device, kernel) pairs whose limit is set; a fixed table, so the lookup never touches the heap. Past its
// capacity the attribute is simply set again on each call (the call is idempotent).
static std::mutex g_attr_mu;
static struct {
  int dev;
  const void* kernel;
} g_attr_done[256];
static int g_attr_n = 0;

vxg_status smem_attr(const void* kernel, int bytes) {
  int dev = 0;
  VXG_CUDA(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lk(g_attr_mu);
  for (int i = 0; i < g_attr_n; i++)
    if (g_attr_done[i].dev == dev && g_attr_done[i].kernel == kernel) return VXG_OK;
  VXG_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
  if (g_attr_n < 256) g_attr_done[g_attr_n++] = {dev, kernel};
  return VXG_OK;
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return (EncodeTiledFn) nullptr;
    return (EncodeTiledFn)p;
  }();
  return fn;
}

vxg_status make_tmap_2d_u8(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t row_stride,
                           uint32_t box_rows, uint32_t box_cols) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) {
    set_error("cuTensorMapEncodeTiled is unavailable");
    return VXG_ERR_CUDA;
  }
  if (((uintptr_t)base & 15) || (row_stride & 15)) {
    set_error("tensor map: base and row stride must be 16-byte aligned");
    return VXG_ERR_ARG;
  }
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {row_stride};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (%d)", (int)r);
    return VXG_ERR_CUDA;
  }
  return VXG_OK;
}

vxg_status make_tmap_2d_f32(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t row_stride,
                            uint32_t box_rows, uint32_t box_cols, bool swizzled) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) {
    set_error("cuTensorMapEncodeTiled is unavailable");
    return VXG_ERR_CUDA;
  }
  if (((uintptr_t)base & 15) || (row_stride & 15)) {
    set_error("tensor map: base and row stride must be 16-byte aligned");
    return VXG_ERR_ARG;
  }
  CUtensorMapSwizzle sw = CU_TENSOR_MAP_SWIZZLE_NONE;
  if (swizzled) {
    switch (box_cols * 4) {  // the swizzle span equals the box's inner extent
      case 32: sw = CU_TENSOR_MAP_SWIZZLE_32B; break;
      case 64: sw = CU_TENSOR_MAP_SWIZZLE_64B; break;
      case 128: sw = CU_TENSOR_MAP_SWIZZLE_128B; break;
      default: set_error("tensor map: f32 box of %u columns has no matching swizzle", box_cols); return VXG_ERR_ARG;
    }
  } else if ((box_cols * 4) % 16 != 0 || box_cols > 256) {
    set_error("tensor map: unswizzled f32 box of %u columns is not a multiple of 16 bytes", box_cols);
    return VXG_ERR_ARG;
  }
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {row_stride};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled (f32) failed (%d)", (int)r);
    return VXG_ERR_CUDA;
  }
  return VXG_OK;
}

static std::atomic<unsigned long long> g_launches{0};
void note_launch(int n) { g_launches.fetch_add((unsigned long long)n, std::memory_order_relaxed); }

cudaMemPool_t scratch_pool() {
  static std::mutex mu;
  static cudaMemPool_t pools[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lk(mu);
  if (!pools[dev]) {
    cudaMemPoolProps props = {};
    props.allocType = cudaMemAllocationTypePinned;
    props.location.type = cudaMemLocationTypeDevice;
    props.location.id = dev;
    cudaMemPool_t p = nullptr;
    if (cudaMemPoolCreate(&p, &props) != cudaSuccess) {
      cudaGetLastError();
      return nullptr;
    }
    uint64_t keep = ~0ull;
    cudaMemPoolSetAttribute(p, cudaMemPoolAttrReleaseThreshold, &keep);
    pools[dev] = p;
  }
  return pools[dev];
}

int sm_count() {
  int dev = 0, n = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 1;
}

}  // namespace vxg

extern "C" {

const char* vxg_last_error(void) { return vxg::g_last_error.c_str(); }

const char* vxg_version(void) { return "0.1.0"; }

unsigned long long vxg_kernel_launches(void) { return vxg::g_launches.load(std::memory_order_relaxed); }

vxg_status vxg_device_status(int* code) {
  if (!code) {
    vxg::set_error("code is NULL");
    return VXG_ERR_ARG;
  }
  int* st = vxg::device_status();
  if (!st) {
    vxg::set_error("no CUDA device");
    return VXG_ERR_CUDA;
  }
  VXG_CUDA(cudaDeviceSynchronize());
  VXG_CUDA(cudaMemcpy(code, st, sizeof(int), cudaMemcpyDeviceToHost));
  VXG_CUDA(cudaMemset(st, 0, sizeof(int)));
  return VXG_OK;
}

}  // extern "C"
