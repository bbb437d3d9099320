// Host-side plumbing shared by the CUDA sources: status codes, the thread-local last-error string (the reference
// FFI's convention, crates/voxrt-ffi/src/lib.rs:61-73), the per-device status word that kernels write on a
// bounded-wait timeout, and tensor-map creation through the driver entry point.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <string>

#include "../../include/vxg.h"

namespace vxg {

void set_error(const char* fmt, ...);
void clear_error();

// Device status word of the current device (allocated on first use, zero-initialised). Kernels write a nonzero
// VXG_DEV_* code on a bounded-wait timeout or an internal check failure.
int* device_status();

enum : int {
  VXG_DEV_OK = 0,
  VXG_DEV_TIMEOUT_PRODUCER = 0x101,
  VXG_DEV_TIMEOUT_UNPACK = 0x102,
  VXG_DEV_TIMEOUT_MMA = 0x103,
  VXG_DEV_TIMEOUT_EPILOGUE = 0x104,
  VXG_DEV_TIMEOUT_DRAIN = 0x105,
  VXG_DEV_TIMEOUT_ATTN = 0x201,
  VXG_DEV_ATTN_PMAX = 0x202,   // a probability row's maximum was not exactly 1 (non-finite scores)
};

inline vxg_status cuda_fail(cudaError_t e, const char* what) {
  set_error("%s: %s", what, cudaGetErrorString(e));
  return e == cudaErrorMemoryAllocation ? VXG_ERR_OOM : VXG_ERR_CUDA;
}

#define VXG_CUDA(call)                                         \
  do {                                                         \
    cudaError_t e_ = (call);                                   \
    if (e_ != cudaSuccess) return ::vxg::cuda_fail(e_, #call); \
  } while (0)

#define VXG_ARG(cond, ...)          \
  do {                              \
    if (!(cond)) {                  \
      ::vxg::set_error(__VA_ARGS__); \
      return VXG_ERR_ARG;           \
    }                               \
  } while (0)

// 2D tensor map over a row-major [rows, cols] matrix of 1-byte elements with a (box_rows x box_cols) box and the
// 128-byte swizzle (box_cols * 1 B must be 128 for that swizzle).
vxg_status make_tmap_2d_u8(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t row_stride,
                           uint32_t box_rows, uint32_t box_cols);

// 2D tensor map over a row-major f32 [rows, cols] matrix with a (box_rows x box_cols) box. Swizzled: box_cols of
// 8, 16 or 32 select the 32-, 64- or 128-byte swizzle (the swizzle span equals one box row); unswizzled: any box
// row that is a multiple of 16 bytes lands row-major in shared memory.
vxg_status make_tmap_2d_f32(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t row_stride,
                            uint32_t box_rows, uint32_t box_cols, bool swizzled = true);

int sm_count();

// The library's stream-ordered memory pool on the current device, created on first use with an unlimited release
// threshold: per-call scratch (cudaMallocFromPoolAsync / cudaFreeAsync) reuses memory the pool already holds instead
// of mapping and unmapping device memory on every call. Null if the pool cannot be created.
cudaMemPool_t scratch_pool();

// Raise a kernel's dynamic shared-memory limit to `bytes` once per (device, kernel); thread-safe. The attribute
// belongs to the current device's context, so a process driving several GPUs sets it on each.
vxg_status smem_attr(const void* kernel, int bytes);

// Count of kernels this library has launched (process-wide), for the benchmark's launch accounting.
void note_launch(int n = 1);

}  // namespace vxg
