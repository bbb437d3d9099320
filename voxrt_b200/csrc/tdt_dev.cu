// Encoder projection of the TDT decoder on the GPU: Decoder::project_encoder (crates/voxrt/src/decoder.rs:123-134)
// = linear (tensor.rs:98-127) of the encoder frames [t, d_model] to [t, hidden]. For t >= 2 the reference takes the
// tile_rows lane order, which the subsampling's linear kernel implements; for t == 1 it takes gemv order
// (gemv_portable, tensor.rs:285-303: dot_lanes8 for rows below out/4*4, a plain 8-lane sum for the rest), done here
// by one thread per output row.
#include "internal.h"
#include "tdt.h"

namespace vxg {
namespace tdt {

__global__ void gemv_lanes8_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                   const float* __restrict__ b, float* __restrict__ y, int out_f, int in_f) {
  const int o = blockIdx.x * blockDim.x + threadIdx.x;
  if (o >= out_f) return;
  const float* wr = w + (size_t)o * in_f;
  const int o4 = out_f / 4 * 4, n8 = in_f / 8 * 8;
  float r;
  if (o < o4) {  // dot_lanes8 (tensor.rs:267-281)
    float a[4] = {0.f, 0.f, 0.f, 0.f}, bb[4] = {0.f, 0.f, 0.f, 0.f};
    for (int c = 0; c < n8; c += 8)
#pragma unroll
      for (int l = 0; l < 4; l++) {
        a[l] = __fmaf_rn(x[c + l], wr[c + l], a[l]);
        bb[l] = __fmaf_rn(x[c + 4 + l], wr[c + 4 + l], bb[l]);
      }
    r = __fadd_rn(__fadd_rn(__fadd_rn(a[0], bb[0]), __fadd_rn(a[1], bb[1])),
                  __fadd_rn(__fadd_rn(a[2], bb[2]), __fadd_rn(a[3], bb[3])));
    for (int c = n8; c < in_f; c++) r = __fadd_rn(r, __fmul_rn(x[c], wr[c]));
  } else {  // dot (tensor.rs:79-95): eight lanes over 8-column chunks, summed in lane order from -0.0, then the tail
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int c = 0; c < n8; c += 8)
#pragma unroll
      for (int k = 0; k < 8; k++) acc[k] = __fadd_rn(acc[k], __fmul_rn(x[c + k], wr[c + k]));
    float s = -0.0f;
#pragma unroll
    for (int k = 0; k < 8; k++) s = __fadd_rn(s, acc[k]);
    for (int c = n8; c < in_f; c++) s = __fadd_rn(s, __fmul_rn(x[c], wr[c]));
    r = s;
  }
  y[o] = __fadd_rn(r, b ? b[o] : 0.0f);
}

}  // namespace tdt
}  // namespace vxg

using namespace vxg;

extern "C" vxg_status vxg_tdt_project_device(const vxg_tdt* t, const float* enc, int frames, float* proj,
                                             void* stream) {
  clear_error();
  VXG_ARG(t && enc && proj && frames >= 1, "bad arguments");
  const tdt::Decoder& D = t->d;
  VXG_ARG(D.enc_w_dev != nullptr, "decoder was created without a device (desc.device = -1)");
  int cur = -1;
  VXG_CUDA(cudaGetDevice(&cur));
  VXG_ARG(cur == D.device, "current device %d is not the decoder's device %d", cur, D.device);
  cudaStream_t st = (cudaStream_t)stream;
  if (frames >= 2) return linear_lanes(enc, D.enc_w_dev, D.enc_b_dev, proj, frames, D.hidden, D.d_model, 0, st);
  tdt::gemv_lanes8_kernel<<<(D.hidden + 127) / 128, 128, 0, st>>>(enc, D.enc_w_dev, D.enc_b_dev, proj, D.hidden,
                                                                   D.d_model);
  note_launch();
  VXG_CUDA(cudaGetLastError());
  return VXG_OK;
}
