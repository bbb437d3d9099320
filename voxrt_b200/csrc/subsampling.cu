// f32 dw-striding Conv2d x8 subsampling front end, bit-identical to the reference.
//
// Reference: Subsampling::forward (crates/voxrt/src/subsampling.rs:109-204), channels-last [T, F, C]:
//   conv0 1 -> C (3x3, stride 2, pad 1) + ReLU; 2 x [depthwise 3x3 stride 2 (no activation); pointwise C x C
//   (`linear`) + ReLU]; final linear F3*C -> d_model (+ bias).
// Convs: start from the bias, taps kt outer / kf inner, out-of-range taps skipped, `o += w * v` (multiply then
// add). `linear` for n >= 2 rows is tile_rows_portable (tensor.rs:233-260): per output four fused lanes over
// 4-column steps (lane l takes columns c = l mod 4), then hsum4 = (l0+l1)+(l2+l3), the tail, the bias.
//
// conv0 is recomputed inside the first depthwise conv for each of its 9 taps (the same arithmetic gives the same
// bits), which avoids writing and re-reading the 4x larger conv0 output. The GEMMs run on CUDA cores: the lane
// order is part of the parity contract and tensor-core (TF32) arithmetic would change it.
#include <cuda_runtime.h>

#include <algorithm>
#include <vector>

#include "common.h"
#include "internal.h"

namespace vxg {
namespace sub {

constexpr int C = 256;  // subsampling channels

__host__ __device__ inline int out_len(int n) { return (n + 2 - 3) / 2 + 1; }  // k 3, stride 2, pad 1

// Tiles: R2 = 2 output rows of the first depthwise conv (5 conv0 rows with halo) x 32 channels per block; the
// conv0 tile and the feats rows it reads are staged in shared memory, every value computed once.
constexpr int CR2 = 2, CC = 32, CT1 = 2 * CR2 + 1, CIN = 4 * CR2 + 3;
constexpr int MAX_MELS = 256;

// y1[t2, f2, c] = dw1(relu(conv0(feats))): blockIdx.x = (utterance-local t2 tile, channel group) over a tile table.
__global__ void __launch_bounds__(256) conv0_dw1_kernel(const float* __restrict__ feats, const int* __restrict__ in_off,
                                                        const int* __restrict__ in_len, const int* __restrict__ y_off,
                                                        const int* __restrict__ tile_u, const int* __restrict__ tile_t,
                                                        int n_mels, const float* __restrict__ w0,
                                                        const float* __restrict__ b0, const float* __restrict__ wd,
                                                        const float* __restrict__ bd, float* __restrict__ y1) {
  extern __shared__ float sm[];
  const int f1n = out_len(n_mels), f2n = out_len(f1n);
  float* fs = sm;                    // [CIN][n_mels] feats rows
  float* x0 = sm + CIN * MAX_MELS;   // [CT1][f1n][CC] conv0 + ReLU
  const int u = tile_u[blockIdx.x], t20 = tile_t[blockIdx.x], c0 = blockIdx.y * CC;
  const int t = in_len[u], t1n = out_len(t), t2n = out_len(t1n);
  const int t10 = 2 * t20 - 1, it0 = 2 * t10 - 1;  // first conv0 row / first feats row of the tile
  const float* fu = feats + (size_t)in_off[u] * n_mels;
  const int tid = threadIdx.x;
  for (int i = tid; i < CIN * n_mels; i += 256) {
    const int r = i / n_mels, m = i % n_mels, it = it0 + r;
    fs[r * n_mels + m] = (it >= 0 && it < t) ? __ldg(fu + (size_t)it * n_mels + m) : 0.0f;
  }
  __syncthreads();
  const int c = tid % CC, grp = tid / CC;  // 8 groups
  {
    float w[9];
#pragma unroll
    for (int k = 0; k < 9; k++) w[k] = __ldg(w0 + k * C + c0 + c);
    const float b = __ldg(b0 + c0 + c);
    for (int i = grp; i < CT1 * f1n; i += 256 / CC) {
      const int r = i / f1n, f1 = i % f1n, t1 = t10 + r;
      float x = b;  // subsampling.rs:117-139: bias, taps kt outer / kf inner, skip out of range, o += w * v
      if (t1 >= 0 && t1 < t1n) {
#pragma unroll
        for (int kt = 0; kt < 3; kt++) {
          const int it = 2 * t1 + kt - 1;
          if (it < 0 || it >= t) continue;
#pragma unroll
          for (int kf = 0; kf < 3; kf++) {
            const int i_f = 2 * f1 + kf - 1;
            if (i_f < 0 || i_f >= n_mels) continue;
            x = __fadd_rn(x, __fmul_rn(w[kt * 3 + kf], fs[(it - it0) * n_mels + i_f]));
          }
        }
      }
      x0[(r * f1n + f1) * CC + c] = fmaxf(x, 0.0f);
    }
  }
  __syncthreads();
  float w[9];
#pragma unroll
  for (int k = 0; k < 9; k++) w[k] = __ldg(wd + k * C + c0 + c);
  const float b = __ldg(bd + c0 + c);
  for (int i = grp; i < CR2 * f2n; i += 256 / CC) {
    const int r2 = i / f2n, f2 = i % f2n, o2 = t20 + r2;
    if (o2 >= t2n) continue;
    float o = b;  // subsampling.rs:144-173
#pragma unroll
    for (int kt = 0; kt < 3; kt++) {
      const int t1 = 2 * o2 + kt - 1;
      if (t1 < 0 || t1 >= t1n) continue;
#pragma unroll
      for (int kf = 0; kf < 3; kf++) {
        const int f1 = 2 * f2 + kf - 1;
        if (f1 < 0 || f1 >= f1n) continue;
        o = __fadd_rn(o, __fmul_rn(w[kt * 3 + kf], x0[((t1 - t10) * f1n + f1) * CC + c]));
      }
    }
    y1[((size_t)(y_off[u] + o2) * f2n + f2) * C + c0 + c] = o;
  }
}

// Depthwise 3x3 stride 2 over [T, F, C] (subsampling.rs:144-173): R3 = 4 output rows x 32 channels per block with the
// 9 input rows staged in shared memory.
constexpr int DR = 4, DT = 2 * DR + 1;

__global__ void __launch_bounds__(256) dw_kernel(const float* __restrict__ x, const int* __restrict__ x_off,
                                                 const int* __restrict__ x_len, const int* __restrict__ y_off,
                                                 const int* __restrict__ tile_u, const int* __restrict__ tile_t,
                                                 int fin, const float* __restrict__ wd, const float* __restrict__ bd,
                                                 float* __restrict__ y) {
  extern __shared__ float xs[];  // [DT][fin][CC]
  const int u = tile_u[blockIdx.x], to0 = tile_t[blockIdx.x], c0 = blockIdx.y * CC;
  const int tc = x_len[u], to = out_len(tc), fo = out_len(fin);
  const int ti0 = 2 * to0 - 1;
  const float* xu = x + (size_t)x_off[u] * fin * C;
  const int tid = threadIdx.x, c = tid % CC, grp = tid / CC;
  for (int i = grp; i < DT * fin; i += 256 / CC) {
    const int r = i / fin, f = i % fin, it = ti0 + r;
    xs[i * CC + c] = (it >= 0 && it < tc) ? __ldg(xu + ((size_t)it * fin + f) * C + c0 + c) : 0.0f;
  }
  __syncthreads();
  float w[9];
#pragma unroll
  for (int k = 0; k < 9; k++) w[k] = __ldg(wd + k * C + c0 + c);
  const float b = __ldg(bd + c0 + c);
  for (int i = grp; i < DR * fo; i += 256 / CC) {
    const int r = i / fo, of = i % fo, ot = to0 + r;
    if (ot >= to) continue;
    float o = b;
#pragma unroll
    for (int kt = 0; kt < 3; kt++) {
      const int it = 2 * ot + kt - 1;
      if (it < 0 || it >= tc) continue;
#pragma unroll
      for (int kf = 0; kf < 3; kf++) {
        const int i_f = 2 * of + kf - 1;
        if (i_f < 0 || i_f >= fin) continue;
        o = __fadd_rn(o, __fmul_rn(w[kt * 3 + kf], xs[((it - ti0) * fin + i_f) * CC + c]));
      }
    }
    y[((size_t)(y_off[u] + ot) * fo + of) * C + c0 + c] = o;
  }
}

// ---------------------------------------------------------------------------- f32 GEMM in the lane order
// y[m, n] = hsum4(lane sums) + bias[n] (+ ReLU), x [M, K], w [N, K] row-major, K % 4 == 0.
// Block: 32 rows x 256 outputs, 256 threads; thread (ty, tx) owns rows 4ty..4ty+3 and outputs tx + 32j (j < 8),
// each with four lane accumulators. Activation loads are warp-wide broadcasts; weight tiles are padded so the
// 16-byte loads of eight consecutive output rows are bank-conflict free.
constexpr int LBM = 32, LBN = 256, LBK = 16, LPAD = 4;

__device__ __forceinline__ void cp16(float* dst, const float* src, bool ok) {
  const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(dst));
  const int sz = ok ? 16 : 0;  // src-size 0 zero-fills
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(src), "r"(sz) : "memory");
}

__global__ void __launch_bounds__(256) linear_lanes_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                                           const float* __restrict__ bias, float* __restrict__ y,
                                                           int M, int N, int K, int relu) {
  __shared__ __align__(16) float xs[2][LBM][LBK + LPAD];
  __shared__ __align__(16) float ws[2][LBN][LBK + LPAD];
  const int tid = threadIdx.x, ty = tid >> 5, tx = tid & 31;
  const int m0 = blockIdx.y * LBM, n0 = blockIdx.x * LBN;
  float acc[4][8][4];
#pragma unroll
  for (int a = 0; a < 4; a++)
#pragma unroll
    for (int b = 0; b < 8; b++)
#pragma unroll
      for (int l = 0; l < 4; l++) acc[a][b][l] = 0.0f;
  auto load = [&](int kt, int buf) {
    const int k0 = kt * LBK;
    if (tid < LBM * LBK / 4) {  // 128 threads: x tile
      const int r = tid / (LBK / 4), c4 = (tid % (LBK / 4)) * 4;
      const bool ok = m0 + r < M;
      cp16(&xs[buf][r][c4], x + (size_t)(ok ? m0 + r : 0) * K + k0 + c4, ok);
    }
#pragma unroll
    for (int i = 0; i < LBN * LBK / 4 / 256; i++) {  // 4 per thread: w tile
      const int e = tid + i * 256;
      const int r = e / (LBK / 4), c4 = (e % (LBK / 4)) * 4;
      const bool ok = n0 + r < N;
      cp16(&ws[buf][r][c4], w + (size_t)(ok ? n0 + r : 0) * K + k0 + c4, ok);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  const int nk = K / LBK;
  load(0, 0);
  for (int kt = 0; kt < nk; kt++) {
    const int buf = kt & 1;
    if (kt + 1 < nk) {
      load(kt + 1, buf ^ 1);
      asm volatile("cp.async.wait_group 1;" ::: "memory");
    } else {
      asm volatile("cp.async.wait_group 0;" ::: "memory");
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < LBK; kk += 4) {
      float4 xv[4];
#pragma unroll
      for (int a = 0; a < 4; a++) xv[a] = *reinterpret_cast<const float4*>(&xs[buf][ty * 4 + a][kk]);
#pragma unroll
      for (int b = 0; b < 8; b++) {
        const float4 wv = *reinterpret_cast<const float4*>(&ws[buf][tx + 32 * b][kk]);
#pragma unroll
        for (int a = 0; a < 4; a++) {  // acc[l] = fma(w[c + l], x[c + l], acc[l])
          acc[a][b][0] = __fmaf_rn(wv.x, xv[a].x, acc[a][b][0]);
          acc[a][b][1] = __fmaf_rn(wv.y, xv[a].y, acc[a][b][1]);
          acc[a][b][2] = __fmaf_rn(wv.z, xv[a].z, acc[a][b][2]);
          acc[a][b][3] = __fmaf_rn(wv.w, xv[a].w, acc[a][b][3]);
        }
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int a = 0; a < 4; a++) {
    const int m = m0 + ty * 4 + a;
    if (m >= M) continue;
#pragma unroll
    for (int b = 0; b < 8; b++) {
      const int n = n0 + tx + 32 * b;
      if (n >= N) continue;
      // hsum4(acc) + tail (0: K % 4 == 0) + bias
      float v = __fadd_rn(__fadd_rn(acc[a][b][0], acc[a][b][1]), __fadd_rn(acc[a][b][2], acc[a][b][3]));
      v = __fadd_rn(v, 0.0f);
      v = __fadd_rn(v, bias ? __ldg(bias + n) : 0.0f);
      if (relu) v = fmaxf(v, 0.0f);
      y[(size_t)m * N + n] = v;
    }
  }
}

}  // namespace sub
}  // namespace vxg

using namespace vxg;

namespace vxg {

vxg_status linear_lanes(const float* x, const float* w, const float* bias, float* y, int M, int N, int K, int relu,
                        cudaStream_t st) {
  if (M <= 0) return VXG_OK;
  VXG_ARG(K % sub::LBK == 0, "linear: K (%d) must be a multiple of %d", K, sub::LBK);
  VXG_ARG(((uintptr_t)x & 15) == 0 && ((uintptr_t)w & 15) == 0, "linear: 16-byte alignment");
  dim3 grid((N + sub::LBN - 1) / sub::LBN, (M + sub::LBM - 1) / sub::LBM);
  sub::linear_lanes_kernel<<<grid, 256, 0, st>>>(x, w, bias, y, M, N, K, relu);
  note_launch();
  VXG_CUDA(cudaGetLastError());
  return VXG_OK;
}

}  // namespace vxg

extern "C" {

int vxg_sub_out_frames(int t_in) { return sub::out_len(sub::out_len(sub::out_len(t_in))); }

vxg_status vxg_linear_f32(const float* x, int M, int K, const float* w, const float* bias, int N, int relu, float* y,
                          void* stream) {
  clear_error();
  VXG_ARG(x && w && y && M >= 0 && N > 0 && K > 0, "bad arguments");
  VXG_ARG(M != 1, "single-row linear uses the reference's gemv order, which this kernel does not implement");
  return linear_lanes(x, w, bias, y, M, N, K, relu, (cudaStream_t)stream);
}

size_t vxg_subsampling_workspace_bytes(const int* t_in, int n_utt, int n_mels) {
  if (!t_in || n_utt <= 0) return 0;
  size_t r2 = 0, r3 = 0, tiles = 0;
  for (int u = 0; u < n_utt; u++) {
    const int t1 = sub::out_len(t_in[u]), t2 = sub::out_len(t1), t3 = sub::out_len(t2);
    r2 += t2;
    r3 += t3;
    tiles += (t2 + sub::CR2 - 1) / sub::CR2 + (t3 + sub::DR - 1) / sub::DR;
  }
  const int f1 = sub::out_len(n_mels), f2 = sub::out_len(f1), f3 = sub::out_len(f2);
  const size_t a = ((r2 * f2 * sub::C * 4 + 255) & ~size_t(255)) * 2;  // y1, z1
  const size_t b = ((r3 * f3 * sub::C * 4 + 255) & ~size_t(255)) * 2;  // y2, z2
  return a + b + (size_t)(6 * n_utt + 2 * tiles + 64) * 4;
}

vxg_status vxg_subsampling(const float* feats, const int* t_in, int n_utt, int n_mels, const float* conv0_w,
                           const float* conv0_b, const float* dw1_w, const float* dw1_b, const float* pw1_w,
                           const float* pw1_b, const float* dw2_w, const float* dw2_b, const float* pw2_w,
                           const float* pw2_b, const float* lin_w, const float* lin_b, int d_model, float* out,
                           void* workspace, size_t ws_bytes, void* stream) {
  clear_error();
  VXG_ARG(feats && t_in && n_utt > 0 && conv0_w && conv0_b && dw1_w && dw1_b && pw1_w && pw1_b && dw2_w && dw2_b &&
              pw2_w && pw2_b && lin_w && lin_b && out && workspace,
          "NULL pointer");
  VXG_ARG(n_mels % 8 == 0 && n_mels <= sub::MAX_MELS, "n_mels must be a multiple of 8, at most 256");
  if (ws_bytes < vxg_subsampling_workspace_bytes(t_in, n_utt, n_mels)) {
    set_error("workspace too small");
    return VXG_ERR_ARG;
  }
  const int f1 = sub::out_len(n_mels), f2 = sub::out_len(f1), f3 = sub::out_len(f2);
  std::vector<int> tab(6 * n_utt);  // in_off, in_len, off2, len2, off3, len3 | conv tiles (u, t2) | dw tiles (u, t3)
  std::vector<int> cu, ct, du, dt;
  int in_rows = 0, r2 = 0, r3 = 0;
  for (int u = 0; u < n_utt; u++) {
    VXG_ARG(t_in[u] > 0, "empty utterance %d", u);
    const int t1 = sub::out_len(t_in[u]), t2 = sub::out_len(t1), t3 = sub::out_len(t2);
    if (t3 < 2) {
      set_error("utterance %d: %d input frames give %d output frame(s); single-frame outputs use the reference's "
                "gemv order, which is not implemented",
                u, t_in[u], t3);
      return VXG_ERR_UNSUPPORTED;
    }
    tab[u] = in_rows;
    tab[n_utt + u] = t_in[u];
    tab[2 * n_utt + u] = r2;
    tab[3 * n_utt + u] = t2;
    tab[4 * n_utt + u] = r3;
    tab[5 * n_utt + u] = t3;
    for (int x = 0; x < t2; x += sub::CR2) {
      cu.push_back(u);
      ct.push_back(x);
    }
    for (int x = 0; x < t3; x += sub::DR) {
      du.push_back(u);
      dt.push_back(x);
    }
    in_rows += t_in[u];
    r2 += t2;
    r3 += t3;
  }
  const int nct = (int)cu.size(), ndt = (int)du.size();
  tab.insert(tab.end(), cu.begin(), cu.end());
  tab.insert(tab.end(), ct.begin(), ct.end());
  tab.insert(tab.end(), du.begin(), du.end());
  tab.insert(tab.end(), dt.begin(), dt.end());
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  const size_t sy1 = ((size_t)r2 * f2 * sub::C * 4 + 255) & ~size_t(255);
  const size_t sy2 = ((size_t)r3 * f3 * sub::C * 4 + 255) & ~size_t(255);
  float* y1 = reinterpret_cast<float*>(ws);
  float* z1 = reinterpret_cast<float*>(ws + sy1);
  float* y2 = reinterpret_cast<float*>(ws + 2 * sy1);
  float* z2 = reinterpret_cast<float*>(ws + 2 * sy1 + sy2);
  int* d_tab = reinterpret_cast<int*>(ws + 2 * sy1 + 2 * sy2);
  cudaStream_t st = (cudaStream_t)stream;
  VXG_CUDA(cudaMemcpyAsync(d_tab, tab.data(), tab.size() * 4, cudaMemcpyHostToDevice, st));
  const int* cut = d_tab + 6 * n_utt;
  const size_t smem1 = (size_t)(sub::CIN * sub::MAX_MELS + sub::CT1 * f1 * sub::CC) * 4;
  const size_t smem2 = (size_t)sub::DT * f2 * sub::CC * 4;
  vxg_status s = smem_attr((const void*)sub::conv0_dw1_kernel,
                           (sub::CIN * sub::MAX_MELS + sub::CT1 * (sub::MAX_MELS / 2) * sub::CC) * 4);
  if (s != VXG_OK || (s = smem_attr((const void*)sub::dw_kernel, sub::DT * (sub::MAX_MELS / 4) * sub::CC * 4)) != VXG_OK)
    return s;
  sub::conv0_dw1_kernel<<<dim3(nct, sub::C / sub::CC), 256, smem1, st>>>(
      feats, d_tab, d_tab + n_utt, d_tab + 2 * n_utt, cut, cut + nct, n_mels, conv0_w, conv0_b, dw1_w, dw1_b, y1);
  note_launch();
  VXG_CUDA(cudaGetLastError());
  s = linear_lanes(y1, pw1_w, pw1_b, z1, r2 * f2, sub::C, sub::C, 1, st);
  if (s != VXG_OK) return s;
  sub::dw_kernel<<<dim3(ndt, sub::C / sub::CC), 256, smem2, st>>>(z1, d_tab + 2 * n_utt, d_tab + 3 * n_utt,
                                                                  d_tab + 4 * n_utt, cut + 2 * nct, cut + 2 * nct + ndt,
                                                                  f2, dw2_w, dw2_b, y2);
  note_launch();
  VXG_CUDA(cudaGetLastError());
  if ((s = linear_lanes(y2, pw2_w, pw2_b, z2, r3 * f3, sub::C, sub::C, 1, st)) != VXG_OK) return s;
  return linear_lanes(z2, lin_w, lin_b, out, r3, d_model, f3 * sub::C, 0, st);
}

}  // extern "C"
