// f32 dw-striding Conv2d x8 subsampling front end, bit-identical to the reference.
//
// Reference: Subsampling::forward (crates/voxrt/src/subsampling.rs:109-204), channels-last [T, F, C]:
//   conv0 1 -> C (3x3, stride 2, pad 1) + ReLU; 2 x [depthwise 3x3 stride 2 (no activation); pointwise C x C
//   (`linear`) + ReLU]; final linear F3*C -> d_model (+ bias).
// Convs: start from the bias, taps kt outer / kf inner, out-of-range taps skipped, `o += w * v` (multiply then
// add). `linear` for n >= 2 rows is tile_rows_portable (tensor.rs:233-260): per output four fused lanes over
// 4-column steps (lane l takes columns c = l mod 4), then hsum4 = (l0+l1)+(l2+l3), the tail, the bias.
//
// conv0 and the first depthwise conv run in one kernel: the conv0 tile (plus halo rows) lives in shared memory only,
// which avoids writing and re-reading the 4x larger conv0 output. The pointwise convs and the final linear run on
// CUDA cores: the lane order is part of the parity contract and tensor-core (TF32) arithmetic would change it.
#include <cuda_runtime.h>

#include <algorithm>
#include <vector>

#include "common.h"
#include "internal.h"

namespace vxg {
namespace sub {

constexpr int C = 256;  // subsampling channels

__host__ __device__ inline int out_len(int n) { return (n + 2 - 3) / 2 + 1; }  // k 3, stride 2, pad 1

// Tiles: R2 = 2 output rows of the first depthwise conv (5 conv0 rows with halo) x 64 channels per block; the
// conv0 tile and the feats rows it reads are staged in shared memory, every value computed once. Each thread owns
// a channel pair (8-byte loads and stores) and runs the reference's multiply-then-add steps on both channels.
constexpr int CR2 = 2, CC = 64, CT1 = 2 * CR2 + 1, CIN = 4 * CR2 + 3;
constexpr int MAX_MELS = 256;

__device__ __forceinline__ uint64_t p2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
// Multiply-then-add on channel pairs as two scalar round-to-nearest operations each. The packed f32x2 forms are
// not used here: ptxas contracts a packed mul.rn feeding a packed add.rn into one fused multiply-add (checked on
// sm_100a), which would skip the product's rounding that the reference's `o += w * v` performs.
__device__ __forceinline__ uint64_t p2mul(uint64_t a, uint64_t b) {
  float a0, a1, b0, b1;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a0), "=f"(a1) : "l"(a));
  asm("mov.b64 {%0, %1}, %2;" : "=f"(b0), "=f"(b1) : "l"(b));
  return p2(__fmul_rn(a0, b0), __fmul_rn(a1, b1));
}
__device__ __forceinline__ uint64_t p2add(uint64_t a, uint64_t b) {
  float a0, a1, b0, b1;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a0), "=f"(a1) : "l"(a));
  asm("mov.b64 {%0, %1}, %2;" : "=f"(b0), "=f"(b1) : "l"(b));
  return p2(__fadd_rn(a0, b0), __fadd_rn(a1, b1));
}
__device__ __forceinline__ uint64_t p2relu(uint64_t v) {
  float a, b;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
  return p2(fmaxf(a, 0.0f), fmaxf(b, 0.0f));
}

// y1[t2, f2, c] = dw1(relu(conv0(feats))): blockIdx.x = (utterance-local t2 tile) over a tile table,
// blockIdx.y = 64-channel group.
__global__ void __launch_bounds__(256) conv0_dw1_kernel(const float* __restrict__ feats, const int* __restrict__ in_off,
                                                        const int* __restrict__ in_len, const int* __restrict__ y_off,
                                                        const int* __restrict__ tile_u, const int* __restrict__ tile_t,
                                                        int n_mels, const float* __restrict__ w0,
                                                        const float* __restrict__ b0, const float* __restrict__ wd,
                                                        const float* __restrict__ bd, float* __restrict__ y1) {
  extern __shared__ float sm[];
  const int f1n = out_len(n_mels), f2n = out_len(f1n);
  float* fs = sm;                                              // [CIN][n_mels] feats rows
  uint64_t* x0 = reinterpret_cast<uint64_t*>(sm + CIN * MAX_MELS);  // [CT1][f1n][CC/2] conv0 + ReLU, channel pairs
  const int u = tile_u[blockIdx.x], t20 = tile_t[blockIdx.x], c0 = blockIdx.y * CC;
  const int t = in_len[u], t1n = out_len(t), t2n = out_len(t1n);
  const int t10 = 2 * t20 - 1, it0 = 2 * t10 - 1;  // first conv0 row / first feats row of the tile
  const float* fu = feats + (size_t)in_off[u] * n_mels;
  const int tid = threadIdx.x;
  for (int i = tid; i < CIN * n_mels; i += 256) {
    const int r = i / n_mels, m = i - r * n_mels, it = it0 + r;
    fs[i] = (it >= 0 && it < t) ? __ldg(fu + (size_t)it * n_mels + m) : 0.0f;
  }
  __syncthreads();
  const int cp = tid & 31, grp = tid >> 5;  // channel pair, position group (8)
  const int c = c0 + 2 * cp;
  {
    uint64_t w[9];
#pragma unroll
    for (int k = 0; k < 9; k++) w[k] = p2(__ldg(w0 + k * C + c), __ldg(w0 + k * C + c + 1));
    const uint64_t b = p2(__ldg(b0 + c), __ldg(b0 + c + 1));
    for (int r = 0; r < CT1; r++) {
      const int t1 = t10 + r;
      const bool row_in = t1 >= 0 && t1 < t1n;
      for (int f1 = grp; f1 < f1n; f1 += 8) {
        uint64_t x = b;  // subsampling.rs:117-139: bias, taps kt outer / kf inner, skip out of range, o += w * v
        if (row_in) {
#pragma unroll
          for (int kt = 0; kt < 3; kt++) {
            const int it = 2 * t1 + kt - 1;
            if (it < 0 || it >= t) continue;
            const float* fr = fs + (it - it0) * n_mels;
#pragma unroll
            for (int kf = 0; kf < 3; kf++) {
              const int i_f = 2 * f1 + kf - 1;
              if (i_f < 0 || i_f >= n_mels) continue;
              const float v = fr[i_f];
              x = p2add(x, p2mul(w[kt * 3 + kf], p2(v, v)));
            }
          }
        }
        x0[(r * f1n + f1) * (CC / 2) + cp] = p2relu(x);
      }
    }
  }
  __syncthreads();
  uint64_t w[9];
#pragma unroll
  for (int k = 0; k < 9; k++) w[k] = p2(__ldg(wd + k * C + c), __ldg(wd + k * C + c + 1));
  const uint64_t b = p2(__ldg(bd + c), __ldg(bd + c + 1));
  for (int r2 = 0; r2 < CR2; r2++) {
    const int o2 = t20 + r2;
    if (o2 >= t2n) break;
    for (int f2 = grp; f2 < f2n; f2 += 8) {
      uint64_t o = b;  // subsampling.rs:144-173
#pragma unroll
      for (int kt = 0; kt < 3; kt++) {
        const int t1 = 2 * o2 + kt - 1;
        if (t1 < 0 || t1 >= t1n) continue;
#pragma unroll
        for (int kf = 0; kf < 3; kf++) {
          const int f1 = 2 * f2 + kf - 1;
          if (f1 < 0 || f1 >= f1n) continue;
          o = p2add(o, p2mul(w[kt * 3 + kf], x0[((t1 - t10) * f1n + f1) * (CC / 2) + cp]));
        }
      }
      *reinterpret_cast<uint64_t*>(y1 + ((size_t)(y_off[u] + o2) * f2n + f2) * C + c) = o;
    }
  }
}

// Depthwise 3x3 stride 2 over [T, F, C] (subsampling.rs:144-173): R3 = 4 output rows x 64 channels per block with the
// 9 input rows staged in shared memory as channel pairs.
constexpr int DR = 4, DT = 2 * DR + 1;

__global__ void __launch_bounds__(256) dw_kernel(const float* __restrict__ x, const int* __restrict__ x_off,
                                                 const int* __restrict__ x_len, const int* __restrict__ y_off,
                                                 const int* __restrict__ tile_u, const int* __restrict__ tile_t,
                                                 int fin, const float* __restrict__ wd, const float* __restrict__ bd,
                                                 float* __restrict__ y) {
  extern __shared__ float xsm[];
  uint64_t* xs = reinterpret_cast<uint64_t*>(xsm);  // [DT][fin][CC/2]
  const int u = tile_u[blockIdx.x], to0 = tile_t[blockIdx.x], c0 = blockIdx.y * CC;
  const int tc = x_len[u], to = out_len(tc), fo = out_len(fin);
  const int ti0 = 2 * to0 - 1;
  const float* xu = x + (size_t)x_off[u] * fin * C;
  const int tid = threadIdx.x, cp = tid & 31, grp = tid >> 5;
  const int c = c0 + 2 * cp;
  for (int r = 0; r < DT; r++) {
    const int it = ti0 + r;
    const bool ok = it >= 0 && it < tc;
    for (int f = grp; f < fin; f += 8)
      xs[(r * fin + f) * (CC / 2) + cp] =
          ok ? __ldg(reinterpret_cast<const unsigned long long*>(xu + ((size_t)it * fin + f) * C + c)) : 0ull;
  }
  __syncthreads();
  uint64_t w[9];
#pragma unroll
  for (int k = 0; k < 9; k++) w[k] = p2(__ldg(wd + k * C + c), __ldg(wd + k * C + c + 1));
  const uint64_t b = p2(__ldg(bd + c), __ldg(bd + c + 1));
  for (int r = 0; r < DR; r++) {
    const int ot = to0 + r;
    if (ot >= to) break;
    for (int of = grp; of < fo; of += 8) {
      uint64_t o = b;
#pragma unroll
      for (int kt = 0; kt < 3; kt++) {
        const int it = 2 * ot + kt - 1;
        if (it < 0 || it >= tc) continue;
#pragma unroll
        for (int kf = 0; kf < 3; kf++) {
          const int i_f = 2 * of + kf - 1;
          if (i_f < 0 || i_f >= fin) continue;
          o = p2add(o, p2mul(w[kt * 3 + kf], xs[((it - ti0) * fin + i_f) * (CC / 2) + cp]));
        }
      }
      *reinterpret_cast<uint64_t*>(y + ((size_t)(y_off[u] + ot) * fo + of) * C + c) = o;
    }
  }
}

// linear (tile_rows_portable order): output (m, n) = hsum4 of four FMA chains, chain l accumulating
// fma(w[n][k], x[m][k], acc_l) over k = l, l + 4, ..., then (l0 + l1) + (l2 + l3), the tail, the bias.
// Here the four chains of an output live in four threads (lanes i, i+8, i+16, i+24 of a warp), each thread carries
// one chain for 8 rows x 8 columns, and the chains are summed at the end with two shuffles in the reference's order.
// Tiles: 64 rows x 64 columns x 32 k per block, staged k-major in shared memory (transposed on the way in) so that a
// thread's 8 rows / 8 columns at one k are two 16-byte loads; column pairs run as packed f32x2 FMAs.
constexpr int FBM = 64, FBN = 64, FBK = 32, FST = FBM + 4;  // FST: k-row stride in floats

__device__ __forceinline__ uint64_t f2pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2unpack(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t f2fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}

__global__ void __launch_bounds__(256, 2) linear_lanes_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                                              const float* __restrict__ bias, float* __restrict__ y,
                                                              int M, int N, int K, int relu) {
  __shared__ __align__(16) float xs[2][FBK][FST];
  __shared__ __align__(16) float ws[2][FBK][FST];
  const int tid = threadIdx.x, lid = tid & 31, bm = tid >> 5;
  const int l = lid >> 3, bn = lid & 7;  // chain, column block
  const int m0 = blockIdx.y * FBM, n0 = blockIdx.x * FBN;
  uint64_t acc[8][4];  // [row][column pair]: columns 4bn + {0,1}, {2,3}, 32 + 4bn + {0,1}, {2,3}
#pragma unroll
  for (int i = 0; i < 8; i++)
#pragma unroll
    for (int j = 0; j < 4; j++) acc[i][j] = 0ull;
  float4 gx[2], gw[2];
  auto gload = [&](int k0) {  // two float4 of x and of w per thread: row e >> 3, k offset (e & 7) * 4
#pragma unroll
    for (int i = 0; i < 2; i++) {
      const int e = tid + i * 256, r = e >> 3, kq = (e & 7) * 4;
      gx[i] = m0 + r < M ? __ldg(reinterpret_cast<const float4*>(x + (size_t)(m0 + r) * K + k0 + kq))
                         : make_float4(0.f, 0.f, 0.f, 0.f);
      gw[i] = n0 + r < N ? __ldg(reinterpret_cast<const float4*>(w + (size_t)(n0 + r) * K + k0 + kq))
                         : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  };
  auto sstore = [&](int buf) {  // transpose to k-major
#pragma unroll
    for (int i = 0; i < 2; i++) {
      const int e = tid + i * 256, r = e >> 3, kq = (e & 7) * 4;
      xs[buf][kq + 0][r] = gx[i].x;
      xs[buf][kq + 1][r] = gx[i].y;
      xs[buf][kq + 2][r] = gx[i].z;
      xs[buf][kq + 3][r] = gx[i].w;
      ws[buf][kq + 0][r] = gw[i].x;
      ws[buf][kq + 1][r] = gw[i].y;
      ws[buf][kq + 2][r] = gw[i].z;
      ws[buf][kq + 3][r] = gw[i].w;
    }
  };
  const int nk = K / FBK;
  gload(0);
  sstore(0);
  __syncthreads();
  for (int kt = 0; kt < nk; kt++) {
    const int buf = kt & 1;
    if (kt + 1 < nk) gload((kt + 1) * FBK);
#pragma unroll
    for (int i = 0; i < FBK / 4; i++) {
      const int k = 4 * i + l;  // this thread's chain visits k = l mod 4, in increasing order
      const float4 xa = *reinterpret_cast<const float4*>(&xs[buf][k][8 * bm]);
      const float4 xb = *reinterpret_cast<const float4*>(&xs[buf][k][8 * bm + 4]);
      const float4 wa = *reinterpret_cast<const float4*>(&ws[buf][k][4 * bn]);
      const float4 wb = *reinterpret_cast<const float4*>(&ws[buf][k][32 + 4 * bn]);
      const uint64_t w01 = f2pack(wa.x, wa.y), w23 = f2pack(wa.z, wa.w);
      const uint64_t w45 = f2pack(wb.x, wb.y), w67 = f2pack(wb.z, wb.w);
      const float xr[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
#pragma unroll
      for (int r = 0; r < 8; r++) {  // acc = fma(w[n][k], x[m][k], acc)
        const uint64_t x2 = f2pack(xr[r], xr[r]);
        acc[r][0] = f2fma(w01, x2, acc[r][0]);
        acc[r][1] = f2fma(w23, x2, acc[r][1]);
        acc[r][2] = f2fma(w45, x2, acc[r][2]);
        acc[r][3] = f2fma(w67, x2, acc[r][3]);
      }
    }
    if (kt + 1 < nk) sstore(buf ^ 1);
    __syncthreads();
  }
  // hsum4 = (l0 + l1) + (l2 + l3): lanes bn + 8l hold chain l of the same outputs
#pragma unroll
  for (int r = 0; r < 8; r++) {
    const int m = m0 + 8 * bm + r;
#pragma unroll
    for (int j = 0; j < 4; j++) {
      float v[2];
      f2unpack(acc[r][j], v[0], v[1]);
#pragma unroll
      for (int e = 0; e < 2; e++) {
        float s01 = __fadd_rn(v[e], __shfl_xor_sync(0xffffffffu, v[e], 8));    // l0+l1 | l2+l3
        float t = __fadd_rn(s01, __shfl_xor_sync(0xffffffffu, s01, 16));       // (l0+l1)+(l2+l3)
        const int n = n0 + (j < 2 ? 4 * bn + 2 * j : 32 + 4 * bn + 2 * (j - 2)) + e;
        if (l == (r & 3) && m < M && n < N) {  // one of the four lanes stores (spread over r)
          t = __fadd_rn(t, 0.0f);
          t = __fadd_rn(t, bias ? __ldg(bias + n) : 0.0f);
          if (relu) t = fmaxf(t, 0.0f);
          y[(size_t)m * N + n] = t;
        }
      }
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
  VXG_ARG(K % sub::FBK == 0, "linear: K (%d) must be a multiple of %d", K, sub::FBK);
  VXG_ARG(((uintptr_t)x & 15) == 0 && ((uintptr_t)w & 15) == 0, "linear: 16-byte alignment");
  dim3 grid((N + sub::FBN - 1) / sub::FBN, (M + sub::FBM - 1) / sub::FBM);
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
  const size_t smem1 = (size_t)(sub::CIN * sub::MAX_MELS + sub::CT1 * f1 * sub::CC) * 4;  // f32 feats + pairs
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
