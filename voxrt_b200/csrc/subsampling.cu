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
#include "ptx.cuh"

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
  // Interior tile with 128 mel bins: every feats row and conv0 row of the tile is in range, so the only skipped
  // taps are those left of frequency 0 (f1 == 0 / f2 == 0, kf == 0, warp-uniform: grp == 0, j == 0). Same
  // operations in the same order as the general path below, with constant offsets and no per-tap checks.
  if (n_mels == 128 && t10 >= 1 && 2 * (t10 + CT1 - 1) + 1 < t && t10 + CT1 - 1 < t1n && t20 + CR2 - 1 < t2n) {
    constexpr int F0 = 128, F1 = 64, F2 = 32;
    float wa[9], wb[9];
#pragma unroll
    for (int k = 0; k < 9; k++) wa[k] = __ldg(w0 + k * C + c), wb[k] = __ldg(w0 + k * C + c + 1);
    const float ba = __ldg(b0 + c), bb = __ldg(b0 + c + 1);
    float2* x0f = reinterpret_cast<float2*>(x0);
#pragma unroll 1
    for (int r = 0; r < CT1; r++) {
      const float* fr = fs + 2 * r * F0;  // feats rows 2r, 2r + 1, 2r + 2 of the tile feed conv0 row r
#pragma unroll
      for (int j = 0; j < F1 / 8; j++) {
        const int f1 = grp + 8 * j;
        float xa = ba, xb = bb;
#pragma unroll
        for (int kt = 0; kt < 3; kt++)
#pragma unroll
          for (int kf = 0; kf < 3; kf++) {
            if (j == 0 && kf == 0 && grp == 0) continue;  // frequency -1
            const float v = fr[kt * F0 + 2 * f1 + kf - 1];
            xa = __fadd_rn(xa, __fmul_rn(wa[kt * 3 + kf], v));
            xb = __fadd_rn(xb, __fmul_rn(wb[kt * 3 + kf], v));
          }
        x0f[(r * F1 + f1) * (CC / 2) + cp] = make_float2(fmaxf(xa, 0.0f), fmaxf(xb, 0.0f));
      }
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < 9; k++) wa[k] = __ldg(wd + k * C + c), wb[k] = __ldg(wd + k * C + c + 1);
    const float da = __ldg(bd + c), db = __ldg(bd + c + 1);
#pragma unroll
    for (int r2 = 0; r2 < CR2; r2++) {
      float* yrow = y1 + ((size_t)(y_off[u] + t20 + r2) * F2) * C + c;
#pragma unroll
      for (int j = 0; j < F2 / 8; j++) {
        const int f2 = grp + 8 * j;
        float oa = da, ob = db;
#pragma unroll
        for (int kt = 0; kt < 3; kt++)
#pragma unroll
          for (int kf = 0; kf < 3; kf++) {
            if (j == 0 && kf == 0 && grp == 0) continue;  // conv0 frequency -1
            const float2 v = x0f[((2 * r2 + kt) * F1 + 2 * f2 + kf - 1) * (CC / 2) + cp];
            oa = __fadd_rn(oa, __fmul_rn(wa[kt * 3 + kf], v.x));
            ob = __fadd_rn(ob, __fmul_rn(wb[kt * 3 + kf], v.y));
          }
        *reinterpret_cast<float2*>(yrow + (size_t)f2 * C) = make_float2(oa, ob);
      }
    }
    return;
  }
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
  if (fin == 32) {  // the model's width (128 mel bins): every staging load in flight before the shared stores
    constexpr int FPT = 32 / 8;  // frequencies per thread and row
    uint64_t v[DT * FPT];
#pragma unroll
    for (int r = 0; r < DT; r++) {
      const int it = ti0 + r;
      const bool ok = it >= 0 && it < tc;
#pragma unroll
      for (int k = 0; k < FPT; k++)
        v[r * FPT + k] = ok ? __ldg(reinterpret_cast<const unsigned long long*>(xu + ((size_t)it * 32 + grp + 8 * k) * C + c))
                            : 0ull;
    }
#pragma unroll
    for (int r = 0; r < DT; r++)
#pragma unroll
      for (int k = 0; k < FPT; k++) xs[(r * 32 + grp + 8 * k) * (CC / 2) + cp] = v[r * FPT + k];
  } else {
    for (int r = 0; r < DT; r++) {
      const int it = ti0 + r;
      const bool ok = it >= 0 && it < tc;
      for (int f = grp; f < fin; f += 8)
        xs[(r * fin + f) * (CC / 2) + cp] =
            ok ? __ldg(reinterpret_cast<const unsigned long long*>(xu + ((size_t)it * fin + f) * C + c)) : 0ull;
    }
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
// The chains are split between two adjacent lanes: lane parity p runs the chain pair (2p, 2p + 1) as packed f32x2
// FMAs on 8-byte shared loads of x[m][4i + 2p ..] and w[n][4i + 2p ..], for an 8 x 8 block of outputs (rows
// rb + 4j, columns cb + 4j' of its warp's 32 x 32 patch); at the end each lane forms its pair sum and one shuffle
// with the partner gives (l0 + l1) + (l2 + l3). Rows and columns interleaved by 4 with a 36-float row pitch keep
// every shared load conflict-free (the 8 words a load instruction touches fall in distinct bank pairs).
// Block tile 128 x 64, K in 32-wide steps through a 3-stage cp.async ring; one 256-thread block per SM with the
// next step's fragments loaded into registers while the current step's FMAs run.
constexpr int LBM = 128, LBN = 64, LBK = 32, LST = LBK + 4, LSTAGES = 3;
constexpr int LSTAGE_F = (LBM + LBN) * LST;  // floats per stage
constexpr int LIN_SMEM = LSTAGES * LSTAGE_F * 4;

__device__ __forceinline__ uint64_t lds64(uint32_t a) {
  uint64_t v;
  asm volatile("ld.shared.b64 %0, [%1];" : "=l"(v) : "r"(a));
  return v;
}
__device__ __forceinline__ uint64_t f2fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ void f2unpack(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}

__global__ void __launch_bounds__(256, 1) linear_pairs_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                                              const float* __restrict__ bias, float* __restrict__ y,
                                                              int M, int N, int K, int relu) {
  extern __shared__ __align__(16) float lsm[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int p = lane & 1, rb = (lane >> 1) & 3, cb = lane >> 3;
  const int wr = (warp & 3) * 32, wc = (warp >> 2) * 32;  // the warp's 32 x 32 patch of the block tile
  const int m0 = blockIdx.y * LBM, n0 = blockIdx.x * LBN;
  const uint32_t s0 = smem_u32(lsm);
  // stage loader: 128 x rows and 64 w rows of 32 floats = 1536 16-byte chunks, six per thread
  auto load = [&](int stage, int k0) {
    const uint32_t sb = s0 + (uint32_t)(stage * LSTAGE_F * 4);
#pragma unroll
    for (int i = 0; i < 6; i++) {
      const int e = tid + i * 256, r = e >> 3, q = e & 7;  // r < 128: x row; else w row r - 128
      if (r < LBM) {
        const bool ok = m0 + r < M;
        cp_async16_zfill(sb + (uint32_t)((r * LST + q * 4) * 4), x + (size_t)(ok ? m0 + r : 0) * K + k0 + q * 4, ok);
      } else {
        const int rw = r - LBM;
        const bool ok = n0 + rw < N;
        cp_async16_zfill(sb + (uint32_t)((r * LST + q * 4) * 4), w + (size_t)(ok ? n0 + rw : 0) * K + k0 + q * 4, ok);
      }
    }
  };
  uint64_t acc[8][8];  // [row j][column j']: chains (2p, 2p + 1)
#pragma unroll
  for (int j = 0; j < 8; j++)
#pragma unroll
    for (int jj = 0; jj < 8; jj++) acc[j][jj] = 0ull;
  // this lane's first row / column word inside a stage (row rb + 4j at +4j*LST, column likewise), chain pair 2p
  const uint32_t xoff = (uint32_t)(((wr + rb) * LST + 2 * p) * 4);
  const uint32_t woff = (uint32_t)(((LBM + wc + cb) * LST + 2 * p) * 4);
  const int nk = K / LBK;
  load(0, 0);
  cp_async_commit();
  if (nk > 1) load(1, LBK);
  cp_async_commit();
  for (int kt = 0; kt < nk; kt++) {
    cp_async_wait_1();  // stage kt has landed (this thread's copies) ...
    __syncthreads();    // ... and everyone's; stage (kt + 2) % 3 was last read in step kt - 1
    if (kt + 2 < nk) load((kt + 2) % LSTAGES, (kt + 2) * LBK);
    cp_async_commit();
    const uint32_t sb = s0 + (uint32_t)((kt % LSTAGES) * LSTAGE_F * 4);
    const uint32_t xb = sb + xoff, wb = sb + woff;
    uint64_t xf[2][8], wf[2][8];
#pragma unroll
    for (int j = 0; j < 8; j++) {
      xf[0][j] = lds64(xb + (uint32_t)(4 * j * LST * 4));
      wf[0][j] = lds64(wb + (uint32_t)(4 * j * LST * 4));
    }
#pragma unroll
    for (int i = 0; i < LBK / 4; i++) {
      const int c = i & 1;
      if (i + 1 < LBK / 4) {  // next step's fragments while this step's FMAs run
#pragma unroll
        for (int j = 0; j < 8; j++) {
          xf[c ^ 1][j] = lds64(xb + (uint32_t)((4 * j * LST + 4 * (i + 1)) * 4));
          wf[c ^ 1][j] = lds64(wb + (uint32_t)((4 * j * LST + 4 * (i + 1)) * 4));
        }
      }
#pragma unroll
      for (int j = 0; j < 8; j++)
#pragma unroll
        for (int jj = 0; jj < 8; jj++) acc[j][jj] = f2fma(wf[c][jj], xf[c][j], acc[j][jj]);
    }
  }
  cp_async_wait_all();
  // pair sums, then (l0 + l1) + (l2 + l3) across the lane pair: lane p = 0 finishes rows j < 4, p = 1 rows j >= 4
  float bj[8];
#pragma unroll
  for (int jj = 0; jj < 8; jj++) {
    const int n = n0 + wc + cb + 4 * jj;
    bj[jj] = (bias && n < N) ? __ldg(bias + n) : 0.0f;
  }
#pragma unroll
  for (int j = 0; j < 4; j++) {
    const int jo = p ? j + 4 : j;  // the row this lane finishes
    const int m = m0 + wr + rb + 4 * jo;
#pragma unroll
    for (int jj = 0; jj < 8; jj++) {
      float a0, a1, b0, b1;
      f2unpack(acc[j][jj], a0, a1);
      f2unpack(acc[j + 4][jj], b0, b1);
      const float mine_lo = __fadd_rn(a0, a1), mine_hi = __fadd_rn(b0, b1);  // pair sums of rows j and j + 4
      const float other = __shfl_xor_sync(0xffffffffu, p ? mine_lo : mine_hi, 1);
      float t = p ? __fadd_rn(other, mine_hi) : __fadd_rn(mine_lo, other);  // (l0 + l1) + (l2 + l3)
      t = __fadd_rn(t, 0.0f);                                                // the (empty) tail
      const int n = n0 + wc + cb + 4 * jj;
      if (m < M && n < N) {
        t = __fadd_rn(t, bj[jj]);
        if (relu) t = fmaxf(t, 0.0f);
        y[(size_t)m * N + n] = t;
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
  VXG_ARG(K % sub::LBK == 0, "linear: K (%d) must be a multiple of %d", K, sub::LBK);
  VXG_ARG(((uintptr_t)x & 15) == 0 && ((uintptr_t)w & 15) == 0, "linear: 16-byte alignment");
  vxg_status s = smem_attr((const void*)sub::linear_pairs_kernel, sub::LIN_SMEM);
  if (s != VXG_OK) return s;
  VXG_ARG((M + sub::LBM - 1) / sub::LBM <= 65535, "linear: M = %d rows exceeds the grid", M);
  dim3 grid((N + sub::LBN - 1) / sub::LBN, (M + sub::LBM - 1) / sub::LBM);
  sub::linear_pairs_kernel<<<grid, 256, sub::LIN_SMEM, st>>>(x, w, bias, y, M, N, K, relu);
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
