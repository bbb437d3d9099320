// Ternary-weight x int8-activation GEMM on the sm_100a tensor cores (tcgen05.mma kind::i8).
//
// Reference semantics (crates/voxrt/src/kernels/mod.rs:166-210, x86.rs:91-154): for every output (t, o)
//   acc = 0; for g in groups: acc = fma(float(S_g), sx[t,g] * sw[o,g], acc);  y = epilogue(old, acc)
// with S_g the exact int32 dot product over the group. The int32 sums come from the tensor cores; the float chain
// runs in the epilogue warps in the reference's group order, so the result is bit-identical.
//
// Persistent, warp-specialised CTA (one per SM, 640 threads), tile = 128 tokens x 128 weight rows:
//   warps 0-15   epilogue: warp w owns TMEM lanes 32*(w%4)..+32 (its tokens) and columns 32*(w/4)..+32 of the
//                tile. Per group it tcgen05.lds the sums, re-arms the buffer and runs the FMA chain on packed f32x2
//                pairs; per tile it applies Store / SiLU / AddScaled (+bias) into a 128-byte-swizzled staging tile
//                that a TMA bulk store writes out (AddScaled's old values arrive the same way, by TMA load).
//   warp 16      TMA producer: activation tile (128 x 128 B, 128-byte swizzle) and the weight tile per K-chunk of
//                128 into a 3-stage ring: either 2-bit codes (128 rows x 32 B, bulk copy) or int8 rows (TMA).
//   warp 17      TMEM allocator + MMA issuer: 4 x (M128 N128 K32) per chunk into one of four per-group int32
//                accumulator buffers (all 512 TMEM columns), commit -> stage free / group ready.
//   warps 18-19  2-bit weights only: unpack codes -> int8 {-1,0,+1} (one PRMT per 4 weights) into the UMMA
//                K-major 128-byte-swizzled layout.
// Exact int -> float without a conversion instruction: every accumulator buffer is pre-set to 0x4B400000 (the
// float 1.5 * 2^23) and the MMA accumulates onto it, so for |S| < 2^22 the result's bits are the float
// 1.5 * 2^23 + S and one subtraction of 1.5 * 2^23 recovers float(S) exactly.
#include <cuda_fp16.h>

#include <algorithm>
#include <cstring>
#include <functional>
#include <thread>
#include <vector>

#include "common.h"
#include "internal.h"
#include "math.cuh"
#include "ptx.cuh"

namespace vxg {
namespace gemm {

constexpr int BM = 128;  // tokens per tile (TMEM lanes)
constexpr int BN = 128;  // weight rows per tile (TMEM columns per buffer)
constexpr int BK = 128;  // K per stage: one 128-byte swizzle row
constexpr int STAGES = 3;
constexpr int EPI_WARPS = 16;
constexpr int PROD_WARP = 16, MMA_WARP = 17, UNPACK_WARP0 = 18, UNPACK_WARPS = 2;
constexpr int THREADS = 20 * 32;
constexpr int NBUF = 4;  // per-group TMEM accumulator buffers
constexpr int REG_LO = 32, REG_HI = 112;
constexpr uint32_t TMEM_COLS = NBUF * BN;
constexpr uint32_t A_BYTES = BM * BK;       // 16 KB
constexpr uint32_t BU_BYTES = BN * BK;      // 16 KB int8 weights
constexpr uint32_t BP_BYTES = BN * BK / 4;  // 4 KB packed codes
constexpr int MAX_NG = 32;                  // K / G groups per output (the model has at most 4096 / 128)
constexpr uint32_t SW_BYTES = 2 * MAX_NG * BN * 4;       // double-buffered weight-scale slice per tile
constexpr uint32_t STG_BYTES = EPI_WARPS * 32 * 32 * 4;  // output staging: 32 rows x 32 f32 per warp
constexpr uint32_t SMEM_BYTES =
    STAGES * (A_BYTES + BU_BYTES + BP_BYTES) + SW_BYTES + STG_BYTES + 1024 /*align*/ + 512 /*barriers*/;
constexpr uint32_t IDESC = idesc_i8(BM, BN);
constexpr uint32_t MAGIC = 0x4B400000u;  // bits of 1.5 * 2^23

struct Params {
  const float* sx;       // [M, ng]
  const uint8_t* codes;  // 2-bit mode: [n_tiles][K/128][BN][32]
  const float* swT;      // [n_tiles][ng][BN], one contiguous slice per output tile
  const float* bias;     // [N] or null
  float* y;              // [M, N]
  int32_t* sums;         // [M, N, ng] or null
  int* status;
  int M, N, K, G;
  int ep;
  float ep_scale;
  int tma_store;  // y via TMA (N % 4 == 0, aligned); otherwise direct stores
};

// 16 two-bit codes (bit layout chosen by the repack) -> 16 int8 trits, one PRMT per 4 weights.
// Code c selects byte c of 0x000100FF: 0 -> -1, 1 -> 0, 2 -> +1.
__device__ __forceinline__ uint4 unpack16(uint32_t w) {
  const uint32_t a = w & 0x33333333u;
  const uint32_t b = (w >> 2) & 0x33333333u;
  uint4 o;
  o.x = __byte_perm(0x000100FFu, 0u, a);
  o.y = __byte_perm(0x000100FFu, 0u, b);
  o.z = __byte_perm(0x000100FFu, 0u, a >> 16);
  o.w = __byte_perm(0x000100FFu, 0u, b >> 16);
  return o;
}

__device__ __forceinline__ uint64_t pack2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void unpack2(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
// Packed pairs of IEEE round-to-nearest f32 operations (sm_100 f32x2): each lane is exactly the scalar op.
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}

__device__ __forceinline__ float apply_ep(int ep, float es, float a, float old) {
  if (ep == VXG_EP_SILU) return silu_fast(a);
  if (ep == VXG_EP_ADD_SCALED) return __fmaf_rn(es, a, old);
  return a;
}

template <bool PACKED>
__global__ void __launch_bounds__(THREADS, 1)
    ternary_gemm_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_w,
                        const __grid_constant__ CUtensorMap tmap_y, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sBu = sA + STAGES * A_BYTES;
  float* sStg = reinterpret_cast<float*>(sBu + STAGES * BU_BYTES);  // 1024-aligned (TMA swizzle atoms)
  uint8_t* sBp = reinterpret_cast<uint8_t*>(sStg) + STG_BYTES;
  float* sSW = reinterpret_cast<float*>(sBp + STAGES * BP_BYTES);
  uint64_t* bars = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(sSW) + SW_BYTES);
  uint64_t* full = bars;                 // producer -> unpackers / MMA (TMA + bulk bytes)
  uint64_t* unpacked = bars + STAGES;    // unpackers -> MMA (2-bit mode)
  uint64_t* empty = bars + 2 * STAGES;   // MMA commit -> producer
  uint64_t* tfull = bars + 3 * STAGES;   // MMA commit -> epilogue (per TMEM buffer)
  uint64_t* tempty = tfull + NBUF;       // epilogue warps -> MMA
  uint64_t* ybar = tempty + NBUF;        // per epilogue warp: AddScaled old-value tile landed
  uint64_t* drain = ybar + EPI_WARPS;    // MMA drain on the error path
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&unpacked[s], UNPACK_WARPS * 32);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < NBUF; b++) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], EPI_WARPS);
    }
    for (int w = 0; w < EPI_WARPS; w++) mbar_init(&ybar[w], 1);
    mbar_init(drain, 1);
    fence_mbar_init();
  }
  if (warp == PROD_WARP && lane == 0) {
    prefetch_tmap(&tmap_x);
    if (!PACKED) prefetch_tmap(&tmap_w);
  }
  if (warp == MMA_WARP) {
    tmem_alloc(tmem_holder, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  if (warp < EPI_WARPS) {  // arm every accumulator buffer with the offset the MMA accumulates onto
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    for (int b = 0; b < NBUF; b++) tmem_st32_const(tmem_base + lane_base + (uint32_t)(b * BN + (warp >> 2) * 32), MAGIC);
    tmem_wait_st();
    tc_fence_before();
  }
  __syncthreads();
  tc_fence_after();

  const int ng = p.K / p.G, cpg = p.G / BK, nchunks = p.K / BK;
  const int m_tiles = (p.M + BM - 1) / BM, n_tiles = (p.N + BN - 1) / BN;
  const int total = m_tiles * n_tiles;

  // Register split: the launch gives 640 x 96; warpgroup 4 (producer, MMA, unpackers) drops to REG_LO and the four
  // epilogue warpgroups rise to REG_HI. The total must stay within the launch budget or the increase never completes.
  static_assert(128 * REG_LO + 512 * REG_HI <= THREADS * 96, "register split exceeds the launch budget");
  if (warp >= EPI_WARPS) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(REG_LO) : "memory");
  if (warp == PROD_WARP) {
    // ------------------------------------------------------------------------------------------ producer
    if (elect_one()) {
      int it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x) {
        const int mt = tile / n_tiles, nt = tile % n_tiles;
        for (int c = 0; c < nchunks; c++, it++) {
          const int s = it % STAGES;
          if (!mbar_wait(&empty[s], ((it / STAGES) & 1) ^ 1, p.status, VXG_DEV_TIMEOUT_PRODUCER)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[s], A_BYTES + (PACKED ? BP_BYTES : BU_BYTES));
          tma_load_2d(sA + s * A_BYTES, &tmap_x, c * BK, mt * BM, &full[s]);
          if (PACKED)
            bulk_load(sBp + s * BP_BYTES, p.codes + ((size_t)nt * nchunks + c) * BP_BYTES, BP_BYTES, &full[s]);
          else
            tma_load_2d(sBu + s * BU_BYTES, &tmap_w, c * BK, nt * BN, &full[s]);
        }
      }
      // every load issued must land before the CTA exits (normally all were consumed)
      for (int k = it > STAGES ? it - STAGES : 0; k < it; k++)
        mbar_wait(&full[k % STAGES], (k / STAGES) & 1, p.status, VXG_DEV_TIMEOUT_DRAIN);
    }
  } else if (warp == MMA_WARP) {
    // ----------------------------------------------------------------------------------------------- MMA
    if (elect_one()) {
      int it = 0, gi = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x) {
        for (int g = 0; g < ng && ok; g++, gi++) {
          const int b = gi % NBUF;
          if (!mbar_wait(&tempty[b], ((gi / NBUF) & 1) ^ 1, p.status, VXG_DEV_TIMEOUT_MMA)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d = tmem_base + (uint32_t)(b * BN);
          for (int cc = 0; cc < cpg; cc++, it++) {
            const int s = it % STAGES;
            if (!mbar_wait(PACKED ? &unpacked[s] : &full[s], (it / STAGES) & 1, p.status, VXG_DEV_TIMEOUT_MMA)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint64_t ad = umma_desc_sw128(smem_u32(sA + s * A_BYTES));
            const uint64_t bd = umma_desc_sw128(smem_u32(sBu + s * BU_BYTES));
#pragma unroll
            for (int k = 0; k < BK / 32; k++) mma_i8(d, ad + (uint64_t)(2 * k), bd + (uint64_t)(2 * k), IDESC, 1u);
            mma_commit(&empty[s]);
          }
          if (ok) mma_commit(&tfull[b]);
        }
      }
      if (!ok) {  // wait for every MMA issued so far before TMEM is released
        mma_commit(drain);
        mbar_wait(drain, 0, p.status, VXG_DEV_TIMEOUT_DRAIN);
      }
    }
  } else if (warp >= UNPACK_WARP0) {
    // ------------------------------------------------------------------------------ unpackers (2-bit mode)
    if (PACKED) {
      const int u = threadIdx.x - UNPACK_WARP0 * 32;
      int it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x) {
        for (int c = 0; c < nchunks; c++, it++) {
          const int s = it % STAGES;
          if (!mbar_wait(&full[s], (it / STAGES) & 1, p.status, VXG_DEV_TIMEOUT_UNPACK)) {
            ok = false;
            break;
          }
          const uint4* src = reinterpret_cast<const uint4*>(sBp + s * BP_BYTES);
          uint8_t* dst = sBu + s * BU_BYTES;
#pragma unroll 2
          for (int wq = u; wq < BN * 2; wq += UNPACK_WARPS * 32) {  // 4 code words = half a row per step
            const uint4 w4 = src[wq];
            const uint32_t r = (uint32_t)(wq >> 1), c0 = (uint32_t)((wq & 1) * 4);
            *reinterpret_cast<uint4*>(dst + sw128_offset(r, c0 + 0)) = unpack16(w4.x);
            *reinterpret_cast<uint4*>(dst + sw128_offset(r, c0 + 1)) = unpack16(w4.y);
            *reinterpret_cast<uint4*>(dst + sw128_offset(r, c0 + 2)) = unpack16(w4.z);
            *reinterpret_cast<uint4*>(dst + sw128_offset(r, c0 + 3)) = unpack16(w4.w);
          }
          fence_proxy_async_smem();
          mbar_arrive(&unpacked[s]);
        }
      }
    }
  }
  } else {
    // ------------------------------------------------------------------------------------------- epilogue
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(REG_HI) : "memory");
    const int q = warp & 3;   // TMEM lane quarter = the warp's 32 tokens
    const int cs = warp >> 2; // 32-column slice of the tile
    float* stg = sStg + warp * 32 * 32;
    auto issue_scales = [&](int tile, int buf) {
      const float* src = p.swT + (size_t)(tile % n_tiles) * ng * BN;
      float* dst = sSW + buf * MAX_NG * BN;
      for (int ch = threadIdx.x; ch < ng * BN / 4; ch += EPI_WARPS * 32) cp_async16(dst + ch * 4, src + ch * 4);
    };
    const uint64_t negm = pack2(-12582912.0f, -12582912.0f);
    int gi = 0, lt = 0, yloads = 0;
    bool ok = true;
    issue_scales(blockIdx.x, 0);
    cp_async_commit();
    for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x, lt++) {
      named_bar_sync(1, EPI_WARPS * 32);  // buffer (lt+1)&1 (tile lt-1) is no longer read
      if (tile + (int)gridDim.x < total) issue_scales(tile + gridDim.x, (lt + 1) & 1);
      cp_async_commit();
      cp_async_wait_1();
      named_bar_sync(1, EPI_WARPS * 32);  // this tile's slice landed for every thread
      const int mt = tile / n_tiles, nt = tile % n_tiles;
      const int row0 = mt * BM + q * 32, col0 = nt * BN + cs * 32;
      const int row = row0 + lane;
      const bool row_ok = row < p.M;
      if (p.tma_store && p.ep == VXG_EP_ADD_SCALED && lane == 0) {  // old values for the residual add
        bulk_wait_read_all();
        mbar_arrive_expect_tx(&ybar[warp], 32 * 32 * 4);
        tma_load_2d(stg, &tmap_y, col0, row0, &ybar[warp]);
      }
      const float* swt = sSW + (lt & 1) * MAX_NG * BN + cs * 32;
      const float* sxr = p.sx + (size_t)(row_ok ? row : 0) * ng;
      float sx_next = row_ok ? __ldg(sxr) : 0.0f;
      uint64_t acc[16];  // f32x2 pairs: columns (2i, 2i+1) of the slice
#pragma unroll
      for (int i = 0; i < 16; i++) acc[i] = 0ull;
      for (int g = 0; g < ng; g++, gi++) {
        const float sxv = sx_next;
        if (g + 1 < ng && row_ok) sx_next = __ldg(sxr + g + 1);
        const int b = gi % NBUF;
        if (!mbar_wait(&tfull[b], (gi / NBUF) & 1, p.status, VXG_DEV_TIMEOUT_EPILOGUE)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(b * BN + cs * 32);
        const uint64_t sx2 = pack2(sxv, sxv);
        const float* swg = swt + g * BN;
#pragma unroll
        for (int h = 0; h < 2; h++) {  // two 16-column halves keep only 16 sums live
          uint32_t S[16];
          tmem_ld16(taddr + h * 16, S);
          tmem_wait_ld();
          tmem_st16_const(taddr + h * 16, MAGIC);  // re-arm for a later group
          if (h == 1) {
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[b]);
          }
#pragma unroll
          for (int c = 0; c < 16; c += 4) {
            const float4 w4 = *reinterpret_cast<const float4*>(swg + h * 16 + c);
            const uint64_t p01 = mul2(sx2, pack2(w4.x, w4.y));
            const uint64_t p23 = mul2(sx2, pack2(w4.z, w4.w));
            const uint64_t f01 = add2(pack2(__uint_as_float(S[c]), __uint_as_float(S[c + 1])), negm);
            const uint64_t f23 = add2(pack2(__uint_as_float(S[c + 2]), __uint_as_float(S[c + 3])), negm);
            const int a = (h * 16 + c) / 2;
            acc[a] = fma2(f01, p01, acc[a]);
            acc[a + 1] = fma2(f23, p23, acc[a + 1]);
          }
          if (p.sums && row_ok) {
            for (int c = 0; c < 16; c++) {
              const int o = col0 + h * 16 + c;
              if (o < p.N) p.sums[((size_t)row * p.N + o) * ng + g] = (int32_t)(S[c] - MAGIC);
            }
          }
        }
      }
      if (!ok) break;
      if (p.tma_store) {
        if (p.ep == VXG_EP_ADD_SCALED) {
          if (!mbar_wait(&ybar[warp], yloads & 1, p.status, VXG_DEV_TIMEOUT_EPILOGUE)) {
            ok = false;
            break;
          }
          yloads++;
        } else {
          if (lane == 0) bulk_wait_read_all();  // previous tile's store has read the staging tile
          __syncwarp();
        }
#pragma unroll
        for (int j = 0; j < 8; j++) {
          float* cell = stg + lane * 32 + ((j ^ (lane & 7)) << 2);  // 128-byte swizzle, 16-byte chunk j
          float v[4];
          unpack2(acc[2 * j], v[0], v[1]);
          unpack2(acc[2 * j + 1], v[2], v[3]);
          float4 old = make_float4(0.f, 0.f, 0.f, 0.f);
          if (p.ep == VXG_EP_ADD_SCALED) old = *reinterpret_cast<const float4*>(cell);
          const float ov[4] = {old.x, old.y, old.z, old.w};
#pragma unroll
          for (int k = 0; k < 4; k++) {
            float a = apply_ep(p.ep, p.ep_scale, v[k], ov[k]);
            const int o = col0 + 4 * j + k;
            if (p.bias && o < p.N) a = __fadd_rn(a, __ldg(p.bias + o));
            v[k] = a;
          }
          *reinterpret_cast<float4*>(cell) = make_float4(v[0], v[1], v[2], v[3]);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(&tmap_y, stg, col0, row0);
          bulk_commit();
        }
      } else if (row_ok) {
        float* yrow = p.y + (size_t)row * p.N;
#pragma unroll
        for (int j = 0; j < 16; j++) {
          float v[2];
          unpack2(acc[j], v[0], v[1]);
#pragma unroll
          for (int k = 0; k < 2; k++) {
            const int o = col0 + 2 * j + k;
            if (o < p.N) {
              float a = apply_ep(p.ep, p.ep_scale, v[k], p.ep == VXG_EP_ADD_SCALED ? yrow[o] : 0.0f);
              if (p.bias) a = __fadd_rn(a, __ldg(p.bias + o));
              yrow[o] = a;
            }
          }
        }
      }
    }
    if (lane == 0) bulk_wait_all();
    cp_async_wait_all();
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == MMA_WARP) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

}  // namespace gemm
}  // namespace vxg

using namespace vxg;

// ------------------------------------------------------------------------------------------------- C ABI

extern "C" {

int vxg_ternary_out_pad(int out) { return (out + gemm::BN - 1) / gemm::BN * gemm::BN; }

size_t vxg_ternary_codes_bytes(int out, int in) {
  if (out <= 0 || in <= 0) return 0;
  return (size_t)vxg_ternary_out_pad(out) * (size_t)in / 4;
}

size_t vxg_ternary_i8_bytes(int out, int in) {
  if (out <= 0 || in <= 0) return 0;
  return (size_t)vxg_ternary_out_pad(out) * (size_t)in;
}

size_t vxg_ternary_scales_count(int out, int in, int group) {
  if (out <= 0 || in <= 0 || group <= 0) return 0;
  return (size_t)(in / group) * (size_t)vxg_ternary_out_pad(out);
}

// trits.rs:7-27 decode: 5 base-3 digits per byte, least significant first, trit = digit - 1 (table per byte).
static void decode_row(const uint8_t* pk, int in, int8_t* row) {
  static const struct Table {
    int8_t t[256][5];
    Table() {
      for (int b = 0; b < 256; b++) {
        int v = b;
        for (int k = 0; k < 5; k++) {
          t[b][k] = (int8_t)(v % 3 - 1);
          v /= 3;
        }
      }
    }
  } T;
  const int full = in / 5;
  for (int i = 0; i < full; i++) std::memcpy(row + 5 * i, T.t[pk[i]], 5);
  for (int k = 0; k < in - 5 * full; k++) row[5 * full + k] = T.t[pk[full]][k];
}

// Run f(r0, r1) over row ranges on up to 32 host threads.
static void for_rows(int n, const std::function<void(int, int)>& f) {
  int nt = (int)std::min(32u, std::max(1u, std::thread::hardware_concurrency()));
  nt = std::max(1, std::min(nt, n / 128));
  if (nt == 1) {
    f(0, n);
    return;
  }
  std::vector<std::thread> th;
  const int chunk = (n + nt - 1) / nt;
  for (int i = 0; i < nt; i++)
    if (i * chunk < n) th.emplace_back(f, i * chunk, std::min(n, (i + 1) * chunk));
  for (auto& t : th) t.join();
}

// Bit position of element e (0..15) of a 16-element word: matches unpack16's PRMT selectors.
static inline int code_pos(int e) {
  const int q = e >> 2, j = e & 3;
  return (q & 2 ? 16 : 0) + (q & 1 ? 2 : 0) + 4 * j;
}

vxg_status vxg_ternary_repack(const uint8_t* qweight, const uint16_t* scales_f16, int out, int in, int group,
                              uint8_t* codes, float* scales_t) {
  clear_error();
  VXG_ARG(qweight && scales_f16 && codes && scales_t, "NULL pointer");
  VXG_ARG(out > 0 && in > 0 && group > 0, "bad shape out=%d in=%d group=%d", out, in, group);
  VXG_ARG(in % gemm::BK == 0 && group % gemm::BK == 0 && in % group == 0,
          "in (%d) and group (%d) must be multiples of 128 with group | in", in, group);
  const int out_pad = vxg_ternary_out_pad(out), rb = (in + 4) / 5, ng = in / group, nch = in / gemm::BK;
  uint32_t* words = reinterpret_cast<uint32_t*>(codes);
  int pos[16];
  for (int e = 0; e < 16; e++) pos[e] = code_pos(e);
  for_rows(out_pad, [&](int r0, int r1) {
    std::vector<int8_t> row(in);
    for (int r = r0; r < r1; r++) {
      if (r < out)
        decode_row(qweight + (size_t)r * rb, in, row.data());
      else
        std::fill(row.begin(), row.end(), (int8_t)0);
      const int nt = r / gemm::BN, rr = r % gemm::BN;
      for (int c = 0; c < nch; c++)
        for (int w = 0; w < 8; w++) {
          uint32_t word = 0;
          for (int e = 0; e < 16; e++) word |= (uint32_t)(row[c * 128 + w * 16 + e] + 1) << pos[e];
          words[(((size_t)nt * nch + c) * gemm::BN + rr) * 8 + w] = word;
        }
    }
  });
  for (int r = 0; r < out_pad; r++)  // tile-major [out_pad/128][ng][128]: one contiguous slice per output tile
    for (int g = 0; g < ng; g++)
      scales_t[((size_t)(r / gemm::BN) * ng + g) * gemm::BN + r % gemm::BN] =
          r < out ? __half2float(__ushort_as_half(scales_f16[(size_t)r * ng + g])) : 0.0f;
  return VXG_OK;
}

vxg_status vxg_ternary_repack_i8(const uint8_t* qweight, const uint16_t* scales_f16, int out, int in, int group,
                                 int8_t* w_rows, float* scales_t) {
  clear_error();
  VXG_ARG(qweight && scales_f16 && w_rows && scales_t, "NULL pointer");
  VXG_ARG(out > 0 && in > 0 && group > 0, "bad shape out=%d in=%d group=%d", out, in, group);
  VXG_ARG(in % gemm::BK == 0 && group % gemm::BK == 0 && in % group == 0,
          "in (%d) and group (%d) must be multiples of 128 with group | in", in, group);
  const int out_pad = vxg_ternary_out_pad(out), rb = (in + 4) / 5, ng = in / group;
  for_rows(out_pad, [&](int r0, int r1) {
    for (int r = r0; r < r1; r++) {
      int8_t* row = w_rows + (size_t)r * in;
      if (r < out)
        decode_row(qweight + (size_t)r * rb, in, row);
      else
        std::memset(row, 0, in);
    }
  });
  for (int r = 0; r < out_pad; r++)
    for (int g = 0; g < ng; g++)
      scales_t[((size_t)(r / gemm::BN) * ng + g) * gemm::BN + r % gemm::BN] =
          r < out ? __half2float(__ushort_as_half(scales_f16[(size_t)r * ng + g])) : 0.0f;
  return VXG_OK;
}

}  // extern "C"

vxg_status vxg::gemm_launch(bool packed, const int8_t* x, const float* sx, const void* w, const float* scales_t,
                            int M, int N, int K, int G, vxg_epilogue ep, float ep_scale, const float* bias, float* y,
                            int32_t* group_sums, cudaStream_t stream) {
  clear_error();
  VXG_ARG(x && sx && w && scales_t && y, "NULL pointer");
  VXG_ARG(M > 0 && N > 0 && K > 0 && G > 0, "bad shape M=%d N=%d K=%d G=%d", M, N, K, G);
  VXG_ARG(K % gemm::BK == 0 && G % gemm::BK == 0 && K % G == 0,
          "K (%d) and G (%d) must be multiples of 128 with G | K", K, G);
  if (K / G > gemm::MAX_NG || K > 32768) {
    set_error("K / G = %d groups (max %d) or K = %d (max 32768) not supported", K / G, gemm::MAX_NG, K);
    return VXG_ERR_UNSUPPORTED;
  }
  VXG_ARG(ep == VXG_EP_STORE || ep == VXG_EP_SILU || ep == VXG_EP_ADD_SCALED, "bad epilogue %d", (int)ep);
  VXG_ARG(((uintptr_t)x & 15) == 0 && ((uintptr_t)w & 15) == 0 && ((uintptr_t)scales_t & 15) == 0,
          "x, weights and scales_t must be 16-byte aligned");
  int* status = device_status();
  VXG_ARG(status != nullptr, "no CUDA device");
  CUtensorMap tx, tw, ty;
  vxg_status st = make_tmap_2d_u8(&tx, x, (uint64_t)M, (uint64_t)K, (uint64_t)K, gemm::BM, gemm::BK);
  if (st != VXG_OK) return st;
  if (!packed) {
    st = make_tmap_2d_u8(&tw, w, (uint64_t)vxg_ternary_out_pad(N), (uint64_t)K, (uint64_t)K, gemm::BN, gemm::BK);
    if (st != VXG_OK) return st;
  } else {
    tw = tx;  // unused
  }
  const int tma_store = (N % 4 == 0) && (((uintptr_t)y & 15) == 0);
  if (tma_store) {
    st = make_tmap_2d_f32(&ty, y, (uint64_t)M, (uint64_t)N, (uint64_t)N * 4, 32);
    if (st != VXG_OK) return st;
  } else {
    ty = tx;  // unused
  }
  {
    const vxg_status sa =
        smem_attr(packed ? (const void*)gemm::ternary_gemm_kernel<true> : (const void*)gemm::ternary_gemm_kernel<false>,
                  (int)gemm::SMEM_BYTES);
    if (sa != VXG_OK) return sa;
  }
  gemm::Params p;
  p.sx = sx;
  p.codes = packed ? static_cast<const uint8_t*>(w) : nullptr;
  p.swT = scales_t;
  p.bias = bias;
  p.y = y;
  p.sums = group_sums;
  p.status = status;
  p.M = M;
  p.N = N;
  p.K = K;
  p.G = G;
  p.ep = (int)ep;
  p.ep_scale = ep_scale;
  p.tma_store = tma_store;
  const int tiles = ((M + gemm::BM - 1) / gemm::BM) * ((N + gemm::BN - 1) / gemm::BN);
  const int grid = std::min(tiles, sm_count());
  if (packed)
    gemm::ternary_gemm_kernel<true><<<grid, gemm::THREADS, gemm::SMEM_BYTES, stream>>>(tx, tw, ty, p);
  else
    gemm::ternary_gemm_kernel<false><<<grid, gemm::THREADS, gemm::SMEM_BYTES, stream>>>(tx, tw, ty, p);
  note_launch();
  VXG_CUDA(cudaGetLastError());
  return VXG_OK;
}

extern "C" {

vxg_status vxg_gemm_ternary_i8(const int8_t* x, const float* sx, const uint8_t* codes, const float* scales_t, int M,
                               int N, int K, int G, vxg_epilogue ep, float ep_scale, const float* bias, float* y,
                               int32_t* group_sums, void* stream) {
  return gemm_launch(true, x, sx, codes, scales_t, M, N, K, G, ep, ep_scale, bias, y, group_sums,
                     (cudaStream_t)stream);
}

vxg_status vxg_gemm_ternary_i8w(const int8_t* x, const float* sx, const int8_t* w_rows, const float* scales_t,
                                int M, int N, int K, int G, vxg_epilogue ep, float ep_scale, const float* bias,
                                float* y, int32_t* group_sums, void* stream) {
  return gemm_launch(false, x, sx, w_rows, scales_t, M, N, K, G, ep, ep_scale, bias, y, group_sums,
                     (cudaStream_t)stream);
}

}  // extern "C"
