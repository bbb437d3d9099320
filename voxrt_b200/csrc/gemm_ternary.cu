// Ternary-weight x int8-activation GEMM on the sm_100a tensor cores (tcgen05.mma kind::i8).
//
// Reference semantics (crates/voxrt/src/kernels/mod.rs:166-210, x86.rs:91-154): for every output (t, o)
//   acc = 0; for g in groups: acc = fma(float(S_g), sx[t,g] * sw[o,g], acc);  y = epilogue(old, acc)
// with S_g the exact int32 dot product over the group. The int32 sums come from the tensor cores; the float chain
// runs in the epilogue warps in the reference's group order, so the result is bit-identical.
//
// Persistent, warp-specialised CTA (one per SM), tile = 128 tokens x 128 weight rows. Each CTA owns a
// contiguous range of tiles in weight-tile-major order, so consecutive tiles share their weight rows:
//   resident mode (K <= 1024): the CTA keeps the tile's whole weight slab (128 rows x K int8, <= 128 KB) in shared
//                memory and only streams activations; the slab is refilled when the weight tile changes, chunk by
//                chunk, so the first tile of a slab overlaps its own fill. 2-bit codes are unpacked in the SM once
//                per slab instead of once per tile.
//   streaming mode (K > 1024): activation and weight chunks stream together through a 4-stage ring.
// Roles:
//   warps 0-15   epilogue: warp w owns TMEM lanes 32*(w%4)..+32 (its tokens) and columns 32*(w/4)..+32 of the tile.
//                Per group it loads the sums (tcgen05.ld), re-arms the buffer and runs the FMA chain on packed f32x2
//                pairs; per tile it applies the epilogue and writes through 1 KB staging quarters with TMA stores
//                (or, for the fused SiLU -> int8 epilogue, stores int8 codes and per-row scales directly).
//   warp 16      TMA producer (activation chunks, weight chunks / code chunks).
//   warp 17      TMEM allocator + MMA issuer: 4 x (M128 N128 K32) per chunk into one of four per-group int32
//                accumulator buffers (all 512 TMEM columns), commit -> stage free / group ready / slab chunk free.
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
constexpr int BK = 128;  // K per chunk: one 128-byte swizzle row
constexpr int EPI_WARPS = 8;      // two warpgroups; warp w: TMEM lanes 32*(w%4).., columns 64*(w/4)..
constexpr int EPI_COLS = BN / (EPI_WARPS / 4);  // 64 columns per epilogue warp
constexpr int PROD_WARP = 8, MMA_WARP = 9, UNPACK_WARP0 = 10, UNPACK_WARPS = 2;
constexpr int THREADS = 12 * 32;  // three whole warpgroups (setmaxnreg acts per warpgroup)
constexpr int LAUNCH_REGS = 168;  // 65536 / 384 rounded down to the allocation unit
constexpr int REG_LO = 120, REG_HI = 192;
static_assert(4 * 32 * REG_LO + EPI_WARPS * 32 * REG_HI <= THREADS * LAUNCH_REGS,
              "register split exceeds the launch budget");
constexpr int NBUF = 4;  // per-group TMEM accumulator buffers
constexpr uint32_t TMEM_COLS = NBUF * BN;
constexpr int KRES = kGemmResidentK;  // largest K whose weight slab stays resident
constexpr int RES_STAGES = 4;   // activation ring, resident mode
constexpr int STR_STAGES = 4;   // activation + weight ring, streaming mode
constexpr int CODE_SLOTS = 2;   // code chunks in flight while a slab fills
constexpr int MAX_NG = 32;      // K / G groups per output (the model has at most 4096 / 128)
constexpr int MAX_CHUNKS = KRES / BK;
constexpr uint32_t A_BYTES = BM * BK;       // 16 KB
constexpr uint32_t BU_BYTES = BN * BK;      // 16 KB int8 weights per chunk
constexpr uint32_t BP_BYTES = BN * BK / 4;  // 4 KB packed codes per chunk
constexpr uint32_t Q_BYTES = 32 * 8 * 4;    // one staging quarter: 32 rows x 8 f32
constexpr uint32_t STG_BYTES = EPI_WARPS * 2 * Q_BYTES;  // two quarters per warp: 16 KB
// resident:  [slab 8 x 16 KB][A ring 4 x 16 KB][code slots 2 x 4 KB][staging 16 KB][sw slice 4 KB]
// streaming: [ring 4 x (A 16 KB + B 16 KB)][code slots 4 x 4 KB][staging 16 KB][sw slice 16 KB]
constexpr uint32_t RES_MAIN = MAX_CHUNKS * BU_BYTES + RES_STAGES * A_BYTES + CODE_SLOTS * BP_BYTES;
constexpr uint32_t STR_MAIN = STR_STAGES * (A_BYTES + BU_BYTES) + STR_STAGES * BP_BYTES;
constexpr uint32_t RES_SW = (KRES / BK) * BN * 4, STR_SW = MAX_NG * BN * 4;
constexpr uint32_t BAR_BYTES = 1024;
constexpr uint32_t RES_SMEM = RES_MAIN + STG_BYTES + RES_SW + BAR_BYTES;
constexpr uint32_t STR_SMEM = STR_MAIN + STG_BYTES + STR_SW + BAR_BYTES;
constexpr uint32_t SMEM_BYTES = (RES_SMEM > STR_SMEM ? RES_SMEM : STR_SMEM) + 1024 /*align*/;
static_assert(SMEM_BYTES <= 232448, "shared memory budget");
constexpr uint32_t IDESC = idesc_i8(BM, BN);
constexpr uint32_t MAGIC = 0x4B400000u;  // bits of 1.5 * 2^23

constexpr int EP_SILU_Q = kGemmSiluQuant;  // SiLU then per-(row, 128-column) int8 quantisation

struct Params {
  const float* sx;       // [M, ng]
  const uint8_t* codes;  // 2-bit mode: [n_tiles][K/128][BN][32]
  const float* swT;      // [n_tiles][ng][BN], one contiguous slice per output tile
  const float* bias;     // [N] or null
  float* y;              // [M, N]
  int8_t* q;             // EP_SILU_Q: [M, N] int8
  float* qs;             // EP_SILU_Q: [M, N/128]
  int32_t* sums;         // [M, N, ng] or null
  int* status;
  int M, N, K, G;
  int ep;
  float ep_scale;
  int tma_store;  // y via TMA (N % 4 == 0, aligned); otherwise direct stores
  int resident;   // weight slab resident (K <= KRES)
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

// One 128 x 128 chunk: 4 KB of codes (row r: 8 words) -> 16 KB int8 in the 128-byte-swizzled K-major layout.
// `u` indexes the unpacking threads (0 .. UNPACK_WARPS*32-1); each handles 2 rows' halves per pass.
__device__ __forceinline__ void unpack_chunk(const uint8_t* src, uint8_t* dst, int u) {
  const uint4* s4 = reinterpret_cast<const uint4*>(src);
#pragma unroll
  for (int i = 0; i < (BN * 2) / (UNPACK_WARPS * 32); i++) {
    const int wq = u + i * UNPACK_WARPS * 32;  // 4 code words = half a row
    const uint4 w4 = s4[wq];
    const uint32_t r = (uint32_t)(wq >> 1), c0 = (uint32_t)((wq & 1) * 4);
    *reinterpret_cast<uint4*>(dst + sw128_offset(r, c0 + 0)) = unpack16(w4.x);
    *reinterpret_cast<uint4*>(dst + sw128_offset(r, c0 + 1)) = unpack16(w4.y);
    *reinterpret_cast<uint4*>(dst + sw128_offset(r, c0 + 2)) = unpack16(w4.z);
    *reinterpret_cast<uint4*>(dst + sw128_offset(r, c0 + 3)) = unpack16(w4.w);
  }
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

template <int EP>
__device__ __forceinline__ float apply_ep(float es, float a, float old) {
  if constexpr (EP == VXG_EP_SILU) return silu_fast(a);
  if constexpr (EP == VXG_EP_ADD_SCALED) return __fmaf_rn(es, a, old);
  return a;
}

constexpr int HC = EPI_COLS / 2;  // columns per TMEM load (half of a warp's slice)

__device__ __forceinline__ void tmem_ld_half(uint32_t taddr, uint32_t (&r)[32]) { tmem_ld32(taddr, r); }
__device__ __forceinline__ void tmem_ld_half(uint32_t taddr, uint32_t (&r)[16]) { tmem_ld16(taddr, r); }
__device__ __forceinline__ void tmem_rearm(uint32_t taddr) {
#pragma unroll
  for (int k = 0; k < EPI_COLS / 32; k++) tmem_st32_const(taddr + 32 * k, MAGIC);
}

// Work split: CTA b owns tiles [b*T/G, (b+1)*T/G) of the weight-tile-major order (tile t -> nt = t / m_tiles,
// mt = t % m_tiles).
__device__ __forceinline__ void tile_range(int total, int& t0, int& t1) {
  t0 = (int)((long long)blockIdx.x * total / gridDim.x);
  t1 = (int)((long long)(blockIdx.x + 1) * total / gridDim.x);
}

// Shared-memory map, fixed per mode at compile time so every address is the base plus a constant.
template <bool RES>
struct Smem {
  static constexpr uint32_t SLAB = 0;                                             // resident: 8 x 16 KB
  static constexpr uint32_t A = RES ? MAX_CHUNKS * BU_BYTES : 0;                  // stage s at A + s * A_STRIDE
  static constexpr uint32_t A_STRIDE = RES ? A_BYTES : A_BYTES + BU_BYTES;
  static constexpr uint32_t B = RES ? 0 : A_BYTES;                                 // streaming: stage s at B + s * A_STRIDE
  static constexpr int STAGES = RES ? RES_STAGES : STR_STAGES;
  static constexpr uint32_t CODE = A + STAGES * A_STRIDE;                          // code slots, 4 KB each
  static constexpr uint32_t MAIN = RES ? RES_MAIN : STR_MAIN;
  static constexpr uint32_t STG = MAIN;
  static constexpr uint32_t SW = STG + STG_BYTES;
  static constexpr uint32_t BARS = SW + (RES ? RES_SW : STR_SW);
  static_assert(CODE + (RES ? CODE_SLOTS : STR_STAGES) * BP_BYTES <= MAIN, "layout");
  static_assert(BARS + BAR_BYTES <= SMEM_BYTES - 1024, "layout");
};
// barrier indices inside the BARS block
enum : int {
  B_AFULL = 0,                       // [4] producer -> MMA / unpackers: stage landed (TMA tx)
  B_AEMPTY = 4,                      // [4] MMA commit -> producer
  B_UNPACKED = 8,                    // [4] streaming 2-bit: unpackers -> MMA
  B_CFULL = 12,                      // [2] resident 2-bit fill: code slot landed
  B_CEMPTY = 14,                     // [2] resident 2-bit fill: code slot read
  B_BREADY = 16,                     // [8] resident: slab chunk filled (one phase per slab)
  B_BFREE = B_BREADY + MAX_CHUNKS,   // [8] resident: slab chunk no longer read (MMA commit)
  B_TFULL = B_BFREE + MAX_CHUNKS,    // [4] MMA commit -> epilogue (per TMEM buffer)
  B_TEMPTY = B_TFULL + NBUF,         // [4] epilogue warps -> MMA
  B_YBAR = B_TEMPTY + NBUF,          // [16] per epilogue warp: AddScaled old-value quarter landed
  B_DRAIN = B_YBAR + EPI_WARPS,      // MMA drain
  B_COUNT = B_DRAIN + 1
};
static_assert(B_COUNT * 8 + 16 <= (int)BAR_BYTES, "barrier block");

template <bool PACKED, bool RES, int EP, bool TMA_STORE>
__global__ void __launch_bounds__(THREADS, 1)
    ternary_gemm_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_w,
                        const __grid_constant__ CUtensorMap tmap_y, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  using L = Smem<RES>;
  constexpr bool res = RES;
  constexpr int stages = L::STAGES;
  uint8_t* const sSlab = smem + L::SLAB;
  uint8_t* const sA = smem + L::A;
  uint8_t* const sBu = smem + L::B;
  uint8_t* const sCode = smem + L::CODE;
  constexpr uint32_t a_stride = L::A_STRIDE, b_stride = L::A_STRIDE;
  float* const sStg = reinterpret_cast<float*>(smem + L::STG);
  float* const sSW = reinterpret_cast<float*>(smem + L::SW);
  uint64_t* const bars = reinterpret_cast<uint64_t*>(smem + L::BARS);
  uint64_t* const afull = bars + B_AFULL;
  uint64_t* const aempty = bars + B_AEMPTY;
  uint64_t* const unpacked = bars + B_UNPACKED;
  uint64_t* const cfull = bars + B_CFULL;
  uint64_t* const cempty = bars + B_CEMPTY;
  uint64_t* const bready = bars + B_BREADY;
  uint64_t* const bfree = bars + B_BFREE;
  uint64_t* const tfull = bars + B_TFULL;
  uint64_t* const tempty = bars + B_TEMPTY;
  uint64_t* const ybar = bars + B_YBAR;
  uint64_t* const drain = bars + B_DRAIN;
  uint32_t* const tmem_holder = reinterpret_cast<uint32_t*>(bars + B_COUNT);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < 4; s++) {
      mbar_init(&afull[s], 1);
      mbar_init(&aempty[s], 1);
      mbar_init(&unpacked[s], UNPACK_WARPS * 32);
    }
    for (int r = 0; r < CODE_SLOTS; r++) {
      mbar_init(&cfull[r], 1);
      mbar_init(&cempty[r], UNPACK_WARPS * 32);
    }
    for (int c = 0; c < MAX_CHUNKS; c++) {
      mbar_init(&bready[c], PACKED ? UNPACK_WARPS * 32 : 1);
      mbar_init(&bfree[c], 1);
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
    for (int b = 0; b < NBUF; b++)
      for (int h = 0; h < EPI_COLS / 32; h++)
        tmem_st32_const(tmem_base + lane_base + (uint32_t)(b * BN + (warp >> 2) * EPI_COLS + h * 32), MAGIC);
    tmem_wait_st();
    tc_fence_before();
  }
  __syncthreads();
  tc_fence_after();

  const int ng = p.K / p.G, cpg = p.G / BK, nchunks = p.K / BK;
  const int m_tiles = (p.M + BM - 1) / BM, n_tiles = (p.N + BN - 1) / BN;
  int t0, t1;
  tile_range(m_tiles * n_tiles, t0, t1);

  if (warp >= EPI_WARPS) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(REG_LO) : "memory");
    if (warp == PROD_WARP) {
      // ------------------------------------------------------------------------------------------ producer
      if (elect_one()) {
        int it = 0, ci = 0, slab = -1, cur_nt = -1;
        bool ok = true;
        for (int t = t0; t < t1 && ok; t++) {
          const int nt = t / m_tiles, mt = t % m_tiles;
          const bool fill = res && nt != cur_nt;
          if (fill) {
            slab++;
            cur_nt = nt;
          }
          for (int c = 0; c < nchunks; c++, it++) {
            if (fill) {
              if (PACKED) {  // code chunk c of the new slab -> a code slot (unpacked into the slab by warps 18-21)
                const int r = ci % CODE_SLOTS;
                if (!mbar_wait(&cempty[r], ((ci / CODE_SLOTS) & 1) ^ 1, p.status, VXG_DEV_TIMEOUT_PRODUCER)) {
                  ok = false;
                  break;
                }
                mbar_arrive_expect_tx(&cfull[r], BP_BYTES);
                bulk_load(sCode + r * BP_BYTES, p.codes + ((size_t)nt * nchunks + c) * BP_BYTES, BP_BYTES, &cfull[r]);
                ci++;
              } else {  // int8 rows straight into slab chunk c once the previous slab's MMAs are done with it
                if (slab > 0 &&
                    !mbar_wait(&bfree[c], (slab - 1) & 1, p.status, VXG_DEV_TIMEOUT_PRODUCER)) {
                  ok = false;
                  break;
                }
                mbar_arrive_expect_tx(&bready[c], BU_BYTES);
                tma_load_2d(sSlab + c * BU_BYTES, &tmap_w, c * BK, nt * BN, &bready[c]);
              }
            }
            const int s = it % stages;
            if (!mbar_wait(&aempty[s], ((it / stages) & 1) ^ 1, p.status, VXG_DEV_TIMEOUT_PRODUCER)) {
              ok = false;
              break;
            }
            if (res) {
              mbar_arrive_expect_tx(&afull[s], A_BYTES);
              tma_load_2d(sA + s * a_stride, &tmap_x, c * BK, mt * BM, &afull[s]);
            } else {
              mbar_arrive_expect_tx(&afull[s], A_BYTES + (PACKED ? BP_BYTES : BU_BYTES));
              tma_load_2d(sA + s * a_stride, &tmap_x, c * BK, mt * BM, &afull[s]);
              if (PACKED)
                bulk_load(sCode + s * BP_BYTES, p.codes + ((size_t)nt * nchunks + c) * BP_BYTES, BP_BYTES,
                          &afull[s]);
              else
                tma_load_2d(sBu + s * b_stride, &tmap_w, c * BK, nt * BN, &afull[s]);
            }
          }
        }
        // every load issued must land before the CTA exits (normally all were consumed)
        for (int k = it > stages ? it - stages : 0; k < it; k++)
          mbar_wait(&afull[k % stages], (k / stages) & 1, p.status, VXG_DEV_TIMEOUT_DRAIN);
        if (res && PACKED)
          for (int k = ci > CODE_SLOTS ? ci - CODE_SLOTS : 0; k < ci; k++)
            mbar_wait(&cfull[k % CODE_SLOTS], (k / CODE_SLOTS) & 1, p.status, VXG_DEV_TIMEOUT_DRAIN);
        if (res && !PACKED && slab >= 0)
          for (int c = 0; c < nchunks; c++) mbar_wait(&bready[c], slab & 1, p.status, VXG_DEV_TIMEOUT_DRAIN);
      }
    } else if (warp == MMA_WARP) {
      // --------------------------------------------------------------------------------------------- MMA
      if (elect_one()) {
        int it = 0, gi = 0, slab = -1, cur_nt = -1;
        bool ok = true;
        for (int t = t0; t < t1 && ok; t++) {
          const int nt = t / m_tiles;
          if (nt != cur_nt) {
            slab++;
            cur_nt = nt;
          }
          const bool last_of_slab = res && (t + 1 == t1 || (t + 1) / m_tiles != nt);
          for (int g = 0; g < ng && ok; g++, gi++) {
            const int b = gi % NBUF;
            if (!mbar_wait(&tempty[b], ((gi / NBUF) & 1) ^ 1, p.status, VXG_DEV_TIMEOUT_MMA)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t d = tmem_base + (uint32_t)(b * BN);
            for (int cc = 0; cc < cpg; cc++, it++) {
              const int c = g * cpg + cc, s = it % stages;
              uint64_t* ready = (!res && PACKED) ? &unpacked[s] : &afull[s];
              if (!mbar_wait(ready, (it / stages) & 1, p.status, VXG_DEV_TIMEOUT_MMA) ||
                  (res && !mbar_wait(&bready[c], slab & 1, p.status, VXG_DEV_TIMEOUT_MMA))) {
                ok = false;
                break;
              }
              tc_fence_after();
              const uint64_t ad = umma_desc_sw128(smem_u32(sA + s * a_stride));
              const uint64_t bd = umma_desc_sw128(smem_u32(res ? sSlab + c * BU_BYTES : sBu + s * b_stride));
#pragma unroll
              for (int k = 0; k < BK / 32; k++) mma_i8(d, ad + (uint64_t)(2 * k), bd + (uint64_t)(2 * k), IDESC, 1u);
              mma_commit(&aempty[s]);
              if (last_of_slab) mma_commit(&bfree[c]);
            }
            if (ok) mma_commit(&tfull[b]);
          }
        }
        // wait for every MMA issued so far before TMEM is released (and before the error path gives up)
        mma_commit(drain);
        mbar_wait(drain, 0, p.status, VXG_DEV_TIMEOUT_DRAIN);
      }
    } else if (PACKED) {
      // ------------------------------------------------------------------------------ unpackers (2-bit mode)
      const int u = threadIdx.x - UNPACK_WARP0 * 32;
      bool ok = true;
      if (res) {
        int ci = 0, slab = -1, cur_nt = -1;
        for (int t = t0; t < t1 && ok; t++) {
          const int nt = t / m_tiles;
          if (nt == cur_nt) continue;
          slab++;
          cur_nt = nt;
          for (int c = 0; c < nchunks; c++, ci++) {
            const int r = ci % CODE_SLOTS;
            if (!mbar_wait(&cfull[r], (ci / CODE_SLOTS) & 1, p.status, VXG_DEV_TIMEOUT_UNPACK) ||
                (slab > 0 && !mbar_wait(&bfree[c], (slab - 1) & 1, p.status, VXG_DEV_TIMEOUT_UNPACK))) {
              ok = false;
              break;
            }
            unpack_chunk(sCode + r * BP_BYTES, sSlab + c * BU_BYTES, u);
            fence_proxy_async_smem();
            mbar_arrive(&cempty[r]);
            mbar_arrive(&bready[c]);
          }
        }
      } else {
        int it = 0;
        for (int t = t0; t < t1 && ok; t++) {
          for (int c = 0; c < nchunks; c++, it++) {
            const int s = it % stages;
            if (!mbar_wait(&afull[s], (it / stages) & 1, p.status, VXG_DEV_TIMEOUT_UNPACK)) {
              ok = false;
              break;
            }
            unpack_chunk(sCode + s * BP_BYTES, sBu + s * b_stride, u);
            fence_proxy_async_smem();
            mbar_arrive(&unpacked[s]);
          }
        }
      }
    }
  } else {
    // ------------------------------------------------------------------------------------------- epilogue
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(REG_HI) : "memory");
    const int q = warp & 3;    // TMEM lane quarter = the warp's 32 tokens
    const int cs = warp >> 2;  // 64-column half of the tile
    float* stg = sStg + warp * (2 * Q_BYTES / 4);
    const uint64_t negm = pack2(-12582912.0f, -12582912.0f);
    int gi = 0, lt = 0, cur_nt = -1, yloads = 0;
    bool ok = true;
    for (int t = t0; t < t1 && ok; t++, lt++) {
      const int nt = t / m_tiles, mt = t % m_tiles;
      if (nt != cur_nt) {  // this weight tile's scale slice [ng][128] -> shared memory
        named_bar_sync(1, EPI_WARPS * 32);  // nobody still reads the previous slice
        const float4* src = reinterpret_cast<const float4*>(p.swT + (size_t)nt * ng * BN);
        for (int i = threadIdx.x; i < ng * BN / 4; i += EPI_WARPS * 32) reinterpret_cast<float4*>(sSW)[i] = __ldg(src + i);
        named_bar_sync(1, EPI_WARPS * 32);
        cur_nt = nt;
      }
      const int row0 = mt * BM + q * 32, col0 = nt * BN + cs * EPI_COLS;
      const int row = row0 + lane;
      const bool row_ok = row < p.M;
      const float* sxr = p.sx + (size_t)(row_ok ? row : 0) * ng;
      float sx_next = row_ok ? __ldg(sxr) : 0.0f;
      uint64_t acc[EPI_COLS / 2];  // f32x2 pairs: columns (2i, 2i+1) of the warp's slice
#pragma unroll
      for (int i = 0; i < EPI_COLS / 2; i++) acc[i] = 0ull;
      const uint32_t tlane = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(cs * EPI_COLS);
      // Software pipeline over half-slices: the load of the next half is in flight while the current one is
      // consumed; a group's buffer is re-armed once both halves are in registers and released after the re-arm
      // has landed.
      uint32_t R0[HC], R1[HC];
      if (!mbar_wait(&tfull[gi % NBUF], (gi / NBUF) & 1, p.status, VXG_DEV_TIMEOUT_EPILOGUE)) break;
      tc_fence_after();
      tmem_ld_half(tlane + (uint32_t)((gi % NBUF) * BN), R0);
      for (int g = 0; g < ng; g++, gi++) {
        const float sxv = sx_next;
        if (g + 1 < ng && row_ok) sx_next = __ldg(sxr + g + 1);
        const uint32_t tb = tlane + (uint32_t)((gi % NBUF) * BN);
        const uint64_t sx2 = pack2(sxv, sxv);
        const float* swg = sSW + g * BN + cs * EPI_COLS;
        tmem_wait_ld();                 // R0 = first half of the warp's columns of group g
        tmem_ld_half(tb + HC, R1);      // second half in flight
#pragma unroll
        for (int c = 0; c < HC; c += 4) {
          const float4 w4 = *reinterpret_cast<const float4*>(swg + c);
          const uint64_t p01 = mul2(sx2, pack2(w4.x, w4.y));
          const uint64_t p23 = mul2(sx2, pack2(w4.z, w4.w));
          const uint64_t f01 = add2(pack2(__uint_as_float(R0[c]), __uint_as_float(R0[c + 1])), negm);
          const uint64_t f23 = add2(pack2(__uint_as_float(R0[c + 2]), __uint_as_float(R0[c + 3])), negm);
          acc[c / 2] = fma2(f01, p01, acc[c / 2]);
          acc[c / 2 + 1] = fma2(f23, p23, acc[c / 2 + 1]);
        }
        if (p.sums && row_ok)
          for (int c = 0; c < HC; c++)
            if (col0 + c < p.N) p.sums[((size_t)row * p.N + col0 + c) * ng + g] = (int32_t)(R0[c] - MAGIC);
        tmem_wait_ld();                 // R1 landed: the whole group is in registers
        tmem_rearm(tb);                 // re-arm the warp's columns for a later group
        if (g + 1 < ng) {               // next group's first half in flight while this one finishes
          const int bn = (gi + 1) % NBUF;
          if (!mbar_wait(&tfull[bn], ((gi + 1) / NBUF) & 1, p.status, VXG_DEV_TIMEOUT_EPILOGUE)) {
            ok = false;
            break;
          }
          tc_fence_after();
          tmem_ld_half(tlane + (uint32_t)(bn * BN), R0);
        }
#pragma unroll
        for (int c = 0; c < HC; c += 4) {
          const float4 w4 = *reinterpret_cast<const float4*>(swg + HC + c);
          const uint64_t p01 = mul2(sx2, pack2(w4.x, w4.y));
          const uint64_t p23 = mul2(sx2, pack2(w4.z, w4.w));
          const uint64_t f01 = add2(pack2(__uint_as_float(R1[c]), __uint_as_float(R1[c + 1])), negm);
          const uint64_t f23 = add2(pack2(__uint_as_float(R1[c + 2]), __uint_as_float(R1[c + 3])), negm);
          acc[HC / 2 + c / 2] = fma2(f01, p01, acc[HC / 2 + c / 2]);
          acc[HC / 2 + c / 2 + 1] = fma2(f23, p23, acc[HC / 2 + c / 2 + 1]);
        }
        if (p.sums && row_ok)
          for (int c = 0; c < HC; c++)
            if (col0 + HC + c < p.N) p.sums[((size_t)row * p.N + col0 + HC + c) * ng + g] = (int32_t)(R1[c] - MAGIC);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[gi % NBUF]);
      }
      if (!ok) break;
      if constexpr (EP == EP_SILU_Q) {
        // SiLU, then quantize_group over the row's 128 columns of this tile (the 2 warps sharing lane quarter q).
        // Values stay in the accumulator registers throughout.
        float amax = 0.0f;
#pragma unroll
        for (int j = 0; j < EPI_COLS / 2; j++) {
          float v0, v1;
          unpack2(acc[j], v0, v1);
          v0 = silu_fast(v0);
          v1 = silu_fast(v1);
          amax = fmaxf(amax, fmaxf(fabsf(v0), fabsf(v1)));
          acc[j] = pack2(v0, v1);
        }
        constexpr int CSQ = EPI_WARPS / 4;  // warps sharing a lane quarter
        float* ex = sStg + (lt & 1) * (4 * CSQ * 32) + q * (CSQ * 32);  // [q][cs][lane], double-buffered by tile
        ex[cs * 32 + lane] = amax;
        named_bar_sync(2 + q, CSQ * 32);
#pragma unroll
        for (int k = 0; k < CSQ; k++) amax = fmaxf(amax, ex[k * 32 + lane]);
        const float s = quant_scale(amax);
        const float inv = __fdiv_rn(1.0f, s);
        if (row_ok) {
          uint4* dst = reinterpret_cast<uint4*>(p.q + (size_t)row * p.N + col0);
#pragma unroll
          for (int hq = 0; hq < EPI_COLS / 16; hq++) {
            uint32_t wq[4];
#pragma unroll
            for (int j = 0; j < 4; j++) {
              float v0, v1, v2, v3;
              unpack2(acc[hq * 8 + 2 * j], v0, v1);
              unpack2(acc[hq * 8 + 2 * j + 1], v2, v3);
              wq[j] = ((uint32_t)quant_code(v0, inv) & 0xFFu) | (((uint32_t)quant_code(v1, inv) & 0xFFu) << 8) |
                      (((uint32_t)quant_code(v2, inv) & 0xFFu) << 16) | (((uint32_t)quant_code(v3, inv) & 0xFFu) << 24);
            }
            dst[hq] = make_uint4(wq[0], wq[1], wq[2], wq[3]);
          }
          if (cs == 0) p.qs[(size_t)row * (p.N / BN) + nt] = s;
        }
      } else {
        // eight 8-column quarters; with TMA stores they go through two alternating 1 KB staging buffers, otherwise
        // (N % 4 != 0 or an unaligned y) straight to global memory
        float* yrow = p.y + (size_t)(row_ok ? row : 0) * p.N;
#pragma unroll
        for (int k = 0; k < EPI_COLS / 8; k++) {
          float* qb = stg + (k & 1) * (Q_BYTES / 4);
          // row `lane` of a quarter: 32 B = two 16-byte chunks, swapped on rows with bit 2 set (32-byte swizzle)
          float* c0p = qb + lane * 8 + (((lane >> 2) & 1) << 2);
          float* c1p = qb + lane * 8 + ((((lane >> 2) & 1) ^ 1) << 2);
          const int o0 = col0 + 8 * k;
          if constexpr (TMA_STORE) {
            if (lane == 0) bulk_wait_read_1();  // the store issued from this buffer two quarters ago has read it
            __syncwarp();
          }
          float ov[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
          if constexpr (EP == VXG_EP_ADD_SCALED) {  // old values for the residual add
            if constexpr (TMA_STORE) {
              if (lane == 0) {
                mbar_arrive_expect_tx(&ybar[warp], Q_BYTES);
                tma_load_2d(qb, &tmap_y, o0, row0, &ybar[warp]);
              }
              if (!mbar_wait(&ybar[warp], yloads & 1, p.status, VXG_DEV_TIMEOUT_EPILOGUE)) {
                ok = false;
                break;
              }
              yloads++;
              const float4 a = *reinterpret_cast<const float4*>(c0p), b4 = *reinterpret_cast<const float4*>(c1p);
              ov[0] = a.x, ov[1] = a.y, ov[2] = a.z, ov[3] = a.w, ov[4] = b4.x, ov[5] = b4.y, ov[6] = b4.z, ov[7] = b4.w;
            } else if (row_ok) {
              for (int e = 0; e < 8; e++)
                if (o0 + e < p.N) ov[e] = yrow[o0 + e];
            }
          }
          float v[8];
          unpack2(acc[4 * k], v[0], v[1]);
          unpack2(acc[4 * k + 1], v[2], v[3]);
          unpack2(acc[4 * k + 2], v[4], v[5]);
          unpack2(acc[4 * k + 3], v[6], v[7]);
#pragma unroll
          for (int e = 0; e < 8; e++) {
            float a = apply_ep<EP>(p.ep_scale, v[e], ov[e]);
            if (p.bias && o0 + e < p.N) a = __fadd_rn(a, __ldg(p.bias + o0 + e));
            v[e] = a;
          }
          if constexpr (TMA_STORE) {
            *reinterpret_cast<float4*>(c0p) = make_float4(v[0], v[1], v[2], v[3]);
            *reinterpret_cast<float4*>(c1p) = make_float4(v[4], v[5], v[6], v[7]);
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              tma_store_2d(&tmap_y, qb, o0, row0);
              bulk_commit();
            }
          } else if (row_ok) {
            for (int e = 0; e < 8; e++)
              if (o0 + e < p.N) yrow[o0 + e] = v[e];
          }
        }
      }
    }
    if (lane == 0) bulk_wait_all();
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == MMA_WARP) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

template <bool PACKED, bool RES>
const void* kernel_for_ep(int ep, bool tma_store) {
  if (!tma_store) {  // y rows not 16-byte multiples (N % 4 != 0) or unaligned: direct stores
    switch (ep) {
      case VXG_EP_SILU: return (const void*)ternary_gemm_kernel<PACKED, RES, VXG_EP_SILU, false>;
      case VXG_EP_ADD_SCALED: return (const void*)ternary_gemm_kernel<PACKED, RES, VXG_EP_ADD_SCALED, false>;
      case EP_SILU_Q: return (const void*)ternary_gemm_kernel<PACKED, RES, EP_SILU_Q, false>;
      default: return (const void*)ternary_gemm_kernel<PACKED, RES, VXG_EP_STORE, false>;
    }
  }
  switch (ep) {
    case VXG_EP_SILU: return (const void*)ternary_gemm_kernel<PACKED, RES, VXG_EP_SILU, true>;
    case VXG_EP_ADD_SCALED: return (const void*)ternary_gemm_kernel<PACKED, RES, VXG_EP_ADD_SCALED, true>;
    case EP_SILU_Q: return (const void*)ternary_gemm_kernel<PACKED, RES, EP_SILU_Q, false>;
    default: return (const void*)ternary_gemm_kernel<PACKED, RES, VXG_EP_STORE, true>;
  }
}

// One instantiation per (weight format, slab mode, epilogue, store path): each carries only its own epilogue code.
const void* kernel_for(bool packed, bool resident, int ep, bool tma_store) {
  return packed ? (resident ? kernel_for_ep<true, true>(ep, tma_store) : kernel_for_ep<true, false>(ep, tma_store))
                : (resident ? kernel_for_ep<false, true>(ep, tma_store) : kernel_for_ep<false, false>(ep, tma_store));
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

// The setmaxnreg split assumes the kernel was compiled to LAUNCH_REGS registers per thread; with fewer the register
// increase in the epilogue warps could never complete, so refuse to launch instead.
static vxg_status check_launch_regs(const void* kernel) {
  cudaFuncAttributes fa;
  VXG_CUDA(cudaFuncGetAttributes(&fa, kernel));
  if (fa.numRegs < gemm::LAUNCH_REGS) {
    set_error("ternary GEMM compiled to %d registers per thread; its register split needs %d", fa.numRegs,
              gemm::LAUNCH_REGS);
    return VXG_ERR_UNSUPPORTED;
  }
  return VXG_OK;
}

vxg_status vxg::gemm_launch(bool packed, const int8_t* x, const float* sx, const void* w, const float* scales_t,
                            int M, int N, int K, int G, int ep, float ep_scale, const float* bias, float* y,
                            int8_t* q, float* q_scales, int32_t* group_sums, cudaStream_t stream) {
  clear_error();
  VXG_ARG(x && sx && w && scales_t, "NULL pointer");
  VXG_ARG(M > 0 && N > 0 && K > 0 && G > 0, "bad shape M=%d N=%d K=%d G=%d", M, N, K, G);
  VXG_ARG(K % gemm::BK == 0 && G % gemm::BK == 0 && K % G == 0,
          "K (%d) and G (%d) must be multiples of 128 with G | K", K, G);
  if (K / G > gemm::MAX_NG || K > 32768) {
    set_error("K / G = %d groups (max %d) or K = %d (max 32768) not supported", K / G, gemm::MAX_NG, K);
    return VXG_ERR_UNSUPPORTED;
  }
  const bool silu_q = ep == gemm::EP_SILU_Q;
  VXG_ARG(ep == VXG_EP_STORE || ep == VXG_EP_SILU || ep == VXG_EP_ADD_SCALED || silu_q, "bad epilogue %d", ep);
  if (silu_q) {
    VXG_ARG(q && q_scales, "NULL output");
    VXG_ARG(N % gemm::BN == 0 && ((uintptr_t)q & 15) == 0, "int8 output needs N %% 128 == 0 and 16-byte alignment");
  } else {
    VXG_ARG(y != nullptr, "NULL output");
  }
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
  const int tma_store = !silu_q && (N % 4 == 0) && (((uintptr_t)y & 15) == 0);
  if (tma_store) {
    st = make_tmap_2d_f32(&ty, y, (uint64_t)M, (uint64_t)N, (uint64_t)N * 4, 32, 8);
    if (st != VXG_OK) return st;
  } else {
    ty = tx;  // unused
  }
  const bool resident = K <= gemm::KRES;
  const void* kfn = gemm::kernel_for(packed, resident, ep, tma_store != 0);
  if ((st = check_launch_regs(kfn)) != VXG_OK) return st;
  if ((st = smem_attr(kfn, (int)gemm::SMEM_BYTES)) != VXG_OK) return st;
  gemm::Params p;
  p.sx = sx;
  p.codes = packed ? static_cast<const uint8_t*>(w) : nullptr;
  p.swT = scales_t;
  p.bias = bias;
  p.y = y;
  p.q = q;
  p.qs = q_scales;
  p.sums = group_sums;
  p.status = status;
  p.M = M;
  p.N = N;
  p.K = K;
  p.G = G;
  p.ep = ep;
  p.ep_scale = ep_scale;
  p.tma_store = tma_store;
  p.resident = resident;
  const int tiles = ((M + gemm::BM - 1) / gemm::BM) * ((N + gemm::BN - 1) / gemm::BN);
  const int grid = std::min(tiles, sm_count());
  void* args[] = {&tx, &tw, &ty, &p};
  VXG_CUDA(cudaLaunchKernel(kfn, dim3(grid), dim3(gemm::THREADS), args, gemm::SMEM_BYTES, stream));
  note_launch();
  VXG_CUDA(cudaGetLastError());
  return VXG_OK;
}

extern "C" {

vxg_status vxg_gemm_ternary_i8(const int8_t* x, const float* sx, const uint8_t* codes, const float* scales_t, int M,
                               int N, int K, int G, vxg_epilogue ep, float ep_scale, const float* bias, float* y,
                               int32_t* group_sums, void* stream) {
  return gemm_launch(true, x, sx, codes, scales_t, M, N, K, G, (int)ep, ep_scale, bias, y, nullptr, nullptr,
                     group_sums, (cudaStream_t)stream);
}

vxg_status vxg_gemm_ternary_i8w(const int8_t* x, const float* sx, const int8_t* w_rows, const float* scales_t,
                                int M, int N, int K, int G, vxg_epilogue ep, float ep_scale, const float* bias,
                                float* y, int32_t* group_sums, void* stream) {
  return gemm_launch(false, x, sx, w_rows, scales_t, M, N, K, G, (int)ep, ep_scale, bias, y, nullptr, nullptr,
                     group_sums, (cudaStream_t)stream);
}

vxg_status vxg_gemm_ternary_silu_q(const int8_t* x, const float* sx, const uint8_t* codes, const float* scales_t,
                                   int M, int N, int K, int G, int8_t* q, float* q_scales, void* stream) {
  return gemm_launch(true, x, sx, codes, scales_t, M, N, K, G, gemm::EP_SILU_Q, 0.0f, nullptr, nullptr, q, q_scales,
                     nullptr, (cudaStream_t)stream);
}

vxg_status vxg_gemm_ternary_silu_q_w(const int8_t* x, const float* sx, const int8_t* w_rows, const float* scales_t,
                                     int M, int N, int K, int G, int8_t* q, float* q_scales, void* stream) {
  return gemm_launch(false, x, sx, w_rows, scales_t, M, N, K, G, gemm::EP_SILU_Q, 0.0f, nullptr, nullptr, q,
                     q_scales, nullptr, (cudaStream_t)stream);
}

}  // extern "C"
