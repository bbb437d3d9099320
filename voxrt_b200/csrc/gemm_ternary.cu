// Ternary-weight x int8-activation GEMM on the sm_100a tensor cores (tcgen05.mma kind::i8).
//
// Reference semantics (crates/voxrt/src/kernels/mod.rs:166-210, x86.rs:91-154): for every output (t, o)
//   acc = 0; for g in groups: acc = fma(float(S_g), sx[t,g] * sw[o,g], acc);  y = epilogue(old, acc)
// with S_g the exact int32 dot product over the group. The int32 sums come from the tensor cores; the float chain
// runs in the epilogue warps in the reference's group order, so the result is bit-identical.
//
// The chain costs, per output and 128-wide group, one int -> float conversion (exact: |S| < 2^24), one scale
// product and one FMA. The product and the FMA run as packed f32x2 instructions on column pairs (each lane rounded
// exactly like the scalar form), so an epilogue thread issues 64 arithmetic instructions per group for its 32
// columns. Measured on B200, the epilogue is bound less by that arithmetic than by the shared-memory pipe (the
// broadcast loads of the weight scales: 8-byte loads, which sm_100 serves far faster than 16-byte broadcasts) and
// by the output stores, which share that pipe with the TMA traffic:
//   * 16 epilogue warps (four per scheduler) of 32 columns each hide each other's TMEM-load latency;
//   * a group's TMEM buffer goes back to the MMA as soon as its sums are in registers (the first MMA of every
//     group overwrites the buffer, so nothing is cleared or re-armed); four buffers use all 512 columns;
//   * the per-row activation scales of a tile arrive in shared memory by TMA with the tile's first chunk, so the
//     group loop reads them with one shared load per 8 groups and never waits on global memory;
//   * a finished tile is stored straight from registers, one 32-byte vector store per 8 columns;
//   * two MMA-issuing threads on different schedulers take alternate groups, so the tensor pipe is not limited by
//     one thread's issue latency (4 MMAs + 2 commits per 272 clocks of tensor work).
//
// Persistent CTA (one per SM), tile = 128 tokens x 128 weight rows. Each CTA owns a contiguous range of tiles in
// weight-tile-major order, so consecutive tiles share their weight rows:
//   resident mode (K <= 1024): the CTA keeps the tile's whole weight slab (128 rows x K int8, <= 128 KB) in shared
//                memory and only streams activations; the slab is refilled when the weight tile changes, chunk by
//                chunk, so the first tile of a slab overlaps its own fill. 2-bit codes are unpacked in the SM once
//                per slab instead of once per tile.
//   streaming mode (K > 1024): activation and weight chunks stream together through a 4-stage ring.
// Roles (640 threads, five warpgroups):
//   warps 0-15   epilogue: warp w owns TMEM lanes 32*(w%4)..+32 (its tokens) and columns 32*(w/4)..+32 of the tile.
//   warp 16      TMA producer (activation chunks, per-tile activation scales, weight chunks / code chunks).
//   warps 17-18  MMA issuers (TMEM allocation by warp 17): even and odd groups, 4 x (M128 N128 K32) per chunk.
//   warp 19      2-bit weights only: unpacks codes -> int8 {-1,0,+1} (one PRMT per 4 weights) into the UMMA
//                K-major 128-byte-swizzled layout.
// TMEM (512 columns): four 128-column int32 group buffers.
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
constexpr int EPI_WARPS = 16;  // four warpgroups; warp w: TMEM lanes 32*(w%4).., columns 32*(w/4)..
constexpr int EPI_COLS = BN / (EPI_WARPS / 4);  // 32 columns per epilogue warp
constexpr int PIECES = EPI_COLS / 8;            // 8-column output pieces per warp and tile
constexpr int PROD_WARP = 16, MMA_WARP0 = 17, UNPACK_WARP0 = 19, UNPACK_WARPS = 1;
constexpr int THREADS = 20 * 32;  // five whole warpgroups (setmaxnreg acts per warpgroup)
constexpr int LAUNCH_REGS = 96;   // 65536 / 640 rounded down to the allocation unit
constexpr int REG_LO = 64, REG_HI = 104;
static_assert((THREADS - EPI_WARPS * 32) * REG_LO + EPI_WARPS * 32 * REG_HI <= THREADS * LAUNCH_REGS,
              "register split exceeds the launch budget");
constexpr int MAX_NBUF = 4;                     // per-group TMEM buffers (all 512 columns)
constexpr uint32_t TMEM_COLS = 512;
constexpr int KRES = kGemmResidentK;  // largest K whose weight slab stays resident
constexpr int RES_STAGES = 4;   // activation ring, resident mode
constexpr int STR_STAGES = 4;   // activation + weight ring, streaming mode
constexpr int CODE_SLOTS = 2;   // code chunks in flight while a slab fills
constexpr int MAX_NG = 32;      // K / G groups per output (the model has at most 4096 / 128)
constexpr int MAX_CHUNKS = KRES / BK;
constexpr uint32_t A_BYTES = BM * BK;       // 16 KB
constexpr uint32_t BU_BYTES = BN * BK;      // 16 KB int8 weights per chunk
constexpr uint32_t BP_BYTES = BN * BK / 4;  // 4 KB packed codes per chunk
constexpr uint32_t XCH_BYTES = 2 * 4 * 4 * 32 * 4;  // SiLU -> int8 row maxima: [tile parity][quarter][slice][lane]
// resident:  [slab 8 x 16 KB][A ring 4 x 16 KB][code slots 2 x 4 KB][sx 2 x 4 KB][sw 4 KB][bias 512 B][xch 4 KB]
// streaming: [ring 4 x (A 16 KB + B 16 KB)][code slots 4 x 4 KB][sx 2 x 16 KB][sw 16 KB][bias 512 B][xch 4 KB]
constexpr uint32_t RES_MAIN = MAX_CHUNKS * BU_BYTES + RES_STAGES * A_BYTES + CODE_SLOTS * BP_BYTES;
constexpr uint32_t STR_MAIN = STR_STAGES * (A_BYTES + BU_BYTES) + STR_STAGES * BP_BYTES;
constexpr uint32_t RES_NG = KRES / BK, STR_NG = MAX_NG;  // groups per output the layout provides for
constexpr uint32_t BAR_BYTES = 1024;
constexpr uint32_t tail_bytes(uint32_t ng) { return 2 * BM * ng * 4 + ng * BN * 4 + BN * 4 + XCH_BYTES + BAR_BYTES; }
constexpr uint32_t RES_SMEM = RES_MAIN + tail_bytes(RES_NG);
constexpr uint32_t STR_SMEM = STR_MAIN + tail_bytes(STR_NG);
constexpr uint32_t SMEM_BYTES = (RES_SMEM > STR_SMEM ? RES_SMEM : STR_SMEM) + 1024 /*align*/;
static_assert(SMEM_BYTES <= 232448, "shared memory budget");
constexpr uint32_t IDESC = idesc_i8(BM, BN);

constexpr int EP_SILU_Q = kGemmSiluQuant;  // SiLU then per-(row, 128-column) int8 quantisation
constexpr int EP_QK_Q = kGemmQKQuant;      // q|k|v projection: per-head int8 Q and K, f32 V
constexpr int EP_GLU = kGemmGlu;           // pointwise_conv1 with interleaved rows: GLU of each 32-column slice

struct Params {
  const float* sx;       // [M, ng]
  const uint8_t* codes;  // 2-bit mode: [n_tiles][K/128][BN][32]
  const float* swT;      // [n_tiles][ng][BN], one contiguous slice per output tile
  const float* bias;     // [N] or null
  float* y;              // [M, N]
  int8_t* q;             // EP_SILU_Q: [M, N] int8
  float* qs;             // EP_SILU_Q: [M, N/128]
  QkQuant qk;            // EP_QK_Q: the attention's per-head int8 Q (+bias_u, +bias_v) and K
  int32_t* sums;         // [M, N, ng] or null
  int* status;
  int M, N, K, G;
  int ep;
  float ep_scale;
  int sx_tma;  // per-tile activation scales by TMA (ng % 4 == 0, 16-byte aligned); otherwise loaded per group
  // TMA swizzle of the scale tile (rows of ng floats): 16-byte chunk bits [4..] of a byte offset are XORed with its
  // bits [7..] under this mask (1, 3, 7 for rows of 32, 64, 128 bytes; 0: none). One row per lane, so without it
  // the lanes of a quarter-warp read the same banks whenever a row spans a multiple of 128 bytes' worth of banks.
  uint32_t sx_swz;
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
#pragma unroll 4
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

__device__ __forceinline__ float4 lds128(uint32_t a) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(a));
  return v;
}
// 8-byte shared load returning the pair packed for the f32x2 instructions. Every lane of a warp reads the same
// address here (a broadcast), which the 8-byte form serves much faster than the 16-byte one on sm_100.
__device__ __forceinline__ uint64_t lds64(uint32_t a) {
  uint64_t v;
  asm volatile("ld.shared.b64 %0, [%1];" : "=l"(v) : "r"(a));
  return v;
}
__device__ __forceinline__ float lds32(uint32_t a) {
  float v;
  asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(a));
  return v;
}
// One 32-byte store (sm_100 256-bit vector store); the address must be 32-byte aligned.
__device__ __forceinline__ void stg256(float* p, const float (&v)[8]) {
  asm volatile("st.global.v8.f32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(p), "f"(v[0]), "f"(v[1]),
               "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7])
               : "memory");
}

template <int EP>
__device__ __forceinline__ float apply_ep(float es, float a, float old) {
  if constexpr (EP == VXG_EP_SILU) return silu_fast(a);
  if constexpr (EP == VXG_EP_ADD_SCALED) return __fmaf_rn(es, a, old);
  return a;
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
  static constexpr uint32_t NG = RES ? RES_NG : STR_NG;
  static constexpr uint32_t SX = MAIN;                    // [2 tile parities][BM rows][ng] f32
  static constexpr uint32_t SX_BYTES = BM * NG * 4;       // one parity's buffer
  static constexpr uint32_t SW = SX + 2 * SX_BYTES;       // [ng][BN] f32
  static constexpr uint32_t BIAS = SW + NG * BN * 4;      // [BN] f32
  static constexpr uint32_t XCH = BIAS + BN * 4;
  static constexpr uint32_t BARS = XCH + XCH_BYTES;
  static_assert(CODE + (RES ? CODE_SLOTS : STR_STAGES) * BP_BYTES <= MAIN, "layout");
  static_assert(BARS + BAR_BYTES <= SMEM_BYTES - 1024, "layout");
  static_assert(SX % 1024 == 0 && SX_BYTES % 1024 == 0 && SW % 16 == 0 && BIAS % 16 == 0, "alignment (SX: TMA swizzle atom)");
};
// barrier indices inside the BARS block
enum : int {
  B_AFULL = 0,                         // [4] producer -> MMA / unpacker: stage landed (TMA tx)
  B_AEMPTY = 4,                        // [4] MMA commit -> producer
  B_UNPACKED = 8,                      // [4] streaming 2-bit: unpacker -> MMA
  B_CFULL = 12,                        // [2] resident 2-bit fill: code slot landed
  B_CEMPTY = 14,                       // [2] resident 2-bit fill: code slot read
  B_BREADY = 16,                       // [8] resident: slab chunk filled (one phase per slab)
  B_BFREE = B_BREADY + MAX_CHUNKS,     // [8] resident: slab chunk no longer read (both issuers commit)
  B_TFULL = B_BFREE + MAX_CHUNKS,      // [4] MMA commit -> epilogue (per TMEM buffer)
  B_TEMPTY = B_TFULL + MAX_NBUF,       // [4] epilogue warps -> MMA
  B_SXFULL = B_TEMPTY + MAX_NBUF,      // [2] tile's activation scales landed (per tile parity)
  B_SXEMPTY = B_SXFULL + 2,            // [2] epilogue warps done with a tile's scales
  B_SWSYNC = B_SXEMPTY + 2,            // epilogue threads: weight-scale slice swap
  B_QX = B_SWSYNC + 1,                 // [4] SiLU -> int8: the four warps of a lane quarter exchanged row maxima
  B_DRAIN = B_QX + 4,                  // MMA drain (both issuers)
  B_COUNT = B_DRAIN + 1
};
static_assert(B_COUNT * 8 + 16 <= (int)BAR_BYTES, "barrier block");

template <bool PACKED, bool RES, int EP, bool VEC, bool UNR>
__global__ void __launch_bounds__(THREADS, 1)
    ternary_gemm_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_w,
                        const __grid_constant__ CUtensorMap tmap_sx, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  using L = Smem<RES>;
  constexpr bool res = RES;
  constexpr int stages = L::STAGES;
  constexpr int NBUF = MAX_NBUF;  // per-group TMEM buffers, 128 columns each
  uint8_t* const sSlab = smem + L::SLAB;
  uint8_t* const sA = smem + L::A;
  uint8_t* const sBu = smem + L::B;
  uint8_t* const sCode = smem + L::CODE;
  constexpr uint32_t a_stride = L::A_STRIDE, b_stride = L::A_STRIDE;
  float* const sSW = reinterpret_cast<float*>(smem + L::SW);
  float* const sBias = reinterpret_cast<float*>(smem + L::BIAS);
  float* const sXch = reinterpret_cast<float*>(smem + L::XCH);
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
  uint64_t* const sxfull = bars + B_SXFULL;
  uint64_t* const sxempty = bars + B_SXEMPTY;
  uint64_t* const swsync = bars + B_SWSYNC;
  uint64_t* const qx = bars + B_QX;
  uint64_t* const drain = bars + B_DRAIN;
  uint32_t* const tmem_holder = reinterpret_cast<uint32_t*>(bars + B_COUNT);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < 4; s++) {
      mbar_init(&afull[s], 1);
      mbar_init(&aempty[s], 1);
      mbar_init(&unpacked[s], UNPACK_WARPS * 32);
      mbar_init(&qx[s], 4 * 32);
    }
    for (int r = 0; r < CODE_SLOTS; r++) {
      mbar_init(&cfull[r], 1);
      mbar_init(&cempty[r], UNPACK_WARPS * 32);
    }
    for (int c = 0; c < MAX_CHUNKS; c++) {
      mbar_init(&bready[c], PACKED ? UNPACK_WARPS * 32 : 1);
      mbar_init(&bfree[c], 2);
    }
    for (int b = 0; b < MAX_NBUF; b++) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], EPI_WARPS);
    }
    for (int k = 0; k < 2; k++) {
      mbar_init(&sxfull[k], 1);
      mbar_init(&sxempty[k], EPI_WARPS);
    }
    mbar_init(swsync, EPI_WARPS * 32);
    mbar_init(drain, 2);
    fence_mbar_init();
  }
  if (warp == PROD_WARP && lane == 0) {
    prefetch_tmap(&tmap_x);
    if (!PACKED) prefetch_tmap(&tmap_w);
    if (p.sx_tma) prefetch_tmap(&tmap_sx);
  }
  if (warp == MMA_WARP0) {
    tmem_alloc(tmem_holder, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  const int ng = p.K / p.G, cpg = p.G / BK, nchunks = p.K / BK;
  const int m_tiles = (p.M + BM - 1) / BM, n_tiles = (p.N + BN - 1) / BN;
  int t0, t1;
  tile_range(m_tiles * n_tiles, t0, t1);

  if (warp >= EPI_WARPS) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(REG_LO) : "memory");
    if (warp == PROD_WARP) {
      // ------------------------------------------------------------------------------------------ producer
      if (elect_one()) {
        int it = 0, ci = 0, slab = -1, cur_nt = -1, lt = 0;
        bool ok = true;
        for (int t = t0; t < t1 && ok; t++, lt++) {
          const int nt = t / m_tiles, mt = t % m_tiles;
          const bool fill = res && nt != cur_nt;
          if (fill) {
            slab++;
            cur_nt = nt;
          }
          if (p.sx_tma) {  // the tile's activation scales, once the tile two back has released the buffer
            const int par = lt & 1;
            if (lt >= 2 && !mbar_wait(&sxempty[par], ((lt >> 1) - 1) & 1, p.status, VXG_DEV_TIMEOUT_PRODUCER)) break;
            mbar_arrive_expect_tx(&sxfull[par], (uint32_t)(BM * ng * 4));
            tma_load_2d(smem + L::SX + par * L::SX_BYTES, &tmap_sx, 0, mt * BM, &sxfull[par]);
          }
          for (int c = 0; c < nchunks; c++, it++) {
            if (fill) {
              if (PACKED) {  // code chunk c of the new slab -> a code slot (unpacked into the slab by warp 19)
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
        if (p.sx_tma)
          for (int k = lt > 2 ? lt - 2 : 0; k < lt; k++)
            mbar_wait(&sxfull[k & 1], (k >> 1) & 1, p.status, VXG_DEV_TIMEOUT_DRAIN);
        if (res && PACKED)
          for (int k = ci > CODE_SLOTS ? ci - CODE_SLOTS : 0; k < ci; k++)
            mbar_wait(&cfull[k % CODE_SLOTS], (k / CODE_SLOTS) & 1, p.status, VXG_DEV_TIMEOUT_DRAIN);
        if (res && !PACKED && slab >= 0)
          for (int c = 0; c < nchunks; c++) mbar_wait(&bready[c], slab & 1, p.status, VXG_DEV_TIMEOUT_DRAIN);
      }
    } else if (warp == MMA_WARP0 || warp == MMA_WARP0 + 1) {
      // -------------------------------------------------------------------------------------- MMA issuers
      const int me = warp - MMA_WARP0;  // takes the groups gi with gi % 2 == me
      // Two issuers only when a group is one chunk: each then waits on a ring stage at most one phase ahead of the
      // barrier (its group's TMEM buffer is free only once the group four back was consumed). A group of several
      // chunks would let the second issuer wait two phases ahead, where a parity wait cannot tell the phases apart,
      // so then issuer 0 takes every group (issuer 1 still commits the slab releases the barriers count).
      const bool two = cpg == 1;
      if (elect_one()) {
        int gi = 0, slab = -1, cur_nt = -1;
        bool ok = true;
        for (int t = t0; t < t1 && ok; t++) {
          const int nt = t / m_tiles;
          if (nt != cur_nt) {
            slab++;
            cur_nt = nt;
          }
          const bool last_of_slab = res && (t + 1 == t1 || (t + 1) / m_tiles != nt);
          for (int g = 0; g < ng && ok; g++, gi++) {
            if (two ? (gi & 1) != me : me != 0) continue;
            const int b = gi % NBUF;
            if (!mbar_wait(&tempty[b], ((gi / NBUF) & 1) ^ 1, p.status, VXG_DEV_TIMEOUT_MMA)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t d = tmem_base + (uint32_t)(b * BN);
            for (int cc = 0; cc < cpg; cc++) {
              const int it = gi * cpg + cc, c = g * cpg + cc, s = it % stages;
              uint64_t* ready = (!res && PACKED) ? &unpacked[s] : &afull[s];
              if (!mbar_wait(ready, (it / stages) & 1, p.status, VXG_DEV_TIMEOUT_MMA) ||
                  (res && !mbar_wait(&bready[c], slab & 1, p.status, VXG_DEV_TIMEOUT_MMA))) {
                ok = false;
                break;
              }
              const uint64_t ad = umma_desc_sw128(smem_u32(sA + s * a_stride));
              const uint64_t bd = umma_desc_sw128(smem_u32(res ? sSlab + c * BU_BYTES : sBu + s * b_stride));
#pragma unroll
              for (int k = 0; k < BK / 32; k++)  // the group's first MMA overwrites the buffer
                mma_i8(d, ad + (uint64_t)(2 * k), bd + (uint64_t)(2 * k), IDESC, (cc | k) != 0 ? 1u : 0u);
              mma_commit(&aempty[s]);
            }
            if (ok) mma_commit(&tfull[b]);
          }
          // both issuers release the slab's chunks after their last MMAs on it (the barriers count two)
          if (ok && last_of_slab)
            for (int c = 0; c < nchunks; c++) mma_commit(&bfree[c]);
        }
        // wait for every MMA issued so far (by both threads) before TMEM is released
        mma_commit(drain);
        mbar_wait(drain, 0, p.status, VXG_DEV_TIMEOUT_DRAIN);
      }
    } else if (PACKED && warp == UNPACK_WARP0) {
      // ------------------------------------------------------------------------------- unpacker (2-bit mode)
      const int u = lane;
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
    const int cs = warp >> 2;  // 32-column slice of the tile
    const bool leader = lane == 0;
    const uint32_t tq = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(cs * EPI_COLS);
    const uint32_t swa = smem_u32(sSW) + (uint32_t)(cs * EPI_COLS * 4);
    const uint32_t sxbase0 = smem_u32(smem + L::SX);                // parity 0 buffer (1024-byte aligned)
    const uint32_t sxrow = (uint32_t)((q * 32 + lane) * ng * 4);     // this row's byte offset in a buffer
    const uint32_t swz = p.sx_swz;
    auto sx_at = [&](uint32_t base, uint32_t off) { return base + (off ^ (((off >> 7) & swz) << 4)); };
    const uint32_t tfull_a = smem_u32(tfull), tempty_a = smem_u32(tempty);
    const uint32_t bias_a = smem_u32(sBias) + (uint32_t)(cs * EPI_COLS * 4);
    const bool has_bias = p.bias != nullptr;

    // TMEM buffer of the next group: tb (address), bo (its barriers' byte offset), tph (phase), bi (index)
    uint32_t tb = tq, bo = 0, tph = 0;
    int bi = 0, lt = 0, cur_nt = -1, nsw = 0;
    int qxn = 0;  // quantiser exchanges done (their parity selects the buffer and the barrier phase)
    int cur_row0 = 0, cur_col0 = 0;  // the current tile's first row of this quarter and first column of the slice
    bool ok = true;
    // One group: wait for its sums, move them to registers, hand the buffer back to the MMA, and advance the FMA
    // chain of the warp's 32 columns by one step. The chain runs on packed pairs (f32x2: two columns per
    // instruction, each lane rounded exactly like the scalar fma / mul); the int32 sums convert exactly (|S| < 2^24).
    // `swg` is the shared address of the group's weight scales for this slice, `sxv` the row's activation scale.
    auto group = [&](uint64_t (&acc)[EPI_COLS / 2], uint32_t swg, float sxv, int g) -> bool {
      if (!mbar_wait_a(tfull_a + bo, tph, p.status, VXG_DEV_TIMEOUT_EPILOGUE)) return false;
      tc_fence_after();
      uint32_t R[EPI_COLS];
      tmem_ld32(tb, R);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (leader) mbar_arrive_a(tempty_a + bo);  // the sums are in registers: the MMA may refill the buffer
      if (bi == NBUF - 1) {
        bi = 0, tb = tq, bo = 0, tph ^= 1u;
      } else {
        bi++, tb += BN, bo += 8;
      }
      const uint64_t sx2 = pk2(sxv, sxv);
#pragma unroll
      for (int c = 0; c < EPI_COLS; c += 2) {
        const uint64_t pr = fmul2(sx2, lds64(swg + (uint32_t)(c * 4)));
        acc[c / 2] = ffma2(pk2(__int2float_rn((int)R[c]), __int2float_rn((int)R[c + 1])), pr, acc[c / 2]);
      }
      if constexpr (!UNR) {  // debug output of the integer group sums (generic path only)
        if (p.sums) {
          const int row = cur_row0 + lane;
          if (row < p.M)
            for (int c = 0; c < EPI_COLS; c++)
              if (cur_col0 + c < p.N) p.sums[((size_t)row * p.N + cur_col0 + c) * ng + g] = (int32_t)R[c];
        }
      }
      return true;
    };

    for (int t = t0; t < t1 && ok; t++, lt++) {
      const int nt = t / m_tiles, mt = t % m_tiles;
      if (nt != cur_nt) {  // this weight tile's scale slice [ng][128] (and bias) -> shared memory
        mbar_arrive(swsync);  // nobody still reads the previous slice
        if (!mbar_wait(swsync, (nsw++) & 1, p.status, VXG_DEV_TIMEOUT_EPILOGUE)) break;
        const float4* src = reinterpret_cast<const float4*>(p.swT + (size_t)nt * ng * BN);
        for (int i = threadIdx.x; i < ng * BN / 4; i += EPI_WARPS * 32) reinterpret_cast<float4*>(sSW)[i] = __ldg(src + i);
        if (has_bias && threadIdx.x < BN) {
          const int o = nt * BN + threadIdx.x;
          sBias[threadIdx.x] = o < p.N ? __ldg(p.bias + o) : 0.0f;
        }
        mbar_arrive(swsync);
        if (!mbar_wait(swsync, (nsw++) & 1, p.status, VXG_DEV_TIMEOUT_EPILOGUE)) break;
        cur_nt = nt;
      }
      cur_row0 = mt * BM + q * 32;
      cur_col0 = nt * BN + cs * EPI_COLS;
      const int row = cur_row0 + lane;
      const bool row_ok = row < p.M;
      const int par = lt & 1;
      const uint32_t sxbase = sxbase0 + (uint32_t)(par * L::SX_BYTES);
      if (p.sx_tma && !mbar_wait(&sxfull[par], (lt >> 1) & 1, p.status, VXG_DEV_TIMEOUT_EPILOGUE)) break;
      uint64_t acc2[EPI_COLS / 2];
#pragma unroll
      for (int i = 0; i < EPI_COLS / 2; i++) acc2[i] = 0ull;  // +0.0f in both halves
      if constexpr (UNR) {
        // ng % 8 == 0 and the scales came by TMA: blocks of 8 groups, the row's 8 activation scales in registers
        // and every shared offset a constant.
        for (int g8 = 0; g8 < ng && ok; g8 += 8) {
          const uint32_t swb = swa + (uint32_t)(g8 * BN * 4), sxo = sxrow + (uint32_t)(g8 * 4);
          const float4 sa = lds128(sx_at(sxbase, sxo)), sb = lds128(sx_at(sxbase, sxo + 16u));
          const float sxr[8] = {sa.x, sa.y, sa.z, sa.w, sb.x, sb.y, sb.z, sb.w};
#pragma unroll
          for (int gg = 0; gg < 8; gg++) {
            if (!group(acc2, swb + (uint32_t)(gg * BN * 4), sxr[gg], g8 + gg)) {
              ok = false;
              break;
            }
          }
        }
      } else {
        const float* sxg = p.sx + (size_t)(row_ok ? row : 0) * ng;
        for (int g = 0; g < ng && ok; g++) {
          const float sxv = p.sx_tma ? lds32(sx_at(sxbase, sxrow + (uint32_t)(g * 4))) : (row_ok ? __ldg(sxg + g) : 0.0f);
          if (!group(acc2, swa + (uint32_t)(g * BN * 4), sxv, g)) {
            ok = false;
            break;
          }
        }
      }
      if (!ok) break;
      if (p.sx_tma) {  // the scales of this tile are no longer read
        __syncwarp();
        if (leader) mbar_arrive(&sxempty[par]);
      }
      float acc[EPI_COLS];
#pragma unroll
      for (int i = 0; i < EPI_COLS / 2; i++) upk2(acc2[i], acc[2 * i], acc[2 * i + 1]);
      // quantize_group over the row's 128 columns of this tile (the 4 warps sharing lane quarter q exchange their
      // maxima through shared memory), codes to dst (32 bytes of this warp's columns) and the scale to *sdst (warp
      // cs = 0). Values stay in registers throughout.
      auto quant_row = [&](float (&val)[EPI_COLS], float amax, int8_t* dst, float* sdst) -> bool {
        float* ex = sXch + (qxn & 1) * (4 * 4 * 32) + q * (4 * 32);  // [exchange parity][q][cs][lane]
        ex[cs * 32 + lane] = amax;
        mbar_arrive(&qx[q]);
        if (!mbar_wait(&qx[q], (uint32_t)(qxn & 1), p.status, VXG_DEV_TIMEOUT_EPILOGUE)) return false;
        qxn++;
#pragma unroll
        for (int k = 0; k < 4; k++) amax = fmaxf(amax, ex[k * 32 + lane]);
        const float s = quant_scale(amax);
        const float inv = __fdiv_rn(1.0f, s);
        uint32_t wq[EPI_COLS / 4];
        // amax == 0 or a normal-range amax: inv is finite and |v * inv| <= 127 (1 + 2^-23), so the shifter's
        // low byte is already the clamped code (two's complement); otherwise the general quant_code.
        if (__all_sync(0xffffffffu, amax == 0.0f || amax >= 2e-36f)) {
#pragma unroll
          for (int j = 0; j < EPI_COLS / 4; j++) {
            const uint32_t c0 = __float_as_uint(__fadd_rn(__fmul_rn(val[4 * j + 0], inv), 12582912.0f));
            const uint32_t c1 = __float_as_uint(__fadd_rn(__fmul_rn(val[4 * j + 1], inv), 12582912.0f));
            const uint32_t c2 = __float_as_uint(__fadd_rn(__fmul_rn(val[4 * j + 2], inv), 12582912.0f));
            const uint32_t c3 = __float_as_uint(__fadd_rn(__fmul_rn(val[4 * j + 3], inv), 12582912.0f));
            wq[j] = __byte_perm(__byte_perm(c0, c1, 0x0040), __byte_perm(c2, c3, 0x0040), 0x5410);
          }
        } else {
#pragma unroll
          for (int j = 0; j < EPI_COLS / 4; j++)
            wq[j] = ((uint32_t)quant_code(val[4 * j], inv) & 0xFFu) |
                    (((uint32_t)quant_code(val[4 * j + 1], inv) & 0xFFu) << 8) |
                    (((uint32_t)quant_code(val[4 * j + 2], inv) & 0xFFu) << 16) |
                    (((uint32_t)quant_code(val[4 * j + 3], inv) & 0xFFu) << 24);
        }
        if (row_ok) {
          uint4* d4 = reinterpret_cast<uint4*>(dst);
          d4[0] = make_uint4(wq[0], wq[1], wq[2], wq[3]);
          d4[1] = make_uint4(wq[4], wq[5], wq[6], wq[7]);
          if (cs == 0) *sdst = s;
        }
        return true;
      };
      if constexpr (EP == EP_SILU_Q) {
        // SiLU, then the quantiser. When every argument of the warp is in the range where silu_fast takes no branch
        // (checked on min / max reductions, NaN caught by max.NaN), the branch-free form runs; otherwise the
        // general one.
        float mn = fabsf(acc[0]), mx = mn, lo = acc[0];
#pragma unroll
        for (int j = 1; j < EPI_COLS; j++) {
          mn = fminf(mn, fabsf(acc[j]));
          mx = max_nan(mx, fabsf(acc[j]));
          lo = fminf(lo, acc[j]);
        }
        const bool inrange = mn > 1e-30f && mx < 1e30f && lo > -85.0f;
        float amax = 0.0f;
        if (__all_sync(0xffffffffu, inrange)) {
#pragma unroll
          for (int j = 0; j < EPI_COLS; j += 2) {
            silu2_inrange(acc[j], acc[j + 1]);
            amax = fmaxf(amax, fmaxf(fabsf(acc[j]), fabsf(acc[j + 1])));
          }
        } else {  // fully unrolled too: a runtime index would move acc to local memory
#pragma unroll
          for (int j = 0; j < EPI_COLS; j++) {
            acc[j] = silu_fast(acc[j]);
            amax = fmaxf(amax, fabsf(acc[j]));
          }
        }
        if (!quant_row(acc, amax, p.q + (size_t)row * p.N + cur_col0, p.qs + (size_t)row * (p.N / BN) + nt)) break;
      } else if constexpr (EP == EP_GLU) {
        // pointwise_conv1 whose weight rows were interleaved at load time: the warp's 32 columns are 16 GLU value
        // channels (64 nt + 16 cs + j) followed by their 16 gates, so each thread holds a and b of 16 channels of
        // its row: glu_row (tensor.rs:936-940) a * sigmoid_fast(b), stored to y [M, N / 2]. The branch-free sigmoid
        // runs when every gate of the warp is > -85 (identical results there).
        bool fast = true;
#pragma unroll
        for (int j = 0; j < EPI_COLS / 2; j++) fast = fast && acc[EPI_COLS / 2 + j] > -85.0f;
        float o[EPI_COLS / 2];
        if (__all_sync(0xffffffffu, fast)) {
#pragma unroll
          for (int j = 0; j < EPI_COLS / 2; j++) o[j] = __fmul_rn(acc[j], sigmoid_inrange(acc[EPI_COLS / 2 + j]));
        } else {
#pragma unroll
          for (int j = 0; j < EPI_COLS / 2; j++) o[j] = __fmul_rn(acc[j], sigmoid_fast(acc[EPI_COLS / 2 + j]));
        }
        if (row_ok) {
          float* yr = p.y + (size_t)row * (p.N / 2) + nt * (BN / 2) + cs * (EPI_COLS / 2);
          const float o0[8] = {o[0], o[1], o[2], o[3], o[4], o[5], o[6], o[7]};
          const float o1[8] = {o[8], o[9], o[10], o[11], o[12], o[13], o[14], o[15]};
          stg256(yr, o0);
          stg256(yr + 8, o1);
        }
      } else if (EP == EP_QK_Q && nt < 2 * p.qk.heads) {
        // q|k|v projection, q or k head: the attention's operands straight from the accumulators (encoder.rs:
        // 349-377): Qu = quant(q + bias_u), Qv = quant(q + bias_v), K = quant(k), one group per (row, head), laid
        // out [head][row][128] with scales [head][row].
        const int hh = nt < p.qk.heads ? nt : nt - p.qk.heads;
        const size_t o = ((size_t)hh * p.M + (row_ok ? row : 0)) * BN + cs * EPI_COLS;
        const size_t so = (size_t)hh * p.M + (row_ok ? row : 0);
        if (nt < p.qk.heads) {
          bool good = true;
#pragma unroll 1
          for (int pass = 0; pass < 2 && good; pass++) {
            const float4* bias4 = reinterpret_cast<const float4*>((pass == 0 ? p.qk.bu : p.qk.bv) + hh * BN +
                                                                  cs * EPI_COLS);
            float a[EPI_COLS];
            float amax = 0.0f;
#pragma unroll
            for (int j = 0; j < EPI_COLS / 4; j++) {
              const float4 b4 = __ldg(bias4 + j);
              a[4 * j + 0] = __fadd_rn(acc[4 * j + 0], b4.x);
              a[4 * j + 1] = __fadd_rn(acc[4 * j + 1], b4.y);
              a[4 * j + 2] = __fadd_rn(acc[4 * j + 2], b4.z);
              a[4 * j + 3] = __fadd_rn(acc[4 * j + 3], b4.w);
            }
#pragma unroll
            for (int j = 0; j < EPI_COLS; j++) amax = fmaxf(amax, fabsf(a[j]));
            good = quant_row(a, amax, (pass == 0 ? p.qk.qu : p.qk.qv) + o, (pass == 0 ? p.qk.squ : p.qk.sqv) + so);
          }
          if (!good) break;
        } else {
          float amax = 0.0f;
#pragma unroll
          for (int j = 0; j < EPI_COLS; j++) amax = fmaxf(amax, fabsf(acc[j]));
          if (!quant_row(acc, amax, p.qk.kh + o, p.qk.sk + so)) break;
        }
      } else {
        // y = ep(acc) (+ bias), stored straight from registers: each thread writes its row's 32 columns (one
        // 128-byte line per thread in the vector form).
        const int ncol = ::max(0, ::min(EPI_COLS, p.N - cur_col0));
        float* yrow = p.y + (size_t)(row_ok ? row : 0) * p.N + cur_col0;
#pragma unroll
        for (int k = 0; k < PIECES; k++) {
          float v[8];
#pragma unroll
          for (int e = 0; e < 8; e++) v[e] = acc[8 * k + e];
          if constexpr (EP == VXG_EP_ADD_SCALED) {
#pragma unroll
            for (int e = 0; e < 8; e++) {
              const float old = (row_ok && 8 * k + e < ncol) ? yrow[8 * k + e] : 0.0f;
              v[e] = __fmaf_rn(p.ep_scale, v[e], old);
            }
          } else if constexpr (EP == VXG_EP_SILU) {
#pragma unroll
            for (int e = 0; e < 8; e++) v[e] = silu_fast(v[e]);
          }
          if (has_bias) {
            const float4 b0 = lds128(bias_a + (uint32_t)(32 * k)), b1 = lds128(bias_a + (uint32_t)(32 * k + 16));
            v[0] = __fadd_rn(v[0], b0.x), v[1] = __fadd_rn(v[1], b0.y), v[2] = __fadd_rn(v[2], b0.z);
            v[3] = __fadd_rn(v[3], b0.w), v[4] = __fadd_rn(v[4], b1.x), v[5] = __fadd_rn(v[5], b1.y);
            v[6] = __fadd_rn(v[6], b1.z), v[7] = __fadd_rn(v[7], b1.w);
          }
          if (!row_ok || 8 * k >= ncol) continue;
          if constexpr (VEC) {
            stg256(yrow + 8 * k, v);  // N % 8 == 0: all 8 columns are in range
          } else {
#pragma unroll
            for (int e = 0; e < 8; e++)
              if (8 * k + e < ncol) yrow[8 * k + e] = v[e];
          }
        }
      }
    }
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == MMA_WARP0) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

template <bool PACKED, bool RES>
const void* kernel_for_ep(int ep, bool vec, bool unr) {
  if (!unr) {  // generic group loop (ng % 8 != 0, scales not by TMA, or the group sums wanted): scalar stores
    switch (ep) {
      case VXG_EP_SILU: return (const void*)ternary_gemm_kernel<PACKED, RES, VXG_EP_SILU, false, false>;
      case VXG_EP_ADD_SCALED: return (const void*)ternary_gemm_kernel<PACKED, RES, VXG_EP_ADD_SCALED, false, false>;
      case EP_SILU_Q: return (const void*)ternary_gemm_kernel<PACKED, RES, EP_SILU_Q, false, false>;
      case EP_QK_Q: return (const void*)ternary_gemm_kernel<PACKED, RES, EP_QK_Q, false, false>;
      case EP_GLU: return nullptr;  // needs the unrolled group loop and vector stores
      default: return (const void*)ternary_gemm_kernel<PACKED, RES, VXG_EP_STORE, false, false>;
    }
  }
  if (!vec) {  // y rows not 32-byte multiples (N % 8 != 0) or an unaligned y: scalar stores
    switch (ep) {
      case VXG_EP_SILU: return (const void*)ternary_gemm_kernel<PACKED, RES, VXG_EP_SILU, false, true>;
      case VXG_EP_ADD_SCALED: return (const void*)ternary_gemm_kernel<PACKED, RES, VXG_EP_ADD_SCALED, false, true>;
      case EP_SILU_Q: return (const void*)ternary_gemm_kernel<PACKED, RES, EP_SILU_Q, false, true>;
      case EP_QK_Q: return (const void*)ternary_gemm_kernel<PACKED, RES, EP_QK_Q, false, true>;
      case EP_GLU: return nullptr;
      default: return (const void*)ternary_gemm_kernel<PACKED, RES, VXG_EP_STORE, false, true>;
    }
  }
  switch (ep) {
    case EP_GLU: return (const void*)ternary_gemm_kernel<PACKED, RES, EP_GLU, true, true>;
    case VXG_EP_SILU: return (const void*)ternary_gemm_kernel<PACKED, RES, VXG_EP_SILU, true, true>;
    case VXG_EP_ADD_SCALED: return (const void*)ternary_gemm_kernel<PACKED, RES, VXG_EP_ADD_SCALED, true, true>;
    case EP_SILU_Q: return (const void*)ternary_gemm_kernel<PACKED, RES, EP_SILU_Q, false, true>;
    case EP_QK_Q: return (const void*)ternary_gemm_kernel<PACKED, RES, EP_QK_Q, true, true>;
    default: return (const void*)ternary_gemm_kernel<PACKED, RES, VXG_EP_STORE, true, true>;
  }
}

// One instantiation per (weight format, slab mode, epilogue, store width, group loop): each carries only its own
// epilogue code.
const void* kernel_for(bool packed, bool resident, int ep, bool vec, bool unr) {
  return packed ? (resident ? kernel_for_ep<true, true>(ep, vec, unr) : kernel_for_ep<true, false>(ep, vec, unr))
                : (resident ? kernel_for_ep<false, true>(ep, vec, unr) : kernel_for_ep<false, false>(ep, vec, unr));
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
                            int8_t* q, float* q_scales, int32_t* group_sums, cudaStream_t stream, const QkQuant* qk) {
  clear_error();
  VXG_ARG(x && sx && w && scales_t, "NULL pointer");
  VXG_ARG(M > 0 && N > 0 && K > 0 && G > 0, "bad shape M=%d N=%d K=%d G=%d", M, N, K, G);
  VXG_ARG(K % gemm::BK == 0 && G % gemm::BK == 0 && K % G == 0,
          "K (%d) and G (%d) must be multiples of 128 with G | K", K, G);
  if (K / G > gemm::MAX_NG || K > 32768 || G > 16384) {  // |group sum| <= 128 * G must stay below 2^22
    set_error("K / G = %d groups (max %d), K = %d (max 32768) or G = %d (max 16384) not supported", K / G,
              gemm::MAX_NG, K, G);
    return VXG_ERR_UNSUPPORTED;
  }
  const bool silu_q = ep == gemm::EP_SILU_Q;
  const bool qk_q = ep == gemm::EP_QK_Q;
  const bool glu = ep == gemm::EP_GLU;
  VXG_ARG(ep == VXG_EP_STORE || ep == VXG_EP_SILU || ep == VXG_EP_ADD_SCALED || silu_q || qk_q || glu,
          "bad epilogue %d", ep);
  if (glu)
    VXG_ARG(N % gemm::BN == 0 && bias == nullptr && group_sums == nullptr && y && ((uintptr_t)y & 31) == 0,
            "GLU epilogue: N %% 128 == 0, 32-byte aligned y [M, N/2], no bias or group sums");
  if (qk_q) {
    VXG_ARG(qk && qk->bu && qk->bv && qk->qu && qk->qv && qk->kh && qk->squ && qk->sqv && qk->sk && y,
            "q|k quantising epilogue: NULL buffer");
    VXG_ARG(qk->heads > 0 && N == 3 * qk->heads * gemm::BN && bias == nullptr && group_sums == nullptr,
            "q|k quantising epilogue: N must be 3 x heads x 128, no bias or group sums");
    VXG_ARG((((uintptr_t)qk->qu | (uintptr_t)qk->qv | (uintptr_t)qk->kh | (uintptr_t)qk->bu | (uintptr_t)qk->bv) &
             15) == 0,
            "q|k quantising epilogue: 16-byte aligned buffers required");
  }
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
  CUtensorMap tx, tw, tsx;
  vxg_status st = make_tmap_2d_u8(&tx, x, (uint64_t)M, (uint64_t)K, (uint64_t)K, gemm::BM, gemm::BK);
  if (st != VXG_OK) return st;
  if (!packed) {
    st = make_tmap_2d_u8(&tw, w, (uint64_t)vxg_ternary_out_pad(N), (uint64_t)K, (uint64_t)K, gemm::BN, gemm::BK);
    if (st != VXG_OK) return st;
  } else {
    tw = tx;  // unused
  }
  const int ng = K / G;
  const int sx_tma = (ng % 4 == 0) && (((uintptr_t)sx & 15) == 0);
  // rows of 32, 64 or 128 bytes take the matching TMA swizzle (the reads apply the same XOR); others none
  const uint32_t sx_swz = !sx_tma ? 0u : ng == 8 ? 1u : ng == 16 ? 3u : ng == 32 ? 7u : 0u;
  if (sx_tma) {
    st = make_tmap_2d_f32(&tsx, sx, (uint64_t)M, (uint64_t)ng, (uint64_t)ng * 4, gemm::BM, (uint32_t)ng, sx_swz != 0);
    if (st != VXG_OK) return st;
  } else {
    tsx = tx;  // unused
  }
  const bool vec = !silu_q && (N % 8 == 0) && (((uintptr_t)y & 31) == 0);
  const bool resident = K <= gemm::KRES;
  const bool unr = sx_tma && ng % 8 == 0 && group_sums == nullptr;
  const void* kfn = gemm::kernel_for(packed, resident, ep, vec, unr);
  if (!kfn) {
    set_error("epilogue %d needs K / G a multiple of 8 and 16-byte aligned activation scales", ep);
    return VXG_ERR_UNSUPPORTED;
  }
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
  p.sx_tma = sx_tma;
  p.sx_swz = sx_swz;
  if (qk_q) p.qk = *qk;
  const int tiles = ((M + gemm::BM - 1) / gemm::BM) * ((N + gemm::BN - 1) / gemm::BN);
  const int grid = std::min(tiles, sm_count());
  void* args[] = {&tx, &tw, &tsx, &p};
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

vxg_status vxg_gemm_ternary_qkv_quant(const int8_t* x, const float* sx, const uint8_t* codes, const float* scales_t,
                                      int M, int heads, int K, int G, const float* bias_u, const float* bias_v,
                                      int8_t* qu, int8_t* qv, int8_t* kh, float* squ, float* sqv, float* sk, float* y,
                                      void* stream) {
  clear_error();
  VXG_ARG(heads > 0 && heads <= 64, "heads = %d out of range", heads);
  QkQuant qk;
  qk.bu = bias_u;
  qk.bv = bias_v;
  qk.qu = qu;
  qk.qv = qv;
  qk.kh = kh;
  qk.squ = squ;
  qk.sqv = sqv;
  qk.sk = sk;
  qk.heads = heads;
  return gemm_launch(true, x, sx, codes, scales_t, M, 3 * heads * gemm::BN, K, G, gemm::EP_QK_Q, 0.0f, nullptr, y,
                     nullptr, nullptr, nullptr, (cudaStream_t)stream, &qk);
}

int vxg_glu_source_row(int r, int n) {
  if (n <= 0 || n % 128 != 0 || r < 0 || r >= n) return -1;
  return glu_interleave_row(r, n / 2);
}

vxg_status vxg_gemm_ternary_glu(const int8_t* x, const float* sx, const uint8_t* codes, const float* scales_t, int M,
                                int N, int K, int G, float* y, void* stream) {
  clear_error();
  VXG_ARG(N > 0 && N % 128 == 0, "GLU projection width %d must be a multiple of 128", N);
  return gemm_launch(true, x, sx, codes, scales_t, M, N, K, G, gemm::EP_GLU, 0.0f, nullptr, y, nullptr, nullptr,
                     nullptr, (cudaStream_t)stream);
}

}  // extern "C"
