// Ternary-weight x int8-activation GEMM on the sm_100a tensor cores (tcgen05.mma kind::i8).
//
// Reference semantics (crates/voxrt/src/kernels/mod.rs:166-210, x86.rs:91-154): for every output (t, o)
//   acc = 0; for g in groups: acc = fma(float(S_g), sx[t,g] * sw[o,g], acc);  y = epilogue(old, acc)
// with S_g the exact int32 dot product over the 128-column group. The int32 sums come from the tensor cores; the
// float chain runs in the epilogue warps in the reference's group order, so the result is bit-identical.
//
// Persistent, warp-specialised CTA (one per SM), tile = 128 tokens x 128 weight rows:
//   warp 0       TMA producer: activation tile (128 x 128 B, 128-byte swizzle) + packed 2-bit weight tile
//                (128 rows x 32 B) per K-chunk of 128, into a 4-stage shared-memory ring;
//   warp 1       TMEM allocator + MMA issuer: 4 x (M128 N128 K32) per chunk into one of two per-group int32
//                accumulator buffers in TMEM (256 columns), commit -> stage free / group ready;
//   warps 2-7    weight unpackers: 2-bit codes -> int8 {-1,0,+1} (one PRMT per 4 weights) written straight into
//                the UMMA K-major 128-byte-swizzled layout;
//   warps 8-15   epilogue: tcgen05.ld the group sums (warp w reads TMEM lanes 32*(w%4)..+32, columns by half),
//                release the buffer, run the per-group FMA chain in registers, and after the last group apply
//                Store / SiLU / AddScaled (+bias) and store f32.
#include <cuda_fp16.h>

#include <algorithm>
#include <cstring>
#include <vector>

#include "common.h"
#include "math.cuh"
#include "ptx.cuh"

namespace vxg {
namespace gemm {

constexpr int BM = 128;  // tokens per tile (TMEM lanes)
constexpr int BN = 128;  // weight rows per tile (TMEM columns per buffer)
constexpr int BK = 128;  // K per stage: one 128-byte swizzle row
constexpr int STAGES = 4;
constexpr int THREADS = 512;
constexpr int UNPACK_WARP0 = 2, UNPACK_WARPS = 6;
constexpr int EPI_WARP0 = 8, EPI_WARPS = 8;
constexpr int REG_LO = 56, REG_HI = 200;
constexpr uint32_t TMEM_COLS = 2 * BN;
constexpr uint32_t A_BYTES = BM * BK;        // 16 KB
constexpr uint32_t BU_BYTES = BN * BK;       // 16 KB int8 weights
constexpr uint32_t BP_BYTES = BN * BK / 4;   // 4 KB packed codes
constexpr uint32_t SMEM_BYTES = STAGES * (A_BYTES + BU_BYTES + BP_BYTES) + 1024 /*align*/ + 256 /*barriers*/;
constexpr uint32_t IDESC = idesc_i8(BM, BN);

struct Params {
  const float* sx;       // [M, ng]
  const uint8_t* codes;  // [n_tiles][K/128][BN][32]
  const float* swT;      // [ng][N_pad]
  const float* bias;     // [N] or null
  float* y;              // [M, N]
  int32_t* sums;         // [M, N, ng] or null
  int* status;
  int M, N, K, G, N_pad;
  int ep;
  float ep_scale;
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

__global__ void __launch_bounds__(THREADS, 1) ternary_gemm_kernel(const __grid_constant__ CUtensorMap tmap_x,
                                                                   const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sBu = sA + STAGES * A_BYTES;
  uint8_t* sBp = sBu + STAGES * BU_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sBp + STAGES * BP_BYTES);
  uint64_t* full = bars;                  // producer -> unpackers (TMA + bulk bytes)
  uint64_t* unpacked = bars + STAGES;     // unpackers -> MMA
  uint64_t* empty = bars + 2 * STAGES;    // MMA commit -> producer
  uint64_t* tfull = bars + 3 * STAGES;    // MMA commit -> epilogue (per TMEM buffer)
  uint64_t* tempty = tfull + 2;           // epilogue -> MMA
  uint64_t* drain = tempty + 2;           // MMA drain on the error path
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&unpacked[s], UNPACK_WARPS * 32);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; b++) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], EPI_WARPS * 32);
    }
    mbar_init(drain, 1);
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) prefetch_tmap(&tmap_x);
  if (warp == 1) {
    tmem_alloc(tmem_holder, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  // Register split (must sum to the launch budget 512 x 128 = 65536, or the increase never completes):
  // warpgroups 0-1 (producer, MMA, unpackers) drop to REG_LO, warpgroups 2-3 (epilogue) rise to REG_HI.
  static_assert(THREADS * 128 == 256 * REG_LO + 256 * REG_HI, "register split must equal the launch budget");

  const int ng = p.K / p.G, cpg = p.G / BK, nchunks = p.K / BK;
  const int m_tiles = (p.M + BM - 1) / BM, n_tiles = (p.N + BN - 1) / BN;
  const int total = m_tiles * n_tiles;

  if (warp < EPI_WARP0) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(REG_LO) : "memory");
  if (warp == 0) {
    // ------------------------------------------------------------------------------------------ producer
    if (elect_one()) {
      int it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x) {
        const int mt = tile / n_tiles, nt = tile % n_tiles;
        for (int c = 0; c < nchunks; c++, it++) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1, p.status, VXG_DEV_TIMEOUT_PRODUCER)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[s], A_BYTES + BP_BYTES);
          tma_load_2d(sA + s * A_BYTES, &tmap_x, c * BK, mt * BM, &full[s]);
          bulk_load(sBp + s * BP_BYTES, p.codes + ((size_t)nt * nchunks + c) * BP_BYTES, BP_BYTES, &full[s]);
        }
      }
      // Drain: every load issued must land before the CTA exits (normally the unpackers consumed them all).
      for (int k = it > STAGES ? it - STAGES : 0; k < it; k++)
        mbar_wait(&full[k % STAGES], (k / STAGES) & 1, p.status, VXG_DEV_TIMEOUT_DRAIN);
    }
  } else if (warp == 1) {
    // ----------------------------------------------------------------------------------------------- MMA
    if (elect_one()) {
      int it = 0, gi = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x) {
        for (int g = 0; g < ng && ok; g++, gi++) {
          const int b = gi & 1;
          if (!mbar_wait(&tempty[b], ((gi >> 1) & 1) ^ 1, p.status, VXG_DEV_TIMEOUT_MMA)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d = tmem_base + (uint32_t)(b * BN);
          for (int cc = 0; cc < cpg; cc++, it++) {
            const int s = it % STAGES;
            if (!mbar_wait(&unpacked[s], (it / STAGES) & 1, p.status, VXG_DEV_TIMEOUT_MMA)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint64_t ad = umma_desc_sw128(smem_u32(sA + s * A_BYTES));
            const uint64_t bd = umma_desc_sw128(smem_u32(sBu + s * BU_BYTES));
#pragma unroll
            for (int k = 0; k < BK / 32; k++)
              mma_i8(d, ad + (uint64_t)(2 * k), bd + (uint64_t)(2 * k), IDESC, (cc | k) != 0 ? 1u : 0u);
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
  } else if (warp < UNPACK_WARP0 + UNPACK_WARPS) {
    // ------------------------------------------------------------------------------------------ unpackers
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
        const uint32_t* src = reinterpret_cast<const uint32_t*>(sBp + s * BP_BYTES);
        uint8_t* dst = sBu + s * BU_BYTES;
        for (int wi = u; wi < BN * 8; wi += UNPACK_WARPS * 32) {
          const uint4 v = unpack16(src[wi]);
          *reinterpret_cast<uint4*>(dst + sw128_offset((uint32_t)(wi >> 3), (uint32_t)(wi & 7))) = v;
        }
        fence_proxy_async_smem();
        mbar_arrive(&unpacked[s]);
      }
    }
  }
  } else {
    // ------------------------------------------------------------------------------------------- epilogue
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(REG_HI) : "memory");
    const int ew = warp - EPI_WARP0;      // 0..7
    const int q = warp & 3;               // TMEM lane quarter this warp may access
    const int half = ew >> 2;             // column half of the 128-wide tile
    int gi = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x) {
      const int mt = tile / n_tiles, nt = tile % n_tiles;
      const int row = mt * BM + q * 32 + lane;
      const int col0 = nt * BN + half * 64;
      const bool row_ok = row < p.M;
      float acc[64];
#pragma unroll
      for (int c = 0; c < 64; c++) acc[c] = 0.0f;
      for (int g = 0; g < ng; g++, gi++) {
        const int b = gi & 1;
        if (!mbar_wait(&tfull[b], (gi >> 1) & 1, p.status, VXG_DEV_TIMEOUT_EPILOGUE)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const float sxv = row_ok ? __ldg(p.sx + (size_t)row * ng + g) : 0.0f;
        const float* swp = p.swT + (size_t)g * p.N_pad + col0;
        const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(b * BN + half * 64);
#pragma unroll
        for (int hh = 0; hh < 2; hh++) {
          uint32_t S[32];
          tmem_ld32(taddr + hh * 32, S);
          tmem_wait_ld();
          if (hh == 1) {
            tc_fence_before();
            mbar_arrive(&tempty[b]);
          }
#pragma unroll
          for (int c = 0; c < 32; c += 4) {
            const float4 w4 = __ldg(reinterpret_cast<const float4*>(swp + hh * 32 + c));
            const float wv[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
            for (int j = 0; j < 4; j++)
              acc[hh * 32 + c + j] =
                  __fmaf_rn(__int2float_rn((int)S[c + j]), __fmul_rn(sxv, wv[j]), acc[hh * 32 + c + j]);
          }
          if (p.sums && row_ok) {
            for (int c = 0; c < 32; c++) {
              const int o = col0 + hh * 32 + c;
              if (o < p.N) p.sums[((size_t)row * p.N + o) * ng + g] = (int32_t)S[c];
            }
          }
        }
      }
      if (!ok || !row_ok) continue;
      float* yrow = p.y + (size_t)row * p.N;
#pragma unroll
      for (int c = 0; c < 64; c += 4) {
        const int o = col0 + c;
        if (o >= p.N) break;
        float v[4];
#pragma unroll
        for (int j = 0; j < 4; j++) {
          float a = acc[c + j];
          if (p.ep == VXG_EP_SILU) {
            a = silu_fast(a);
          } else if (p.ep == VXG_EP_ADD_SCALED) {
            a = (o + j < p.N) ? __fmaf_rn(p.ep_scale, a, yrow[o + j]) : 0.0f;
          }
          if (p.bias && o + j < p.N) a = __fadd_rn(a, __ldg(p.bias + o + j));
          v[j] = a;
        }
        if (o + 4 <= p.N && (p.N & 3) == 0) {
          *reinterpret_cast<float4*>(yrow + o) = make_float4(v[0], v[1], v[2], v[3]);
        } else {
          for (int j = 0; j < 4 && o + j < p.N; j++) yrow[o + j] = v[j];
        }
      }
    }
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
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

size_t vxg_ternary_scales_count(int out, int in, int group) {
  if (out <= 0 || in <= 0 || group <= 0) return 0;
  return (size_t)(in / group) * (size_t)vxg_ternary_out_pad(out);
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
  std::vector<int8_t> row(in);
  uint32_t* words = reinterpret_cast<uint32_t*>(codes);
  for (int r = 0; r < out_pad; r++) {
    if (r < out) {  // trits.rs:7-27: 5 base-3 digits per byte, least significant first, trit = digit - 1
      const uint8_t* pk = qweight + (size_t)r * rb;
      for (int i = 0; i < in; i++) {
        unsigned v = pk[i / 5];
        for (int k = 0; k < i % 5; k++) v /= 3;
        row[i] = (int8_t)((int)(v % 3) - 1);
      }
    } else {
      std::fill(row.begin(), row.end(), (int8_t)0);
    }
    const int nt = r / gemm::BN, rr = r % gemm::BN;
    for (int c = 0; c < nch; c++)
      for (int w = 0; w < 8; w++) {
        uint32_t word = 0;
        for (int e = 0; e < 16; e++) word |= (uint32_t)(row[c * 128 + w * 16 + e] + 1) << code_pos(e);
        words[(((size_t)nt * nch + c) * gemm::BN + rr) * 8 + w] = word;
      }
  }
  for (int g = 0; g < ng; g++)
    for (int r = 0; r < out_pad; r++)
      scales_t[(size_t)g * out_pad + r] =
          r < out ? __half2float(__ushort_as_half(scales_f16[(size_t)r * ng + g])) : 0.0f;
  return VXG_OK;
}

vxg_status vxg_gemm_ternary_i8(const int8_t* x, const float* sx, const uint8_t* codes, const float* scales_t, int M,
                               int N, int K, int G, vxg_epilogue ep, float ep_scale, const float* bias, float* y,
                               int32_t* group_sums, void* stream) {
  clear_error();
  VXG_ARG(x && sx && codes && scales_t && y, "NULL pointer");
  VXG_ARG(M > 0 && N > 0 && K > 0 && G > 0, "bad shape M=%d N=%d K=%d G=%d", M, N, K, G);
  VXG_ARG(K % gemm::BK == 0 && G % gemm::BK == 0 && K % G == 0,
          "K (%d) and G (%d) must be multiples of 128 with G | K", K, G);
  VXG_ARG(ep == VXG_EP_STORE || ep == VXG_EP_SILU || ep == VXG_EP_ADD_SCALED, "bad epilogue %d", (int)ep);
  VXG_ARG(((uintptr_t)x & 15) == 0 && ((uintptr_t)codes & 15) == 0 && ((uintptr_t)scales_t & 15) == 0,
          "x, codes and scales_t must be 16-byte aligned");
  int* status = device_status();
  VXG_ARG(status != nullptr, "no CUDA device");
  CUtensorMap tmap;
  vxg_status st = make_tmap_2d_u8(&tmap, x, (uint64_t)M, (uint64_t)K, (uint64_t)K, gemm::BM, gemm::BK);
  if (st != VXG_OK) return st;
  static bool attr_set = false;
  if (!attr_set) {
    VXG_CUDA(cudaFuncSetAttribute(gemm::ternary_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)gemm::SMEM_BYTES));
    attr_set = true;
  }
  gemm::Params p;
  p.sx = sx;
  p.codes = codes;
  p.swT = scales_t;
  p.bias = bias;
  p.y = y;
  p.sums = group_sums;
  p.status = status;
  p.M = M;
  p.N = N;
  p.K = K;
  p.G = G;
  p.N_pad = vxg_ternary_out_pad(N);
  p.ep = (int)ep;
  p.ep_scale = ep_scale;
  const int tiles = ((M + gemm::BM - 1) / gemm::BM) * ((N + gemm::BN - 1) / gemm::BN);
  const int grid = std::min(tiles, sm_count());
  gemm::ternary_gemm_kernel<<<grid, gemm::THREADS, gemm::SMEM_BYTES, (cudaStream_t)stream>>>(tmap, p);
  VXG_CUDA(cudaGetLastError());
  return VXG_OK;
}

}  // extern "C"
