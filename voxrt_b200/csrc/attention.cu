// int8 relative-position multi-head attention core on sm_100a (tcgen05.mma kind::i8, scores and P*V in TMEM).
//
// Reference: attn_core_int8 (crates/voxrt/src/encoder.rs:317-534) with its int8 context (VOXRT_ATTN_CTX default).
// Per utterance of t frames and per head (dh = 128):
//   Qu[i] = quant(q_i + bias_u), Qv[i] = quant(q_i + bias_v), K[j] = quant(k_j)   (one group per row, :349-377)
//   R[p]  = quant(rel_k[p])  for positions p = t-1-i+j                             (:378-390)
//   Vt[c] = quant(v[0..t, c]) one group over all frames (zeros to t16)             (:391-402)
//   s1[i,j] = fma(float(Qu_i.K_j), squ_i*sk_j, 0); s2[i,j] = fma(float(Qv_i.R_p), sqv_i*srel_p, 0)
//   row i: v_j = (s1 + s2) * scaling; max = max_j v_j; e_j = exp_poly(v_j - max);
//          sum = hsum4(4 lane chains over j = l mod 4) + in-order tail;  P = quant(e) (scale 1/127)
//   out[i,c] = fma(float(P_i.Vt_c), (s_p/sum)*sv_c, 0)                               (:489-502)
// Every float step above is reproduced exactly; the int32 dot products come from the tensor cores.
//
// One kernel per layer after the quantisation prep: attn_fused_kernel keeps every score on chip. Per (128 queries,
// head) it runs the S1 and S2-band tiles on tcgen05 into TMEM twice: pass 1 for the row maxima, pass 2 (recomputing
// the same scores) for e = exp_poly(v - max), the int8 P tile, the reference's four lane-chain sums in key order and
// P * V^T on tcgen05; then the context epilogue.
//
// Batched layout: utterances are stacked along the token axis (offset off[u], length len[u]); the relative table
// rel_k is shared by the batch (positions Tmax-1 .. -(Tmax-1)), row Tmax - t + p of it is utterance row p.
#include <cuda_runtime.h>

#include <algorithm>
#include <vector>

#include "common.h"
#include "internal.h"
#include "math.cuh"
#include "ptx.cuh"

namespace vxg {
namespace attn {

constexpr int DH = 128;      // head dim
constexpr int BQ = kAttnBQ;  // query rows per CTA
constexpr int BKV = 128;     // keys per tile
constexpr uint32_t MAGIC = 0x4B400000u;
constexpr uint32_t TSTRIDE = 68;  // words per row of the band de-skew staging (conflict-free both ways)

struct Params {
  const int* tile_utt;  // per query tile: utterance
  const int* tile_q0;   // per query tile: first query row within the utterance
  const int* off;       // [U] token offset
  const int* len;       // [U] frames
  const int* voff;      // [U] key offset in the transposed V (multiple of 16)
  const float* squ;     // [H][Mtot]
  const float* sqv;
  const float* sk;
  const float* srelT;  // [H][NP]
  const float* sv;     // [H][U][128]
  float* ctx;          // [Mtot, H*128] f32 or null
  int8_t* ctx_q;       // [Mtot, H*128] int8 or null (quantised per head for the output projection)
  float* ctx_s;        // [Mtot, H]
  int* status;
  int Mtot, NP, tmax, H, U;
  float scaling;
};

__device__ __forceinline__ float exact_i2f(uint32_t s_plus_magic) {  // |S| < 2^22: exact
  return __fsub_rn(__uint_as_float(s_plus_magic), 12582912.0f);
}

// exp_poly (math.cuh) of two arguments x <= 88 that are not NaN (here v - rowmax <= 0): the upper clamp cannot act
// and the lower clamp is a plain max. The fused multiply-adds and the exact subtraction of the shifter run as packed
// f32x2 instructions (each half rounded like the scalar step; fma(-n, c, y) computed as fma(n, -c, y)); the
// shifter rounding of y * log2(e) and the final p * 2^n stay scalar (a packed multiply feeding a packed add may be
// contracted into one FMA, which would skip the product's rounding: a mismatch against the oracle showed it).
__device__ __forceinline__ void exp2_le88(float x0, float x1, float& e0, float& e1) {
  const float y0 = fmaxf(x0, -87.0f), y1 = fmaxf(x1, -87.0f);
  const float t0 = __fadd_rn(__fmul_rn(y0, 1.44269504088896340736f), 12582912.0f);
  const float t1 = __fadd_rn(__fmul_rn(y1, 1.44269504088896340736f), 12582912.0f);
  const uint64_t n = fadd2(pk2(t0, t1), pk2(-12582912.0f, -12582912.0f));  // exact
  uint64_t r = ffma2(n, pk2(-0.69314575f, -0.69314575f), pk2(y0, y1));
  r = ffma2(n, pk2(-1.4286068e-6f, -1.4286068e-6f), r);
  uint64_t q = pk2(1.0f / 720.0f, 1.0f / 720.0f);
  q = ffma2(q, r, pk2(1.0f / 120.0f, 1.0f / 120.0f));
  q = ffma2(q, r, pk2(1.0f / 24.0f, 1.0f / 24.0f));
  q = ffma2(q, r, pk2(1.0f / 6.0f, 1.0f / 6.0f));
  q = ffma2(q, r, pk2(0.5f, 0.5f));
  q = ffma2(q, r, pk2(1.0f, 1.0f));
  q = ffma2(q, r, pk2(1.0f, 1.0f));
  float q0, q1;
  upk2(q, q0, q1);
  e0 = __fmul_rn(q0, __int_as_float((__float_as_int(t0) - 0x4B400000 + 127) << 23));
  e1 = __fmul_rn(q1, __int_as_float((__float_as_int(t1) - 0x4B400000 + 127) << 23));
}

// ------------------------------------------------------------------------------------------- fused kernel
// One work item = (128 query rows, head). Pass 1 walks the key tiles computing the scores v in TMEM / registers and
// keeps only the row maxima; pass 2 walks them again, recomputing the same v, and turns them into e, the int8 P
// tile (shared memory) and the reference's four lane-chain sums, while tcgen05 accumulates P * V^T in TMEM. No
// score leaves the SM. Persistent: CTA b takes items b, b + gridDim.x, ... (item w = query tile w % n_tiles of head
// w / n_tiles); every barrier phase and ring slot runs on across passes and items.
//
// Roles: warp 0 issues the TMA loads (Qu/Qv per item; per key tile K, the 128 relative positions the tile's band adds
// to a 3-slot ring, and in pass 2 the Vt tile), warp 1 the MMAs, warps 2-3 stage the key and band scales, warps 4-11
// are the epilogue: warp (quarter q = warp & 3, half hf) owns TMEM lanes / query rows 32 q .. 32 q + 31 and the 32-key
// chunks c = hf and c = 2 + hf of every tile. The lane-chain sums run over the keys in order, so each row's four
// chain values pass from one warp of the pair to the other after every chunk (named barriers, producer / consumer).
constexpr int F_THREADS = 384;
constexpr int F_EPI0 = 4, F_EPI = 8;
constexpr int F_RSLOTS = 3;
constexpr uint32_t F_OFF_QU = 0;
constexpr uint32_t F_OFF_QV = F_OFF_QU + BQ * DH;
constexpr uint32_t F_OFF_K = F_OFF_QV + BQ * DH;               // 2 x [128 keys][128 dh]
constexpr uint32_t F_OFF_R = F_OFF_K + 2 * BKV * DH;           // 3 x [128 positions][128 dh]
constexpr uint32_t F_OFF_V = F_OFF_R + F_RSLOTS * BKV * DH;    // Vt [128 dh][128 keys]
constexpr uint32_t F_OFF_P = F_OFF_V + DH * BKV;               // P [128 rows][128 keys]
constexpr uint32_t F_OFF_T = F_OFF_P + BQ * BKV;               // per epilogue warp: [32][TSTRIDE] words
constexpr uint32_t F_OFF_KS = F_OFF_T + F_EPI * 32 * TSTRIDE * 4;  // [2][128] key scales
constexpr uint32_t F_OFF_RS = F_OFF_KS + 2 * BKV * 4;              // [2][256] band scales
constexpr uint32_t F_OFF_MX = F_OFF_RS + 2 * 2 * BKV * 4;          // [2 halves][128] row maxima
constexpr uint32_t F_OFF_CH = F_OFF_MX + 2 * BQ * 4;               // [128] float4 lane-chain sums
constexpr uint32_t F_OFF_TL = F_OFF_CH + BQ * 16;                  // [128] float4 e of keys t4 .. t-1
constexpr uint32_t F_OFF_BAR = F_OFF_TL + BQ * 16;
constexpr uint32_t F_SMEM = F_OFF_BAR + 256 + 1024;
static_assert(F_SMEM <= 232448, "fused attention shared memory");
static_assert(F_OFF_V % 1024 == 0 && F_OFF_P % 1024 == 0 && F_OFF_R % 1024 == 0, "swizzle atoms");
// TMEM columns: S1 [0,128), S2 band [128,384) (positions of ring chunks k and k+1), O [384,512)
constexpr uint32_t F_TM_S1 = 0, F_TM_S2 = 128, F_TM_O = 384, F_TMEM = 512;
constexpr int F_BAR_EPI = 1, F_BAR_A = 2, F_BAR_B = 6;  // named barriers: all epilogue warps; handoffs per quarter

__global__ void __launch_bounds__(F_THREADS, 1)
    attn_fused_kernel(const __grid_constant__ CUtensorMap tm_qu, const __grid_constant__ CUtensorMap tm_qv,
                      const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_r,
                      const __grid_constant__ CUtensorMap tm_v, const Params p, int n_tiles) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + F_OFF_BAR);
  uint64_t* q_full = bars + 0;
  uint64_t* q_empty = bars + 1;
  uint64_t* k_full = bars + 2;   // [2]
  uint64_t* k_empty = bars + 4;  // [2]
  uint64_t* r_full = bars + 6;   // [3]
  uint64_t* r_empty = bars + 9;  // [3]
  uint64_t* v_full = bars + 12;
  uint64_t* v_empty = bars + 13;
  uint64_t* s_full = bars + 14;
  uint64_t* s_empty = bars + 15;
  uint64_t* sc_full = bars + 16;   // [2]
  uint64_t* sc_empty = bars + 18;  // [2]
  uint64_t* p_full = bars + 20;
  uint64_t* p_empty = bars + 21;
  uint64_t* o_full = bars + 22;
  uint64_t* o_empty = bars + 23;
  uint64_t* drain = bars + 24;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 25);
  float* sKs = reinterpret_cast<float*>(smem + F_OFF_KS);
  float* sRs = reinterpret_cast<float*>(smem + F_OFF_RS);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_items = n_tiles * p.H;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int s = 0; s < 2; s++) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&sc_full[s], 64);
      mbar_init(&sc_empty[s], F_EPI * 32);
    }
    for (int s = 0; s < F_RSLOTS; s++) {
      mbar_init(&r_full[s], 1);
      mbar_init(&r_empty[s], 1);
    }
    mbar_init(v_full, 1);
    mbar_init(v_empty, 1);
    mbar_init(s_full, 1);
    mbar_init(s_empty, F_EPI * 32);
    mbar_init(p_full, F_EPI * 32);
    mbar_init(p_empty, 1);
    mbar_init(o_full, 1);
    mbar_init(o_empty, 4 * 32);
    mbar_init(drain, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, F_TMEM);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == 0) {
    // ------------------------------------------------------------------------------------- TMA producer
    // Per pass, for s = 0 .. nkt: ring chunk s (positions rel0 + 128 s ..), then K tile s - 1, then (pass 2) Vt tile
    // s - 2; Vt tile nkt - 1 last. MMA S(k) needs chunks k, k + 1 and K tile k; P*V(k) needs Vt tile k.
    if (elect_one()) {
      bool ok = true;
      int gk = 0, gr = 0, gv = 0, n = 0;
      for (int w = blockIdx.x; w < n_items && ok; w += gridDim.x, n++) {
        const int tile = w % n_tiles, h = w / n_tiles;
        const int u = p.tile_utt[tile], i0 = p.tile_q0[tile];
        const int t = p.len[u], off = p.off[u], nkt = (t + BKV - 1) / BKV;
        const int rel0 = p.tmax - 1 - i0 - (BQ - 1);
        if (n > 0 && !mbar_wait(q_empty, (n - 1) & 1, p.status, VXG_DEV_TIMEOUT_ATTN)) break;
        mbar_arrive_expect_tx(q_full, 2 * BQ * DH);
        tma_load_2d(smem + F_OFF_QU, &tm_qu, 0, h * p.Mtot + off + i0, q_full);
        tma_load_2d(smem + F_OFF_QV, &tm_qv, 0, h * p.Mtot + off + i0, q_full);
        for (int pass = 0; pass < 2 && ok; pass++) {
          for (int s = 0; s <= nkt + 1 && ok; s++) {
            if (s <= nkt) {
              const int slot = gr % F_RSLOTS;
              if (!mbar_wait(&r_empty[slot], ((gr / F_RSLOTS) & 1) ^ 1, p.status, VXG_DEV_TIMEOUT_ATTN)) {
                ok = false;
                break;
              }
              mbar_arrive_expect_tx(&r_full[slot], BKV * DH);
              tma_load_2d(smem + F_OFF_R + slot * BKV * DH, &tm_r, h * DH, rel0 + s * BKV, &r_full[slot]);
              gr++;
            }
            if (s >= 1 && s <= nkt) {
              const int b = gk & 1;
              if (!mbar_wait(&k_empty[b], ((gk >> 1) & 1) ^ 1, p.status, VXG_DEV_TIMEOUT_ATTN)) {
                ok = false;
                break;
              }
              mbar_arrive_expect_tx(&k_full[b], BKV * DH);
              tma_load_2d(smem + F_OFF_K + b * BKV * DH, &tm_k, 0, h * p.Mtot + off + (s - 1) * BKV, &k_full[b]);
              gk++;
            }
            if (pass == 1 && s >= 2) {
              if (!mbar_wait(v_empty, (gv & 1) ^ 1, p.status, VXG_DEV_TIMEOUT_ATTN)) {
                ok = false;
                break;
              }
              mbar_arrive_expect_tx(v_full, DH * BKV);
              tma_load_2d(smem + F_OFF_V, &tm_v, p.voff[u] + (s - 2) * BKV, h * DH, v_full);
              gv++;
            }
          }
        }
      }
      // every load issued must land before the CTA exits
      if (n > 0) mbar_wait(q_full, (n - 1) & 1, p.status, VXG_DEV_TIMEOUT_DRAIN);
      for (int x = gr > F_RSLOTS ? gr - F_RSLOTS : 0; x < gr; x++)
        mbar_wait(&r_full[x % F_RSLOTS], (x / F_RSLOTS) & 1, p.status, VXG_DEV_TIMEOUT_DRAIN);
      for (int x = gk > 2 ? gk - 2 : 0; x < gk; x++)
        mbar_wait(&k_full[x & 1], (x >> 1) & 1, p.status, VXG_DEV_TIMEOUT_DRAIN);
      if (gv > 0) mbar_wait(v_full, (gv - 1) & 1, p.status, VXG_DEV_TIMEOUT_DRAIN);
    }
  } else if (warp == 1) {
    // -------------------------------------------------------------------------------------- MMA issuer
    if (elect_one()) {
      bool ok = true;
      int gk = 0, gr = 0, gv = 0, gs = 0, n = 0;
      const uint64_t dqu = umma_desc_sw128(smem_u32(smem + F_OFF_QU));
      const uint64_t dqv = umma_desc_sw128(smem_u32(smem + F_OFF_QV));
      const uint64_t dpm = umma_desc_sw128(smem_u32(smem + F_OFF_P));
      const uint64_t dvt = umma_desc_sw128(smem_u32(smem + F_OFF_V));
      // O += P * Vt^T for key tile kk of item n (P and Vt tiles in shared memory)
      auto pv = [&](int kk) {
        if (kk == 0 && n > 0 && !mbar_wait(o_empty, (n - 1) & 1, p.status, VXG_DEV_TIMEOUT_ATTN)) return false;
        if (!mbar_wait(v_full, gv & 1, p.status, VXG_DEV_TIMEOUT_ATTN) ||
            !mbar_wait(p_full, gv & 1, p.status, VXG_DEV_TIMEOUT_ATTN))
          return false;
        tc_fence_after();
#pragma unroll
        for (int x = 0; x < 4; x++)
          mma_i8(tmem + F_TM_O, dpm + 2 * x, dvt + 2 * x, idesc_i8(128, 128), (kk | x) != 0 ? 1u : 0u);
        mma_commit(p_empty);
        mma_commit(v_empty);
        gv++;
        return true;
      };
      for (int w = blockIdx.x; w < n_items && ok; w += gridDim.x, n++) {
        const int tile = w % n_tiles;
        const int nkt = (p.len[p.tile_utt[tile]] + BKV - 1) / BKV;
        if (!mbar_wait(q_full, n & 1, p.status, VXG_DEV_TIMEOUT_ATTN)) break;
        for (int pass = 0; pass < 2 && ok; pass++) {
          const int rb = gr;  // ring index of this pass's chunk 0
          for (int k = 0; k < nkt; k++, gk++, gs++) {
            const int s0 = (rb + k) % F_RSLOTS, s1 = (rb + k + 1) % F_RSLOTS, b = gk & 1;
            if ((k == 0 && !mbar_wait(&r_full[s0], ((rb + k) / F_RSLOTS) & 1, p.status, VXG_DEV_TIMEOUT_ATTN)) ||
                !mbar_wait(&r_full[s1], ((rb + k + 1) / F_RSLOTS) & 1, p.status, VXG_DEV_TIMEOUT_ATTN) ||
                !mbar_wait(&k_full[b], (gk >> 1) & 1, p.status, VXG_DEV_TIMEOUT_ATTN) ||
                !mbar_wait(s_empty, (gs & 1) ^ 1, p.status, VXG_DEV_TIMEOUT_ATTN)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint64_t dk = umma_desc_sw128(smem_u32(smem + F_OFF_K + b * BKV * DH));
            const uint64_t dr0 = umma_desc_sw128(smem_u32(smem + F_OFF_R + s0 * BKV * DH));
            const uint64_t dr1 = umma_desc_sw128(smem_u32(smem + F_OFF_R + s1 * BKV * DH));
#pragma unroll
            for (int x = 0; x < 4; x++)
              mma_i8(tmem + F_TM_S1, dqu + 2 * x, dk + 2 * x, idesc_i8(128, 128), x ? 1u : 0u);
#pragma unroll
            for (int x = 0; x < 4; x++) {
              mma_i8(tmem + F_TM_S2, dqv + 2 * x, dr0 + 2 * x, idesc_i8(128, 128), x ? 1u : 0u);
              mma_i8(tmem + F_TM_S2 + 128, dqv + 2 * x, dr1 + 2 * x, idesc_i8(128, 128), x ? 1u : 0u);
            }
            mma_commit(s_full);
            mma_commit(&k_empty[b]);
            mma_commit(&r_empty[s0]);
            if (k == nkt - 1) mma_commit(&r_empty[s1]);
            if (pass == 1 && k >= 1 && !pv(k - 1)) {
              ok = false;
              break;
            }
          }
          gr = rb + nkt + 1;
          if (ok && pass == 1) {
            if (!pv(nkt - 1)) {
              ok = false;
              break;
            }
            mma_commit(o_full);
          }
        }
        if (ok) mma_commit(q_empty);  // the item's Q tiles are no longer read
      }
      mma_commit(drain);
      mbar_wait(drain, 0, p.status, VXG_DEV_TIMEOUT_DRAIN);
    }
  } else if (warp < F_EPI0) {
    // --------------------------------------------------------------------------------- scale loaders
    const int lt = threadIdx.x - 2 * 32;  // 0..63
    int g = 0;
    bool ok = true;
    for (int w = blockIdx.x; w < n_items && ok; w += gridDim.x) {
      const int tile = w % n_tiles, h = w / n_tiles;
      const int u = p.tile_utt[tile], i0 = p.tile_q0[tile];
      const int t = p.len[u], off = p.off[u], nkt = (t + BKV - 1) / BKV;
      const int rel0 = p.tmax - 1 - i0 - (BQ - 1);
      const float* skh = p.sk + (size_t)h * p.Mtot + off;
      const float* srh = p.srelT + (size_t)h * p.NP;
      for (int step = 0; step < 2 * nkt; step++, g++) {
        const int k = step % nkt, b = g & 1;
        if (!mbar_wait(&sc_empty[b], ((g >> 1) & 1) ^ 1, p.status, VXG_DEV_TIMEOUT_ATTN)) {
          ok = false;
          break;
        }
        for (int x = lt; x < BKV; x += 64) {
          const int j = k * BKV + x;
          sKs[b * BKV + x] = j < t ? __ldg(skh + j) : 0.0f;
        }
        for (int x = lt; x < 2 * BKV; x += 64) {
          const int r = rel0 + k * BKV + x;
          sRs[b * 2 * BKV + x] = (r >= 0 && r < p.NP) ? __ldg(srh + r) : 0.0f;
        }
        mbar_arrive(&sc_full[b]);
      }
    }
  } else {
    // ---------------------------------------------------------------------------------------- epilogue
    const int ew = warp - F_EPI0;
    const int q = warp & 3, hf = ew >> 2;
    const int r = q * 32 + lane;
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    float* stg = reinterpret_cast<float*>(smem + F_OFF_T) + ew * 32 * TSTRIDE;
    float* sMx = reinterpret_cast<float*>(smem + F_OFF_MX);
    float4* sCh = reinterpret_cast<float4*>(smem + F_OFF_CH);
    float4* sTl = reinterpret_cast<float4*>(smem + F_OFF_TL);
    const uint32_t prow = smem_u32(smem + F_OFF_P) + (uint32_t)r * 128u;
    const float inv127 = __fdiv_rn(1.0f, __fdiv_rn(1.0f, 127.0f));  // 1 / (absmax 1 / 127): every P row's max is 1
    int g = 0, gp = 0, n = 0;  // key-tile steps (both passes), pass-2 steps, items
    // After a failed wait (the error is recorded in p.status) the remaining waits are skipped, but every named
    // barrier below is still passed in the same order by every epilogue warp, so no warp is left waiting.
    bool ok = true;
    auto wait = [&](uint64_t* bar, uint32_t parity) {
      if (ok && !mbar_wait(bar, parity, p.status, VXG_DEV_TIMEOUT_ATTN)) ok = false;
    };
    // this thread's query-row scales of item w (0 outside the utterance); item w + gridDim.x's are loaded while item
    // w runs, so an item's epilogue does not start with a global round trip
    auto row_scales = [&](int w, float& su, float& sv) {
      su = sv = 0.0f;
      if (w >= n_items) return;
      const int tile = w % n_tiles, h = w / n_tiles, u = p.tile_utt[tile], i = p.tile_q0[tile] + r;
      if (i < p.len[u]) {
        const int gi = h * p.Mtot + p.off[u] + i;
        su = __ldg(p.squ + gi);
        sv = __ldg(p.sqv + gi);
      }
    };
    float squ_next, sqv_next;
    row_scales(blockIdx.x, squ_next, sqv_next);
    for (int w = blockIdx.x; w < n_items; w += gridDim.x, n++) {
      const int tile = w % n_tiles, h = w / n_tiles;
      const int u = p.tile_utt[tile], i0 = p.tile_q0[tile];
      const int t = p.len[u], off = p.off[u], nkt = (t + BKV - 1) / BKV;
      const int t4 = t & ~3;
      const int i = i0 + r;
      const bool valid = i < t;
      const float squ = squ_next, sqv = sqv_next;
      row_scales(w + gridDim.x, squ_next, sqv_next);
      // The unscaled scores a + b of this row for the 32 keys of chunk c of the key tile in TMEM (ring buffer b of
      // the scales), as 16 packed pairs: a = fma(float(S1), squ*sk, 0), b = fma(float(S2), sqv*srel, 0); the score
      // is v = (a + b) * scaling (encoder.rs:404-470). Packed f32x2 steps round each half like the scalar step, and
      // no packed product here feeds a packed add (the products feed FMAs as multiplicands).
      const uint64_t su2 = pk2(squ, squ), sv2 = pk2(sqv, sqv), nmag = pk2(-12582912.0f, -12582912.0f),
                     zero2 = pk2(0.0f, 0.0f);
      auto sums = [&](int c, int b, bool release, uint64_t (&sum)[16]) {
        uint32_t s1[32], bl[32], bh[32];
        tmem_ld32(tmem + lane_base + F_TM_S1 + c * 32, s1);
        const uint32_t band = F_TM_S2 + (uint32_t)(96 - 32 * q + 32 * c);  // 64 band columns of this warp
        tmem_ld32(tmem + lane_base + band, bl);
        tmem_ld32(tmem + lane_base + band + 32, bh);
        tmem_wait_ld();
        if (release) {
          tc_fence_before();
          mbar_arrive(s_empty);
        }
        // undo the diagonal skew: each thread writes its row's window (stride 68) and reads back columns
        // 31 - lane .. 62 - lane of it, so only the 16-byte pieces that overlap that range are written, and a thread
        // reads only its own row (program order, no warp barrier)
#pragma unroll
        for (int m = 0; m < 32; m += 4) {
          if (m + 3 >= 31 - lane)
            *reinterpret_cast<uint4*>(stg + lane * TSTRIDE + m) = make_uint4(bl[m], bl[m + 1], bl[m + 2], bl[m + 3]);
          if (m <= 31 - lane)
            *reinterpret_cast<uint4*>(stg + lane * TSTRIDE + 32 + m) = make_uint4(bh[m], bh[m + 1], bh[m + 2], bh[m + 3]);
        }
        const float4* ks4 = reinterpret_cast<const float4*>(sKs + b * BKV + c * 32);
        const float* rs = sRs + b * 2 * BKV + c * 32 + (BQ - 1) - r;
        const float* sk = stg + lane * (TSTRIDE - 1) + 31;
#pragma unroll
        for (int m = 0; m < 16; m++) {
          const float4 kq = ks4[m >> 1];
          const float2 kp = (m & 1) ? make_float2(kq.z, kq.w) : make_float2(kq.x, kq.y);
          const uint64_t f1 = fadd2(pk2(__uint_as_float(s1[2 * m] + MAGIC), __uint_as_float(s1[2 * m + 1] + MAGIC)), nmag);
          const uint64_t a2 = ffma2(f1, fmul2(su2, pk2(kp.x, kp.y)), zero2);
          const uint32_t t0 = __float_as_uint(sk[2 * m]), t1 = __float_as_uint(sk[2 * m + 1]);
          const uint64_t f2 = fadd2(pk2(__uint_as_float(t0 + MAGIC), __uint_as_float(t1 + MAGIC)), nmag);
          const uint64_t b2 = ffma2(f2, fmul2(sv2, pk2(rs[2 * m], rs[2 * m + 1])), zero2);
          sum[m] = fadd2(a2, b2);
        }
      };

      // ---- pass 1: row maxima. max_j (u_j * scaling) = (max_j u_j) * scaling exactly: scaling > 0 and rounding
      // is monotone, so the maximum of the unscaled sums is taken and scaled once.
      float mx = -INFINITY;
      for (int k = 0; k < nkt; k++, g++) {
        const int b = g & 1;
        wait(s_full, g & 1);
        wait(&sc_full[b], (g >> 1) & 1);
        tc_fence_after();
#pragma unroll 1
        for (int cc = 0; cc < 2; cc++) {
          const int c = 2 * cc + hf;
          uint64_t u[16];
          sums(c, b, cc == 1, u);
          const int j0 = k * BKV + c * 32;
          if (j0 + 32 <= t) {
#pragma unroll
            for (int m = 0; m < 16; m++) {
              float lo, hi;
              upk2(u[m], lo, hi);
              mx = fmaxf(mx, fmaxf(lo, hi));
            }
          } else {
#pragma unroll
            for (int m = 0; m < 16; m++) {
              float lo, hi;
              upk2(u[m], lo, hi);
              if (j0 + 2 * m < t) mx = fmaxf(mx, lo);
              if (j0 + 2 * m + 1 < t) mx = fmaxf(mx, hi);
            }
          }
        }
        mbar_arrive(&sc_empty[b]);
      }
      mx = __fmul_rn(mx, p.scaling);
      sMx[hf * BQ + r] = mx;
      named_bar_sync(F_BAR_EPI, F_EPI * 32);
      mx = fmaxf(sMx[r], sMx[BQ + r]);
      if (hf == 0 && valid && !(fabsf(mx) <= 3.402823466e38f)) atomicCAS(p.status, 0, VXG_DEV_ATTN_PMAX);

      // ---- pass 2: e, P, lane chains (exp_row_scaled_portable, tensor.rs:810-826), O += P * V^T
      for (int k = 0; k < nkt; k++, g++) {
        const int b = g & 1;
        wait(s_full, g & 1);
        wait(&sc_full[b], (g >> 1) & 1);
        tc_fence_after();
#pragma unroll 1
        for (int cc = 0; cc < 2; cc++) {
          const int c = 2 * cc + hf;
          const int idx = 4 * k + c;  // chunk index in key order
          float v[32];
          {
            uint64_t u[16];
            sums(c, b, cc == 1, u);
#pragma unroll
            for (int m = 0; m < 16; m++) {
              upk2(u[m], v[2 * m], v[2 * m + 1]);
              v[2 * m] = __fmul_rn(v[2 * m], p.scaling);
              v[2 * m + 1] = __fmul_rn(v[2 * m + 1], p.scaling);
            }
          }
          const int j0 = k * BKV + c * 32;
          uint32_t wq[8];
          if (valid && j0 + 32 <= t) {
            // every key of the chunk is in range: v - max <= 0 (max is the row's maximum, scores are finite), so
            // e in [0, 1], e * 127 <= 127 and the shifter's low byte is quant_code's code
#pragma unroll
            for (int m = 0; m < 32; m += 2) exp2_le88(__fsub_rn(v[m], mx), __fsub_rn(v[m + 1], mx), v[m], v[m + 1]);
#pragma unroll
            for (int m = 0; m < 8; m++) {  // the code is the low byte of fl(e * inv + 1.5 * 2^23)
              uint32_t x[4];
#pragma unroll
              for (int k2 = 0; k2 < 4; k2++)
                x[k2] = __float_as_uint(__fadd_rn(__fmul_rn(v[4 * m + k2], inv127), 12582912.0f));
              wq[m] = __byte_perm(__byte_perm(x[0], x[1], 0x0040), __byte_perm(x[2], x[3], 0x0040), 0x5410);
            }
          } else {
#pragma unroll
            for (int m = 0; m < 32; m++) v[m] = (valid && j0 + m < t) ? exp_poly(__fsub_rn(v[m], mx)) : 0.0f;
#pragma unroll
            for (int m = 0; m < 8; m++)
              wq[m] = ((uint32_t)quant_code(v[4 * m], inv127) & 0xFFu) |
                      (((uint32_t)quant_code(v[4 * m + 1], inv127) & 0xFFu) << 8) |
                      (((uint32_t)quant_code(v[4 * m + 2], inv127) & 0xFFu) << 16) |
                      (((uint32_t)quant_code(v[4 * m + 3], inv127) & 0xFFu) << 24);
          }
          if (cc == 0) wait(p_empty, (gp & 1) ^ 1);  // P*V of the previous key tile has read the P tile
          // row r's 32 codes of chunk c: 16-byte units 2c, 2c + 1 of the 128B-swizzled P row
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(prow + ((((uint32_t)(2 * c)) ^ (uint32_t)(r & 7)) << 4)),
                       "r"(wq[0]), "r"(wq[1]), "r"(wq[2]), "r"(wq[3])
                       : "memory");
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(prow + ((((uint32_t)(2 * c + 1)) ^ (uint32_t)(r & 7)) << 4)),
                       "r"(wq[4]), "r"(wq[5]), "r"(wq[6]), "r"(wq[7])
                       : "memory");
          // lane chains: chain l sums e_j, j = l mod 4, j < t4, in increasing j; the chunk before this one (the
          // other warp of the pair) hands the four running sums over
          if (idx > 0) named_bar_sync(hf ? F_BAR_A + q : F_BAR_B + q, 64);
          float4 ch = idx > 0 ? sCh[r] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
          if (j0 + 32 <= t4) {
#pragma unroll
            for (int m = 0; m < 32; m += 4) {
              ch.x = __fadd_rn(ch.x, v[m]);
              ch.y = __fadd_rn(ch.y, v[m + 1]);
              ch.z = __fadd_rn(ch.z, v[m + 2]);
              ch.w = __fadd_rn(ch.w, v[m + 3]);
            }
          } else {
#pragma unroll
            for (int m = 0; m < 32; m += 4) {
              if (j0 + m < t4) {
                ch.x = __fadd_rn(ch.x, v[m]);
                ch.y = __fadd_rn(ch.y, v[m + 1]);
                ch.z = __fadd_rn(ch.z, v[m + 2]);
                ch.w = __fadd_rn(ch.w, v[m + 3]);
              }
            }
            if (t4 < t && j0 <= t4 && t4 < j0 + 32) {  // the tail keys t4 .. t-1 (added after the chains, in order)
              float tl[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
              for (int m = 0; m < 32; m += 4)
                if (j0 + m == t4) tl[0] = v[m], tl[1] = v[m + 1], tl[2] = v[m + 2];
              sTl[r] = make_float4(tl[0], tl[1], tl[2], 0.0f);
            }
          }
          sCh[r] = ch;
          if (idx < 4 * nkt - 1) named_bar_arrive(hf ? F_BAR_B + q : F_BAR_A + q, 64);
        }
        mbar_arrive(&sc_empty[b]);
        fence_proxy_async_smem();
        mbar_arrive(p_full);
        gp++;
      }
      named_bar_sync(F_BAR_EPI, F_EPI * 32);  // final chain sums and tails are in shared memory
      if (hf == 0) {
        // ------------------------------------------------------------------ context epilogue (lane quarter q)
        float inv = 0.0f;
        if (valid) {  // sum = hsum4(chains) + the tail j in [t4, t) in order
          const float4 ch = sCh[r];
          float sum = __fadd_rn(__fadd_rn(ch.x, ch.y), __fadd_rn(ch.z, ch.w));
          const float4 tl = sTl[r];
          if (t4 < t) sum = __fadd_rn(sum, tl.x);
          if (t4 + 1 < t) sum = __fadd_rn(sum, tl.y);
          if (t4 + 2 < t) sum = __fadd_rn(sum, tl.z);
          inv = __fdiv_rn(1.0f, sum);
        }
        wait(o_full, n & 1);
        tc_fence_after();
        const float sp = __fmul_rn(__fdiv_rn(1.0f, 127.0f), inv);  // P scale, 1/sum (:494-501)
        const float* svh = p.sv + ((size_t)h * p.U + u) * DH;
        const size_t orow = (size_t)(off + (valid ? i : 0));
        const int dmod = p.H * DH;
        // out[c] = fma(float(O[c]), sp * sv[c], 0); pass A: absmax (and the f32 context), pass B: int8 codes
        float amax = 0.0f;
#pragma unroll 1
        for (int c = 0; c < DH; c += 32) {
          uint32_t o[32];
          tmem_ld32(tmem + lane_base + F_TM_O + c, o);
          tmem_wait_ld();
#pragma unroll
          for (int m = 0; m < 32; m += 4) {
            float vv[4];
#pragma unroll
            for (int k2 = 0; k2 < 4; k2++) {
              vv[k2] = __fmaf_rn(__int2float_rn((int)o[m + k2]), __fmul_rn(sp, __ldg(svh + c + m + k2)), 0.0f);
              amax = fmaxf(amax, fabsf(vv[k2]));
            }
            if (valid && p.ctx)
              *reinterpret_cast<float4*>(p.ctx + orow * dmod + h * DH + c + m) = make_float4(vv[0], vv[1], vv[2], vv[3]);
          }
        }
        if (p.ctx_q) {
          const float qs = quant_scale(amax);
          const float qinv = __fdiv_rn(1.0f, qs);
#pragma unroll 1
          for (int c = 0; c < DH; c += 32) {
            uint32_t o[32];
            tmem_ld32(tmem + lane_base + F_TM_O + c, o);
            tmem_wait_ld();
            uint32_t qw[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
            for (int m = 0; m < 32; m++) {
              const float vv = __fmaf_rn(__int2float_rn((int)o[m]), __fmul_rn(sp, __ldg(svh + c + m)), 0.0f);
              qw[m >> 2] |= ((uint32_t)quant_code(vv, qinv) & 0xFFu) << (8 * (m & 3));
            }
            if (valid) {
              uint4* dst = reinterpret_cast<uint4*>(p.ctx_q + orow * dmod + h * DH + c);
              dst[0] = make_uint4(qw[0], qw[1], qw[2], qw[3]);
              dst[1] = make_uint4(qw[4], qw[5], qw[6], qw[7]);
            }
          }
          if (valid) p.ctx_s[orow * p.H + h] = qs;
        }
        tc_fence_before();
        mbar_arrive(o_empty);
      }
    }
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, F_TMEM);
  }
}

// ------------------------------------------------------------------------------------------- prep kernels

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Quantise 4 values per lane (one 128-wide group per warp); returns the scale, writes 4 codes as one word.
__device__ __forceinline__ float quant128(const float (&v)[4], int8_t* dst, int lane) {
  float a = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
  a = warp_max(a);
  const float s = quant_scale(a);
  const float inv = __fdiv_rn(1.0f, s);
  uint32_t w = 0;
#pragma unroll
  for (int k = 0; k < 4; k++) w |= ((uint32_t)quant_code(v[k], inv) & 0xFFu) << (8 * k);
  *reinterpret_cast<uint32_t*>(dst + lane * 4) = w;
  return s;
}

// Qu = quant(q + bias_u), Qv = quant(q + bias_v), K = quant(k) per (token, head): encoder.rs:353-377.
__global__ void prep_qk_kernel(const float* __restrict__ qkv, int ld, int Mtot, int H, const float* __restrict__ bu,
                               const float* __restrict__ bv, int8_t* QU, int8_t* QV, int8_t* KH, float* squ,
                               float* sqv, float* sk) {
  const int lane = threadIdx.x & 31;
  const int nw = gridDim.x * (blockDim.x >> 5);
  for (int pr = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); pr < Mtot * H; pr += nw) {
    const int row = pr / H, h = pr % H;
    const float4 q4 = *reinterpret_cast<const float4*>(qkv + (size_t)row * ld + h * DH + lane * 4);
    const float4 k4 = *reinterpret_cast<const float4*>(qkv + (size_t)row * ld + H * DH + h * DH + lane * 4);
    const float4 u4 = *reinterpret_cast<const float4*>(bu + h * DH + lane * 4);
    const float4 v4 = *reinterpret_cast<const float4*>(bv + h * DH + lane * 4);
    const float qa[4] = {q4.x, q4.y, q4.z, q4.w}, ub[4] = {u4.x, u4.y, u4.z, u4.w}, vb[4] = {v4.x, v4.y, v4.z, v4.w};
    float a[4], b[4];
#pragma unroll
    for (int k = 0; k < 4; k++) {
      a[k] = __fadd_rn(qa[k], ub[k]);
      b[k] = __fadd_rn(qa[k], vb[k]);
    }
    const float kk[4] = {k4.x, k4.y, k4.z, k4.w};
    const size_t o = ((size_t)h * Mtot + row) * DH;
    const float s1 = quant128(a, QU + o, lane);
    const float s2 = quant128(b, QV + o, lane);
    const float s3 = quant128(kk, KH + o, lane);
    if (lane == 0) {
      squ[(size_t)h * Mtot + row] = s1;
      sqv[(size_t)h * Mtot + row] = s2;
      sk[(size_t)h * Mtot + row] = s3;
    }
  }
}

// R = quant(rel_k row, head slice) with transposed scales (encoder.rs:378-390).
__global__ void prep_rel_kernel(const float* __restrict__ rel, int NP, int H, int8_t* R, float* srelT) {
  const int lane = threadIdx.x & 31;
  const int nw = gridDim.x * (blockDim.x >> 5);
  for (int pr = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); pr < NP * H; pr += nw) {
    const int row = pr / H, h = pr % H;
    const float4 r4 = *reinterpret_cast<const float4*>(rel + (size_t)row * H * DH + h * DH + lane * 4);
    const float v[4] = {r4.x, r4.y, r4.z, r4.w};
    const float s = quant128(v, R + (size_t)row * H * DH + h * DH, lane);
    if (lane == 0) srelT[(size_t)h * NP + row] = s;
  }
}

// Vt[c] = quant(v[0..t, c]) over all frames (one group of t16, zero padded): encoder.rs:391-402. Two passes over the
// utterance's 64-row chunks (the batch plan's conv tiles), one block of 256 threads per (chunk, head):
// prep_v_max_kernel writes each chunk's column maxima of |v|; prep_v_quant_kernel combines the utterance's
// partials (max is order-free), quantises its chunk and writes it transposed through shared memory.
constexpr int VCH = 64;  // rows per chunk (= kConvTR)
__global__ void __launch_bounds__(256) prep_v_max_kernel(const float* __restrict__ qkv, int ld, int H,
                                                         const int* __restrict__ off, const int* __restrict__ len,
                                                         const int* __restrict__ tile_u,
                                                         const int* __restrict__ tile_r, float* __restrict__ part) {
  // thread (warp w, lane L) reads channels 4L .. 4L+3 of rows w, w + 8, ... (coalesced float4 rows, all in flight)
  __shared__ float red[8][DH];
  const int i = blockIdx.x, h = blockIdx.y, lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int u = tile_u[i], r0 = tile_r[i];
  const int n = min(VCH, len[u] - r0);
  const float* tile = qkv + (size_t)(off[u] + r0) * ld + 2 * H * DH + h * DH;
  float4 v[VCH / 8];
#pragma unroll
  for (int m = 0; m < VCH / 8; m++) {
    const int r = w + 8 * m;
    v[m] = r < n ? __ldg(reinterpret_cast<const float4*>(tile + (size_t)r * ld) + lane) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  float4 am = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int m = 0; m < VCH / 8; m++) {
    am.x = fmaxf(am.x, fabsf(v[m].x));
    am.y = fmaxf(am.y, fabsf(v[m].y));
    am.z = fmaxf(am.z, fabsf(v[m].z));
    am.w = fmaxf(am.w, fabsf(v[m].w));
  }
  reinterpret_cast<float4*>(red[w])[lane] = am;
  __syncthreads();
  if (threadIdx.x < DH) {
    float a = red[0][threadIdx.x];
#pragma unroll
    for (int k = 1; k < 8; k++) a = fmaxf(a, red[k][threadIdx.x]);
    part[((size_t)i * H + h) * DH + threadIdx.x] = a;
  }
}

// One block of 256 threads per (chunk, head): the chunk's 64 x 128 f32 tile comes in by coalesced float4 loads (all
// in flight) and is staged row-major in shared memory; thread (c, half) then reads channel c down 32 rows (a
// conflict-free column read), quantises with the channel's scale and writes its 32 codes as two 16-byte stores.
constexpr int VQ_THREADS = 256;
__global__ void __launch_bounds__(VQ_THREADS) prep_v_quant_kernel(const float* __restrict__ qkv, int ld, int H, int U,
                                                                  const int* __restrict__ off,
                                                                  const int* __restrict__ len,
                                                                  const int* __restrict__ voff,
                                                                  const int* __restrict__ tile_u,
                                                                  const int* __restrict__ tile_r,
                                                                  const float* __restrict__ part, int Mv, int8_t* VT,
                                                                  float* sv) {
  __shared__ __align__(16) float vt[VCH][DH];
  __shared__ float sinv[DH];
  const int i = blockIdx.x, h = blockIdx.y, tid = threadIdx.x;
  const int u = tile_u[i], r0 = tile_r[i], t = len[u];
  const int n = min(VCH, t - r0);
  const float* tile = qkv + (size_t)(off[u] + r0) * ld + 2 * H * DH + h * DH;
  float4 v[VCH * DH / 4 / VQ_THREADS];
#pragma unroll
  for (int m = 0; m < VCH * DH / 4 / VQ_THREADS; m++) {
    const int idx = tid + m * VQ_THREADS, r = idx / (DH / 4), c4 = idx % (DH / 4);
    v[m] = r < n ? __ldg(reinterpret_cast<const float4*>(tile + (size_t)r * ld) + c4) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  if (tid < DH) {
    const int first = i - r0 / VCH, nch = (t + VCH - 1) / VCH;
    float amax = 0.0f;
    for (int k = 0; k < nch; k++) amax = fmaxf(amax, part[((size_t)(first + k) * H + h) * DH + tid]);
    const float sc = quant_scale(amax);
    sinv[tid] = __fdiv_rn(1.0f, sc);
    if (r0 == 0) sv[((size_t)h * U + u) * DH + tid] = sc;
  }
#pragma unroll
  for (int m = 0; m < VCH * DH / 4 / VQ_THREADS; m++) {
    const int idx = tid + m * VQ_THREADS;
    reinterpret_cast<float4*>(&vt[idx / (DH / 4)][0])[idx % (DH / 4)] = v[m];
  }
  __syncthreads();
  const int c = tid % DH, half = tid / DH;  // rows 32 half .. 32 half + 31 of channel c
  const float inv = sinv[c];
  uint32_t w[8];
#pragma unroll
  for (int k = 0; k < 8; k++) {
    uint32_t x = 0;
#pragma unroll
    for (int b = 0; b < 4; b++) x |= ((uint32_t)quant_code(vt[half * 32 + 4 * k + b][c], inv) & 0xFFu) << (8 * b);
    w[k] = x;
  }
  const int nb = min(VCH, ((t + 15) & ~15) - r0);  // bytes of this chunk inside the 16-padded row (multiple of 16)
  int8_t* dst = VT + (size_t)h * DH * Mv + (size_t)c * Mv + voff[u] + r0 + half * 32;
  if (half * 32 < nb) *reinterpret_cast<uint4*>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
  if (half * 32 + 16 < nb) *reinterpret_cast<uint4*>(dst + 16) = make_uint4(w[4], w[5], w[6], w[7]);
}

}  // namespace attn
}  // namespace vxg

using namespace vxg;

namespace {

struct AttnLayout {
  size_t qu, qv, kh, squ, sqv, sk, r, srel, vt, sv, vpart, total;
};

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

AttnLayout attn_layout(int Mtot, int tmax, int U, int H, int Mv) {
  const int vchunks = (Mtot + attn::VCH - 1) / attn::VCH + U;  // >= the plan's 64-row tiles
  AttnLayout L;
  const int NP = 2 * tmax - 1;
  size_t o = 0;
  auto take = [&](size_t bytes) {
    size_t at = o;
    o += align256(bytes);
    return at;
  };
  L.qu = take((size_t)H * Mtot * attn::DH);
  L.qv = take((size_t)H * Mtot * attn::DH);
  L.kh = take((size_t)H * Mtot * attn::DH);
  L.squ = take((size_t)H * Mtot * 4);
  L.sqv = take((size_t)H * Mtot * 4);
  L.sk = take((size_t)H * Mtot * 4);
  L.r = take((size_t)NP * H * attn::DH);
  L.srel = take((size_t)H * NP * 4);
  L.vt = take((size_t)H * attn::DH * Mv);
  L.sv = take((size_t)H * U * attn::DH * 4);
  L.vpart = take((size_t)vchunks * H * attn::DH * 4);
  L.total = o;
  return L;
}

}  // namespace

namespace vxg {

void batch_plan(BatchPlan& b, const int* len, int n, int tmax) {
  b.n_utt = n;
  b.tmax = tmax;
  b.rows = 0;
  b.Mv = 0;
  std::vector<int> off(n), ln(n), voff(n), au, aq, cu, cr;
  for (int u = 0; u < n; u++) {
    off[u] = b.rows;
    ln[u] = len[u];
    voff[u] = b.Mv;
    b.rows += len[u];
    b.Mv += (len[u] + 15) & ~15;
    for (int q0 = 0; q0 < len[u]; q0 += kAttnBQ) {
      au.push_back(u);
      aq.push_back(q0);
    }
    for (int r0 = 0; r0 < len[u]; r0 += kConvTR) {
      cu.push_back(u);
      cr.push_back(r0);
    }
  }
  // Attention query tiles, costliest first (key tiles of the utterance, then rows in the tile): both attention
  // kernels hand out (tile, head) items in table order, so the last, partly filled wave holds the cheapest items.
  // Any order is valid: every tile's results go to its own rows.
  {
    std::vector<int> ord(au.size());
    for (size_t i = 0; i < ord.size(); i++) ord[i] = (int)i;
    auto key_tiles = [&](int i) { return (len[au[i]] + attn::BKV - 1) / attn::BKV; };
    auto rows_in = [&](int i) { return std::min(kAttnBQ, len[au[i]] - aq[i]); };
    std::stable_sort(ord.begin(), ord.end(), [&](int a, int c) {
      const int ka = key_tiles(a), kc = key_tiles(c);
      return ka != kc ? ka > kc : rows_in(a) > rows_in(c);
    });
    std::vector<int> su(ord.size()), sq(ord.size());
    for (size_t i = 0; i < ord.size(); i++) su[i] = au[ord[i]], sq[i] = aq[ord[i]];
    au.swap(su);
    aq.swap(sq);
  }
  b.att_tiles = (int)au.size();
  b.conv_tiles = (int)cu.size();
  b.tab.clear();
  auto put = [&](const std::vector<int>& v) {
    int at = (int)b.tab.size();
    b.tab.insert(b.tab.end(), v.begin(), v.end());
    return at;
  };
  b.o_off = put(off);
  b.o_len = put(ln);
  b.o_voff = put(voff);
  b.o_att_u = put(au);
  b.o_att_q = put(aq);
  b.o_conv_u = put(cu);
  b.o_conv_r = put(cr);
}

size_t attention_ws_bytes(int rows, int tmax, int n_utt, int heads, int Mv) {
  return attn_layout(rows, tmax, n_utt, heads, Mv).total;
}

QkQuant attention_qk_buffers(const BatchPlan& b, int heads, void* workspace) {
  const AttnLayout L = attn_layout(b.rows, b.tmax, b.n_utt, heads, b.Mv);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  QkQuant q;
  q.qu = (int8_t*)(ws + L.qu);
  q.qv = (int8_t*)(ws + L.qv);
  q.kh = (int8_t*)(ws + L.kh);
  q.squ = (float*)(ws + L.squ);
  q.sqv = (float*)(ws + L.sqv);
  q.sk = (float*)(ws + L.sk);
  q.heads = heads;
  return q;
}

vxg_status attention_run(const BatchPlan& b, const int* dtab, const float* qkv, int ld_qkv, const float* rel_k,
                         const float* bias_u, const float* bias_v, int heads, float scaling, float* ctx,
                         int8_t* ctx_q, float* ctx_s, void* workspace, size_t ws_bytes, cudaStream_t st,
                         bool qk_ready) {
  const int Mtot = b.rows, tmax = b.tmax, n_utt = b.n_utt, n_tiles = b.att_tiles, NP = 2 * tmax - 1, Mv = b.Mv;
  AttnLayout L = attn_layout(Mtot, tmax, n_utt, heads, Mv);
  if (ws_bytes < L.total) {
    set_error("attention workspace too small: %zu < %zu bytes", ws_bytes, L.total);
    return VXG_ERR_ARG;
  }
  int* status = device_status();
  VXG_ARG(status != nullptr, "no CUDA device");
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  const int* d_off = dtab + b.o_off;
  const int* d_len = dtab + b.o_len;
  const int* d_voff = dtab + b.o_voff;
  int8_t *QU = (int8_t*)(ws + L.qu), *QV = (int8_t*)(ws + L.qv), *KH = (int8_t*)(ws + L.kh);
  float *squ = (float*)(ws + L.squ), *sqv = (float*)(ws + L.sqv), *sk = (float*)(ws + L.sk);
  int8_t* R = (int8_t*)(ws + L.r);
  float* srelT = (float*)(ws + L.srel);
  int8_t* VT = (int8_t*)(ws + L.vt);
  float* sv = (float*)(ws + L.sv);
  const int nblk = std::max(1, std::min(sm_count() * 8, (Mtot * heads + 7) / 8));
  if (!qk_ready) {
    attn::prep_qk_kernel<<<nblk, 256, 0, st>>>(qkv, ld_qkv, Mtot, heads, bias_u, bias_v, QU, QV, KH, squ, sqv, sk);
    note_launch();
  }
  attn::prep_rel_kernel<<<std::max(1, std::min(sm_count() * 8, (NP * heads + 7) / 8)), 256, 0, st>>>(
      rel_k, NP, heads, R, srelT);
  note_launch();
  static_assert(attn::VCH == kConvTR, "V prep chunks are the plan's 64-row tiles");
  {
    const dim3 grid(b.conv_tiles, heads);
    const int* tu = dtab + b.o_conv_u;
    const int* tr = dtab + b.o_conv_r;
    float* part = (float*)(ws + L.vpart);
    attn::prep_v_max_kernel<<<grid, 256, 0, st>>>(qkv, ld_qkv, heads, d_off, d_len, tu, tr, part);
    attn::prep_v_quant_kernel<<<grid, attn::VQ_THREADS, 0, st>>>(qkv, ld_qkv, heads, n_utt, d_off, d_len, d_voff, tu,
                                                                 tr, part, Mv, VT, sv);
    note_launch(2);
  }
  VXG_CUDA(cudaGetLastError());
  CUtensorMap tqu, tqv, tk, tr, tv;
  vxg_status s;
  if ((s = make_tmap_2d_u8(&tqu, QU, (uint64_t)heads * Mtot, attn::DH, attn::DH, attn::BQ, attn::DH)) != VXG_OK) return s;
  if ((s = make_tmap_2d_u8(&tqv, QV, (uint64_t)heads * Mtot, attn::DH, attn::DH, attn::BQ, attn::DH)) != VXG_OK) return s;
  if ((s = make_tmap_2d_u8(&tk, KH, (uint64_t)heads * Mtot, attn::DH, attn::DH, attn::BKV, attn::DH)) != VXG_OK) return s;
  if ((s = make_tmap_2d_u8(&tr, R, (uint64_t)NP, (uint64_t)heads * attn::DH, (uint64_t)heads * attn::DH,
                           attn::BKV, attn::DH)) != VXG_OK)
    return s;
  if ((s = make_tmap_2d_u8(&tv, VT, (uint64_t)heads * attn::DH, (uint64_t)Mv, (uint64_t)Mv, attn::DH,
                           attn::BKV)) != VXG_OK)
    return s;
  if ((s = smem_attr((const void*)attn::attn_fused_kernel, (int)attn::F_SMEM)) != VXG_OK) return s;
  attn::Params p;
  p.tile_utt = dtab + b.o_att_u;
  p.tile_q0 = dtab + b.o_att_q;
  p.off = d_off;
  p.len = d_len;
  p.voff = d_voff;
  p.squ = squ;
  p.sqv = sqv;
  p.sk = sk;
  p.srelT = srelT;
  p.sv = sv;
  p.ctx = ctx;
  p.ctx_q = ctx_q;
  p.ctx_s = ctx_s;
  p.status = status;
  p.Mtot = Mtot;
  p.NP = NP;
  p.tmax = tmax;
  p.H = heads;
  p.U = n_utt;
  p.scaling = scaling;
  const int grid = std::min(n_tiles * heads, sm_count());
  attn::attn_fused_kernel<<<grid, attn::F_THREADS, attn::F_SMEM, st>>>(tqu, tqv, tk, tr, tv, p, n_tiles);
  note_launch();
  VXG_CUDA(cudaGetLastError());
  return VXG_OK;
}

}  // namespace vxg

extern "C" {

size_t vxg_attention_workspace_bytes(int rows, int tmax, int n_utt, int heads) {
  if (rows <= 0 || tmax <= 0 || n_utt <= 0 || heads <= 0) return 0;
  const int Mv = rows + 16 * n_utt;
  const int n_tiles = rows / attn::BQ + n_utt;
  const int n_conv = rows / kConvTR + n_utt;
  return ((attention_ws_bytes(rows, tmax, n_utt, heads, Mv) + 255) & ~size_t(255)) +
         (size_t)(3 * n_utt + 2 * n_tiles + 2 * n_conv) * 4 + 256;
}

vxg_status vxg_attention_i8(const float* qkv, int ld_qkv, const float* rel_k, int tmax, const int* off,
                            const int* len, int n_utt, const float* bias_u, const float* bias_v, int heads,
                            int head_dim, float scaling, float* ctx, int8_t* ctx_q, float* ctx_s, void* workspace,
                            size_t ws_bytes, void* stream) {
  clear_error();
  VXG_ARG(qkv && rel_k && off && len && bias_u && bias_v && workspace, "NULL pointer");
  VXG_ARG(head_dim == attn::DH, "head_dim must be 128 (got %d)", head_dim);
  VXG_ARG(heads > 0 && n_utt > 0 && tmax > 0, "bad sizes");
  VXG_ARG(ctx || ctx_q, "no output requested");
  VXG_ARG(!ctx_q || ctx_s, "ctx_q needs ctx_s");
  VXG_ARG(ld_qkv >= 3 * heads * attn::DH && ld_qkv % 4 == 0 && ((uintptr_t)qkv & 15) == 0,
          "qkv rows must hold q|k|v (3 * heads * 128 floats) with a 16-byte aligned stride");
  VXG_ARG(((uintptr_t)rel_k & 15) == 0 && ((uintptr_t)ctx & 15) == 0 && ((uintptr_t)ctx_q & 15) == 0, "alignment");
  int expect = 0;
  for (int u = 0; u < n_utt; u++) {
    VXG_ARG(len[u] > 0 && len[u] <= tmax, "utterance %d: len %d tmax %d", u, len[u], tmax);
    VXG_ARG(off[u] == expect, "utterances must be stacked in order without gaps (utterance %d at %d, expected %d)",
            u, off[u], expect);
    expect += len[u];
  }
  BatchPlan b;
  batch_plan(b, len, n_utt, tmax);
  const size_t att = (attention_ws_bytes(b.rows, tmax, n_utt, heads, b.Mv) + 255) & ~size_t(255);
  if (ws_bytes < att + b.tab.size() * 4) {
    set_error("workspace too small: %zu < %zu bytes", ws_bytes, att + b.tab.size() * 4);
    return VXG_ERR_ARG;
  }
  cudaStream_t st = (cudaStream_t)stream;
  int* dtab = reinterpret_cast<int*>(static_cast<uint8_t*>(workspace) + att);
  VXG_CUDA(cudaMemcpyAsync(dtab, b.tab.data(), b.tab.size() * 4, cudaMemcpyHostToDevice, st));
  return attention_run(b, dtab, qkv, ld_qkv, rel_k, bias_u, bias_v, heads, scaling, ctx, ctx_q, ctx_s, workspace,
                       att, st);
}

}  // extern "C"
