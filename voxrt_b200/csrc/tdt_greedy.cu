// TDT greedy decode on the GPU: Decoder::greedy (crates/voxrt/src/decoder.rs:204-266) for many utterances at once.
//
// Every utterance ("lane") takes exactly the steps of the reference's loop; the lanes advance in lockstep rounds so
// that one pass over the weights serves all of them. A round is
//   plan        lanes whose prediction-network output is stale (a token was emitted) and lanes not yet done;
//   pred step   for the stale lanes (Decoder::pred_step, decoder.rs:136-175): embedding row, per layer the int8
//               products W_ih q(x) + b and W_hh q(h) (gemm_single, kernels/mod.rs:285-315), the LSTM cell, then the
//               f32 decoder projector (gemv_f16, tensor.rs:529-600, dot_lanes8 order);
//   joint       for every unfinished lane (Decoder::joint, decoder.rs:178-192): relu(enc_t + g), int8 quantisation,
//               the int8 head product + bias, argmax over the vocabulary and over the durations;
//   step        the loop's bookkeeping (emission, state swap, symbol count, frame advance).
// The per-lane arithmetic is the host decoder's operation for operation (tdt.cpp): int8 group sums are exact
// integers (here from mma.sync m16n8k32 s8 products), the float chain over groups is
// acc = fma(float(S_g), sq[g] * s_row, acc) in group order, the cell uses the correctly rounded exp / tanh of
// crmath.cuh, and nothing is contracted (-fmad=false; explicit __f*_rn). So emissions are identical to the host's.
//
// Rounds are captured once per call into a CUDA graph and replayed in chunks, kDepth of them queued ahead of the
// host, which reads the number of unfinished lanes after the oldest; the GPU does not wait for the host between
// chunks unless the host falls kDepth - 1 chunks behind.
#include <algorithm>
#include <climits>
#include <cstring>
#include <vector>

#include "common.h"
#include "crmath.cuh"
#include "math.cuh"
#include "tdt.h"

namespace vxg {
namespace tdt {
namespace {

constexpr int kTileRows = 64;   // weight rows per product tile: 4 warps x 16
constexpr int kTileLanes = 64;  // lanes per product tile: 8 n-blocks of 8
constexpr int kProjLanes = 32;  // lanes per projector tile
constexpr int kRoundsPerGraph = 8;
constexpr int kDepth = 4;  // chunks of rounds queued ahead of the host's polling

struct Part {  // partial argmax over one 64-row block: value and row
  float v;
  int i;
};

__device__ __forceinline__ bool better(float v, int i, float bv, int bi) {  // first maximum under a strict '>'
  return v > bv || (v == bv && i < bi);
}

// Everything one round touches. Lane state is indexed by lane u; scratch rows by the lane's position j in the
// compacted list of its phase.
struct Args {
  // model
  const float* emb;
  const int8_t* w_ih[4];
  const int8_t* w_hh[4];
  const float* s_ih[4];
  const float* s_hh[4];
  const float* b[4];
  const float* proj_w;
  const float* proj_b;
  const int8_t* head_w;
  const float* head_s;
  const float* head_b;
  const int* durations;
  int hidden, vocab, n_dur, blank, max_symbols, n_layers, head_rows;
  // lanes
  int U;
  int* list_pred;  // [U] lanes needing a prediction-network step
  int* list_act;   // [U] unfinished lanes
  int* counts;     // [0] = stale lanes, [1] = unfinished lanes
  const int* t;    // frames per lane
  const long long* off;  // first frame row of each lane in proj
  const float* proj;     // [sum t, hidden] projected encoder frames
  int* tf;
  int* sym;
  int* last;
  int* have;  // may be null (single pred steps)
  int* done;
  int* nemit;
  int* cur;   // [U] state selector (greedy), or null
  float* H;   // [U, n_layers, hidden] state
  float* C;
  float* Hn;  // state after the lane's latest pred step
  float* Cn;
  float* G;   // [U, hidden] prediction-network output
  // scratch by list position
  float* gates;  // [U, 4 hidden]
  int8_t* qx;    // [U, hidden]
  int8_t* qh;
  float* sqx;    // [U, hidden / 128]
  float* sqh;
  Part* part;    // [U, head_rows / 64]
  float* dlog;   // [U, n_dur]
  float* logits; // [U, vocab + n_dur] or null
  vxg_emission* out;
  const long long* out_off;  // [U + 1] utterance u's emissions at out + out_off[u], capacity out_off[u + 1] - out_off[u]
};

// ------------------------------------------------------------------------------------------------ plan
// Compacts the lanes of each phase, in lane order. One block of 1024 threads.
__global__ void __launch_bounds__(1024) plan_kernel(Args a) {
  __shared__ int wp[32], wa[32], base[2];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) base[0] = base[1] = 0;
  __syncthreads();
  for (int u0 = 0; u0 < a.U; u0 += 1024) {
    const int u = u0 + tid;
    const bool act = u < a.U && !a.done[u];
    const bool pred = act && !a.have[u];
    const unsigned bp = __ballot_sync(0xffffffffu, pred), ba = __ballot_sync(0xffffffffu, act);
    if (lane == 0) wp[warp] = __popc(bp), wa[warp] = __popc(ba);
    __syncthreads();
    int op = base[0], oa = base[1];
    for (int w = 0; w < warp; w++) op += wp[w], oa += wa[w];
    const unsigned below = (1u << lane) - 1u;
    if (pred) a.list_pred[op + __popc(bp & below)] = u;
    if (act) a.list_act[oa + __popc(ba & below)] = u;
    __syncthreads();
    if (tid == 0) {
      int sp = 0, sa = 0;
      for (int w = 0; w < 32; w++) sp += wp[w], sa += wa[w];
      base[0] += sp, base[1] += sa;
    }
    __syncthreads();
  }
  if (tid == 0) a.counts[0] = base[0], a.counts[1] = base[1];
}

// ------------------------------------------------------------------------------------------------ state
// Greedy mode keeps two state buffers per lane (H/C and Hn/Cn) and a per-lane selector `cur`: a prediction step
// reads the current one and writes the other; an emission flips the selector (decoder.rs:238-240 takes the new
// state) instead of copying it. Without a selector (single steps) H/C are the inputs and Hn/Cn the outputs.
__device__ __forceinline__ bool flipped(const Args& a, int u) { return a.cur && a.cur[u]; }
__device__ __forceinline__ size_t srow(const Args& a, int u, int l) {
  return ((size_t)u * a.n_layers + l) * a.hidden;
}
__device__ __forceinline__ const float* h_in(const Args& a, int u, int l) {
  return (flipped(a, u) ? a.Hn : a.H) + srow(a, u, l);
}
__device__ __forceinline__ const float* c_in(const Args& a, int u, int l) {
  return (flipped(a, u) ? a.Cn : a.C) + srow(a, u, l);
}
__device__ __forceinline__ float* h_out(const Args& a, int u, int l) {
  return (flipped(a, u) ? a.H : a.Hn) + srow(a, u, l);
}
__device__ __forceinline__ float* c_out(const Args& a, int u, int l) {
  return (flipped(a, u) ? a.C : a.Cn) + srow(a, u, l);
}

// ------------------------------------------------------------------------------------------------ quantise
// QuantAct::quantize_layout of one 128-wide group (packed.rs:527-535) by a block of 128 threads, one value each:
// s = amax / 127 (1 if all zero), code = clamp(round_ties_even(v * (1 / s)), -127, 127).
__device__ __forceinline__ void quant_group128(float v, int8_t* q, float* sq, float* red) {
  float m = fabsf(v);
#pragma unroll
  for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  const int w = threadIdx.x >> 5;
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[w] = m;
  __syncthreads();
  const float amax = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
  const float s = quant_scale(amax);
  q[threadIdx.x] = (int8_t)quant_code(v, __fdiv_rn(1.0f, s));
  if (threadIdx.x == 0) *sq = s;
}

// Inputs of LSTM layer l for the stale lanes, quantised: x (layer 0: the embedding row of the last token; above:
// layer l - 1's new h) and the layer's previous h. Layers above 0 get theirs from cell_kernel.
__global__ void __launch_bounds__(128) layer_quant_kernel(Args a, int l) {
  __shared__ float red[4];
  const int h = a.hidden, ng = h / 128, n = a.counts[0];
  for (int w = blockIdx.x; w < n * ng; w += gridDim.x) {
    const int j = w / ng, g = w % ng, u = a.list_pred[j], k = g * 128 + threadIdx.x;
    const float x = l == 0 ? a.emb[(size_t)a.last[u] * h + k] : h_out(a, u, l - 1)[k];
    quant_group128(x, a.qx + (size_t)j * h + g * 128, a.sqx + (size_t)j * ng + g, red);
    quant_group128(h_in(a, u, l)[k], a.qh + (size_t)j * h + g * 128, a.sqh + (size_t)j * ng + g, red);
  }
}

// Joint input of the unfinished lanes: z = max(enc_t + g, 0), quantised (decoder.rs:178-186).
__global__ void __launch_bounds__(128) joint_quant_kernel(Args a) {
  __shared__ float red[4];
  const int h = a.hidden, ng = h / 128, n = a.counts[1];
  for (int w = blockIdx.x; w < n * ng; w += gridDim.x) {
    const int j = w / ng, g = w % ng, u = a.list_act[j], k = g * 128 + threadIdx.x;
    const float e = a.proj[(size_t)(a.off[u] + a.tf[u]) * h + k];
    const float z = fmaxf(__fadd_rn(e, a.G[(size_t)u * h + k]), 0.0f);
    quant_group128(z, a.qx + (size_t)j * h + g * 128, a.sqx + (size_t)j * ng + g, red);
  }
}

// ------------------------------------------------------------------------------------------------ int8 products
__device__ __forceinline__ void mma_s8(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                       uint32_t b1) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"((uint32_t)__cvta_generic_to_shared(dst)),
               "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

// A product tile is 64 weight rows x 64 lanes. Its K loop runs over 128-wide groups ("steps"); each step's weight
// slice [64 rows][128 B] and activation slice [64 lanes][128 B] are brought into one of kStages shared-memory slots
// by cp.async, kStages - 1 steps ahead of the tensor-core work. In a slot, row r's 16-byte chunk c sits at chunk
// c ^ 4 (r & 1), which makes the fragment loads below free of bank conflicts.
constexpr int kStages = 4;
constexpr int kSlotBytes = 2 * 64 * 128;

struct Operand {  // one int8 product: weight rows + row scales, activation codes + group scales
  const int8_t* w;
  const float* ws;
  const int8_t* q;
  const float* sq;
};

__device__ __forceinline__ void load_step(uint8_t* slot, const Operand& o, int r0, int j0, int n, int h, int g) {
  uint8_t* sw = slot;
  uint8_t* sx = slot + 64 * 128;
  for (int i = threadIdx.x; i < 64 * 8; i += blockDim.x) {
    const int r = i >> 3, c = i & 7, pc = (c ^ ((r & 1) << 2)) * 16;
    cp_async16(sw + r * 128 + pc, o.w + (size_t)(r0 + r) * h + g * 128 + c * 16);
    const int jr = min(j0 + r, n - 1);  // lanes past n repeat the last one; their results are not stored
    cp_async16(sx + r * 128 + pc, o.q + (size_t)jr * h + g * 128 + c * 16);
  }
}

template <int NOP>
__device__ __forceinline__ Operand pick(const Operand (&op)[NOP], int i) {  // op[i] without a dynamic local index
  Operand o = op[0];
#pragma unroll
  for (int p = 1; p < NOP; p++)
    if (i == p) o = op[p];
  return o;
}

// Group scales of the tile's lanes, zero past n.
__device__ __forceinline__ void stage_scales(const float* sq, int j0, int n, int ng, float* sqs) {
  for (int i = threadIdx.x; i < 64 * ng; i += blockDim.x) {
    const int r = i / ng;
    sqs[i] = j0 + r < n ? sq[(size_t)(j0 + r) * ng + i % ng] : 0.0f;
  }
}

// gemm_single (kernels/mod.rs:285-315) for one tile and NOP operands summed over the same rows: per operand and
// group the exact int32 sums S_g from m16n8k32 products, then acc = fma(float(S_g), sq[lane][g] * s_row, acc) in
// group order. Warp w owns rows 16w + (gid, gid + 8); acc[op][nb] holds those rows x lanes nb * 8 + 2 tig + {0, 1}
// in the mma accumulator order. Inside a 32-wide product the k order is permuted identically for both operands
// (thread tig carries bytes tig*16 .. tig*16+15 of each 64-byte half group), which leaves every integer sum as it
// is. sqs: [NOP][64][ng] shared scratch for the group scales of the tile's lanes, staged here while the first
// slots load.
template <int NOP>
__device__ __forceinline__ void tile_products(const Operand (&op)[NOP], int r0, int j0, int n, int h,
                                              uint8_t* slots, float* sqs, float (&acc)[NOP][8][4]) {
  const int ng = h / 128, steps = NOP * ng;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, gid = lane >> 2, tig = lane & 3;
  const int swz = (gid & 1) << 2;
  const int nbn = min(8, (n - j0 + 7) >> 3);  // n-blocks holding live lanes
  float s_lo[NOP], s_hi[NOP];
#pragma unroll
  for (int p = 0; p < NOP; p++) {
    s_lo[p] = op[p].ws[r0 + warp * 16 + gid];
    s_hi[p] = op[p].ws[r0 + warp * 16 + gid + 8];
#pragma unroll
    for (int nb = 0; nb < 8; nb++)
#pragma unroll
      for (int e = 0; e < 4; e++) acc[p][nb][e] = 0.0f;
  }
#pragma unroll
  for (int s = 0; s < kStages - 1; s++) {
    if (s < steps) load_step(slots + s * kSlotBytes, pick(op, s / ng), r0, j0, n, h, s % ng);
    cp_async_commit();
  }
#pragma unroll
  for (int p = 0; p < NOP; p++) stage_scales(op[p].sq, j0, n, ng, sqs + p * 64 * ng);  // ordered by the first sync
#pragma unroll 1
  for (int s = 0; s < steps; s++) {
    const int ls = s + kStages - 1;
    if (ls < steps) load_step(slots + (ls % kStages) * kSlotBytes, pick(op, ls / ng), r0, j0, n, h, ls % ng);
    cp_async_commit();
    cp_async_wait<kStages - 1>();
    __syncthreads();
    const uint8_t* sw = slots + (s % kStages) * kSlotBytes;
    const uint8_t* sx = sw + 64 * 128;
    const uint8_t* wl = sw + (warp * 16 + gid) * 128;
    const uint4 lo0 = *reinterpret_cast<const uint4*>(wl + ((tig ^ swz) << 4));
    const uint4 lo1 = *reinterpret_cast<const uint4*>(wl + (((tig + 4) ^ swz) << 4));
    const uint4 hi0 = *reinterpret_cast<const uint4*>(wl + 8 * 128 + ((tig ^ swz) << 4));
    const uint4 hi1 = *reinterpret_cast<const uint4*>(wl + 8 * 128 + (((tig + 4) ^ swz) << 4));
    const int p = s / ng, g = s % ng;
    const float* sq = sqs + (size_t)p * 64 * ng;
#pragma unroll
    for (int hb = 0; hb < 2; hb++) {  // n-blocks 4 hb .. 4 hb + 3, skipped when they hold no live lane
      if (hb * 4 >= nbn) break;
      uint4 x0[4], x1[4];
      int c[4][4];
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const uint8_t* xr = sx + ((hb * 4 + i) * 8 + gid) * 128;
        x0[i] = *reinterpret_cast<const uint4*>(xr + ((tig ^ swz) << 4));
        x1[i] = *reinterpret_cast<const uint4*>(xr + (((tig + 4) ^ swz) << 4));
        c[i][0] = c[i][1] = c[i][2] = c[i][3] = 0;
      }
      // k-outer order: four independent accumulator chains between dependent products
#pragma unroll
      for (int i = 0; i < 4; i++) mma_s8(c[i], lo0.x, hi0.x, lo0.y, hi0.y, x0[i].x, x0[i].y);
#pragma unroll
      for (int i = 0; i < 4; i++) mma_s8(c[i], lo0.z, hi0.z, lo0.w, hi0.w, x0[i].z, x0[i].w);
#pragma unroll
      for (int i = 0; i < 4; i++) mma_s8(c[i], lo1.x, hi1.x, lo1.y, hi1.y, x1[i].x, x1[i].y);
#pragma unroll
      for (int i = 0; i < 4; i++) mma_s8(c[i], lo1.z, hi1.z, lo1.w, hi1.w, x1[i].z, x1[i].w);
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const int nb = hb * 4 + i;
        const float sq0 = sq[(nb * 8 + 2 * tig) * ng + g], sq1 = sq[(nb * 8 + 2 * tig + 1) * ng + g];
#pragma unroll
        for (int q = 0; q < NOP; q++)
          if (q == p) {  // static register indexing: the operand of this step
            acc[q][nb][0] = __fmaf_rn(__int2float_rn(c[i][0]), __fmul_rn(sq0, s_lo[q]), acc[q][nb][0]);
            acc[q][nb][1] = __fmaf_rn(__int2float_rn(c[i][1]), __fmul_rn(sq1, s_lo[q]), acc[q][nb][1]);
            acc[q][nb][2] = __fmaf_rn(__int2float_rn(c[i][2]), __fmul_rn(sq0, s_hi[q]), acc[q][nb][2]);
            acc[q][nb][3] = __fmaf_rn(__int2float_rn(c[i][3]), __fmul_rn(sq1, s_hi[q]), acc[q][nb][3]);
          }
      }
    }
    __syncthreads();  // the slot is refilled kStages - 1 steps later
  }
}

// ------------------------------------------------------------------------------------------------ few lanes
// With few lanes (the end of a batch, or long-form segments) a 64 x 64 product tile staged through a cp.async ring
// leaves most of the GPU idle and pays one memory round trip per 128-wide group. Then the block copies the lanes'
// activation codes into shared memory once, and each warp takes 16 weight rows and loads the m16n8k32 fragments of
// all their groups from global memory at once (16-byte loads in the tile path's permuted k order), so a product
// costs one round trip; the integer sums and the float chain are the tile path's, step for step.
constexpr int kFewLanes = 16;     // two n-blocks of 8 lanes
constexpr int kFewMaxGroups = 5;  // hidden <= 640: every group's fragments fit in registers

__device__ __forceinline__ uint4 ldg16(const void* p) { return __ldg(reinterpret_cast<const uint4*>(p)); }

// Rows 0 .. n-1 of an activation operand ([n][h] int8, contiguous) into shared memory.
__device__ __forceinline__ void stage_rows(const int8_t* q, int n, int h, int8_t* xs) {
  const int chunks = n * h / 16;
  for (int i = threadIdx.x; i < chunks; i += blockDim.x)
    reinterpret_cast<uint4*>(xs)[i] = __ldg(reinterpret_cast<const uint4*>(q) + i);
}

// acc[nb][e] for rows r0 + gid (e < 2) and r0 + gid + 8 (e >= 2), list positions nb * 8 + 2 tig + (e & 1): the
// chain acc = fma(float(S_g), sq[j][g] * s_row, acc) over the NG groups in order, from 0 (gemm_single,
// kernels/mod.rs:285-315). xs: the operand's activation rows in shared memory. Positions past n repeat the last
// one; their scales are 0 and their results unused.
template <int NG>
__device__ __forceinline__ void warp_rows16(const Operand& o, const int8_t* xs, int r0, int n, float (&acc)[2][4]) {
  constexpr int h = NG * 128;
  const int lane = threadIdx.x & 31, gid = lane >> 2, tig = lane & 3;
  const int8_t* wl = o.w + (size_t)(r0 + gid) * h + tig * 16;
  const int8_t* wh = wl + (size_t)8 * h;
  uint4 lo0[NG], lo1[NG], hi0[NG], hi1[NG];
#pragma unroll
  for (int g = 0; g < NG; g++) {  // all groups in flight
    lo0[g] = ldg16(wl + g * 128);
    lo1[g] = ldg16(wl + g * 128 + 64);
    hi0[g] = ldg16(wh + g * 128);
    hi1[g] = ldg16(wh + g * 128 + 64);
  }
  const float s_lo = o.ws[r0 + gid], s_hi = o.ws[r0 + gid + 8];
  const int nbn = n > 8 ? 2 : 1;
#pragma unroll
  for (int nb = 0; nb < 2; nb++) {
#pragma unroll
    for (int e = 0; e < 4; e++) acc[nb][e] = 0.0f;
    if (nb >= nbn) continue;
    const int8_t* xr = xs + min(nb * 8 + gid, n - 1) * h + tig * 16;
    const int j0 = nb * 8 + 2 * tig, j1 = j0 + 1;
#pragma unroll
    for (int g = 0; g < NG; g++) {
      const uint4 x0 = *reinterpret_cast<const uint4*>(xr + g * 128);
      const uint4 x1 = *reinterpret_cast<const uint4*>(xr + g * 128 + 64);
      int c[4] = {0, 0, 0, 0};
      mma_s8(c, lo0[g].x, hi0[g].x, lo0[g].y, hi0[g].y, x0.x, x0.y);
      mma_s8(c, lo0[g].z, hi0[g].z, lo0[g].w, hi0[g].w, x0.z, x0.w);
      mma_s8(c, lo1[g].x, hi1[g].x, lo1[g].y, hi1[g].y, x1.x, x1.y);
      mma_s8(c, lo1[g].z, hi1[g].z, lo1[g].w, hi1[g].w, x1.z, x1.w);
      const float sq0 = j0 < n ? o.sq[(size_t)j0 * NG + g] : 0.0f;
      const float sq1 = j1 < n ? o.sq[(size_t)j1 * NG + g] : 0.0f;
      acc[nb][0] = __fmaf_rn(__int2float_rn(c[0]), __fmul_rn(sq0, s_lo), acc[nb][0]);
      acc[nb][1] = __fmaf_rn(__int2float_rn(c[1]), __fmul_rn(sq1, s_lo), acc[nb][1]);
      acc[nb][2] = __fmaf_rn(__int2float_rn(c[2]), __fmul_rn(sq0, s_hi), acc[nb][2]);
      acc[nb][3] = __fmaf_rn(__int2float_rn(c[3]), __fmul_rn(sq1, s_hi), acc[nb][3]);
    }
  }
}

// gates for the stale lanes, few-lane form: a warp per 16 gate rows.
template <int NG>
__device__ void gates_few(const Args& a, int l, int n, const Operand (&op)[2], int8_t* xs) {
  constexpr int h = NG * 128, rows = 4 * h;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, gid = lane >> 2, tig = lane & 3;
  int8_t* xs1 = xs + kFewLanes * h;
  stage_rows(op[0].q, n, h, xs);
  stage_rows(op[1].q, n, h, xs1);
  __syncthreads();
  for (int t = blockIdx.x * 4 + warp; t < rows / 16; t += gridDim.x * 4) {
    const int r0 = t * 16;
    float ai[2][4], ah[2][4];
    warp_rows16<NG>(op[0], xs, r0, n, ai);
    warp_rows16<NG>(op[1], xs1, r0, n, ah);
    const int rlo = r0 + gid;
    const float b_lo = a.b[l][rlo], b_hi = a.b[l][rlo + 8];
#pragma unroll
    for (int nb = 0; nb < 2; nb++)
#pragma unroll
      for (int e = 0; e < 4; e++) {
        const int j = nb * 8 + 2 * tig + (e & 1), r = rlo + (e >> 1) * 8;
        if (j < n) a.gates[(size_t)j * rows + r] = __fadd_rn(__fadd_rn(ai[nb][e], (e >> 1) ? b_hi : b_lo), ah[nb][e]);
      }
  }
}

// LSTM layer l gates of the stale lanes: gates = (W_ih q(x) + b) + W_hh q(h) (decoder.rs:150-160).
__global__ void __launch_bounds__(128) gates_kernel(Args a, int l) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int h = a.hidden, n = a.counts[0], rows = 4 * h;
  uint8_t* slots = smem;
  float* sqs = reinterpret_cast<float*>(smem + kStages * kSlotBytes);  // [2][64][ng]
  const int nrb = rows / kTileRows, tiles = nrb * ((n + kTileLanes - 1) / kTileLanes);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, gid = lane >> 2, tig = lane & 3;
  const Operand op[2] = {{a.w_ih[l], a.s_ih[l], a.qx, a.sqx}, {a.w_hh[l], a.s_hh[l], a.qh, a.sqh}};
  if (n <= kFewLanes && h <= kFewMaxGroups * 128) {  // block-uniform
    if (n == 0) return;
    int8_t* xs = reinterpret_cast<int8_t*>(smem);  // the lanes' codes of both operands (in the slot area)
    switch (h / 128) {
      case 1: gates_few<1>(a, l, n, op, xs); break;
      case 2: gates_few<2>(a, l, n, op, xs); break;
      case 3: gates_few<3>(a, l, n, op, xs); break;
      case 4: gates_few<4>(a, l, n, op, xs); break;
      default: gates_few<5>(a, l, n, op, xs); break;
    }
    return;
  }
  for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
    const int rb = t % nrb, j0 = (t / nrb) * kTileLanes, r0 = rb * kTileRows;
    float acc[2][8][4];
    tile_products<2>(op, r0, j0, n, h, slots, sqs, acc);
    const int rlo = r0 + warp * 16 + gid;
    const float b_lo = a.b[l][rlo], b_hi = a.b[l][rlo + 8];
#pragma unroll
    for (int nb = 0; nb < 8; nb++)
#pragma unroll
      for (int e = 0; e < 4; e++) {
        const int j = j0 + nb * 8 + 2 * tig + (e & 1), r = rlo + (e >> 1) * 8;
        if (j < n)
          a.gates[(size_t)j * rows + r] = __fadd_rn(__fadd_rn(acc[0][nb][e], (e >> 1) ? b_hi : b_lo), acc[1][nb][e]);
      }
  }
}

// LSTM cell of layer l (decoder.rs:161-171) for the stale lanes, one hidden unit per thread: i = sigmoid,
// f = sigmoid, g = tanh, o = sigmoid; c' = f c + i g; h' = o tanh(c'); then the next layer's inputs, quantised.
__global__ void __launch_bounds__(128) cell_kernel(Args a, int l) {
  __shared__ float red[4];
  const int h = a.hidden, ng = h / 128, n = a.counts[0], nl = a.n_layers;
  for (int w = blockIdx.x; w < n * ng; w += gridDim.x) {
    const int j = w / ng, g = w % ng, u = a.list_pred[j], k = g * 128 + threadIdx.x;
    const float* gt = a.gates + (size_t)j * 4 * h;
    const float i = __fdiv_rn(1.0f, __fadd_rn(1.0f, crm::expf_cr(-gt[k])));
    const float f = __fdiv_rn(1.0f, __fadd_rn(1.0f, crm::expf_cr(-gt[h + k])));
    const float gg = crm::tanhf_cr(gt[2 * h + k]);
    const float o = __fdiv_rn(1.0f, __fadd_rn(1.0f, crm::expf_cr(-gt[3 * h + k])));
    const float cn = __fadd_rn(__fmul_rn(f, c_in(a, u, l)[k]), __fmul_rn(i, gg));
    const float hn = __fmul_rn(o, crm::tanhf_cr(cn));
    c_out(a, u, l)[k] = cn;
    h_out(a, u, l)[k] = hn;
    if (l + 1 < nl) {
      quant_group128(hn, a.qx + (size_t)j * h + g * 128, a.sqx + (size_t)j * ng + g, red);
      quant_group128(h_in(a, u, l + 1)[k], a.qh + (size_t)j * h + g * 128, a.sqh + (size_t)j * ng + g, red);
    }
  }
}

// Decoder projector of the stale lanes (gemv_f16 in dot_lanes8 order, tensor.rs:267-281): per row, lanes l of
// a and b accumulate x[c + l] * w[c + l] and x[c + 4 + l] * w[c + 4 + l] over 8-column steps (fma), then
// ((a0 + b0) + (a1 + b1)) + ((a2 + b2) + (a3 + b3)) + bias. Tiles of 64 rows x 32 lanes; a thread owns 4 rows x
// 2 lanes (rows 8 apart, lanes 2 apart), so that each shared-memory load of a warp reads 8 (weights) or 4
// (activations) distinct 16-byte chunks in distinct banks and feeds 4 or 8 threads. The K loop runs over 64-column
// chunks through a 4-slot cp.async ring; rows are padded to 68 floats. Warps whose lanes are all past n skip the math.
constexpr int kProjChunk = 64, kProjLd = 68, kProjStages = 4;
__global__ void __launch_bounds__(256, 2) proj_kernel(Args a) {
  extern __shared__ __align__(16) uint8_t smem[];
  float* ws = reinterpret_cast<float*>(smem);      // [kProjStages][64][kProjLd]
  float* xs = ws + kProjStages * 64 * kProjLd;      // [kProjStages][32][kProjLd]
  const int h = a.hidden, n = a.counts[0], nl = a.n_layers, chunks = h / kProjChunk;
  const int nrb = h / 64, tiles = nrb * ((n + kProjLanes - 1) / kProjLanes);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rbase = (warp & 1) * 32 + (lane & 7);           // rows rbase + 8 i
  const int lbase = ((warp >> 1) * 4 + (lane >> 3)) * 2;    // lanes lbase + e
  if (n <= kFewLanes) {
    if (n == 0) return;
    // eight threads per output (row, lane): thread l8 runs chain l8 (column c + l8 of every 8-column step), then
    // ((s0 + s4) + (s1 + s5)) + ((s2 + s6) + (s3 + s7)) + bias across the eight by shuffles; four outputs per warp
    const int l8 = lane & 7, nout = h * n, nw = gridDim.x * 8;
    for (int base = (blockIdx.x * 8 + warp) * 4; base < nout; base += nw * 4) {  // warp-uniform trip count
      const int o = base + (lane >> 3);
      float s = 0.0f;
      int row = 0, u = 0;
      if (o < nout) {
        row = o % h;
        u = a.list_pred[o / h];
        const float* x = h_out(a, u, nl - 1);
        const float* w = a.proj_w + (size_t)row * h;
#pragma unroll 8
        for (int c = 0; c < h; c += 8) s = __fmaf_rn(__ldg(x + c + l8), __ldg(w + c + l8), s);
      }
      const float p = __fadd_rn(s, __shfl_down_sync(0xffffffffu, s, 4));  // s_l + s_{l+4}, lanes l8 < 4
      const float q = __fadd_rn(p, __shfl_down_sync(0xffffffffu, p, 1));  // (p0 + p1), (p2 + p3) at l8 = 0, 2
      const float v = __fadd_rn(q, __shfl_down_sync(0xffffffffu, q, 2));  // at l8 = 0
      if (o < nout && l8 == 0) {
        a.G[(size_t)u * h + row] = __fadd_rn(v, a.proj_b[row]);
        if (row == 0 && a.have) a.have[u] = 1;
      }
    }
    return;
  }
  for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
    const int rb = t % nrb, j0 = (t / nrb) * kProjLanes;
    const bool live = j0 + (warp >> 1) * 8 < n;  // warp-uniform
    auto load = [&](int kc) {
      float* wb = ws + (kc % kProjStages) * 64 * kProjLd;
      float* xb = xs + (kc % kProjStages) * kProjLanes * kProjLd;
      for (int i = threadIdx.x; i < 64 * 16; i += 256) {
        const int rr = i >> 4, c4 = i & 15;
        cp_async16(wb + rr * kProjLd + c4 * 4, a.proj_w + (size_t)(rb * 64 + rr) * h + kc * kProjChunk + c4 * 4);
      }
      for (int i = threadIdx.x; i < kProjLanes * 16; i += 256) {
        const int jj = i >> 4, c4 = i & 15, u = a.list_pred[min(j0 + jj, n - 1)];
        cp_async16(xb + jj * kProjLd + c4 * 4, h_out(a, u, nl - 1) + kc * kProjChunk + c4 * 4);
      }
    };
    float acc[4][2][8];
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
      for (int e = 0; e < 2; e++)
#pragma unroll
        for (int q = 0; q < 8; q++) acc[i][e][q] = 0.0f;
#pragma unroll
    for (int kc = 0; kc < kProjStages - 1; kc++) {
      if (kc < chunks) load(kc);
      cp_async_commit();
    }
    for (int kc = 0; kc < chunks; kc++) {
      if (kc + kProjStages - 1 < chunks) load(kc + kProjStages - 1);
      cp_async_commit();
      cp_async_wait<kProjStages - 1>();
      __syncthreads();
      if (live) {
        const float* wb = ws + (kc % kProjStages) * 64 * kProjLd + rbase * kProjLd;
        const float* xb = xs + (kc % kProjStages) * kProjLanes * kProjLd + lbase * kProjLd;
#pragma unroll 1
        for (int c = 0; c < kProjChunk; c += 8) {
          float4 x0[2], x1[2];
#pragma unroll
          for (int e = 0; e < 2; e++) {
            x0[e] = *reinterpret_cast<const float4*>(xb + e * kProjLd + c);
            x1[e] = *reinterpret_cast<const float4*>(xb + e * kProjLd + c + 4);
          }
#pragma unroll
          for (int i = 0; i < 4; i++) {
            const float4 w0 = *reinterpret_cast<const float4*>(wb + i * 8 * kProjLd + c);
            const float4 w1 = *reinterpret_cast<const float4*>(wb + i * 8 * kProjLd + c + 4);
#pragma unroll
            for (int e = 0; e < 2; e++) {
              float* s = acc[i][e];
              s[0] = __fmaf_rn(x0[e].x, w0.x, s[0]);
              s[1] = __fmaf_rn(x0[e].y, w0.y, s[1]);
              s[2] = __fmaf_rn(x0[e].z, w0.z, s[2]);
              s[3] = __fmaf_rn(x0[e].w, w0.w, s[3]);
              s[4] = __fmaf_rn(x1[e].x, w1.x, s[4]);
              s[5] = __fmaf_rn(x1[e].y, w1.y, s[5]);
              s[6] = __fmaf_rn(x1[e].z, w1.z, s[6]);
              s[7] = __fmaf_rn(x1[e].w, w1.w, s[7]);
            }
          }
        }
      }
      __syncthreads();  // the slot is refilled kProjStages - 1 chunks later
    }
    if (!live) continue;
#pragma unroll
    for (int e = 0; e < 2; e++) {
      const int j = j0 + lbase + e;
      if (j >= n) continue;
      const int u = a.list_pred[j];
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const int row = rb * 64 + rbase + 8 * i;
        const float* s = acc[i][e];
        const float v = __fadd_rn(__fadd_rn(__fadd_rn(s[0], s[4]), __fadd_rn(s[1], s[5])),
                                  __fadd_rn(__fadd_rn(s[2], s[6]), __fadd_rn(s[3], s[7])));
        a.G[(size_t)u * h + row] = __fadd_rn(v, a.proj_b[row]);
      }
      if (rb == 0 && rbase == 0 && a.have) a.have[u] = 1;
    }
  }
}

// Joint head of the unfinished lanes (int8 product + bias, decoder.rs:186-191) with the vocabulary argmax folded
// in: each 64-row block leaves its first maximum per lane in `part`; duration logits go to `dlog`.
__global__ void __launch_bounds__(128) head_kernel(Args a) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int h = a.hidden, n = a.counts[1], ng = h / 128, nout = a.vocab + a.n_dur;
  uint8_t* slots = smem;
  float* sqs = reinterpret_cast<float*>(smem + kStages * kSlotBytes);  // [64][ng]
  Part* red = reinterpret_cast<Part*>(sqs + 64 * ng);                  // [4 warps][64 lanes]
  const int nrb = a.head_rows / kTileRows, tiles = nrb * ((n + kTileLanes - 1) / kTileLanes);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, gid = lane >> 2, tig = lane & 3;
  const Operand op[1] = {{a.head_w, a.head_s, a.qx, a.sqx}};
  // few lanes (block-uniform): the lanes' codes staged once, then a warp per 16 rows of each 64-row block
  const bool few = n <= kFewLanes && h <= kFewMaxGroups * 128;
  if (few) {
    if (n == 0) return;
    stage_rows(a.qx, n, h, reinterpret_cast<int8_t*>(slots));
    __syncthreads();
  }
  for (int t = blockIdx.x; t < (few ? nrb : tiles); t += gridDim.x) {
    const int rb = few ? t : t % nrb, j0 = few ? 0 : (t / nrb) * kTileLanes, r0 = rb * kTileRows;
    float acc[1][8][4];
    if (few) {
      float f[2][4];
      const int8_t* xs = reinterpret_cast<const int8_t*>(slots);
      switch (h / 128) {
        case 1: warp_rows16<1>(op[0], xs, r0 + warp * 16, n, f); break;
        case 2: warp_rows16<2>(op[0], xs, r0 + warp * 16, n, f); break;
        case 3: warp_rows16<3>(op[0], xs, r0 + warp * 16, n, f); break;
        case 4: warp_rows16<4>(op[0], xs, r0 + warp * 16, n, f); break;
        default: warp_rows16<5>(op[0], xs, r0 + warp * 16, n, f); break;
      }
#pragma unroll
      for (int nb = 0; nb < 8; nb++)
#pragma unroll
        for (int e = 0; e < 4; e++) acc[0][nb][e] = nb < 2 ? f[nb & 1][e] : 0.0f;
    } else {
      tile_products<1>(op, r0, j0, n, h, slots, sqs, acc);
    }
    const int rlo = r0 + warp * 16 + gid, rhi = rlo + 8;
    const float blo = rlo < nout ? a.head_b[rlo] : 0.0f, bhi = rhi < nout ? a.head_b[rhi] : 0.0f;
    const int nbn = min(8, (n - j0 + 7) >> 3);  // n-blocks holding live lanes (block-uniform)
#pragma unroll
    for (int nb = 0; nb < 8; nb++)
#pragma unroll
      for (int e = 0; e < 2; e++) {
        if (nb >= nbn) continue;
        const int jl = nb * 8 + 2 * tig + e, j = j0 + jl;
        const float ylo = __fadd_rn(acc[0][nb][e], blo), yhi = __fadd_rn(acc[0][nb][2 + e], bhi);
        if (j < n) {
          if (a.logits) {
            if (rlo < nout) a.logits[(size_t)j * nout + rlo] = ylo;
            if (rhi < nout) a.logits[(size_t)j * nout + rhi] = yhi;
          }
          if (rlo >= a.vocab && rlo < nout) a.dlog[(size_t)j * a.n_dur + rlo - a.vocab] = ylo;
          if (rhi >= a.vocab && rhi < nout) a.dlog[(size_t)j * a.n_dur + rhi - a.vocab] = yhi;
        }
        float bv = -INFINITY;
        int bi = INT_MAX;
        if (rlo < a.vocab) bv = ylo, bi = rlo;
        if (rhi < a.vocab && better(yhi, rhi, bv, bi)) bv = yhi, bi = rhi;
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) {  // across gid: the warp's 16 rows
          const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
          const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
          if (better(ov, oi, bv, bi)) bv = ov, bi = oi;
        }
        if (gid == 0) red[warp * kTileLanes + jl] = Part{bv, bi};
      }
    __syncthreads();
    if (threadIdx.x < kTileLanes && j0 + (int)threadIdx.x < n) {
      Part b = red[threadIdx.x];
      for (int w = 1; w < 4; w++) {
        const Part o = red[w * kTileLanes + threadIdx.x];
        if (better(o.v, o.i, b.v, b.i)) b = o;
      }
      a.part[(size_t)(j0 + threadIdx.x) * nrb + rb] = b;
    }
    __syncthreads();
  }
}

// The loop's bookkeeping for each unfinished lane (decoder.rs:222-262), one warp per lane.
__global__ void __launch_bounds__(256) step_kernel(Args a) {
  const int n = a.counts[1], lane = threadIdx.x & 31, nrb = a.head_rows / kTileRows;
  const int nw = blockDim.x / 32;
  for (int j = blockIdx.x * nw + (threadIdx.x >> 5); j < n; j += gridDim.x * nw) {
    float bv = -INFINITY;
    int bi = INT_MAX;
    for (int i = lane; i < nrb; i += 32) {
      const Part p = a.part[(size_t)j * nrb + i];
      if (better(p.v, p.i, bv, bi)) bv = p.v, bi = p.i;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (better(ov, oi, bv, bi)) bv = ov, bi = oi;
    }
    if (lane != 0) continue;
    const int u = a.list_act[j], k = bi;
    int di = 0;
    const float* dl = a.dlog + (size_t)j * a.n_dur;
    for (int i = 1; i < a.n_dur; i++)
      if (dl[i] > dl[di]) di = i;
    const int dur = a.durations[di];
    const int tf = a.tf[u];
    if (k != a.blank) {
      const int ne = a.nemit[u];
      if (ne < a.out_off[u + 1] - a.out_off[u]) a.out[a.out_off[u] + ne] = vxg_emission{k, tf, dur};
      a.nemit[u] = ne + 1;
      a.cur[u] ^= 1;  // the state of the latest prediction step becomes current
      a.have[u] = 0;
      a.last[u] = k;
    }
    const int sym = a.sym[u] + 1;
    int nt = tf + dur;
    if (dur != 0 || sym >= a.max_symbols || k == a.blank) {
      if (dur == 0) nt += 1;
      a.sym[u] = 0;
      if (nt >= a.t[u]) a.done[u] = 1;
    } else {
      a.sym[u] = sym;
    }
    a.tf[u] = nt;
  }
}

__global__ void init_kernel(Args a) {
  for (int u = blockIdx.x * blockDim.x + threadIdx.x; u < a.U; u += gridDim.x * blockDim.x) {
    a.tf[u] = 0;
    a.sym[u] = 0;
    a.last[u] = a.blank;
    a.have[u] = 0;
    a.done[u] = a.t[u] <= 0;
    a.nemit[u] = 0;
    a.cur[u] = 0;
  }
}

__global__ void identity_kernel(int* list, int* counts, long long* off, int* tf, int n) {
  for (int u = blockIdx.x * blockDim.x + threadIdx.x; u < n; u += gridDim.x * blockDim.x) {
    list[u] = u;
    if (off) off[u] = u;
    if (tf) tf[u] = 0;
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) counts[0] = counts[1] = n;
}

size_t gates_smem(int h) { return (size_t)kStages * kSlotBytes + (size_t)2 * 64 * (h / 128) * 4; }
size_t head_smem(int h) {
  return (size_t)kStages * kSlotBytes + (size_t)64 * (h / 128) * 4 + (size_t)4 * kTileLanes * sizeof(Part);
}
size_t proj_smem() { return (size_t)kProjStages * (64 + kProjLanes) * kProjLd * 4; }

// Carves the per-call scratch of U lanes out of one allocation.
struct Scratch {
  size_t bytes = 0;
  std::vector<std::pair<void**, size_t>> parts;
  template <class T>
  void add(T** p, size_t count) {
    parts.push_back({reinterpret_cast<void**>(p), (sizeof(T) * count + 255) / 256 * 256});
    bytes += parts.back().second;
  }
  void bind(void* base) {
    char* c = static_cast<char*>(base);
    for (auto& p : parts) {
      *p.first = c;
      c += p.second;
    }
  }
};

void model_args(const Decoder& D, Args& a) {
  const DevModel& M = D.dev;
  a.emb = M.emb;
  for (int l = 0; l < 4; l++) {
    a.w_ih[l] = M.w_ih[l], a.w_hh[l] = M.w_hh[l], a.s_ih[l] = M.s_ih[l], a.s_hh[l] = M.s_hh[l], a.b[l] = M.b[l];
  }
  a.proj_w = M.proj_w, a.proj_b = M.proj_b, a.head_w = M.head_w, a.head_s = M.head_s, a.head_b = M.head_b;
  a.durations = M.durations;
  a.hidden = D.hidden, a.vocab = D.vocab, a.n_dur = D.n_dur, a.blank = D.blank, a.max_symbols = D.max_symbols;
  a.n_layers = D.n_layers, a.head_rows = M.head_rows;
}

// Scratch shared by every phase, for U lanes.
void add_phase_scratch(Scratch& S, Args& a, int U, int h, int head_rows, int n_dur) {
  S.add(&a.list_pred, U);
  S.add(&a.list_act, U);
  S.add(&a.counts, 4);
  S.add(&a.gates, (size_t)U * 4 * h);
  S.add(&a.qx, (size_t)U * h);
  S.add(&a.qh, (size_t)U * h);
  S.add(&a.sqx, (size_t)U * (h / 128));
  S.add(&a.sqh, (size_t)U * (h / 128));
  S.add(&a.part, (size_t)U * (head_rows / kTileRows));
  S.add(&a.dlog, (size_t)U * n_dur);
}

// The limits are raised once per device and kernel, so to the largest hidden size covered (4096).
vxg_status set_smem_attrs() {
  const int h = 4096;
  vxg_status s = smem_attr(reinterpret_cast<const void*>(gates_kernel), (int)gates_smem(h));
  if (s == VXG_OK) s = smem_attr(reinterpret_cast<const void*>(head_kernel), (int)head_smem(h));
  if (s == VXG_OK) s = smem_attr(reinterpret_cast<const void*>(proj_kernel), (int)proj_smem());
  return s;
}

// Launches of one prediction-network step of the stale lanes (list_pred / counts[0]). Grids are fixed (the lane
// counts live on the device): grid-stride loops over (lane, group) items and persistent loops over product tiles.
int launch_pred(const Args& a, cudaStream_t st, int sms) {
  const int h = a.hidden;
  layer_quant_kernel<<<sms * 8, 128, 0, st>>>(a, 0);
  for (int l = 0; l < a.n_layers; l++) {
    gates_kernel<<<sms * 3, 128, gates_smem(h), st>>>(a, l);
    cell_kernel<<<sms * 8, 128, 0, st>>>(a, l);  // also quantises layer l + 1's inputs
  }
  proj_kernel<<<sms * 2, 256, proj_smem(), st>>>(a);
  return 2 + 2 * a.n_layers;
}

int launch_joint(const Args& a, cudaStream_t st, int sms) {
  joint_quant_kernel<<<sms * 8, 128, 0, st>>>(a);
  head_kernel<<<sms * 3, 128, head_smem(a.hidden), st>>>(a);
  return 2;
}

int launch_round(const Args& a, cudaStream_t st, int sms) {
  plan_kernel<<<1, 1024, 0, st>>>(a);
  int k = 1 + launch_pred(a, st, sms) + launch_joint(a, st, sms);
  step_kernel<<<sms * 2, 256, 0, st>>>(a);
  return k + 1;
}

cudaError_t scratch_alloc(void** p, size_t bytes, cudaStream_t st) {
  cudaMemPool_t pool = scratch_pool();
  return pool ? cudaMallocFromPoolAsync(p, bytes, pool, st) : cudaMallocAsync(p, bytes, st);
}

// The greedy loop's polling resources (a page-locked flag word per queued chunk, one event each, the capture
// stream), created once per host thread and device and kept: allocating page-locked memory per call can stall
// behind the driver's work on other page-locked ranges.
struct PollResources {
  int* flag = nullptr;
  cudaEvent_t ev[kDepth] = {};
  cudaStream_t cs = nullptr;
};
cudaError_t poll_resources(int dev, PollResources** out) {
  static thread_local PollResources per_dev[64];
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  PollResources& r = per_dev[dev];
  cudaError_t e = cudaSuccess;
  if (!r.flag) e = cudaHostAlloc(reinterpret_cast<void**>(&r.flag), kDepth * sizeof(int), cudaHostAllocDefault);
  for (int i = 0; i < kDepth && e == cudaSuccess; i++)
    if (!r.ev[i]) e = cudaEventCreateWithFlags(&r.ev[i], cudaEventDisableTiming);
  if (e == cudaSuccess && !r.cs) e = cudaStreamCreateWithFlags(&r.cs, cudaStreamNonBlocking);
  *out = &r;
  return e;
}

vxg_status check_device(const Decoder& D) {
  if (!D.dev.block) {
    set_error("decoder was created without a device (desc.device = -1)");
    return VXG_ERR_ARG;
  }
  int cur = -1;
  VXG_CUDA(cudaGetDevice(&cur));
  VXG_ARG(cur == D.device, "current device %d is not the decoder's device %d", cur, D.device);
  return VXG_OK;
}

}  // namespace

vxg_status upload_device_model(Decoder& D) {
  const int h = D.hidden, nl = D.n_layers, nout = D.vocab + D.n_dur;
  DevModel& M = D.dev;
  M.head_rows = (nout + kTileRows - 1) / kTileRows * kTileRows;
  Scratch S;
  S.add(&M.emb, (size_t)D.vocab * h);
  for (int l = 0; l < nl; l++) {
    S.add(&M.w_ih[l], (size_t)4 * h * h);
    S.add(&M.w_hh[l], (size_t)4 * h * h);
    S.add(&M.s_ih[l], (size_t)4 * h);
    S.add(&M.s_hh[l], (size_t)4 * h);
    S.add(&M.b[l], (size_t)4 * h);
  }
  S.add(&M.proj_w, (size_t)h * h);
  S.add(&M.proj_b, (size_t)h);
  S.add(&M.head_w, (size_t)M.head_rows * h);
  S.add(&M.head_s, (size_t)M.head_rows);
  S.add(&M.head_b, (size_t)nout);
  S.add(&M.durations, (size_t)D.n_dur);
  VXG_CUDA(cudaMalloc(&M.block, S.bytes));
  VXG_CUDA(cudaMemset(M.block, 0, S.bytes));
  S.bind(M.block);
  auto up = [](void* dst, const void* src, size_t bytes) { return cudaMemcpy(dst, src, bytes, cudaMemcpyHostToDevice); };
  VXG_CUDA(up(M.emb, D.embedding.data(), sizeof(float) * D.embedding.size()));
  for (int l = 0; l < nl; l++) {
    VXG_CUDA(up(M.w_ih[l], D.w_ih[l].rows.data(), (size_t)4 * h * h));
    VXG_CUDA(up(M.w_hh[l], D.w_hh[l].rows.data(), (size_t)4 * h * h));
    VXG_CUDA(up(M.s_ih[l], D.w_ih[l].scale.data(), sizeof(float) * 4 * h));
    VXG_CUDA(up(M.s_hh[l], D.w_hh[l].scale.data(), sizeof(float) * 4 * h));
    VXG_CUDA(up(M.b[l], D.b[l].data(), sizeof(float) * 4 * h));
  }
  VXG_CUDA(up(M.proj_w, D.proj.rows.data(), sizeof(float) * h * h));
  VXG_CUDA(up(M.proj_b, D.proj.bias.data(), sizeof(float) * h));
  VXG_CUDA(up(M.head_w, D.head.rows.data(), (size_t)nout * h));  // pad rows stay zero
  VXG_CUDA(up(M.head_s, D.head.scale.data(), sizeof(float) * nout));
  VXG_CUDA(up(M.head_b, D.head_b.data(), sizeof(float) * nout));
  VXG_CUDA(up(M.durations, D.durations.data(), sizeof(int) * D.n_dur));
  return VXG_OK;
}

void free_device_model(Decoder& D) {
  if (D.dev.block) cudaFree(D.dev.block);
  D.dev = DevModel{};
}

}  // namespace tdt
}  // namespace vxg

using namespace vxg;
using namespace vxg::tdt;

extern "C" {

vxg_status vxg_tdt_pred_step_device(const vxg_tdt* t, int n, const int* tokens, const float* h, const float* c,
                                    float* g, float* h_out, float* c_out, void* stream) {
  clear_error();
  VXG_ARG(t && n >= 0 && (n == 0 || (tokens && h && c && g && h_out && c_out)), "bad arguments");
  const Decoder& D = t->d;
  vxg_status s = check_device(D);
  if (s != VXG_OK || n == 0) return s;
  if ((s = set_smem_attrs()) != VXG_OK) return s;
  cudaStream_t st = (cudaStream_t)stream;
  Args a{};
  model_args(D, a);
  a.U = n;
  a.last = const_cast<int*>(tokens);
  a.H = const_cast<float*>(h), a.C = const_cast<float*>(c), a.Hn = h_out, a.Cn = c_out, a.G = g;
  Scratch S;
  add_phase_scratch(S, a, n, D.hidden, D.dev.head_rows, D.n_dur);
  void* ws = nullptr;
  VXG_CUDA(scratch_alloc(&ws, S.bytes, st));
  S.bind(ws);
  identity_kernel<<<(n + 255) / 256, 256, 0, st>>>(a.list_pred, a.counts, nullptr, nullptr, n);
  const int k = launch_pred(a, st, sm_count());
  note_launch(1 + k);
  const cudaError_t e = cudaGetLastError();
  cudaFreeAsync(ws, st);
  if (e != cudaSuccess) return cuda_fail(e, "vxg_tdt_pred_step_device");
  return VXG_OK;
}

vxg_status vxg_tdt_joint_device(const vxg_tdt* t, int n, const float* enc, const float* g, float* logits,
                                void* stream) {
  clear_error();
  VXG_ARG(t && n >= 0 && (n == 0 || (enc && g && logits)), "bad arguments");
  const Decoder& D = t->d;
  vxg_status s = check_device(D);
  if (s != VXG_OK || n == 0) return s;
  if ((s = set_smem_attrs()) != VXG_OK) return s;
  cudaStream_t st = (cudaStream_t)stream;
  Args a{};
  model_args(D, a);
  a.U = n;
  a.proj = enc, a.G = const_cast<float*>(g), a.logits = logits;
  Scratch S;
  add_phase_scratch(S, a, n, D.hidden, D.dev.head_rows, D.n_dur);
  long long* off = nullptr;
  int* tf = nullptr;
  S.add(&off, n);
  S.add(&tf, n);
  void* ws = nullptr;
  VXG_CUDA(scratch_alloc(&ws, S.bytes, st));
  S.bind(ws);
  a.off = off, a.tf = tf;
  identity_kernel<<<(n + 255) / 256, 256, 0, st>>>(a.list_act, a.counts, off, tf, n);
  const int k = launch_joint(a, st, sm_count());
  note_launch(1 + k);
  const cudaError_t e = cudaGetLastError();
  cudaFreeAsync(ws, st);
  if (e != cudaSuccess) return cuda_fail(e, "vxg_tdt_joint_device");
  return VXG_OK;
}

vxg_status vxg_tdt_greedy_device(const vxg_tdt* t, int n, const float* proj, const int* frames, vxg_emission* out,
                                 const size_t* cap, int* n_out, void* stream) {
  clear_error();
  VXG_ARG(t && n >= 0 && (n == 0 || (frames && cap && n_out)), "bad arguments");
  const Decoder& D = t->d;
  vxg_status s = check_device(D);
  if (s != VXG_OK || n == 0) return s;
  long long total = 0;
  int tmax = 0;
  std::vector<long long> off(2 * (size_t)n + 1);  // frame offsets [n], then emission offsets [n + 1]
  long long* eoff = off.data() + n;
  eoff[0] = 0;
  for (int u = 0; u < n; u++) {
    VXG_ARG(frames[u] >= 0, "utterance %d: negative frame count", u);
    off[u] = total;
    total += frames[u];
    tmax = std::max(tmax, frames[u]);
    eoff[u + 1] = eoff[u] + (long long)cap[u];
  }
  VXG_ARG(proj || total == 0, "NULL proj");
  VXG_ARG(out || eoff[n] == 0, "NULL out");
  if ((s = set_smem_attrs()) != VXG_OK) return s;
  cudaStream_t st = (cudaStream_t)stream;
  const int h = D.hidden, nl = D.n_layers;
  Args a{};
  model_args(D, a);
  a.U = n;
  a.proj = proj, a.out = out;
  Scratch S;
  add_phase_scratch(S, a, n, h, D.dev.head_rows, D.n_dur);
  int* t_dev = nullptr;
  long long* off_dev = nullptr;
  S.add(&t_dev, n);
  S.add(&off_dev, 2 * (size_t)n + 1);
  S.add(&a.tf, n);
  S.add(&a.sym, n);
  S.add(&a.last, n);
  S.add(&a.have, n);
  S.add(&a.done, n);
  S.add(&a.nemit, n);
  S.add(&a.cur, n);
  const size_t state = (size_t)n * nl * h;
  S.add(&a.H, state);
  S.add(&a.C, state);
  S.add(&a.Hn, state);
  S.add(&a.Cn, state);
  S.add(&a.G, (size_t)n * h);
  void* ws = nullptr;
  PollResources* pr = nullptr;
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  vxg_status rc = VXG_OK;
  cudaError_t e = cudaSuccess;
  // a lane takes at most max_symbols rounds per frame
  const long long max_rounds = (long long)tmax * D.max_symbols + 2;
  const long long max_chunks = max_rounds / kRoundsPerGraph + kDepth + 1;
#define STEP(call)                              \
  do {                                          \
    if (e == cudaSuccess) {                     \
      e = (call);                               \
      if (e != cudaSuccess) rc = cuda_fail(e, #call); \
    }                                           \
  } while (0)
  STEP(scratch_alloc(&ws, S.bytes, st));
  STEP(poll_resources(D.device, &pr));
  // host-visible count of unfinished lanes after each chunk, one slot per queued chunk
  int* flag = pr ? pr->flag : nullptr;
  cudaEvent_t* ev = pr ? pr->ev : nullptr;
  cudaStream_t cs = pr ? pr->cs : nullptr;
  if (e == cudaSuccess) {
    S.bind(ws);
    a.t = t_dev, a.off = off_dev, a.out_off = off_dev + n;
  }
  STEP(cudaMemcpyAsync(t_dev, frames, sizeof(int) * n, cudaMemcpyHostToDevice, st));
  STEP(cudaMemcpyAsync(off_dev, off.data(), sizeof(long long) * off.size(), cudaMemcpyHostToDevice, st));
  STEP(cudaMemsetAsync(a.H, 0, sizeof(float) * state, st));
  STEP(cudaMemsetAsync(a.C, 0, sizeof(float) * state, st));
  if (e == cudaSuccess) {
    init_kernel<<<(n + 255) / 256, 256, 0, st>>>(a);
    note_launch();
    STEP(cudaGetLastError());
  }
  int per_round = 0;
  const int sms = sm_count();
  STEP(cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal));
  if (e == cudaSuccess) {
    for (int r = 0; r < kRoundsPerGraph; r++) per_round = launch_round(a, cs, sms);
    const cudaError_t le = cudaGetLastError();
    e = cudaStreamEndCapture(cs, &graph);
    if (le != cudaSuccess) e = le;
    if (e != cudaSuccess) rc = cuda_fail(e, "capturing the decode rounds");
  }
  STEP(cudaGraphInstantiate(&exec, graph, 0));
  // kDepth chunks in flight, then one more per chunk the host sees unfinished: the GPU has kDepth - 1 chunks of
  // rounds queued while the host reads the oldest flag
  long long launched = 0, seen = 0;
  auto launch_chunk = [&](int slot) {
    STEP(cudaGraphLaunch(exec, st));
    STEP(cudaMemcpyAsync(flag + slot, a.counts + 1, sizeof(int), cudaMemcpyDeviceToHost, st));
    STEP(cudaEventRecord(ev[slot], st));
    if (e == cudaSuccess) note_launch(per_round * kRoundsPerGraph);
    launched++;
  };
  for (int i = 0; i < kDepth; i++) launch_chunk(i);
  while (e == cudaSuccess) {
    const int slot = (int)(seen % kDepth);
    STEP(cudaEventSynchronize(ev[slot]));
    if (e != cudaSuccess) break;
    seen++;
    if (flag[slot] == 0) break;
    if (launched >= max_chunks) {
      set_error("vxg_tdt_greedy_device: %lld rounds without finishing (bound %lld)", launched * kRoundsPerGraph,
                max_rounds);
      rc = VXG_ERR_TIMEOUT;
      break;
    }
    launch_chunk(slot);
  }
  STEP(cudaMemcpyAsync(n_out, a.nemit, sizeof(int) * n, cudaMemcpyDeviceToDevice, st));
#undef STEP
  if (ws) cudaFreeAsync(ws, st);
  for (int i = 0; ev && i < kDepth; i++)  // every chunk and flag copy has landed before the next call reuses them
    if (ev[i]) cudaEventSynchronize(ev[i]);
  if (exec) cudaGraphExecDestroy(exec);
  if (graph) cudaGraphDestroy(graph);
  return rc;
}

}  // extern "C"
