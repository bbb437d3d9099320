// TDT decoder state shared by the host greedy loop (tdt.cpp) and the device encoder projection (tdt_dev.cu).
#pragma once
#include <cstdint>
#include <vector>

#include "../../include/vxg.h"

namespace vxg {
namespace tdt {

// Per-row int8 weights for one-token products (the reference's int8_rows layout, decoder.rs:270-303): codes by row
// for the scalar path, and 16-row x 4-column interleaved planes for the AVX-512 VNNI path (one vpdpbusd = 16 rows x
// 4 columns), with each group's code sums for the +128 offset of unsigned activations.
struct I8Rows {
  int out = 0, inp = 0, ng = 0, blocks = 0;
  std::vector<int8_t> rows;    // [out][inp]
  std::vector<float> scale;    // [blocks * 16] row scale (0 in pad rows)
  std::vector<int8_t> q16;     // [blocks][inp / 4][16][4]
  std::vector<int32_t> wsum;   // [blocks][ng][16]
};

// f16 weight matrix for the decoder projector (gemv_f16): f32 rows for the scalar path and 16-row column-major
// blocks ([blocks][inp][16]) for the vector path.
struct F16Rows {
  int out = 0, inp = 0, blocks = 0;
  std::vector<float> rows;  // [out][inp]
  std::vector<float> t16;   // [blocks][inp][16]
  std::vector<float> bias;  // [out]
};

// The prediction network and joint head on the decoder's GPU, for the batched greedy decode (tdt_greedy.cu): the
// int8 rows and row scales of I8Rows (rows padded with zero rows and zero scales to a multiple of 64), the embedding,
// summed LSTM biases, the projector's f32 rows, the head bias and the duration table. One allocation (`block`).
struct DevModel {
  void* block = nullptr;
  float* emb = nullptr;                       // [vocab, hidden]
  int8_t* w_ih[4] = {}, *w_hh[4] = {};        // [4 hidden, hidden]
  float* s_ih[4] = {}, *s_hh[4] = {};         // [4 hidden]
  float* b[4] = {};                           // [4 hidden] b_ih + b_hh
  float* proj_w = nullptr, *proj_b = nullptr; // [hidden, hidden], [hidden]
  int8_t* head_w = nullptr;                   // [head_rows, hidden]
  float* head_s = nullptr, *head_b = nullptr; // [head_rows], [vocab + n_dur]
  int* durations = nullptr;                   // [n_dur]
  int head_rows = 0;
};

struct Decoder;
// Upload / release Decoder::dev on the current device (tdt_greedy.cu).
vxg_status upload_device_model(Decoder& D);
void free_device_model(Decoder& D);

struct Decoder {
  int hidden = 0, vocab = 0, n_dur = 0, blank = 0, max_symbols = 0, d_model = 0, n_layers = 0;
  std::vector<int> durations;
  std::vector<float> embedding;  // [vocab, hidden]
  std::vector<I8Rows> w_ih, w_hh;
  std::vector<std::vector<float>> b;  // b_ih + b_hh per layer
  F16Rows proj;
  I8Rows head;
  std::vector<float> head_b;
  std::vector<float> enc_w, enc_b;  // host copies of the encoder projector
  int device = -1;
  float* enc_w_dev = nullptr;  // [hidden, d_model] on `device`
  float* enc_b_dev = nullptr;
  DevModel dev;
  bool vnni = false;
};

}  // namespace tdt
}  // namespace vxg

struct vxg_tdt {
  vxg::tdt::Decoder d;
};
