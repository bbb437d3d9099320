// Enumerates every f32 input of expf_cr / tanhf_cr (crmath.cuh) whose double-precision evaluation lies within 2^-48 of
// a point halfway between two floats, printing "exp|tanh <input bits hex> <double result hex-float>". Run by
// crmath_gen.py, which resolves each case with exact decimal arithmetic and writes crmath_tables.h.
#include <cstdio>
#include <thread>
#include <vector>
#include <mutex>

#include "crmath.cuh"

using namespace vxg::crm;

int main() {
  const unsigned nt = std::max(1u, std::thread::hardware_concurrency());
  std::mutex mu;
  std::vector<std::thread> th;
  for (unsigned t = 0; t < nt; t++)
    th.emplace_back([&, t] {
      std::vector<char> buf;
      char line[96];
      for (uint64_t b = t; b < (1ull << 32); b += nt) {
        const float x = ffrom((uint32_t)b);
        if (x != x) continue;
        if (x <= 89.0f && x >= -104.0f) {
          const double y = exp_d((double)x);
          if (near_half(y)) {
            const int n = snprintf(line, sizeof line, "exp %08x %a\n", (unsigned)b, y);
            buf.insert(buf.end(), line, line + n);
          }
        }
        if (x > 0.0f && x < 20.0f) {
          const double y = tanh_d((double)x);
          if (near_half(y)) {
            const int n = snprintf(line, sizeof line, "tanh %08x %a\n", (unsigned)b, y);
            buf.insert(buf.end(), line, line + n);
          }
        }
      }
      std::lock_guard<std::mutex> lk(mu);
      fwrite(buf.data(), 1, buf.size(), stdout);
    });
  for (auto& x : th) x.join();
  return 0;
}
