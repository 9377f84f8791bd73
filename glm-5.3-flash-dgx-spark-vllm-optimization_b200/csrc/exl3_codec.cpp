// Host-side (CPU) EXL3 trellis codec: the codebook, tile decode to fp16 and a multi-threaded whole-matrix decode.
// Used to validate checkpoints at load (a sample of tiles decoded on the CPU against the GPU kernels' decode), by
// the exhaustive codebook test, and by tools that need the dequantized weights without a GPU.  The format (tile
// bit order, state windows, mcg codebook, tile positions) is the checkpoint's and is described in ops/exl3.py; the
// reference keeps the same rules in Python (code/fork/kernels/exl3_format_ref.py:1-31).
#include <torch/extension.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <thread>
#include <vector>

namespace g53codec {

// fp16 bits -> double (exact)
double half_to_double(uint16_t h) {
  const int sign = h >> 15, e = (h >> 10) & 31, m = h & 1023;
  double v;
  if (e == 0) v = std::ldexp((double)m, -24);
  else if (e == 31) v = m ? NAN : INFINITY;
  else v = std::ldexp((double)(m | 1024), e - 25);
  return sign ? -v : v;
}

// double -> fp16 bits, round to nearest even (one rounding), overflow to inf
uint16_t double_to_half(double x) {
  if (std::isnan(x)) return 0x7e00;
  const uint16_t sign = std::signbit(x) ? 0x8000 : 0;
  double a = std::fabs(x);
  if (a == 0.0) return sign;
  int e;
  std::frexp(a, &e);                           // a = f * 2^e, f in [0.5, 1)
  int ex = e - 1;                              // a in [2^ex, 2^(ex+1))
  if (ex < -14) ex = -14;                      // subnormal range: quantum 2^-24
  const double q = std::ldexp(1.0, ex - 10);   // spacing of representable values at this exponent
  double r = a / q;                            // integer part = significand (incl. implicit bit when normal)
  double fl = std::floor(r);
  const double rem = r - fl;
  if (rem > 0.5 || (rem == 0.5 && std::fmod(fl, 2.0) != 0.0)) fl += 1.0;
  double v = fl * q;
  if (v >= 65520.0) return sign | 0x7c00;      // rounds to inf
  int e2;
  std::frexp(v, &e2);
  const int E = e2 - 1;
  if (E < -14) return sign | (uint16_t)(v / std::ldexp(1.0, -24));      // subnormal
  const uint16_t mant = (uint16_t)(v / std::ldexp(1.0, E - 10)) - 1024;
  return sign | (uint16_t)((E + 15) << 10) | mant;
}

// codebook value of a 16-bit state: fp16(lo) + fp16(hi) of the masked product, rounded once to fp16
uint16_t codebook(uint32_t s) {
  uint32_t x = (s * 0xCBAC1FEDu) & 0xFFFFFFFFu;
  x = (x & 0x8FFF8FFFu) ^ 0x3B603B60u;
  return double_to_half(half_to_double((uint16_t)(x & 0xffff)) + half_to_double((uint16_t)(x >> 16)));
}

// 16-bit state of value p of a tile (32 uint32 words, circular bitstream from the MSB of word 0)
inline uint32_t state(const uint32_t* w, int p) {
  const int total = 1024, bits = 4;
  const int start = ((p + 1) * bits - 16 + total) % total;
  const int w0 = start / 32, w1 = (w0 + 1) % 32, off = start % 32;
  const uint64_t window = ((uint64_t)w[w0] << 32) | w[w1];
  return (uint32_t)((window >> (48 - off)) & 0xffff);
}

// tile value p -> (row, col) inside the 16 x 16 tile
inline void tile_pos(int p, int& row, int& col) {
  const int l = p / 8, j = p % 8;
  row = 2 * (l % 4) + (j & 1) + 8 * ((j >> 1) & 1);
  col = l / 4 + 8 * (j >> 2);
}

}  // namespace g53codec

// fp16 [65536] (as int16 bits)
torch::Tensor exl3_codebook_cpu() {
  auto out = torch::empty({65536}, torch::dtype(torch::kInt16));
  int16_t* o = out.data_ptr<int16_t>();
  for (uint32_t s = 0; s < 65536; ++s) o[s] = (int16_t)g53codec::codebook(s);
  return out.view(torch::kFloat16);
}

// trellis int16 [K/16, N/16, 64] (CPU) -> W_q fp16 [K, N], tiles decoded on `threads` host threads
torch::Tensor exl3_decode_cpu(const torch::Tensor& trellis, int64_t threads) {
  TORCH_CHECK(trellis.device().is_cpu() && trellis.scalar_type() == torch::kInt16 && trellis.dim() == 3 &&
                  trellis.size(2) == 64,
              "trellis must be a CPU int16 [K/16, N/16, 64] tensor (4-bit codes)");
  auto tr = trellis.contiguous();
  const int64_t KT = tr.size(0), NT = tr.size(1), N = NT * 16;
  auto out = torch::empty({KT * 16, N}, torch::dtype(torch::kInt16));
  const uint32_t* w = reinterpret_cast<const uint32_t*>(tr.data_ptr<int16_t>());
  int16_t* o = out.data_ptr<int16_t>();
  std::vector<uint16_t> cb(65536);
  for (uint32_t s = 0; s < 65536; ++s) cb[s] = g53codec::codebook(s);
  const int nth = (int)std::max<int64_t>(1, std::min<int64_t>(threads > 0 ? threads : 8, KT));
  auto work = [&](int t) {
    for (int64_t kt = t; kt < KT; kt += nth)
      for (int64_t nt = 0; nt < NT; ++nt) {
        const uint32_t* tw = w + (kt * NT + nt) * 32;
        for (int p = 0; p < 256; ++p) {
          int r, c;
          g53codec::tile_pos(p, r, c);
          o[(kt * 16 + r) * N + nt * 16 + c] = (int16_t)cb[g53codec::state(tw, p)];
        }
      }
  };
  std::vector<std::thread> pool;
  for (int t = 0; t < nth; ++t) pool.emplace_back(work, t);
  for (auto& th : pool) th.join();
  return out.view(torch::kFloat16);
}

void register_exl3_codec(pybind11::module& m) {
  m.def("exl3_codebook_cpu", &exl3_codebook_cpu, "EXL3 mcg codebook, fp16 [65536] (host)");
  m.def("exl3_decode_cpu", &exl3_decode_cpu, "EXL3 trellis [K/16, N/16, 64] -> fp16 [K, N] on host threads",
        pybind11::arg("trellis"), pybind11::arg("threads") = 8);
}
