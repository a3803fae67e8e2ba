// synth.cpp — deterministic synthetic .smodel tensors and the X4 packer.
//
// The BASELINE configs are random-init models.  Every value is a pure
// function of (seed, stream, counter) through SplitMix64, so tensors can be
// generated in parallel and any sub-range regenerated identically.
//   q4_0: per block d = fp16(|N(0, sigma)| / 8) (round-half-even from the
//         double), 16 random bytes of nibbles (uniform 0..15);
//   q8_0: per block d = fp16(scale), 32 bytes mapped to -127..127;
//   f32:  N(mean, sigma) through Box-Muller on two uniforms.
// The X4 writer restates tools/silicatepack.py:982-1022.
//
// The same source is also compiled into the CPU oracle's library with
// ZSYNTH_ORACLE defined, which names the entry points zo_synth_* and
// zo_pack_x4: the CPU reference arm then generates identical bytes without
// loading this library.
#include <cmath>
#include <cstring>
#include <thread>
#include <vector>

#include "../../include/zgpu.h"

namespace {

inline uint64_t mix64(uint64_t seed, uint64_t stream, uint64_t ctr) {
  uint64_t z = seed ^ (stream * 0xD1B54A32D192ED03ull);
  z += (ctr + 1) * 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

inline double unit_open(uint64_t r) {  // (0, 1)
  return (static_cast<double>(r >> 11) + 0.5) * (1.0 / 9007199254740992.0);
}

inline double normal_at(uint64_t seed, uint64_t stream, uint64_t i) {
  const double u1 = unit_open(mix64(seed, stream, 2 * i));
  const double u2 = unit_open(mix64(seed, stream, 2 * i + 1));
  return std::sqrt(-2.0 * std::log(u1)) * std::cos(6.283185307179586 * u2);
}

// binary16 nearest-even from a double, with the packer's non-finite -> 0 and
// +-65504 clamp (tools/silicatepack.py float_to_fp16_bytes).
uint16_t f64_to_fp16(double v) {
  if (!std::isfinite(v)) v = 0.0;
  if (v > 65504.0) v = 65504.0;
  if (v < -65504.0) v = -65504.0;
  const uint16_t sign = std::signbit(v) ? 0x8000u : 0u;
  const double a = std::fabs(v);
  if (a == 0.0) return sign;
  int e;
  std::frexp(a, &e);
  const int ub = e - 1;
  const double q = (ub < -14) ? std::ldexp(1.0, -24) : std::ldexp(1.0, ub - 10);
  const double res = std::nearbyint(a / q) * q;
  if (res < std::ldexp(1.0, -14))
    return static_cast<uint16_t>(sign | static_cast<uint16_t>(res / std::ldexp(1.0, -24)));
  int e2;
  const double m2 = std::frexp(res, &e2);
  const uint16_t mant = static_cast<uint16_t>((m2 * 2.0 - 1.0) * 1024.0);
  return static_cast<uint16_t>(sign | static_cast<uint16_t>((e2 - 1 + 15) << 10) | mant);
}

template <class F>
void parallel_rows(uint64_t rows, F &&f) {
  unsigned nt = std::thread::hardware_concurrency();
  if (nt == 0) nt = 1;
  if (nt > 64) nt = 64;
  if (rows < 64 || nt == 1) {
    f(0, rows);
    return;
  }
  std::vector<std::thread> ts;
  const uint64_t per = (rows + nt - 1) / nt;
  for (unsigned t = 0; t < nt; ++t) {
    const uint64_t r0 = t * per, r1 = std::min<uint64_t>(rows, r0 + per);
    if (r0 >= r1) break;
    ts.emplace_back([=, &f] { f(r0, r1); });
  }
  for (auto &t : ts) t.join();
}

}  // namespace

#ifdef ZSYNTH_ORACLE
#define ZSYNTH_NAME(n) zo_##n
#else
#define ZSYNTH_NAME(n) zgpu_##n
#endif

extern "C" {

void ZSYNTH_NAME(synth_q4_0)(uint64_t seed, uint64_t stream, uint64_t rows, uint64_t cols, float sigma,
                     void *out) {
  const uint64_t bpr = cols / 32;
  uint8_t *o = static_cast<uint8_t *>(out);
  parallel_rows(rows, [&](uint64_t r0, uint64_t r1) {
    for (uint64_t r = r0; r < r1; ++r) {
      for (uint64_t b = 0; b < bpr; ++b) {
        const uint64_t i = r * bpr + b;
        uint8_t *blk = o + i * 18;
        const double d = std::fabs(normal_at(seed, 2 * stream, i) * sigma) / 8.0;
        const uint16_t h = f64_to_fp16(d);
        blk[0] = static_cast<uint8_t>(h & 0xFF);
        blk[1] = static_cast<uint8_t>(h >> 8);
        const uint64_t w0 = mix64(seed, 2 * stream + 1, 2 * i);
        const uint64_t w1 = mix64(seed, 2 * stream + 1, 2 * i + 1);
        std::memcpy(blk + 2, &w0, 8);
        std::memcpy(blk + 10, &w1, 8);
      }
    }
  });
}

void ZSYNTH_NAME(synth_q8_0)(uint64_t seed, uint64_t stream, uint64_t rows, uint64_t cols, float scale,
                     void *out) {
  const uint64_t bpr = cols / 32;
  uint8_t *o = static_cast<uint8_t *>(out);
  const uint16_t h = f64_to_fp16(static_cast<double>(scale));
  parallel_rows(rows, [&](uint64_t r0, uint64_t r1) {
    for (uint64_t r = r0; r < r1; ++r) {
      for (uint64_t b = 0; b < bpr; ++b) {
        const uint64_t i = r * bpr + b;
        uint8_t *blk = o + i * 34;
        blk[0] = static_cast<uint8_t>(h & 0xFF);
        blk[1] = static_cast<uint8_t>(h >> 8);
        for (int k = 0; k < 4; ++k) {
          const uint64_t w = mix64(seed, 2 * stream + 1, 4 * i + k);
          for (int j = 0; j < 8; ++j) {
            const uint32_t byte = static_cast<uint32_t>((w >> (8 * j)) & 0xFF);
            const int v = static_cast<int>((byte * 255u) >> 8) - 127;  // -127..127
            blk[2 + 8 * k + j] = static_cast<uint8_t>(static_cast<int8_t>(v));
          }
        }
      }
    }
  });
}

void ZSYNTH_NAME(synth_f32)(uint64_t seed, uint64_t stream, uint64_t n, float mean, float sigma,
                    float *out) {
  for (uint64_t i = 0; i < n; ++i) {
    out[i] = (sigma == 0.0f)
                 ? mean
                 : static_cast<float>(static_cast<double>(mean) +
                                      static_cast<double>(sigma) * normal_at(seed, stream, i));
  }
}

void ZSYNTH_NAME(synth_tokens)(uint64_t seed, uint64_t stream, uint64_t n, uint32_t vocab, uint32_t *out) {
  for (uint64_t i = 0; i < n; ++i) {
    const uint64_t r = mix64(seed, stream, i);
    out[i] = static_cast<uint32_t>(((r >> 32) * static_cast<uint64_t>(vocab)) >> 32);
  }
}

zgpu_status ZSYNTH_NAME(pack_x4)(const void *plain, void *x4, uint64_t rows, uint64_t cols,
                         uint32_t quant) {
  const uint64_t bb = quant == ZGPU_Q4_0 ? 18 : quant == ZGPU_Q8_0 ? 34 : 0;
  if (!bb) return ZGPU_ERR_UNSUPPORTED_QUANT;
  if (!plain || !x4 || rows % 4 || cols % 32 || cols == 0) return ZGPU_ERR_INVALID_ARG;
  const uint64_t bpr = cols / 32, body = bb - 2;
  const uint8_t *src = static_cast<const uint8_t *>(plain);
  uint8_t *dst = static_cast<uint8_t *>(x4);
  parallel_rows(rows / 4, [&](uint64_t g0, uint64_t g1) {
    for (uint64_t g = g0; g < g1; ++g) {
      uint8_t *d = dst + g * bpr * bb * 4;
      for (uint64_t b = 0; b < bpr; ++b) {
        for (uint64_t l = 0; l < 4; ++l) {
          const uint8_t *s = src + ((4 * g + l) * bpr + b) * bb;
          *d++ = s[0];
          *d++ = s[1];
        }
        for (uint64_t l = 0; l < 4; ++l) {
          const uint8_t *s = src + ((4 * g + l) * bpr + b) * bb;
          std::memcpy(d, s + 2, body);
          d += body;
        }
      }
    }
  });
  return ZGPU_OK;
}

}  // extern "C"
