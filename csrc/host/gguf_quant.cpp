// GGUF block quantizers / dequantizers (host C++): F16, Q8_0, Q4_K.
//
// Layouts follow the ggml GGUF specification (the on-disk format must be byte-compatible):
//   Q8_0  block of 32:  fp16 d | int8 qs[32]                         (34 bytes)   x = d * q
//   Q4_K  block of 256: fp16 d | fp16 dmin | u8 scales[12] | u8 qs[128] (144 bytes)
//         8 sub-blocks of 32 with 6-bit scale sc_j and 6-bit min m_j packed in scales[12];
//         x = d * sc_j * q - dmin * m_j, q a 4-bit value; the 64 values of sub-blocks (2i, 2i+1)
//         share qs[32i .. 32i+32): low nibbles -> sub-block 2i, high nibbles -> sub-block 2i+1.
// The reference's own Q4_K code is not spec-compliant (its Java dequantizer ignores the packed
// 6-bit scales, runner/gguf/gollek-gguf-loader/…/gguf/quant/Dequantizer.java:185-209, and the
// native quantizer writes a different symmetric format, runner/llamacpp/gguf-bridge/
// gguf_quantizer.cpp:236-278); this file implements the ggml layout, checked against gguf-py.
//
// The Q4_K quantizer here picks each sub-block's (scale, min) from its range with a short
// refinement (least-squares re-fit of the scale for fixed codes), then packs both to 6 bits
// relative to the super-block maxima.
#include <torch/extension.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>

namespace {

inline uint16_t f32_to_f16_bits(float f) { return c10::Half(f).x; }
inline float f16_bits_to_f32(uint16_t h) {
  c10::Half v;
  v.x = h;
  return static_cast<float>(v);
}

void get_scale_min_k4(int j, const uint8_t* q, uint8_t& sc, uint8_t& m) {
  if (j < 4) {
    sc = q[j] & 63;
    m = q[j + 4] & 63;
  } else {
    sc = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
    m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
  }
}

void pack_scale_min_k4(const uint8_t* sc, const uint8_t* m, uint8_t* q) {
  std::memset(q, 0, 12);
  for (int j = 0; j < 4; ++j) {
    q[j] = (sc[j] & 63) | ((sc[j + 4] >> 4) << 6);
    q[j + 4] = (m[j] & 63) | ((m[j + 4] >> 4) << 6);
  }
  for (int j = 4; j < 8; ++j) q[j + 4] = (sc[j] & 0xF) | ((m[j] & 0xF) << 4);
}

// Fit x ~ s * q - mn with q in [0, 15], mn >= 0 (ggml convention: min stored as positive offset).
void fit_subblock(const float* x, float& s, float& mn) {
  float lo = x[0], hi = x[0];
  for (int i = 1; i < 32; ++i) {
    lo = std::min(lo, x[i]);
    hi = std::max(hi, x[i]);
  }
  lo = std::min(lo, 0.f);
  if (hi <= lo) {
    s = 0.f;
    mn = -lo;
    return;
  }
  s = (hi - lo) / 15.f;
  mn = -lo;
  // two rounds of least-squares refinement of (s, mn) for the current codes
  for (int it = 0; it < 2; ++it) {
    double sq = 0, sqq = 0, sx = 0, sxq = 0;
    for (int i = 0; i < 32; ++i) {
      int q = (int)std::lround((x[i] + mn) / s);
      q = std::min(15, std::max(0, q));
      sq += q;
      sqq += (double)q * q;
      sx += x[i];
      sxq += (double)x[i] * q;
    }
    const double n = 32.0, det = n * sqq - sq * sq;
    if (det <= 0) break;
    const double ns = (n * sxq - sq * sx) / det;
    const double nb = (sx - ns * sq) / n;  // x ~ ns*q + nb  => mn = -nb
    if (ns <= 0 || -nb < 0) break;
    s = (float)ns;
    mn = (float)(-nb);
  }
}

}  // namespace

torch::Tensor quantize_q8_0(torch::Tensor x) {
  x = x.contiguous().to(torch::kFloat);
  const int64_t n = x.numel();
  TORCH_CHECK(n % 32 == 0, "Q8_0 needs a multiple of 32 elements");
  const int64_t nb = n / 32;
  auto out = torch::empty({nb * 34}, torch::kUInt8);
  const float* xp = x.data_ptr<float>();
  uint8_t* o = out.data_ptr<uint8_t>();
  at::parallel_for(0, nb, 256, [&](int64_t b0, int64_t b1) {
    for (int64_t b = b0; b < b1; ++b) {
      const float* v = xp + b * 32;
      float amax = 0.f;
      for (int i = 0; i < 32; ++i) amax = std::max(amax, std::fabs(v[i]));
      const float d = amax / 127.f;
      const float id = d > 0.f ? 1.f / d : 0.f;
      uint8_t* blk = o + b * 34;
      const uint16_t dh = f32_to_f16_bits(d);
      std::memcpy(blk, &dh, 2);
      for (int i = 0; i < 32; ++i) {
        int q = (int)std::lround(v[i] * id);
        q = std::min(127, std::max(-128, q));
        blk[2 + i] = (uint8_t)(int8_t)q;
      }
    }
  });
  return out;
}

torch::Tensor dequantize_q8_0(torch::Tensor raw, int64_t n) {
  TORCH_CHECK(raw.scalar_type() == torch::kUInt8 && raw.is_contiguous(), "raw bytes");
  TORCH_CHECK(n % 32 == 0 && raw.numel() >= n / 32 * 34, "Q8_0 size");
  auto out = torch::empty({n}, torch::kFloat);
  const uint8_t* r = raw.data_ptr<uint8_t>();
  float* o = out.data_ptr<float>();
  at::parallel_for(0, n / 32, 256, [&](int64_t b0, int64_t b1) {
    for (int64_t b = b0; b < b1; ++b) {
      uint16_t dh;
      std::memcpy(&dh, r + b * 34, 2);
      const float d = f16_bits_to_f32(dh);
      for (int i = 0; i < 32; ++i) o[b * 32 + i] = d * (float)(int8_t)r[b * 34 + 2 + i];
    }
  });
  return out;
}

torch::Tensor quantize_q4_k(torch::Tensor x) {
  x = x.contiguous().to(torch::kFloat);
  const int64_t n = x.numel();
  TORCH_CHECK(n % 256 == 0, "Q4_K needs a multiple of 256 elements");
  const int64_t nb = n / 256;
  auto out = torch::empty({nb * 144}, torch::kUInt8);
  const float* xp = x.data_ptr<float>();
  uint8_t* o = out.data_ptr<uint8_t>();
  at::parallel_for(0, nb, 64, [&](int64_t b0, int64_t b1) {
    for (int64_t b = b0; b < b1; ++b) {
      const float* v = xp + b * 256;
      float s[8], mn[8];
      float smax = 0.f, mmax = 0.f;
      for (int j = 0; j < 8; ++j) {
        fit_subblock(v + 32 * j, s[j], mn[j]);
        smax = std::max(smax, s[j]);
        mmax = std::max(mmax, mn[j]);
      }
      const float d = smax / 63.f, dmin = mmax / 63.f;
      uint8_t sc[8], m[8];
      for (int j = 0; j < 8; ++j) {
        sc[j] = d > 0.f ? (uint8_t)std::min(63L, std::lround(s[j] / d)) : 0;
        m[j] = dmin > 0.f ? (uint8_t)std::min(63L, std::lround(mn[j] / dmin)) : 0;
      }
      uint8_t* blk = o + b * 144;
      // store d/dmin rounded to fp16 and quantise against the rounded values
      const uint16_t dh = f32_to_f16_bits(d), dmh = f32_to_f16_bits(dmin);
      std::memcpy(blk, &dh, 2);
      std::memcpy(blk + 2, &dmh, 2);
      pack_scale_min_k4(sc, m, blk + 4);
      const float dr = f16_bits_to_f32(dh), dmr = f16_bits_to_f32(dmh);
      uint8_t* qs = blk + 16;
      std::memset(qs, 0, 128);
      for (int j = 0; j < 8; ++j) {
        const float step = dr * sc[j], off = dmr * m[j];
        const float inv = step > 0.f ? 1.f / step : 0.f;
        for (int i = 0; i < 32; ++i) {
          int q = (int)std::lround((v[32 * j + i] + off) * inv);
          q = std::min(15, std::max(0, q));
          uint8_t& byte = qs[32 * (j / 2) + i];
          byte |= (j & 1) ? (uint8_t)(q << 4) : (uint8_t)q;
        }
      }
    }
  });
  return out;
}

torch::Tensor dequantize_q4_k(torch::Tensor raw, int64_t n) {
  TORCH_CHECK(raw.scalar_type() == torch::kUInt8 && raw.is_contiguous(), "raw bytes");
  TORCH_CHECK(n % 256 == 0 && raw.numel() >= n / 256 * 144, "Q4_K size");
  auto out = torch::empty({n}, torch::kFloat);
  const uint8_t* r = raw.data_ptr<uint8_t>();
  float* o = out.data_ptr<float>();
  at::parallel_for(0, n / 256, 64, [&](int64_t b0, int64_t b1) {
    for (int64_t b = b0; b < b1; ++b) {
      const uint8_t* blk = r + b * 144;
      uint16_t dh, dmh;
      std::memcpy(&dh, blk, 2);
      std::memcpy(&dmh, blk + 2, 2);
      const float d = f16_bits_to_f32(dh), dmin = f16_bits_to_f32(dmh);
      const uint8_t* qs = blk + 16;
      for (int j = 0; j < 8; ++j) {
        uint8_t sc, m;
        get_scale_min_k4(j, blk + 4, sc, m);
        const float d1 = d * sc, m1 = dmin * m;
        for (int i = 0; i < 32; ++i) {
          const uint8_t byte = qs[32 * (j / 2) + i];
          const int q = (j & 1) ? (byte >> 4) : (byte & 0xF);
          o[b * 256 + 32 * j + i] = d1 * q - m1;
        }
      }
    }
  });
  return out;
}
