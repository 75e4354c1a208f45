// GGUF block formats beyond F16 / Q8_0 / Q4_K (host C++): Q4_0, Q4_1, Q5_0, Q5_1 (32-element
// blocks) and the k-quants Q2_K, Q3_K, Q5_K, Q6_K (256-element super-blocks), dequantizers and
// quantizers. Stock llama.cpp files mix these (a "Q4_K_M" file carries Q6_K and Q5_K tensors), so
// loading GGUF files unchanged needs all of them.
//
// Layouts (ggml GGUF specification; the bytes must match what other GGUF tools read and write):
//   Q4_0 (18 B)  fp16 d | u8 qs[16]            x = d * (q - 8),   q = nibble (low: j, high: j + 16)
//   Q4_1 (20 B)  fp16 d | fp16 m | u8 qs[16]   x = d * q + m
//   Q5_0 (22 B)  fp16 d | u32 qh | u8 qs[16]   x = d * (q - 16),  q = nibble | bit j of qh << 4
//   Q5_1 (24 B)  fp16 d | fp16 m | u32 qh | u8 qs[16]             x = d * q + m
//   Q2_K (84 B)  u8 scales[16] | u8 qs[64] | fp16 d | fp16 dmin
//                16 sub-blocks of 16: scales[j] = sc (low 4 bits) | m (high 4 bits),
//                x = d * sc * q - dmin * m, q two bits of qs
//   Q3_K (110 B) u8 hmask[32] | u8 qs[64] | u8 scales[12] | fp16 d
//                16 sub-blocks of 16 with 6-bit scales (packed in 12 bytes, stored + 32),
//                x = d * (s - 32) * (q - 4), q = two bits of qs | hmask bit << 2
//   Q5_K (176 B) fp16 d | fp16 dmin | u8 scales[12] | u8 qh[32] | u8 qs[128]
//                8 sub-blocks of 32, 6-bit scale and min as in Q4_K, q = nibble | qh bit << 4
//   Q6_K (210 B) u8 ql[128] | u8 qh[64] | int8 scales[16] | fp16 d
//                16 sub-blocks of 16, x = d * scale * (q - 32), q = nibble | two qh bits << 4
// Dequantization rounds exactly as the format's reference code does: fp16 scales widened to fp32,
// products evaluated left to right in fp32 with no fused multiply-add (this file is compiled
// with -ffp-contract=off), so the values agree bit for bit with other implementations.
//
// The quantizers are round-to-nearest with a per-(sub-)block range fit; they write valid blocks
// of each format (checked by dequantizing them) and are the requantization path of the converter.
#include <torch/extension.h>
#include <ATen/Parallel.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <string>

namespace {

constexpr int QK = 32;
constexpr int QKK = 256;

inline float h2f(const uint8_t* p) {
  uint16_t h;
  std::memcpy(&h, p, 2);
  c10::Half v;
  v.x = h;
  return static_cast<float>(v);
}
inline void f2h(float f, uint8_t* p) {
  const uint16_t h = c10::Half(f).x;
  std::memcpy(p, &h, 2);
}
inline float round_h(float f) { return static_cast<float>(c10::Half(f)); }

// 6-bit scale / min of sub-block j packed in 12 bytes (Q4_K / Q5_K layout)
inline void scale_min_k4(int j, const uint8_t* q, int& sc, int& m) {
  if (j < 4) {
    sc = q[j] & 63;
    m = q[j + 4] & 63;
  } else {
    sc = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
    m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
  }
}
inline void pack_scale_min_k4(const int* sc, const int* m, uint8_t* q) {
  std::memset(q, 0, 12);
  for (int j = 0; j < 4; ++j) {
    q[j] = (uint8_t)((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
    q[j + 4] = (uint8_t)((m[j] & 63) | ((m[j + 4] >> 4) << 6));
  }
  for (int j = 4; j < 8; ++j) q[j + 4] = (uint8_t)((sc[j] & 0xF) | ((m[j] & 0xF) << 4));
}

// ---------------------------------------------------------------------------- dequantizers
void deq_q4_0(const uint8_t* b, float* y) {
  const float d = h2f(b);
  const uint8_t* qs = b + 2;
  for (int j = 0; j < 16; ++j) {
    y[j] = ((int)(qs[j] & 0xF) - 8) * d;
    y[j + 16] = ((int)(qs[j] >> 4) - 8) * d;
  }
}
void deq_q4_1(const uint8_t* b, float* y) {
  const float d = h2f(b), m = h2f(b + 2);
  const uint8_t* qs = b + 4;
  for (int j = 0; j < 16; ++j) {
    y[j] = (qs[j] & 0xF) * d + m;
    y[j + 16] = (qs[j] >> 4) * d + m;
  }
}
void deq_q5_0(const uint8_t* b, float* y) {
  const float d = h2f(b);
  uint32_t qh;
  std::memcpy(&qh, b + 2, 4);
  const uint8_t* qs = b + 6;
  for (int j = 0; j < 16; ++j) {
    const int h0 = ((qh >> j) << 4) & 0x10, h1 = (qh >> (j + 12)) & 0x10;
    y[j] = (((qs[j] & 0xF) | h0) - 16) * d;
    y[j + 16] = (((qs[j] >> 4) | h1) - 16) * d;
  }
}
void deq_q5_1(const uint8_t* b, float* y) {
  const float d = h2f(b), m = h2f(b + 2);
  uint32_t qh;
  std::memcpy(&qh, b + 4, 4);
  const uint8_t* qs = b + 8;
  for (int j = 0; j < 16; ++j) {
    const int h0 = ((qh >> j) << 4) & 0x10, h1 = (qh >> (j + 12)) & 0x10;
    y[j] = ((qs[j] & 0xF) | h0) * d + m;
    y[j + 16] = ((qs[j] >> 4) | h1) * d + m;
  }
}
void deq_q2_k(const uint8_t* b, float* y) {
  const uint8_t* sc = b;
  const uint8_t* q = b + 16;
  const float d = h2f(b + 80), dmin = h2f(b + 82);
  int is = 0;
  for (int n = 0; n < QKK; n += 128) {
    int shift = 0;
    for (int j = 0; j < 4; ++j) {
      for (int half = 0; half < 2; ++half) {
        const int s = sc[is++];
        const float dl = d * (s & 0xF), ml = dmin * (s >> 4);
        for (int l = 0; l < 16; ++l) *y++ = dl * ((q[l + 16 * half] >> shift) & 3) - ml;
      }
      shift += 2;
    }
    q += 32;
  }
}
// the 16 6-bit Q3_K scales (stored + 32) unpacked from their 12 bytes
void q3k_scales(const uint8_t* s12, int8_t* out) {
  uint32_t aux[4];
  std::memcpy(aux, s12, 12);
  const uint32_t k1 = 0x03030303u, k2 = 0x0f0f0f0fu;
  const uint32_t tmp = aux[2];
  aux[2] = ((aux[0] >> 4) & k2) | (((tmp >> 4) & k1) << 4);
  aux[3] = ((aux[1] >> 4) & k2) | (((tmp >> 6) & k1) << 4);
  aux[0] = (aux[0] & k2) | (((tmp >> 0) & k1) << 4);
  aux[1] = (aux[1] & k2) | (((tmp >> 2) & k1) << 4);
  std::memcpy(out, aux, 16);
}
void deq_q3_k(const uint8_t* b, float* y) {
  const uint8_t* hm = b;
  const uint8_t* q = b + 32;
  int8_t scales[16];
  q3k_scales(b + 96, scales);
  const float d_all = h2f(b + 108);
  int is = 0;
  uint8_t m = 1;
  for (int n = 0; n < QKK; n += 128) {
    int shift = 0;
    for (int j = 0; j < 4; ++j) {
      for (int half = 0; half < 2; ++half) {
        const float dl = d_all * (scales[is++] - 32);
        for (int l = 0; l < 16; ++l) {
          const int li = l + 16 * half;
          *y++ = dl * ((int)((q[li] >> shift) & 3) - ((hm[li] & m) ? 0 : 4));
        }
      }
      shift += 2;
      m <<= 1;
    }
    q += 32;
  }
}
void deq_q5_k(const uint8_t* b, float* y) {
  const float d = h2f(b), dmin = h2f(b + 2);
  const uint8_t* scales = b + 4;
  const uint8_t* qh = b + 16;
  const uint8_t* ql = b + 48;
  int is = 0;
  uint8_t u1 = 1, u2 = 2;
  for (int j = 0; j < QKK; j += 64) {
    int sc, mn;
    scale_min_k4(is, scales, sc, mn);
    const float d1 = d * sc, m1 = dmin * mn;
    scale_min_k4(is + 1, scales, sc, mn);
    const float d2 = d * sc, m2 = dmin * mn;
    for (int l = 0; l < 32; ++l) *y++ = d1 * ((ql[l] & 0xF) + ((qh[l] & u1) ? 16 : 0)) - m1;
    for (int l = 0; l < 32; ++l) *y++ = d2 * ((ql[l] >> 4) + ((qh[l] & u2) ? 16 : 0)) - m2;
    ql += 32;
    is += 2;
    u1 <<= 2;
    u2 <<= 2;
  }
}
void deq_q6_k(const uint8_t* b, float* y) {
  const uint8_t* ql = b;
  const uint8_t* qh = b + 128;
  const int8_t* sc = reinterpret_cast<const int8_t*>(b + 192);
  const float d = h2f(b + 208);
  for (int n = 0; n < QKK; n += 128) {
    for (int l = 0; l < 32; ++l) {
      const int is = l / 16;
      const int q1 = (int)((ql[l] & 0xF) | (((qh[l] >> 0) & 3) << 4)) - 32;
      const int q2 = (int)((ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4)) - 32;
      const int q3 = (int)((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
      const int q4 = (int)((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
      y[l] = d * sc[is] * q1;
      y[l + 32] = d * sc[is + 2] * q2;
      y[l + 64] = d * sc[is + 4] * q3;
      y[l + 96] = d * sc[is + 6] * q4;
    }
    y += 128;
    ql += 64;
    qh += 32;
    sc += 8;
  }
}

// ---------------------------------------------------------------------------- quantizers
// signed value of largest magnitude
inline float signed_amax(const float* x, int n) {
  float a = 0.f, v = 0.f;
  for (int i = 0; i < n; ++i)
    if (std::fabs(x[i]) > a) {
      a = std::fabs(x[i]);
      v = x[i];
    }
  return v;
}
inline int clampi(int v, int lo, int hi) { return std::min(hi, std::max(lo, v)); }

void q_q4_0(const float* x, uint8_t* b) {
  const float d = round_h(signed_amax(x, QK) / -8.f), id = d ? 1.f / d : 0.f;
  f2h(d, b);
  for (int j = 0; j < 16; ++j) {
    const int a = clampi((int)std::lround(x[j] * id) + 8, 0, 15);
    const int c = clampi((int)std::lround(x[j + 16] * id) + 8, 0, 15);
    b[2 + j] = (uint8_t)(a | (c << 4));
  }
}
void q_q4_1(const float* x, uint8_t* b) {
  float lo = x[0], hi = x[0];
  for (int i = 1; i < QK; ++i) lo = std::min(lo, x[i]), hi = std::max(hi, x[i]);
  const float d = round_h((hi - lo) / 15.f), m = round_h(lo), id = d ? 1.f / d : 0.f;
  f2h(d, b);
  f2h(m, b + 2);
  for (int j = 0; j < 16; ++j) {
    const int a = clampi((int)std::lround((x[j] - m) * id), 0, 15);
    const int c = clampi((int)std::lround((x[j + 16] - m) * id), 0, 15);
    b[4 + j] = (uint8_t)(a | (c << 4));
  }
}
void q_q5_0(const float* x, uint8_t* b) {
  const float d = round_h(signed_amax(x, QK) / -16.f), id = d ? 1.f / d : 0.f;
  f2h(d, b);
  uint32_t qh = 0;
  for (int j = 0; j < 16; ++j) {
    const int a = clampi((int)std::lround(x[j] * id) + 16, 0, 31);
    const int c = clampi((int)std::lround(x[j + 16] * id) + 16, 0, 31);
    b[6 + j] = (uint8_t)((a & 0xF) | ((c & 0xF) << 4));
    qh |= (uint32_t)((a >> 4) & 1) << j;
    qh |= (uint32_t)((c >> 4) & 1) << (j + 16);
  }
  std::memcpy(b + 2, &qh, 4);
}
void q_q5_1(const float* x, uint8_t* b) {
  float lo = x[0], hi = x[0];
  for (int i = 1; i < QK; ++i) lo = std::min(lo, x[i]), hi = std::max(hi, x[i]);
  const float d = round_h((hi - lo) / 31.f), m = round_h(lo), id = d ? 1.f / d : 0.f;
  f2h(d, b);
  f2h(m, b + 2);
  uint32_t qh = 0;
  for (int j = 0; j < 16; ++j) {
    const int a = clampi((int)std::lround((x[j] - m) * id), 0, 31);
    const int c = clampi((int)std::lround((x[j + 16] - m) * id), 0, 31);
    b[8 + j] = (uint8_t)((a & 0xF) | ((c & 0xF) << 4));
    qh |= (uint32_t)((a >> 4) & 1) << j;
    qh |= (uint32_t)((c >> 4) & 1) << (j + 16);
  }
  std::memcpy(b + 4, &qh, 4);
}

// x ~ s * q - mn over n values, q in [0, levels], mn >= 0: range fit
inline void range_fit(const float* x, int n, int levels, float& s, float& mn) {
  float lo = x[0], hi = x[0];
  for (int i = 1; i < n; ++i) lo = std::min(lo, x[i]), hi = std::max(hi, x[i]);
  lo = std::min(lo, 0.f);
  s = hi > lo ? (hi - lo) / levels : 0.f;
  mn = -lo;
}

void q_q2_k(const float* x, uint8_t* b) {
  float s[16], mn[16], smax = 0.f, mmax = 0.f;
  for (int j = 0; j < 16; ++j) {
    range_fit(x + 16 * j, 16, 3, s[j], mn[j]);
    smax = std::max(smax, s[j]);
    mmax = std::max(mmax, mn[j]);
  }
  const float d = round_h(smax / 15.f), dmin = round_h(mmax / 15.f);
  f2h(d, b + 80);
  f2h(dmin, b + 82);
  int L[QKK];
  for (int j = 0; j < 16; ++j) {
    const int sc = d ? clampi((int)std::lround(s[j] / d), 0, 15) : 0;
    const int m = dmin ? clampi((int)std::lround(mn[j] / dmin), 0, 15) : 0;
    b[j] = (uint8_t)(sc | (m << 4));
    const float dl = d * sc, ml = dmin * m;
    for (int l = 0; l < 16; ++l)
      L[16 * j + l] = dl ? clampi((int)std::lround((x[16 * j + l] + ml) / dl), 0, 3) : 0;
  }
  // element 16 * sub + l sits in byte (n/128)*32 + (sub%2)*16 + l at shift 2 * ((sub%8)/2)
  uint8_t* q = b + 16;
  std::memset(q, 0, 64);
  for (int i = 0; i < QKK; ++i) {
    const int n = i / 128, r = i % 128, sub = r / 16, l = r % 16;
    q[n * 32 + (sub % 2) * 16 + l] |= (uint8_t)(L[i] << (2 * (sub / 2)));
  }
}
void q_q3_k(const float* x, uint8_t* b) {
  float s[16], amax = 0.f, sv = 0.f;
  for (int j = 0; j < 16; ++j) {
    s[j] = signed_amax(x + 16 * j, 16) / -4.f;
    if (std::fabs(s[j]) > amax) amax = std::fabs(s[j]), sv = s[j];
  }
  const float d = round_h(sv / -32.f);
  f2h(d, b + 108);
  int sc[16], L[QKK];
  for (int j = 0; j < 16; ++j) {
    sc[j] = d ? clampi((int)std::lround(s[j] / d), -32, 31) : 0;
    const float dl = d * sc[j];
    for (int l = 0; l < 16; ++l) L[16 * j + l] = dl ? clampi((int)std::lround(x[16 * j + l] / dl), -4, 3) + 4 : 4;
  }
  // scales: 6-bit (sc + 32); low 4 bits of scales j and j+8 share byte j (j < 8), high 2 bits in bytes 8..11
  uint8_t* s12 = b + 96;
  std::memset(s12, 0, 12);
  for (int j = 0; j < 16; ++j) {
    const int u = sc[j] + 32;
    if (j < 8)
      s12[j] |= (uint8_t)(u & 0xF);
    else
      s12[j - 8] |= (uint8_t)((u & 0xF) << 4);
    s12[8 + (j % 4)] |= (uint8_t)((u >> 4) << (2 * (j / 4)));
  }
  uint8_t* hm = b;
  uint8_t* q = b + 32;
  std::memset(hm, 0, 32);
  std::memset(q, 0, 64);
  for (int i = 0; i < QKK; ++i) {
    const int n = i / 128, r = i % 128, sub = r / 16, l = r % 16;
    const int pos = (sub % 2) * 16 + l;
    q[n * 32 + pos] |= (uint8_t)((L[i] & 3) << (2 * (sub / 2)));
    if (L[i] & 4) hm[pos] |= (uint8_t)(1u << (n * 4 + sub / 2));
  }
}
void q_q5_k(const float* x, uint8_t* b) {
  float s[8], mn[8], smax = 0.f, mmax = 0.f;
  for (int j = 0; j < 8; ++j) {
    range_fit(x + 32 * j, 32, 31, s[j], mn[j]);
    smax = std::max(smax, s[j]);
    mmax = std::max(mmax, mn[j]);
  }
  const float d = round_h(smax / 63.f), dmin = round_h(mmax / 63.f);
  f2h(d, b);
  f2h(dmin, b + 2);
  int sc[8], m[8];
  for (int j = 0; j < 8; ++j) {
    sc[j] = d ? clampi((int)std::lround(s[j] / d), 0, 63) : 0;
    m[j] = dmin ? clampi((int)std::lround(mn[j] / dmin), 0, 63) : 0;
  }
  pack_scale_min_k4(sc, m, b + 4);
  uint8_t* qh = b + 16;
  uint8_t* ql = b + 48;
  std::memset(qh, 0, 32);
  std::memset(ql, 0, 128);
  for (int j = 0; j < 8; ++j) {
    const float dl = d * sc[j], ml = dmin * m[j];
    for (int l = 0; l < 32; ++l) {
      const int q = dl ? clampi((int)std::lround((x[32 * j + l] + ml) / dl), 0, 31) : 0;
      const int pair = j / 2;
      ql[pair * 32 + l] |= (uint8_t)((q & 0xF) << (4 * (j % 2)));
      if (q & 16) qh[l] |= (uint8_t)(1u << j);
    }
  }
}
void q_q6_k(const float* x, uint8_t* b) {
  float s[16], amax = 0.f, sv = 0.f;
  for (int j = 0; j < 16; ++j) {
    s[j] = signed_amax(x + 16 * j, 16) / -32.f;
    if (std::fabs(s[j]) > amax) amax = std::fabs(s[j]), sv = s[j];
  }
  const float d = round_h(sv / -128.f);
  f2h(d, b + 208);
  int8_t* scs = reinterpret_cast<int8_t*>(b + 192);
  uint8_t* ql = b;
  uint8_t* qh = b + 128;
  std::memset(ql, 0, 128);
  std::memset(qh, 0, 64);
  for (int j = 0; j < 16; ++j) {
    const int sc = d ? clampi((int)std::lround(s[j] / d), -128, 127) : 0;
    scs[j] = (int8_t)sc;
    const float dl = d * sc;
    for (int l = 0; l < 16; ++l) {
      const int i = 16 * j + l;
      const int q = dl ? clampi((int)std::lround(x[i] / dl), -32, 31) + 32 : 32;
      // element i: half n = i / 128, r = i % 128, quarter k = r / 32, lane = r % 32
      const int n = i / 128, r = i % 128, k = r / 32, lane = r % 32;
      ql[n * 64 + (k % 2) * 32 + lane] |= (uint8_t)((q & 0xF) << (4 * (k / 2)));
      qh[n * 32 + lane] |= (uint8_t)(((q >> 4) & 3) << (2 * k));
    }
  }
}

struct Fmt {
  int block, bytes;
  void (*deq)(const uint8_t*, float*);
  void (*q)(const float*, uint8_t*);
};

Fmt fmt_of(int64_t t) {
  switch (t) {
    case 2: return {QK, 18, deq_q4_0, q_q4_0};
    case 3: return {QK, 20, deq_q4_1, q_q4_1};
    case 6: return {QK, 22, deq_q5_0, q_q5_0};
    case 7: return {QK, 24, deq_q5_1, q_q5_1};
    case 10: return {QKK, 84, deq_q2_k, q_q2_k};
    case 11: return {QKK, 110, deq_q3_k, q_q3_k};
    case 13: return {QKK, 176, deq_q5_k, q_q5_k};
    case 14: return {QKK, 210, deq_q6_k, q_q6_k};
    default: TORCH_CHECK(false, "ggml type ", t, " is not handled here");
  }
}

}  // namespace

// Dequantize `n` values of ggml type `type` (2 Q4_0, 3 Q4_1, 6 Q5_0, 7 Q5_1, 10 Q2_K, 11 Q3_K,
// 13 Q5_K, 14 Q6_K) from raw block bytes to fp32.
torch::Tensor gguf_dequantize(torch::Tensor raw, int64_t type, int64_t n) {
  const Fmt f = fmt_of(type);
  TORCH_CHECK(raw.dtype() == torch::kUInt8 && raw.is_contiguous() && !raw.is_cuda(), "raw: contiguous CPU uint8");
  TORCH_CHECK(n % f.block == 0, "element count must be a multiple of the block size");
  const int64_t nb = n / f.block;
  TORCH_CHECK(raw.numel() >= nb * f.bytes, "raw buffer too small");
  auto out = torch::empty({n}, torch::kFloat32);
  const uint8_t* src = raw.data_ptr<uint8_t>();
  float* dst = out.data_ptr<float>();
  at::parallel_for(0, nb, 1024, [&](int64_t b0, int64_t b1) {
    for (int64_t b = b0; b < b1; ++b) f.deq(src + b * f.bytes, dst + b * f.block);
  });
  return out;
}

// Quantize fp32 values into ggml blocks of `type`.
torch::Tensor gguf_quantize(torch::Tensor x, int64_t type) {
  const Fmt f = fmt_of(type);
  x = x.contiguous().to(torch::kFloat32).cpu();
  const int64_t n = x.numel();
  TORCH_CHECK(n % f.block == 0, "element count must be a multiple of the block size");
  const int64_t nb = n / f.block;
  auto out = torch::empty({nb * f.bytes}, torch::kUInt8);
  const float* src = x.data_ptr<float>();
  uint8_t* dst = out.data_ptr<uint8_t>();
  at::parallel_for(0, nb, 256, [&](int64_t b0, int64_t b1) {
    for (int64_t b = b0; b < b1; ++b) f.q(src + b * f.block, dst + b * f.bytes);
  });
  return out;
}
