// K9: GGUF-quantized weights on the GPU (sm_100a): Q4_K / Q8_0 GEMV and dequantization.
//
// Weights stay in their ggml block format in HBM ([N rows] x [K/256 Q4_K blocks of 144 B] or
// [K/32 Q8_0 blocks of 34 B]) and are decoded in registers.
//   q4k_gemv   y[m, n] = sum_k x[m, k] W[n, k] for up to 16 tokens (decode): one warp per row group,
//              lane l decodes 8 weights of sub-block l/4 of every super-block (one 8-byte load of
//              packed nibbles + the 6-bit scale/min of that sub-block) and applies them to every
//              token; optional SwiGLU epilogue over gate/up rows interleaved in groups of 64.
//   q8_0_gemv  same for Q8_0 (lm_head / embeddings of Q4_K_M-style checkpoints).
//   q6k_gemv   same for Q6_K (the output matrix and the more-bits attn_v / ffn_down tensors of
//              Q4_K_M files): lane l decodes weights [8l, 8l + 8) of each 210-byte super-block.
//   dequant_*  whole-matrix dequantization to bf16 (prefill: followed by the tcgen05 GEMM).
// Block layouts: ggml spec (see csrc/host/gguf_quant.cpp); the reference decodes these only on
// the CPU (runner/gguf/gollek-gguf-loader/…/gguf/quant/Dequantizer.java, GGUFVectorOps.java:73-88).
#include "../common/common.cuh"
#include "../common/tma_host.h"
#include "launchers.h"

#include <algorithm>
#include <cstdlib>

using namespace gollek;

namespace {

constexpr int kGemvMaxTok = 16;
constexpr int kGemvWarps = 8;

GOLLEK_DEVICE float h2f(const uint8_t* p) {
  __half h;
  *reinterpret_cast<uint16_t*>(&h) = *reinterpret_cast<const uint16_t*>(p);
  return __half2float(h);
}

// Decode the 8 Q4_K weights lane `lane` owns in one 144-byte super-block, from the block's 16-byte
// header (d, dmin, 12 bytes of packed 6-bit scales / mins) and the lane's 8 bytes of nibbles.
GOLLEK_DEVICE uint32_t q4k_sbyte(const uint4& hdr, int i) {  // byte i of the 12 packed scale bytes
  const uint32_t w = i < 4 ? hdr.y : (i < 8 ? hdr.z : hdr.w);
  return (w >> (8 * (i & 3))) & 0xFF;
}

GOLLEK_DEVICE float half_bits(uint32_t bits) {
  __half h;
  *reinterpret_cast<uint16_t*>(&h) = (uint16_t)bits;
  return __half2float(h);
}

GOLLEK_DEVICE void q4k_decode8_regs(const uint4 hdr, const uint2 q, int lane, float* w) {
  const int j = lane >> 2;
  const float d = half_bits(hdr.x & 0xFFFF), dmin = half_bits(hdr.x >> 16);
  uint32_t sv, mv;
  if (j < 4) {
    sv = q4k_sbyte(hdr, j) & 63;
    mv = q4k_sbyte(hdr, j + 4) & 63;
  } else {
    sv = (q4k_sbyte(hdr, j + 4) & 0xF) | ((q4k_sbyte(hdr, j - 4) >> 6) << 4);
    mv = (q4k_sbyte(hdr, j + 4) >> 4) | ((q4k_sbyte(hdr, j) >> 6) << 4);
  }
  const float a = d * (float)sv, b = dmin * (float)mv;
  const uint32_t qq[2] = {q.x, q.y};
  const int shift = (j & 1) ? 4 : 0;
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const uint32_t byte = (qq[e >> 2] >> (8 * (e & 3))) & 0xFF;
    w[e] = a * (float)((byte >> shift) & 0xF) - b;
  }
}

// The GEMV's form of the same decode, without an integer-to-float conversion per weight. The 8
// nibbles n_e become f_e = 1 + n_e / 16 by placing each nibble in the mantissa of 1.0f (one byte
// permute per weight), and the lane's dot product with x over its 8 weights is
//   sum_e (a n_e - b) x_e = 16 a sum_e f_e x_e - (16 a + b) sum_e x_e,
// so a row costs one FMA per weight; sum_e x_e is shared by every row of the warp. a16 = 16 a and
// c = 16 a + b come from the sub-block's scale and min.
// Conversions on the ALU / FMA pipes instead of the conversion unit (measured at 87 % busy when every
// lane converted its block's scales with F2F / I2F): a half's sign, exponent and mantissa moved into
// float position and scaled by 2^112 (the exponent bias difference; exact for every finite half,
// subnormals and zero included), and a small integer through the 2^23 magic constant.
GOLLEK_DEVICE float half_bits_alu(uint32_t h) {
  return __uint_as_float(((h & 0x8000u) << 16) | ((h & 0x7FFFu) << 13)) * 0x1p112f;
}
GOLLEK_DEVICE float small_uint_to_float(uint32_t v) {  // exact for v < 2^23
  return __uint_as_float(0x4B000000u | v) - 8388608.f;
}

GOLLEK_DEVICE void q4k_scales_regs(const uint4 hdr, int lane, float& a16, float& c) {
  const int j = lane >> 2;
  const float d = half_bits_alu(hdr.x & 0xFFFF), dmin = half_bits_alu(hdr.x >> 16);
  uint32_t sv, mv;
  if (j < 4) {
    sv = q4k_sbyte(hdr, j) & 63;
    mv = q4k_sbyte(hdr, j + 4) & 63;
  } else {
    sv = (q4k_sbyte(hdr, j + 4) & 0xF) | ((q4k_sbyte(hdr, j - 4) >> 6) << 4);
    mv = (q4k_sbyte(hdr, j + 4) >> 4) | ((q4k_sbyte(hdr, j) >> 6) << 4);
  }
  a16 = 16.f * (d * small_uint_to_float(sv));
  c = a16 + dmin * small_uint_to_float(mv);
}

GOLLEK_DEVICE void q4k_unpack8_unit(const uint2 q, int lane, float* f) {
  // nibble k of byte e (low for even sub-blocks, high for odd) -> bits 3..6 of that byte, 0x80 set:
  // byte value 0x80 | n << 3 placed as byte 2 under 0x3F gives the float bits 0x3F800000 | n << 19
  const bool hi = ((lane >> 2) & 1) != 0;
  const uint32_t t0 = hi ? (q.x >> 1) : (q.x << 3), t1 = hi ? (q.y >> 1) : (q.y << 3);
  const uint32_t v0 = (t0 & 0x78787878u) | 0x80808080u, v1 = (t1 & 0x78787878u) | 0x80808080u;
  f[0] = __uint_as_float(__byte_perm(v0, 0x3F000000u, 0x7054));
  f[1] = __uint_as_float(__byte_perm(v0, 0x3F000000u, 0x7154));
  f[2] = __uint_as_float(__byte_perm(v0, 0x3F000000u, 0x7254));
  f[3] = __uint_as_float(__byte_perm(v0, 0x3F000000u, 0x7354));
  f[4] = __uint_as_float(__byte_perm(v1, 0x3F000000u, 0x7054));
  f[5] = __uint_as_float(__byte_perm(v1, 0x3F000000u, 0x7154));
  f[6] = __uint_as_float(__byte_perm(v1, 0x3F000000u, 0x7254));
  f[7] = __uint_as_float(__byte_perm(v1, 0x3F000000u, 0x7354));
}

GOLLEK_DEVICE void q4k_decode8(const uint8_t* blk, int lane, float* w) {
  q4k_decode8_regs(*reinterpret_cast<const uint4*>(blk),
                   *reinterpret_cast<const uint2*>(blk + 16 + 32 * (lane >> 3) + (lane & 3) * 8), lane, w);
}

// KS warps share a row pair, each over 1/KS of the super-blocks (partial sums added through shared
// memory): a narrow matrix (4096 rows = 2048 pairs) otherwise gives each SM only ~14 warps, each
// walking a long serial decode-and-FMA chain over all of K.
template <int NT, bool SWIGLU, int KS>
__global__ void __launch_bounds__(kGemvWarps * 32, NT == 1 ? 3 : 1)
    q4k_gemv_kernel(__nv_bfloat16* __restrict__ y, int64_t ldy, const __nv_bfloat16* __restrict__ x, int64_t ldx,
                    const uint8_t* __restrict__ W, int N, int K, int M) {
  // each warp group of KS owns a pair of rows: (n, n + 64) in SwiGLU mode (gate, up), (2i, 2i+1) otherwise
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int pair = blockIdx.x * (kGemvWarps / KS) + warp / KS;
  const int kq = warp % KS;
  int r0, r1;
  if (SWIGLU) {
    const int grp = pair / 64, within = pair % 64;
    r0 = grp * 128 + within;
    r1 = r0 + 64;
  } else {
    r0 = 2 * pair;
    r1 = r0 + 1;
  }
  const bool live = r0 < N;
  if (KS == 1 && !live) return;
  const bool has1 = r1 < N;
  const int nblk = K / 256;
  const int64_t row_bytes = (int64_t)nblk * 144;
  const uint8_t* w0 = W + (int64_t)(live ? r0 : 0) * row_bytes;
  const uint8_t* w1 = W + (int64_t)(has1 ? r1 : (live ? r0 : 0)) * row_bytes;
  float acc0[NT], acc1[NT];
#pragma unroll
  for (int m = 0; m < NT; ++m) acc0[m] = acc1[m] = 0.f;
  const int koff = (lane >> 2) * 32 + (lane & 3) * 8;
  const int qoff = 16 + 32 * (lane >> 3) + (lane & 3) * 8;  // lane's nibbles inside a block
  const int bbeg = live ? kq * nblk / KS : 0, bend = live ? (kq + 1) * nblk / KS : 0;
  // kBU super-blocks per round: their loads are all issued before any is decoded
  constexpr int kBU = 4;
  for (int b0 = bbeg; b0 < bend; b0 += kBU) {
    uint4 h0[kBU], h1[kBU];
    uint2 q0[kBU], q1[kBU];
#pragma unroll
    for (int u = 0; u < kBU; ++u) {
      const int b = min(b0 + u, bend - 1);
      h0[u] = __ldg(reinterpret_cast<const uint4*>(w0 + b * 144));
      h1[u] = __ldg(reinterpret_cast<const uint4*>(w1 + b * 144));
      q0[u] = __ldg(reinterpret_cast<const uint2*>(w0 + b * 144 + qoff));
      q1[u] = __ldg(reinterpret_cast<const uint2*>(w1 + b * 144 + qoff));
    }
#pragma unroll
    for (int u = 0; u < kBU; ++u) {
      const int b = b0 + u;
      if (b >= bend) break;
      float fa[8], fb[8], a0, c0, a1, c1;
      q4k_scales_regs(h0[u], lane, a0, c0);
      q4k_scales_regs(h1[u], lane, a1, c1);
      q4k_unpack8_unit(q0[u], lane, fa);
      q4k_unpack8_unit(q1[u], lane, fb);
#pragma unroll
      for (int m = 0; m < NT; ++m) {
        if (m < M) {
          float xv[8];
          bf16x8_to_float(__ldg(reinterpret_cast<const uint4*>(x + (int64_t)m * ldx + b * 256 + koff)), xv);
          float sx = 0.f, sa = 0.f, sb = 0.f;
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            sx += xv[e];
            sa = fmaf(fa[e], xv[e], sa);
            sb = fmaf(fb[e], xv[e], sb);
          }
          acc0[m] = fmaf(a0, sa, fmaf(-c0, sx, acc0[m]));
          acc1[m] = fmaf(a1, sb, fmaf(-c1, sx, acc1[m]));
        }
      }
    }
  }
  __shared__ float red[KS > 1 ? kGemvWarps : 1][2][NT];
#pragma unroll
  for (int m = 0; m < NT; ++m) {
    if (m < M) {
      float s0 = warp_sum(acc0[m]);
      float s1 = warp_sum(acc1[m]);
      if (KS > 1) {
        if (lane == 0) {
          red[KS > 1 ? warp : 0][0][m] = s0;
          red[KS > 1 ? warp : 0][1][m] = s1;
        }
      } else if (lane == 0) {
        if (SWIGLU) {
          const int on = (r0 / 128) * 64 + r0 % 128;
          y[(int64_t)m * ldy + on] = __float2bfloat16(silu(s0) * s1);
        } else {
          y[(int64_t)m * ldy + r0] = __float2bfloat16(s0);
          if (has1) y[(int64_t)m * ldy + r1] = __float2bfloat16(s1);
        }
      }
    }
  }
  if (KS == 1) return;
  __syncthreads();
  if (!live || kq != 0 || lane >= NT || lane >= M) return;
  // lane m sums token m's KS partials of the pair (in K order)
  const int m = lane;
  float s0 = 0.f, s1 = 0.f;
#pragma unroll
  for (int q = 0; q < KS; ++q) {
    s0 += red[KS > 1 ? warp + q : 0][0][m];
    s1 += red[KS > 1 ? warp + q : 0][1][m];
  }
  if (SWIGLU) {
    const int on = (r0 / 128) * 64 + r0 % 128;
    y[(int64_t)m * ldy + on] = __float2bfloat16(silu(s0) * s1);
  } else {
    y[(int64_t)m * ldy + r0] = __float2bfloat16(s0);
    if (has1) y[(int64_t)m * ldy + r1] = __float2bfloat16(s1);
  }
}

template <int NT>
__global__ void __launch_bounds__(kGemvWarps * 32) q8_0_gemv_kernel(__nv_bfloat16* __restrict__ y, int64_t ldy,
                                                                    const __nv_bfloat16* __restrict__ x, int64_t ldx,
                                                                    const uint8_t* __restrict__ W, int N, int K,
                                                                    int M) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * kGemvWarps + warp;
  if (row >= N) return;
  const int nblk = K / 32;
  const uint8_t* wr = W + (int64_t)row * nblk * 34;
  float acc[NT];
#pragma unroll
  for (int m = 0; m < NT; ++m) acc[m] = 0.f;
  // lane handles 8 weights: block b = i / 4, quarter = i % 4, for i = lane, lane + 32, ...
  for (int i = lane; i < nblk * 4; i += 32) {
    const int b = i >> 2, qtr = i & 3;
    const uint8_t* blk = wr + b * 34;
    const float d = h2f(blk);
    // Q8_0 blocks are 34 bytes, so only 2-byte alignment is guaranteed: load 4 x u16
    const uint16_t* q16 = reinterpret_cast<const uint16_t*>(blk + 2 + qtr * 8);
    float w[8];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const uint16_t v = q16[e];
      w[2 * e] = d * (float)(int8_t)(v & 0xFF);
      w[2 * e + 1] = d * (float)(int8_t)(v >> 8);
    }
#pragma unroll
    for (int m = 0; m < NT; ++m) {
      if (m < M) {
        float xv[8];
        bf16x8_to_float(__ldg(reinterpret_cast<const uint4*>(x + (int64_t)m * ldx + b * 32 + qtr * 8)), xv);
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[m] = fmaf(w[e], xv[e], acc[m]);
      }
    }
  }
#pragma unroll
  for (int m = 0; m < NT; ++m) {
    if (m < M) {
      const float s = warp_sum(acc[m]);
      if (lane == 0) y[(int64_t)m * ldy + row] = __float2bfloat16(s);
    }
  }
}

// The 8 Q6_K weights [8g, 8g + 8) of one 210-byte super-block (ql[128] | qh[64] | int8 scales[16] |
// fp16 d). Element i: half n = i / 128, quarter k = (i % 128) / 32, position p = i % 32; low 4 bits
// from ql[64n + 32(k % 2) + p] (high nibble when k >= 2), 2 high bits from qh[32n + p] at bit 2k,
// scale scales[8n + 2k + p / 16]; w = d * scale * (q - 32). Blocks are only 2-byte aligned.
GOLLEK_DEVICE void q6k_decode8(const uint8_t* blk, int g, float* w) {
  const int i0 = 8 * g;
  const int n = i0 >> 7, r = i0 & 127, k = r >> 5, p0 = r & 31;
  const uint16_t* ql = reinterpret_cast<const uint16_t*>(blk + 64 * n + 32 * (k & 1) + p0);
  const uint16_t* qh = reinterpret_cast<const uint16_t*>(blk + 128 + 32 * n + p0);
  const float d = h2f(blk + 208);
  const float sc = d * (float)reinterpret_cast<const int8_t*>(blk + 192)[8 * n + 2 * k + (p0 >> 4)];
  const int lshift = (k >> 1) * 4, hshift = 2 * k;
#pragma unroll
  for (int e2 = 0; e2 < 4; ++e2) {
    const uint32_t l2 = ql[e2], h2 = qh[e2];
#pragma unroll
    for (int b = 0; b < 2; ++b) {
      const uint32_t lo = ((l2 >> (8 * b)) >> lshift) & 0xF;
      const uint32_t hi = ((h2 >> (8 * b)) >> hshift) & 0x3;
      w[2 * e2 + b] = sc * (float)((int)(lo | (hi << 4)) - 32);
    }
  }
}

template <int NT>
__global__ void __launch_bounds__(kGemvWarps * 32) q6k_gemv_kernel(__nv_bfloat16* __restrict__ y, int64_t ldy,
                                                                   const __nv_bfloat16* __restrict__ x, int64_t ldx,
                                                                   const uint8_t* __restrict__ W, int N, int K,
                                                                   int M) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * kGemvWarps + warp;
  if (row >= N) return;
  const int nblk = K / 256;
  const uint8_t* wr = W + (int64_t)row * nblk * 210;
  float acc[NT];
#pragma unroll
  for (int m = 0; m < NT; ++m) acc[m] = 0.f;
  for (int b = 0; b < nblk; ++b) {
    float w[8];
    q6k_decode8(wr + (int64_t)b * 210, lane, w);
#pragma unroll
    for (int m = 0; m < NT; ++m) {
      if (m < M) {
        float xv[8];
        bf16x8_to_float(__ldg(reinterpret_cast<const uint4*>(x + (int64_t)m * ldx + b * 256 + lane * 8)), xv);
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[m] = fmaf(w[e], xv[e], acc[m]);
      }
    }
  }
#pragma unroll
  for (int m = 0; m < NT; ++m) {
    if (m < M) {
      const float s = warp_sum(acc[m]);
      if (lane == 0) y[(int64_t)m * ldy + row] = __float2bfloat16(s);
    }
  }
}

__global__ void dequant_q6k_kernel(__nv_bfloat16* __restrict__ out, const uint8_t* __restrict__ W, int64_t nblocks) {
  const int lane = threadIdx.x & 31;
  const int64_t wid = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t b = wid; b < nblocks; b += nw) {
    float w[8];
    q6k_decode8(W + b * 210, lane, w);
    *reinterpret_cast<uint4*>(out + b * 256 + lane * 8) = float_to_bf16x8(w);
  }
}

// One 256-weight super-block per warp-iteration: lane l writes its 8 decoded weights.
__global__ void dequant_q4k_kernel(__nv_bfloat16* __restrict__ out, const uint8_t* __restrict__ W,
                                   int64_t nblocks) {
  const int lane = threadIdx.x & 31;
  const int64_t wid = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t b = wid; b < nblocks; b += nw) {
    float w[8];
    q4k_decode8(W + b * 144, lane, w);
    const int koff = (lane >> 2) * 32 + (lane & 3) * 8;
    *reinterpret_cast<uint4*>(out + b * 256 + koff) = float_to_bf16x8(w);
  }
}

__global__ void dequant_q8_0_kernel(__nv_bfloat16* __restrict__ out, const uint8_t* __restrict__ W,
                                    int64_t nblocks) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;  // one quarter block (8 weights)
  if (i >= nblocks * 4) return;
  const int64_t b = i >> 2;
  const int qtr = i & 3;
  const uint8_t* blk = W + b * 34;
  const float d = h2f(blk);
  float w[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) w[e] = d * (float)(int8_t)blk[2 + qtr * 8 + e];
  *reinterpret_cast<uint4*>(out + b * 32 + qtr * 8) = float_to_bf16x8(w);
}

// Embedding rows gathered from a Q8_0 table.
__global__ void embedding_q8_0_kernel(__nv_bfloat16* __restrict__ out, const int* __restrict__ ids,
                                      const uint8_t* __restrict__ table, int d, int vocab) {
  const int t = blockIdx.x;
  int id = ids[t];
  id = id < 0 ? 0 : (id >= vocab ? vocab - 1 : id);
  const uint8_t* row = table + (int64_t)id * (d / 32) * 34;
  for (int i = threadIdx.x; i < d / 8; i += blockDim.x) {
    const uint8_t* blk = row + (i >> 2) * 34;
    const float dd = h2f(blk);
    float w[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) w[e] = dd * (float)(int8_t)blk[2 + (i & 3) * 8 + e];
    *reinterpret_cast<uint4*>(out + (int64_t)t * d + i * 8) = float_to_bf16x8(w);
  }
}

}  // namespace

namespace gollek {

// GOLLEK_GEMV_KSPLIT=0: one warp per row pair over all of K (read at every call)
static bool gemv_ksplit_off() {
  const char* e = getenv("GOLLEK_GEMV_KSPLIT");
  return e && e[0] == '0';
}

void launch_gguf_gemv(void* y, int64_t ldy, const void* x, int64_t ldx, const void* W, int qtype, int N, int K,
                      int M, bool swiglu, cudaStream_t s) {
  throw_if(M < 1 || M > kGemvMaxTok, "gguf gemv: 1..16 tokens");
  throw_if(qtype == 12 && K % 256 != 0, "Q4_K: K must be a multiple of 256");
  throw_if(qtype == 8 && K % 32 != 0, "Q8_0: K must be a multiple of 32");
  throw_if(qtype == 14 && K % 256 != 0, "Q6_K: K must be a multiple of 256");
  throw_if(swiglu && (qtype != 12 || N % 128 != 0), "gguf gemv swiglu: Q4_K with N % 128 == 0");
  const auto* xp = reinterpret_cast<const __nv_bfloat16*>(x);
  auto* yp = reinterpret_cast<__nv_bfloat16*>(y);
  const auto* wp = reinterpret_cast<const uint8_t*>(W);
  if (qtype == 12) {
    const int pairs = (N + 1) / 2;
    // warps per row pair: enough warps for ~32 per SM, each over >= 8 super-blocks
    const int nblk = K / 256;
    int ks = 1;
    while (ks < 4 && pairs * ks < 32 * num_sms() && nblk / (2 * ks) >= 8) ks *= 2;
    if (gemv_ksplit_off()) ks = 1;
    const int grid = (pairs * ks + kGemvWarps - 1) / kGemvWarps;
#define GOLLEK_Q4K(NT, KS)                                                                                     \
  if (M <= NT && ks == KS) {                                                                                  \
    if (swiglu) q4k_gemv_kernel<NT, true, KS><<<grid, kGemvWarps * 32, 0, s>>>(yp, ldy, xp, ldx, wp, N, K, M); \
    else q4k_gemv_kernel<NT, false, KS><<<grid, kGemvWarps * 32, 0, s>>>(yp, ldy, xp, ldx, wp, N, K, M);       \
    check_launch("q4k_gemv");                                                                                 \
    return;                                                                                                   \
  }
    GOLLEK_Q4K(1, 1)
    GOLLEK_Q4K(1, 2)
    GOLLEK_Q4K(1, 4)
    GOLLEK_Q4K(4, 1)
    GOLLEK_Q4K(4, 2)
    GOLLEK_Q4K(4, 4)
    GOLLEK_Q4K(8, 1)
    GOLLEK_Q4K(16, 1)
#undef GOLLEK_Q4K
    ks = 1;  // 8 / 16 tokens: no K split
    const int grid1 = (pairs + kGemvWarps - 1) / kGemvWarps;
    if (M <= 8) {
      if (swiglu) q4k_gemv_kernel<8, true, 1><<<grid1, kGemvWarps * 32, 0, s>>>(yp, ldy, xp, ldx, wp, N, K, M);
      else q4k_gemv_kernel<8, false, 1><<<grid1, kGemvWarps * 32, 0, s>>>(yp, ldy, xp, ldx, wp, N, K, M);
    } else {
      if (swiglu) q4k_gemv_kernel<16, true, 1><<<grid1, kGemvWarps * 32, 0, s>>>(yp, ldy, xp, ldx, wp, N, K, M);
      else q4k_gemv_kernel<16, false, 1><<<grid1, kGemvWarps * 32, 0, s>>>(yp, ldy, xp, ldx, wp, N, K, M);
    }
    check_launch("q4k_gemv");
    return;
  } else if (qtype == 8) {
    const int grid = (N + kGemvWarps - 1) / kGemvWarps;
#define GOLLEK_Q8(NT)                                                                                 \
  if (M <= NT) {                                                                                    \
    q8_0_gemv_kernel<NT><<<grid, kGemvWarps * 32, 0, s>>>(yp, ldy, xp, ldx, wp, N, K, M);          \
    check_launch("q8_0_gemv");                                                                      \
    return;                                                                                         \
  }
    GOLLEK_Q8(1)
    GOLLEK_Q8(4)
    GOLLEK_Q8(8)
    GOLLEK_Q8(16)
#undef GOLLEK_Q8
  } else if (qtype == 14) {
    const int grid = (N + kGemvWarps - 1) / kGemvWarps;
#define GOLLEK_Q6(NT)                                                                                 \
  if (M <= NT) {                                                                                    \
    q6k_gemv_kernel<NT><<<grid, kGemvWarps * 32, 0, s>>>(yp, ldy, xp, ldx, wp, N, K, M);           \
    check_launch("q6k_gemv");                                                                       \
    return;                                                                                         \
  }
    GOLLEK_Q6(1)
    GOLLEK_Q6(4)
    GOLLEK_Q6(8)
    GOLLEK_Q6(16)
#undef GOLLEK_Q6
  }
  throw_if(true, "gguf gemv: unsupported ggml type " + std::to_string(qtype));
}

void launch_gguf_dequant(void* out, const void* W, int qtype, int64_t numel, cudaStream_t s) {
  const auto* wp = reinterpret_cast<const uint8_t*>(W);
  auto* op = reinterpret_cast<__nv_bfloat16*>(out);
  if (qtype == 12) {
    throw_if(numel % 256 != 0, "Q4_K dequant: size");
    const int64_t nb = numel / 256;
    const int grid = (int)std::min<int64_t>((nb + 7) / 8, 148 * 16);
    dequant_q4k_kernel<<<grid, 256, 0, s>>>(op, wp, nb);
  } else if (qtype == 8) {
    throw_if(numel % 32 != 0, "Q8_0 dequant: size");
    const int64_t nq = numel / 8;
    dequant_q8_0_kernel<<<(unsigned)((nq + 255) / 256), 256, 0, s>>>(op, wp, numel / 32);
  } else if (qtype == 14) {
    throw_if(numel % 256 != 0, "Q6_K dequant: size");
    const int64_t nb = numel / 256;
    const int grid = (int)std::min<int64_t>((nb + 7) / 8, 148 * 16);
    dequant_q6k_kernel<<<grid, 256, 0, s>>>(op, wp, nb);
  } else {
    throw_if(true, "gguf dequant: unsupported ggml type " + std::to_string(qtype));
  }
  check_launch("gguf_dequant");
}

void launch_embedding_q8_0(void* out, const int* ids, const void* table, int T, int d, int vocab, cudaStream_t s) {
  throw_if(d % 32 != 0, "Q8_0 embedding: dim must be a multiple of 32");
  if (T == 0) return;
  embedding_q8_0_kernel<<<T, 128, 0, s>>>(reinterpret_cast<__nv_bfloat16*>(out), ids,
                                         reinterpret_cast<const uint8_t*>(table), d, vocab);
  check_launch("embedding_q8_0");
}

}  // namespace gollek
