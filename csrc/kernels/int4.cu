// 4-bit group-quantized weights on the GPU (sm_100a): GPTQ / AWQ / RTN int4 and NF4 (QLoRA).
//
// Canonical layout (every source format is repacked into it at load time):
//   q      uint8 [N, K/2]   row n, byte j = weights k=2j (low nibble) and k=2j+1 (high nibble)
//   scale  bf16  [N, K/g]   one per group of g consecutive k
//   zero   bf16  [N, K/g]   asymmetric int4: w = (q - zero) * scale
//   NF4 (lut != 0):          w = NF4[q] * scale (zero unused), NF4 = the 16 normal-float levels
// Row-major by output row, so tensor-parallel row slices and K slices on group boundaries are
// byte views, as with the GGUF blocks.
//
//   int4_gemv    y[m, n] = Σ_k x[m, k] w[n, k] for up to 8 tokens: one warp per output row (two
//                rows, gate and up, for the SwiGLU variant over rows interleaved in groups of 64);
//                lane l decodes 32 weights per 16-byte load and applies them to every token.
//   int4_dequant bf16 [N, K] (prefill: followed by the tcgen05 GEMM in L2-sized row chunks).
//
// Reference: QLoRA NF4 matmul qlora_fused_matmul (core/optimization/gollek-plugin-qlora/…/qlora/
// binding/QLoraBinding.java:19-46, CPU math QLoraCpuFallback.java:18-119) and the GPTQ/AWQ
// quantizers (core/quantizer/gollek-quantizer-{gptq,awq}); none ships GPU code.
#include "../common/common.cuh"
#include "launchers.h"

using namespace gollek;

namespace {

constexpr int kI4MaxTok = 8;
constexpr int kI4Warps = 8;

// NF4 levels: quantiles of N(0, 1) rescaled to [-1, 1] (Dettmers et al., "QLoRA", 2023, App. E).
__constant__ float kNF4[16] = {-1.0f, -0.6961928009986877f, -0.5250730514526367f, -0.39491748809814453f,
                               -0.28444138169288635f, -0.18477343022823334f, -0.09105003625154495f, 0.0f,
                               0.07958029955625534f, 0.16093020141124725f, 0.24611230194568634f,
                               0.33791524171829224f, 0.44070982933044434f, 0.5626170039176941f,
                               0.7229568362236023f, 1.0f};

// 32 weights of one row, k0 .. k0+31 (16 packed bytes), all in group k0 / g.
// lut_s: the NF4 levels in shared memory (lane-varying indices hit 16 distinct banks, where the
// constant cache would serialise them)
GOLLEK_DEVICE void dequant32(const uint4 q, float s, float z, bool lut, const float* lut_s, float* w) {
  const uint32_t qq[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
  for (int b = 0; b < 16; ++b) {
    const uint32_t byte = (qq[b >> 2] >> (8 * (b & 3))) & 0xFF;
    const int lo = byte & 0xF, hi = byte >> 4;
    if (lut) {
      w[2 * b] = lut_s[lo] * s;
      w[2 * b + 1] = lut_s[hi] * s;
    } else {
      w[2 * b] = ((float)lo - z) * s;
      w[2 * b + 1] = ((float)hi - z) * s;
    }
  }
}

// Partial dot products of one row against M tokens: lane takes 32-weight chunks lane, lane+32, ...
template <int MT>
GOLLEK_DEVICE void row_dot(const uint8_t* __restrict__ qrow, const __nv_bfloat16* __restrict__ srow,
                           const __nv_bfloat16* __restrict__ zrow, const __nv_bfloat16* __restrict__ x,
                           int64_t ldx, int M, int K, int g, bool lut, const float* lut_s, int lane,
                           float* acc) {
  const int chunks = K / 32;
  constexpr int kU = 4;  // chunks per lane per round: their loads are issued before any is decoded
  for (int c0 = lane; c0 < chunks; c0 += 32 * kU) {
    uint4 qv[kU];
    float sv[kU], zv[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int c = min(c0 + 32 * u, chunks - 1);
      const int gi = (c * 32) / g;
      qv[u] = __ldg(reinterpret_cast<const uint4*>(qrow + c * 16));
      sv[u] = __bfloat162float(srow[gi]);
      zv[u] = lut ? 0.f : __bfloat162float(zrow[gi]);
    }
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int c = c0 + 32 * u;
      if (c >= chunks) break;
      const int k0 = c * 32;
      float w[32];
      dequant32(qv[u], sv[u], zv[u], lut, lut_s, w);
#pragma unroll
      for (int m = 0; m < MT; ++m) {
        if (m < M) {
          const __nv_bfloat16* xr = x + (int64_t)m * ldx + k0;
          float xf[8];
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            bf16x8_to_float(__ldg(reinterpret_cast<const uint4*>(xr + 8 * v)), xf);
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[m] = fmaf(xf[e], w[8 * v + e], acc[m]);
          }
        }
      }
    }
  }
}

template <bool SWIGLU>
__global__ void __launch_bounds__(kI4Warps * 32) int4_gemv_kernel(
    __nv_bfloat16* __restrict__ out, int64_t ldo, const __nv_bfloat16* __restrict__ x, int64_t ldx,
    const uint8_t* __restrict__ q, const __nv_bfloat16* __restrict__ scale, const __nv_bfloat16* __restrict__ zero,
    int M, int N_out, int K, int g, int lut) {
  __shared__ float lut_s[16];
  if (threadIdx.x < 16) lut_s[threadIdx.x] = kNF4[threadIdx.x];
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int col = blockIdx.x * kI4Warps + warp;
  if (col >= N_out) return;
  const int ng = K / g;
  float acc[kI4MaxTok], acc2[kI4MaxTok];
#pragma unroll
  for (int m = 0; m < kI4MaxTok; ++m) acc[m] = acc2[m] = 0.f;
  // SwiGLU: output column c reads gate row (c/64)*128 + c%64 and the up row 64 further
  const int n = SWIGLU ? (col / 64) * 128 + col % 64 : col;
  row_dot<kI4MaxTok>(q + (int64_t)n * (K / 2), scale + (int64_t)n * ng, zero ? zero + (int64_t)n * ng : nullptr, x, ldx,
                     M, K, g, lut != 0, lut_s, lane, acc);
  if (SWIGLU)
    row_dot<kI4MaxTok>(q + (int64_t)(n + 64) * (K / 2), scale + (int64_t)(n + 64) * ng,
                       zero ? zero + (int64_t)(n + 64) * ng : nullptr, x, ldx, M, K, g, lut != 0, lut_s, lane, acc2);
#pragma unroll
  for (int m = 0; m < kI4MaxTok; ++m) {
    if (m < M) {
      const float a = warp_sum(acc[m]);
      float r = a;
      if (SWIGLU) r = silu(a) * warp_sum(acc2[m]);
      if (lane == 0) out[(int64_t)m * ldo + col] = __float2bfloat16(r);
    }
  }
}

__global__ void int4_dequant_kernel(__nv_bfloat16* __restrict__ out, const uint8_t* __restrict__ q,
                                    const __nv_bfloat16* __restrict__ scale, const __nv_bfloat16* __restrict__ zero,
                                    int N, int K, int g, int lut) {
  // one thread per 32 weights of a row
  __shared__ float lut_s[16];
  if (threadIdx.x < 16) lut_s[threadIdx.x] = kNF4[threadIdx.x];
  __syncthreads();
  const int chunks = K / 32;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)N * chunks) return;
  const int n = (int)(i / chunks), c = (int)(i % chunks);
  const int k0 = c * 32, gi = k0 / g, ng = K / g;
  const uint4 qv = *reinterpret_cast<const uint4*>(q + (int64_t)n * (K / 2) + k0 / 2);
  const float s = __bfloat162float(scale[(int64_t)n * ng + gi]);
  const float z = lut ? 0.f : __bfloat162float(zero[(int64_t)n * ng + gi]);
  float w[32];
  dequant32(qv, s, z, lut != 0, lut_s, w);
  uint4* dst = reinterpret_cast<uint4*>(out + (int64_t)n * K + k0);
#pragma unroll
  for (int v = 0; v < 4; ++v) dst[v] = float_to_bf16x8(w + 8 * v);
}

}  // namespace

namespace gollek {

void launch_int4_gemv(void* out, int64_t ldo, const void* x, int64_t ldx, const void* q, const void* scale,
                      const void* zero, int M, int N, int K, int g, bool lut, bool swiglu, cudaStream_t s) {
  throw_if(M < 1 || M > kI4MaxTok, "int4 gemv: 1..8 tokens");
  throw_if(K % 32 != 0 || g % 32 != 0 || K % g != 0, "int4: K and the group size must be multiples of 32");
  throw_if(ldx % 8 != 0, "int4 gemv: activation rows must keep 16-byte alignment");
  throw_if(!lut && zero == nullptr, "int4: asymmetric weights need zero points");
  const int n_out = swiglu ? N / 2 : N;
  throw_if(swiglu && N % 128 != 0, "int4 gemv swiglu: N must be a multiple of 128");
  const int grid = (n_out + kI4Warps - 1) / kI4Warps;
  auto* o = reinterpret_cast<__nv_bfloat16*>(out);
  auto* xb = reinterpret_cast<const __nv_bfloat16*>(x);
  auto* qb = reinterpret_cast<const uint8_t*>(q);
  auto* sb = reinterpret_cast<const __nv_bfloat16*>(scale);
  auto* zb = reinterpret_cast<const __nv_bfloat16*>(zero);
  if (swiglu)
    int4_gemv_kernel<true><<<grid, kI4Warps * 32, 0, s>>>(o, ldo, xb, ldx, qb, sb, zb, M, n_out, K, g, lut);
  else
    int4_gemv_kernel<false><<<grid, kI4Warps * 32, 0, s>>>(o, ldo, xb, ldx, qb, sb, zb, M, n_out, K, g, lut);
  check_launch("int4_gemv");
}

void launch_int4_dequant(void* out, const void* q, const void* scale, const void* zero, int N, int K, int g, bool lut,
                         cudaStream_t s) {
  throw_if(K % 32 != 0 || g % 32 != 0 || K % g != 0, "int4: K and the group size must be multiples of 32");
  throw_if(!lut && zero == nullptr, "int4: asymmetric weights need zero points");
  const int64_t threads = (int64_t)N * (K / 32);
  if (threads == 0) return;
  int4_dequant_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, s>>>(
      reinterpret_cast<__nv_bfloat16*>(out), reinterpret_cast<const uint8_t*>(q),
      reinterpret_cast<const __nv_bfloat16*>(scale), reinterpret_cast<const __nv_bfloat16*>(zero), N, K, g, lut);
  check_launch("int4_dequant");
}

}  // namespace gollek
