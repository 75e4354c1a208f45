// Memory-bound fused elementwise kernels (sm_100a):
//   K1  rms_norm / fused_add_rms_norm   (+ residual add, one HBM pass)
//   K2  rope_kv_write                   (QKV split + NeoX RoPE + paged KV-cache scatter)
//   K13 embedding gather
//   silu_mul (SwiGLU on a [gate | up] activation, used by the MoE path)
//
// Reference math: RMSNorm kernel/cuda/gollek-kernel-cuda/…/cuda/binding/CudaCpuFallback.java:181-211,
// SiLU·up :261-290, RoPE runner/safetensor/gollek-safetensor-engine/…/attention/RopeFrequencyCache.java:49-107,
// paged KV write …/attention/FlashAttentionKernel.java:166-194.
#include "../common/common.cuh"
#include "../common/tma_host.h"
#include "launchers.h"

using namespace gollek;

namespace {

constexpr int kNormThreads = 256;

template <int MAXV, bool ADD>
__global__ void __launch_bounds__(kNormThreads) rms_norm_kernel(__nv_bfloat16* __restrict__ out,
                                                                const __nv_bfloat16* __restrict__ x,
                                                                __nv_bfloat16* __restrict__ residual,
                                                                const __nv_bfloat16* __restrict__ w, int d,
                                                                int64_t x_stride, int64_t out_stride, float eps,
                                                                int center) {
  // center != 0: LayerNorm without bias (Cohere): (x - mean) * rsqrt(var + eps) * w
  const int row = blockIdx.x;
  const int nvec = d >> 3;
  const uint4* xr = reinterpret_cast<const uint4*>(x + (int64_t)row * x_stride);
  uint4* rr = ADD ? reinterpret_cast<uint4*>(residual + (int64_t)row * d) : nullptr;
  float v[MAXV][8];
  float ss = 0.f, sum = 0.f;
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    int idx = threadIdx.x + i * kNormThreads;
    if (idx < nvec) {
      bf16x8_to_float(xr[idx], v[i]);
      if (ADD) {
        float r[8];
        bf16x8_to_float(rr[idx], r);
#pragma unroll
        for (int j = 0; j < 8; ++j) v[i][j] += r[j];
        uint4 packed = float_to_bf16x8(v[i]);
        rr[idx] = packed;
        bf16x8_to_float(packed, v[i]);  // normalise the rounded residual, like the oracle
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        ss += v[i][j] * v[i][j];
        sum += v[i][j];
      }
    }
  }
  __shared__ float red[2][kNormThreads / 32];
  ss = warp_sum(ss);
  sum = warp_sum(sum);
  if ((threadIdx.x & 31) == 0) {
    red[0][threadIdx.x >> 5] = ss;
    red[1][threadIdx.x >> 5] = sum;
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < kNormThreads / 32 ? red[0][threadIdx.x] : 0.f;
    float u = threadIdx.x < kNormThreads / 32 ? red[1][threadIdx.x] : 0.f;
    t = warp_sum(t);
    u = warp_sum(u);
    if (threadIdx.x == 0) {
      red[0][0] = t;
      red[1][0] = u;
    }
  }
  __syncthreads();
  const float mean = center ? red[1][0] / (float)d : 0.f;
  const float var = red[0][0] / (float)d - mean * mean;
  const float rs = rsqrtf(fmaxf(var, 0.f) + eps);
  const uint4* wr = reinterpret_cast<const uint4*>(w);
  uint4* orow = reinterpret_cast<uint4*>(out + (int64_t)row * out_stride);
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    int idx = threadIdx.x + i * kNormThreads;
    if (idx < nvec) {
      float wf[8];
      bf16x8_to_float(wr[idx], wf);
#pragma unroll
      for (int j = 0; j < 8; ++j) v[i][j] = (v[i][j] - mean) * rs * wf[j];
      orow[idx] = float_to_bf16x8(v[i]);
    }
  }
}

// ---------------------------------------------------------------------------------------------
// K2: RoPE + paged KV write. One CTA per token.
// ---------------------------------------------------------------------------------------------
// One CTA per token, one warp per head (q heads, then k heads): optional projection bias, optional
// per-head RMSNorm (Qwen3 / Gemma-3 QK-norm: x * rsqrt(mean(x^2) + eps) * w over head_dim), then
// NeoX rotation of the first `rot` dims (rot < D: partial rotary, or a head zero-padded to a
// supported size); dims [rot, D) pass through. Lane l owns rotation pairs (j, j+1) and
// (j+half, j+half+1) for j = 2l + 64i, half = rot / 2. V rows (+ bias) are copied into the cache.
// The cos/sin table rows hold rot values (cos of the rot/2 pairs, then sin).
__global__ void __launch_bounds__(128) rope_kv_write_kernel(
    __nv_bfloat16* __restrict__ q_out, const __nv_bfloat16* __restrict__ qkv, const int* __restrict__ positions,
    const float* __restrict__ cos_sin, __nv_bfloat16* __restrict__ cache, const int* __restrict__ slots, int H,
    int Hk, int D, int block_size, int64_t qkv_stride, int max_pos, const __nv_bfloat16* __restrict__ bias,
    const __nv_bfloat16* __restrict__ q_norm, const __nv_bfloat16* __restrict__ k_norm, float norm_eps,
    int rot, int num_blocks, uint32_t* bounds) {
  const int t = blockIdx.x;
  const int half = rot >> 1;
  int pos = positions[t];
  pos = pos < 0 ? 0 : (pos >= max_pos ? max_pos - 1 : pos);
  const float* cs = cos_sin + (int64_t)pos * rot;
  const __nv_bfloat16* row = qkv + (int64_t)t * qkv_stride;
  int slot = slots ? slots[t] : -1;
  // a slot in a block beyond the pool is reported and its K/V write skipped
  if (slot >= 0 && checked_index(slot / block_size, num_blocks, bounds, -1) < 0) slot = -1;
  const int64_t blk = slot >= 0 ? slot / block_size : 0;
  const int off = slot >= 0 ? slot % block_size : 0;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int kMaxI = 2;  // head_dim <= 256: at most two 64-wide pair groups per lane
  for (int h = warp; h < H + Hk; h += 4) {
    if (h >= H && slot < 0) break;
    const __nv_bfloat16* src = row + h * D;
    float2 x1[kMaxI], x2[kMaxI];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < kMaxI; ++i) {
      const int j = 2 * lane + 64 * i;
      if (j < half) {
        x1[i] = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(src + j));
        x2[i] = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(src + j + half));
        if (bias) {
          const float2 b1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(bias + h * D + j));
          const float2 b2 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(bias + h * D + j + half));
          x1[i].x += b1.x; x1[i].y += b1.y; x2[i].x += b2.x; x2[i].y += b2.y;
        }
        ss += x1[i].x * x1[i].x + x1[i].y * x1[i].y + x2[i].x * x2[i].x + x2[i].y * x2[i].y;
      }
    }
    // pass-through dims [rot, D): at most kPass pairs per lane (D - rot <= 64 * kPass = 256)
    constexpr int kPass = 4;
    float2 xp[kPass];
#pragma unroll
    for (int i = 0; i < kPass; ++i) {
      const int e = rot + 2 * lane + 64 * i;
      if (e < D) {
        xp[i] = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(src + e));
        if (bias) {
          const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(bias + h * D + e));
          xp[i].x += b.x; xp[i].y += b.y;
        }
        ss += xp[i].x * xp[i].x + xp[i].y * xp[i].y;
      }
    }
    const __nv_bfloat16* nw = h < H ? q_norm : k_norm;
    float rs = 1.f;
    if (nw) rs = rsqrtf(warp_sum(ss) / (float)D + norm_eps);
    __nv_bfloat16* dst = h < H ? q_out + ((int64_t)t * H + h) * D
                               : cache + (((blk * 2 + 0) * Hk + (h - H)) * block_size + off) * (int64_t)D;
#pragma unroll
    for (int i = 0; i < kMaxI; ++i) {
      const int j = 2 * lane + 64 * i;
      if (j < half) {
        if (nw) {
          const float2 w1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(nw + j));
          const float2 w2 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(nw + j + half));
          x1[i].x *= rs * w1.x; x1[i].y *= rs * w1.y; x2[i].x *= rs * w2.x; x2[i].y *= rs * w2.y;
        }
        const float c0 = cs[j], c1 = cs[j + 1], s0 = cs[half + j], s1 = cs[half + j + 1];
        *reinterpret_cast<__nv_bfloat162*>(dst + j) =
            __floats2bfloat162_rn(x1[i].x * c0 - x2[i].x * s0, x1[i].y * c1 - x2[i].y * s1);
        *reinterpret_cast<__nv_bfloat162*>(dst + j + half) =
            __floats2bfloat162_rn(x2[i].x * c0 + x1[i].x * s0, x2[i].y * c1 + x1[i].y * s1);
      }
    }
#pragma unroll
    for (int i = 0; i < kPass; ++i) {
      const int e = rot + 2 * lane + 64 * i;
      if (e < D) {
        if (nw) {
          const float2 w = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(nw + e));
          xp[i].x *= rs * w.x; xp[i].y *= rs * w.y;
        }
        *reinterpret_cast<__nv_bfloat162*>(dst + e) = __floats2bfloat162_rn(xp[i].x, xp[i].y);
      }
    }
  }
  if (slot >= 0) {
    const int nv = Hk * D / 8;
    const __nv_bfloat16* vrow = row + (H + Hk) * D;
    for (int i = threadIdx.x; i < nv; i += blockDim.x) {
      const int kh = (i * 8) / D, dd = (i * 8) % D;
      __nv_bfloat16* dst = cache + (((blk * 2 + 1) * Hk + kh) * block_size + off) * (int64_t)D + dd;
      uint4 v = *reinterpret_cast<const uint4*>(vrow + i * 8);
      if (bias) {
        float f[8], b[8];
        bf16x8_to_float(v, f);
        bf16x8_to_float(*reinterpret_cast<const uint4*>(bias + (H + Hk) * D + i * 8), b);
#pragma unroll
        for (int e = 0; e < 8; ++e) f[e] += b[e];
        v = float_to_bf16x8(f);
      }
      *reinterpret_cast<uint4*>(dst) = v;
    }
  }
}

// ---------------------------------------------------------------------------------------------
// K13: embedding gather (vectorised 16-byte copies).
// ---------------------------------------------------------------------------------------------
// scale != 1 multiplies the gathered row (Gemma's sqrt(hidden) embedding normaliser)
__global__ void embedding_kernel(__nv_bfloat16* __restrict__ out, const int* __restrict__ ids,
                                 const __nv_bfloat16* __restrict__ table, int d, int vocab, float scale,
                                 uint32_t* bounds) {
  const int t = blockIdx.x;
  const int raw = ids[t];
  int id = checked_index(raw, vocab, bounds, raw < 0 ? 0 : vocab - 1);
  id = id < 0 ? 0 : (id >= vocab ? vocab - 1 : id);
  const uint4* src = reinterpret_cast<const uint4*>(table + (int64_t)id * d);
  uint4* dst = reinterpret_cast<uint4*>(out + (int64_t)t * d);
  for (int i = threadIdx.x; i < d / 8; i += blockDim.x) {
    if (scale == 1.f) {
      dst[i] = src[i];
    } else {
      float f[8];
      bf16x8_to_float(src[i], f);
#pragma unroll
      for (int e = 0; e < 8; ++e) f[e] *= scale;
      dst[i] = float_to_bf16x8(f);
    }
  }
}

__global__ void silu_mul_kernel(__nv_bfloat16* __restrict__ out, const __nv_bfloat16* __restrict__ x, int d) {
  const int t = blockIdx.y;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;  // vector index (8 elements)
  if (i * 8 >= d) return;
  const __nv_bfloat16* row = x + (int64_t)t * 2 * d;
  float g[8], u[8], o[8];
  bf16x8_to_float(*reinterpret_cast<const uint4*>(row + i * 8), g);
  bf16x8_to_float(*reinterpret_cast<const uint4*>(row + d + i * 8), u);
#pragma unroll
  for (int j = 0; j < 8; ++j) o[j] = silu(g[j]) * u[j];
  *reinterpret_cast<uint4*>(out + (int64_t)t * d + i * 8) = float_to_bf16x8(o);
}

}  // namespace

namespace gollek {

void launch_rms_norm(void* out, const void* x, void* residual, const void* w, int T, int d, int64_t x_stride,
                     int64_t out_stride, float eps, cudaStream_t s, bool center) {
  throw_if(d % 8 != 0 || d > 8 * 4 * kNormThreads, "rms_norm: hidden size must be a multiple of 8, <= 8192");
  throw_if(x_stride % 8 != 0 || out_stride % 8 != 0, "rms_norm: row stride must keep 16-byte alignment");
  if (T == 0) return;
  auto* o = reinterpret_cast<__nv_bfloat16*>(out);
  auto* xp = reinterpret_cast<const __nv_bfloat16*>(x);
  auto* rp = reinterpret_cast<__nv_bfloat16*>(residual);
  auto* wp = reinterpret_cast<const __nv_bfloat16*>(w);
  const int nvec = d / 8;
  const int c = center ? 1 : 0;
#define GOLLEK_NORM(V)                                                                                        \
  if (rp) rms_norm_kernel<V, true><<<T, kNormThreads, 0, s>>>(o, xp, rp, wp, d, x_stride, out_stride, eps, c);  \
  else rms_norm_kernel<V, false><<<T, kNormThreads, 0, s>>>(o, xp, rp, wp, d, x_stride, out_stride, eps, c);
  if (nvec <= kNormThreads) {
    GOLLEK_NORM(1)
  } else if (nvec <= 2 * kNormThreads) {
    GOLLEK_NORM(2)
  } else {
    GOLLEK_NORM(4)
  }
#undef GOLLEK_NORM
  check_launch("rms_norm");
}

void launch_rope_kv_write(void* q_out, const void* qkv, const int* positions, const float* cos_sin, void* cache,
                          const int* slots, int T, int H, int Hk, int D, int block_size, int64_t qkv_stride,
                          int max_pos, const void* bias, const void* q_norm, const void* k_norm, float norm_eps,
                          int rot, cudaStream_t s, int num_blocks) {
  throw_if(D % 16 != 0 || D > 256, "rope_kv_write: head_dim must be a multiple of 16, <= 256");
  throw_if(rot % 4 != 0 || rot > D || D - rot > 256, "rope_kv_write: rotary dims must be a multiple of 4, "
                                                     "<= head_dim, with at most 256 pass-through dims");
  if (T == 0) return;
  rope_kv_write_kernel<<<T, 128, 0, s>>>(reinterpret_cast<__nv_bfloat16*>(q_out),
                                         reinterpret_cast<const __nv_bfloat16*>(qkv), positions, cos_sin,
                                         reinterpret_cast<__nv_bfloat16*>(cache), slots, H, Hk, D, block_size,
                                         qkv_stride, max_pos, reinterpret_cast<const __nv_bfloat16*>(bias),
                                         reinterpret_cast<const __nv_bfloat16*>(q_norm),
                                         reinterpret_cast<const __nv_bfloat16*>(k_norm), norm_eps, rot,
                                         num_blocks, num_blocks > 0 ? bounds_status() : nullptr);
  check_launch("rope_kv_write");
}

void launch_embedding(void* out, const int* ids, const void* table, int T, int d, int vocab, float scale,
                      cudaStream_t s) {
  throw_if(d % 8 != 0, "embedding: dim must be a multiple of 8");
  if (T == 0) return;
  embedding_kernel<<<T, 128, 0, s>>>(reinterpret_cast<__nv_bfloat16*>(out), ids,
                                     reinterpret_cast<const __nv_bfloat16*>(table), d, vocab, scale,
                                     bounds_status());
  check_launch("embedding");
}

void launch_silu_mul(void* out, const void* x, int T, int d, cudaStream_t s) {
  throw_if(d % 8 != 0, "silu_mul: width must be a multiple of 16");
  if (T == 0) return;
  dim3 grid((d / 8 + 127) / 128, T);
  silu_mul_kernel<<<grid, 128, 0, s>>>(reinterpret_cast<__nv_bfloat16*>(out),
                                       reinterpret_cast<const __nv_bfloat16*>(x), d);
  check_launch("silu_mul");
}

}  // namespace gollek
