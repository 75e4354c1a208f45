// fp8 (e4m3) paged KV cache: quantized writes and block dequantization.
//
// Layout: values uint8 [NB, 2, Hk, 16, D] (e4m3 bit patterns, the bf16 cache's layout with one byte
// per value) and scales fp32 [NB, 2, Hk, 16]: one scale per (block, K/V, kv head, token), value =
// e4m3 * scale. A token's scale is fixed when the token is written (its own absmax / 448), so a
// block that fills one decode step at a time never needs requantizing.
//
//   kv_quant_fp8_kernel      the step's K/V rows (bf16 [T, 2, Hk, D], written by the RoPE + KV-write
//                            kernel into a scratch) -> the cache slots of the tokens
//   kv_dequant_blocks_kernel listed blocks -> a bf16 cache of the same layout (prefill attention
//                            over an fp8 cache reads this copy with the bf16 tcgen05 kernel)
// Decode attention reads the fp8 cache directly (attention.cu, tensor-core kernel, FP8 = true).
#include <cuda_fp8.h>

#include "../common/common.cuh"
#include "../common/tma_host.h"
#include "launchers.h"

namespace gollek {

namespace {

constexpr float kE4m3Max = 448.f;

// One warp per (token, K/V, kv head); D = 128: four values per lane.
__global__ void __launch_bounds__(256) kv_quant_fp8_kernel(const __nv_bfloat16* __restrict__ kv,
                                                           const int* __restrict__ slots, uint8_t* __restrict__ cache,
                                                           float* __restrict__ scales, int T, int Hk, int block_size,
                                                           int num_blocks, uint32_t* bounds) {
  constexpr int D = 128;
  const int gw = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (gw >= T * 2 * Hk) return;
  const int t = gw / (2 * Hk), rem = gw % (2 * Hk);
  const int which = rem / Hk, kh = rem % Hk;
  const int slot = slots[t];
  if (slot < 0) return;
  if (checked_index(slot / block_size, num_blocks, bounds, -1) < 0) return;  // beyond the pool: skipped
  const int64_t blk = slot / block_size, off = slot % block_size;
  const __nv_bfloat16* src = kv + ((int64_t)(t * 2 + which) * Hk + kh) * D + lane * 4;
  const uint2 raw = *reinterpret_cast<const uint2*>(src);
  const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.x));
  const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.y));
  const float amax = warp_max(fmaxf(fmaxf(fabsf(a.x), fabsf(a.y)), fmaxf(fabsf(b.x), fabsf(b.y))));
  const float scale = amax > 0.f ? __fdiv_rn(amax, kE4m3Max) : 1.f;
  // x / scale correctly rounded (not x * (1 / scale)): the stored byte is a function of x and
  // scale alone, equal to any IEEE restatement of the rule
  const __nv_fp8x2_storage_t lo = __nv_cvt_float2_to_fp8x2(
      make_float2(__fdiv_rn(a.x, scale), __fdiv_rn(a.y, scale)), __NV_SATFINITE, __NV_E4M3);
  const __nv_fp8x2_storage_t hi = __nv_cvt_float2_to_fp8x2(
      make_float2(__fdiv_rn(b.x, scale), __fdiv_rn(b.y, scale)), __NV_SATFINITE, __NV_E4M3);
  const int64_t row = ((blk * 2 + which) * Hk + kh) * block_size + off;
  reinterpret_cast<uint32_t*>(cache + row * D)[lane] = (uint32_t)lo | ((uint32_t)hi << 16);
  if (lane == 0) scales[row] = scale;
}

// One warp per (listed block, K/V, kv head, token row); D = 128.
__global__ void __launch_bounds__(256) kv_dequant_blocks_kernel(const uint8_t* __restrict__ cache,
                                                                const float* __restrict__ scales,
                                                                const int* __restrict__ ids, int n, int num_blocks,
                                                                int Hk, int block_size,
                                                                __nv_bfloat16* __restrict__ dst) {
  constexpr int D = 128;
  const int64_t gw = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const int64_t per_block = 2ll * Hk * block_size;
  if (gw >= n * per_block) return;
  const int i = (int)(gw / per_block);
  const int64_t r = gw % per_block;  // (K/V, kv head, token) inside the block
  const int id = ids[i];
  if (id < 0 || id >= num_blocks) return;  // table padding: never attended
  const int64_t src_row = (int64_t)id * per_block + r;
  const float s = scales[src_row];
  const uint32_t w = reinterpret_cast<const uint32_t*>(cache + src_row * D)[lane];
  const __half2_raw h0 = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(w & 0xffffu), __NV_E4M3);
  const __half2_raw h1 = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(w >> 16), __NV_E4M3);
  const float2 f0 = __half22float2(*reinterpret_cast<const __half2*>(&h0));
  const float2 f1 = __half22float2(*reinterpret_cast<const __half2*>(&h1));
  __nv_bfloat162 o0 = __floats2bfloat162_rn(f0.x * s, f0.y * s);
  __nv_bfloat162 o1 = __floats2bfloat162_rn(f1.x * s, f1.y * s);
  uint2 out;
  out.x = *reinterpret_cast<uint32_t*>(&o0);
  out.y = *reinterpret_cast<uint32_t*>(&o1);
  *reinterpret_cast<uint2*>(dst + ((int64_t)i * per_block + r) * D + lane * 4) = out;
}

}  // namespace

void launch_kv_quant_fp8(const void* kv, const int* slots, void* cache, float* scales, int T, int Hk, int D,
                         int block_size, cudaStream_t s, int num_blocks) {
  throw_if(D != 128, "fp8 KV cache: head_dim 128 only");
  if (T == 0) return;
  const int64_t warps = (int64_t)T * 2 * Hk;
  kv_quant_fp8_kernel<<<(unsigned)((warps + 7) / 8), 256, 0, s>>>(reinterpret_cast<const __nv_bfloat16*>(kv), slots,
                                                                   reinterpret_cast<uint8_t*>(cache), scales, T, Hk,
                                                                   block_size, num_blocks,
                                                                   num_blocks > 0 ? bounds_status() : nullptr);
  check_launch("kv_quant_fp8");
}

void launch_kv_dequant_blocks(const void* cache, const float* scales, const int* ids, int n, int num_blocks, int Hk,
                              int D, int block_size, void* dst, cudaStream_t s) {
  throw_if(D != 128, "fp8 KV cache: head_dim 128 only");
  if (n == 0) return;
  const int64_t warps = (int64_t)n * 2 * Hk * block_size;
  kv_dequant_blocks_kernel<<<(unsigned)((warps + 7) / 8), 256, 0, s>>>(
      reinterpret_cast<const uint8_t*>(cache), scales, ids, n, num_blocks, Hk, block_size,
      reinterpret_cast<__nv_bfloat16*>(dst));
  check_launch("kv_dequant_blocks");
}

}  // namespace gollek
