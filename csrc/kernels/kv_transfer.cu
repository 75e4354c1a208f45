// KV-cache block transfer for prefill/decode disaggregation (sm_100a).
//
//   kv_gather_blocks   packed[l, i] = cache[l, block_ids[i]]   (one sequence's blocks, every layer)
//   kv_scatter_blocks  cache[l, block_ids[i]] = packed[l, i]
//
// A paged block of one layer is 2 * Hk * block_size * head_dim contiguous bf16 values ([K | V] x
// heads x tokens x dims), so each (layer, block) pair is one contiguous span: one CTA copies it
// with 16-byte loads/stores. The packed tensor [L, n, 2, Hk, block_size, head_dim] is what crosses
// NVLink (a peer copy into the decode GPU) or the network (cluster hand-off); the receiver
// scatters it into the blocks its own allocator assigned.
//
// Reference behaviour: the prefill→decode KV hand-off of
// core/optimization/gollek-plugin-prefill-decode/…/prefilldecode/PrefillDecodeDisaggService.java:1-80 and
// inference/gollek-cluster/…/cluster/CacheHandoffService.java:27-54 (which acknowledges without moving data).
#include "../common/common.cuh"
#include "launchers.h"

using namespace gollek;

namespace {

template <bool GATHER>
__global__ void __launch_bounds__(256) kv_blocks_kernel(__nv_bfloat16* __restrict__ cache, __nv_bfloat16* __restrict__ packed,
                                                        const int* __restrict__ block_ids, int n, int64_t num_blocks,
                                                        int64_t span) {
  const int i = blockIdx.x, l = blockIdx.y;
  const int64_t b = block_ids[i];
  if (b < 0 || b >= num_blocks) return;  // invalid ids are skipped (checked on the host as well)
  uint4* c = reinterpret_cast<uint4*>(cache + ((int64_t)l * num_blocks + b) * span);
  uint4* p = reinterpret_cast<uint4*>(packed + ((int64_t)l * n + i) * span);
  const int64_t nv = span / 8;
  for (int64_t v = threadIdx.x; v < nv; v += blockDim.x) {
    if (GATHER)
      p[v] = c[v];
    else
      c[v] = p[v];
  }
}

// K15 (KV eviction scoring): mean L2 norm of the keys of each listed block over every layer,
// KV head and token. One CTA per block; warp w takes rows (layer, head, token) w, w + 8, ...; a row
// is head_dim contiguous bf16 values read as 16-byte vectors (head_dim <= 256 -> <= 1 vector per
// lane). Keys with small norms draw the most attention (Devoto et al., "A Simple and Effective
// L2 Norm-Based Strategy for KV Cache Compression", EMNLP 2024), so -norm ranks block importance.
__global__ void __launch_bounds__(256) kv_key_norm_kernel(const __nv_bfloat16* __restrict__ cache,
                                                          const int* __restrict__ block_ids, float* __restrict__ out,
                                                          int layers, int64_t num_blocks, int Hk, int bs, int D) {
  __shared__ float part[8];
  const int i = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t b = block_ids[i];
  float acc = 0.f;
  if (b >= 0 && b < num_blocks) {
    const int rows = layers * Hk * bs, vec = D / 8;
    for (int row = warp; row < rows; row += 8) {
      const int l = row / (Hk * bs), rem = row % (Hk * bs);
      // block layout [2, Hk, bs, D]: K is the first half
      const __nv_bfloat16* k = cache + (((int64_t)l * num_blocks + b) * 2 * Hk * bs + rem) * D;
      float ss = 0.f;
      if (lane < vec) {
        float f[8];
        bf16x8_to_float(reinterpret_cast<const uint4*>(k)[lane], f);
#pragma unroll
        for (int e = 0; e < 8; ++e) ss = fmaf(f[e], f[e], ss);
      }
      ss = warp_sum(ss);
      acc += sqrtf(ss);
    }
  }
  if (lane == 0) part[warp] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < 8; ++w) t += part[w];
    out[i] = t / (float)(layers * Hk * bs);
  }
}

}  // namespace

namespace gollek {

void launch_kv_blocks(void* cache, void* packed, const int* block_ids, int n, int layers, int64_t num_blocks,
                      int64_t span, bool gather, cudaStream_t s) {
  throw_if(span % 8 != 0, "kv transfer: block span must be a multiple of 8 elements");
  if (n == 0 || layers == 0) return;
  dim3 grid(n, layers);
  auto* c = reinterpret_cast<__nv_bfloat16*>(cache);
  auto* p = reinterpret_cast<__nv_bfloat16*>(packed);
  if (gather)
    kv_blocks_kernel<true><<<grid, 256, 0, s>>>(c, p, block_ids, n, num_blocks, span);
  else
    kv_blocks_kernel<false><<<grid, 256, 0, s>>>(c, p, block_ids, n, num_blocks, span);
  check_launch("kv block transfer");
}

void launch_kv_key_norms(const void* cache, const int* block_ids, float* out, int n, int layers, int64_t num_blocks,
                         int Hk, int bs, int D, cudaStream_t s) {
  throw_if(D % 8 != 0 || D > 256, "kv key norms: head_dim must be a multiple of 8, at most 256");
  if (n == 0) return;
  kv_key_norm_kernel<<<n, 256, 0, s>>>(reinterpret_cast<const __nv_bfloat16*>(cache), block_ids, out, layers,
                                       num_blocks, Hk, bs, D);
  check_launch("kv_key_norms");
}

}  // namespace gollek
