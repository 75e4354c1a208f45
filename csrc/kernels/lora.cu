// K10: batched multi-LoRA for the serving path (sm_100a).
//
// Tokens of one step are grouped by adapter slot as CSR segments (seg_ptr / tok_idx / seg_slot);
// nothing is physically reordered — kernels gather input rows and scatter output rows by index.
//   shrink:  V[t, 0:R] += x[t, :] · A[slot]^T           A [slots, R, K]  (R = modules x rank)
//            grid (segment, K-split); each warp holds rows of A in registers and streams the
//            segment's tokens from shared memory; fp32 atomics combine the K splits.
//   expand:  Y[t, n] += scale[slot] * sum_r B[slot, n, r] * V[t, roff(n) + r]   B [slots, N, rank]
//            roff(n) selects the module's rank block (fused q/k/v: three column ranges).
// One adapter's weights are read once per segment, independent of how many tokens use it.
//
// Reference semantics: QLoRA fused matmul (W + s·B·A)·x, core/optimization/gollek-plugin-qlora/…/
// QLoraCpuFallback.java:30-119, with per-request adapter routing (runner/safetensor/…/LoraAdapterRouter.java).
#include "../common/common.cuh"
#include "launchers.h"

using namespace gollek;

namespace {

constexpr int kShrinkThreads = 256;
constexpr int kShrinkChunk = 512;   // K elements per CTA (16 per lane)
constexpr int kShrinkTok = 16;      // tokens staged in shared memory at a time

__global__ void __launch_bounds__(kShrinkThreads) lora_shrink_kernel(
    float* __restrict__ V, int ldv, const __nv_bfloat16* __restrict__ x, int64_t ldx,
    const __nv_bfloat16* __restrict__ A, int R, int K, const int* __restrict__ seg_ptr,
    const int* __restrict__ tok_idx, const int* __restrict__ seg_slot) {
  __shared__ __align__(16) __nv_bfloat16 xs[kShrinkTok][kShrinkChunk];
  const int seg = blockIdx.x;
  const int k0 = blockIdx.y * kShrinkChunk;
  const int t0 = seg_ptr[seg], t1 = seg_ptr[seg + 1];
  const int slot = seg_slot[seg];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nwarps = kShrinkThreads / 32;
  const __nv_bfloat16* Aslot = A + (int64_t)slot * R * K;
  // rows of A this warp owns (at most 8 with R <= 64)
  constexpr int kMaxRowsPerWarp = 8;
  float a[kMaxRowsPerWarp][16];
#pragma unroll
  for (int i = 0; i < kMaxRowsPerWarp; ++i) {
    const int r = warp + i * nwarps;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int k = k0 + h * 256 + lane * 8;
      if (r < R && k + 8 <= K) {
        bf16x8_to_float(*reinterpret_cast<const uint4*>(Aslot + (int64_t)r * K + k), &a[i][h * 8]);
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) a[i][h * 8 + e] = 0.f;
      }
    }
  }
  for (int tb = t0; tb < t1; tb += kShrinkTok) {
    const int nt = min(kShrinkTok, t1 - tb);
    __syncthreads();
    for (int i = threadIdx.x; i < nt * (kShrinkChunk / 8); i += blockDim.x) {
      const int tt = i / (kShrinkChunk / 8), c = i % (kShrinkChunk / 8);
      const int k = k0 + c * 8;
      uint4 v = make_uint4(0, 0, 0, 0);
      if (k + 8 <= K) v = *reinterpret_cast<const uint4*>(x + (int64_t)tok_idx[tb + tt] * ldx + k);
      *reinterpret_cast<uint4*>(&xs[tt][c * 8]) = v;
    }
    __syncthreads();
    for (int tt = 0; tt < nt; ++tt) {
      float xv[16];
      bf16x8_to_float(*reinterpret_cast<const uint4*>(&xs[tt][lane * 8]), xv);
      bf16x8_to_float(*reinterpret_cast<const uint4*>(&xs[tt][256 + lane * 8]), xv + 8);
      const int t = tok_idx[tb + tt];
#pragma unroll
      for (int i = 0; i < kMaxRowsPerWarp; ++i) {
        const int r = warp + i * nwarps;
        if (r >= R) break;
        float s = 0.f;
#pragma unroll
        for (int e = 0; e < 16; ++e) s = fmaf(a[i][e], xv[e], s);
        s = warp_sum(s);
        if (lane == 0) atomicAdd(&V[(int64_t)t * ldv + r], s);
      }
    }
  }
}

constexpr int kExpandThreads = 256;
constexpr int kExpandTok = 64;

__global__ void __launch_bounds__(kExpandThreads) lora_expand_kernel(
    __nv_bfloat16* __restrict__ Y, int64_t ldy, const float* __restrict__ V, int ldv,
    const __nv_bfloat16* __restrict__ B, int N, int rank, int n1, int n2, const float* __restrict__ scales,
    const int* __restrict__ seg_ptr, const int* __restrict__ tok_idx, const int* __restrict__ seg_slot) {
  __shared__ float vs[kExpandTok][64];
  const int seg = blockIdx.x;
  const int n = blockIdx.y * kExpandThreads + threadIdx.x;
  const int t0 = seg_ptr[seg], t1 = seg_ptr[seg + 1];
  const int slot = seg_slot[seg];
  const float sc = scales[slot];
  const int roff = n < n1 ? 0 : (n < n2 ? rank : 2 * rank);
  float b[16];
#pragma unroll
  for (int r = 0; r < 16; ++r) b[r] = 0.f;
  if (n < N) {
    const __nv_bfloat16* brow = B + ((int64_t)slot * N + n) * rank;
    for (int r = 0; r < rank; ++r) b[r] = __bfloat162float(brow[r]);
  }
  const int vw = ldv;  // V row width (all modules' ranks)
  for (int tb = t0; tb < t1; tb += kExpandTok) {
    const int nt = min(kExpandTok, t1 - tb);
    __syncthreads();
    for (int i = threadIdx.x; i < nt * vw; i += blockDim.x) {
      const int tt = i / vw, r = i % vw;
      vs[tt][r] = V[(int64_t)tok_idx[tb + tt] * ldv + r];
    }
    __syncthreads();
    if (n < N) {
      for (int tt = 0; tt < nt; ++tt) {
        float y = 0.f;
#pragma unroll
        for (int r = 0; r < 16; ++r) y = fmaf(b[r], vs[tt][roff + r], y);
        __nv_bfloat16* dst = Y + (int64_t)tok_idx[tb + tt] * ldy + n;
        *dst = __float2bfloat16(__bfloat162float(*dst) + sc * y);
      }
    }
  }
}

}  // namespace

namespace gollek {

void launch_lora_shrink(float* V, int ldv, const void* x, int64_t ldx, const void* A, int R, int K,
                        const int* seg_ptr, const int* tok_idx, const int* seg_slot, int num_segs, cudaStream_t s) {
  throw_if(R > 64, "lora shrink: at most 64 rank rows (modules x rank)");
  throw_if(K % 8 != 0, "lora shrink: K must be a multiple of 8");
  if (num_segs == 0) return;
  dim3 grid(num_segs, (K + kShrinkChunk - 1) / kShrinkChunk);
  lora_shrink_kernel<<<grid, kShrinkThreads, 0, s>>>(V, ldv, reinterpret_cast<const __nv_bfloat16*>(x), ldx,
                                                     reinterpret_cast<const __nv_bfloat16*>(A), R, K, seg_ptr,
                                                     tok_idx, seg_slot);
  check_launch("lora_shrink");
}

void launch_lora_expand(void* Y, int64_t ldy, const float* V, int ldv, const void* B, int N, int rank, int n1,
                        int n2, const float* scales, const int* seg_ptr, const int* tok_idx, const int* seg_slot,
                        int num_segs, cudaStream_t s) {
  throw_if(rank > 16, "lora expand: rank must be <= 16");
  throw_if(ldv > 64, "lora expand: at most 64 rank columns");
  if (num_segs == 0) return;
  dim3 grid(num_segs, (N + kExpandThreads - 1) / kExpandThreads);
  lora_expand_kernel<<<grid, kExpandThreads, 0, s>>>(reinterpret_cast<__nv_bfloat16*>(Y), ldy, V, ldv,
                                                     reinterpret_cast<const __nv_bfloat16*>(B), N, rank, n1, n2,
                                                     scales, seg_ptr, tok_idx, seg_slot);
  check_launch("lora_expand");
}

}  // namespace gollek
