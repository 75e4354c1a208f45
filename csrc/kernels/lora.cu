// K10: batched multi-LoRA for the serving path (sm_100a).
//
// Tokens of one step are grouped by adapter slot as CSR segments (seg_ptr / tok_idx / seg_slot);
// nothing is physically reordered — kernels gather input rows and scatter output rows by index.
//   shrink:  V[t, 0:R] = x[t, :] · A[slot]^T            A [slots, R, K]  (R = modules x rank)
//            mma.sync m16n8k16 over 64-token tiles of each segment (16 tokens per warp, the whole
//            K accumulated in registers; no atomics)
//   expand:  Y[t, n] += scale[slot] * sum_r B[slot, n, r] * V[t, roff(n) + r]   B [slots, N, rank]
//            roff(n) selects the module's rank block (fused q/k/v: three column ranges).
// Both launch one CTA (column) per 64-token tile, so a popular adapter's tokens spread over the
// GPU instead of serialising in one CTA.
//
// Reference semantics: QLoRA fused matmul (W + s·B·A)·x, core/optimization/gollek-plugin-qlora/…/
// QLoraCpuFallback.java:30-119, with per-request adapter routing (runner/safetensor/…/LoraAdapterRouter.java).
#include "../common/common.cuh"
#include "launchers.h"

using namespace gollek;

namespace {

constexpr int kLoraTile = 64;  // tokens of one adapter segment per CTA (tiles built on the host)

GOLLEK_DEVICE void mma_bf16_m16n8k16(float* d, const uint32_t* a, const uint32_t* b) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

// shrink: V[t, 0:R] = x[t, :] . A[slot]^T on tensor cores. CTA = one 64-token tile of a segment;
// per 64-wide K chunk the tile's x rows and the adapter's A rows are staged in shared memory with
// 16-byte loads (the next chunk prefetched into registers), then warp w runs its 16 tokens as the
// M = 16 rows of mma m16n8k16 against the R <= 64 rank rows (up to 8 n-tiles). K is split over
// blockIdx.y; partial sums are added to the zeroed V atomically.
constexpr int kTileK = 64;
constexpr int kTilePad = kTileK + 8;  // row pitch in shared memory (bf16): staggers the banks

__global__ void __launch_bounds__(128) lora_shrink_kernel(
    float* __restrict__ V, int ldv, const __nv_bfloat16* __restrict__ x, int64_t ldx,
    const __nv_bfloat16* __restrict__ A, int R, int K, const int* __restrict__ seg_ptr,
    const int* __restrict__ tok_idx, const int* __restrict__ seg_slot, const int2* __restrict__ tiles) {
  __shared__ __align__(16) __nv_bfloat16 xs[kLoraTile][kTilePad];
  __shared__ __align__(16) __nv_bfloat16 as[64][kTilePad];
  __shared__ int ts[kLoraTile];
  const int2 tile = tiles[blockIdx.x];
  const int seg = tile.x, p0 = tile.y;
  const int nt_tok = min(p0 + kLoraTile, seg_ptr[seg + 1]) - p0;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, q = lane & 3;
  // K split over blockIdx.y: [kb, ke) in kTileK chunks; partial sums are added to V atomically
  const int per = (K / kTileK + gridDim.y - 1) / gridDim.y * kTileK;
  const int kb = blockIdx.y * per, ke = min(K, kb + per);
  const __nv_bfloat16* As = A + (int64_t)seg_slot[seg] * R * K;
  for (int i = tid; i < kLoraTile; i += 128) ts[i] = i < nt_tok ? tok_idx[p0 + i] : -1;
  const int nt = (R + 7) >> 3;
  float c[8][4];
#pragma unroll
  for (int j = 0; j < 8; ++j) c[j][0] = c[j][1] = c[j][2] = c[j][3] = 0.f;
  __syncthreads();
  // each thread stages 4 x-vectors and up to 4 A-vectors (16 bytes) per chunk; the next chunk's are
  // loaded into registers while this chunk is multiplied
  uint4 xv[4], av[4];
  auto load = [&](int k0) {
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int i = tid + 128 * u, r = i >> 3, v = i & 7;
      xv[u] = ts[r] >= 0 ? *reinterpret_cast<const uint4*>(x + (int64_t)ts[r] * ldx + k0 + 8 * v)
                         : make_uint4(0, 0, 0, 0);
      av[u] = r < R ? *reinterpret_cast<const uint4*>(As + (int64_t)r * K + k0 + 8 * v) : make_uint4(0, 0, 0, 0);
    }
  };
  if (kb < ke) load(kb);
  for (int k0 = kb; k0 < ke; k0 += kTileK) {
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int i = tid + 128 * u, r = i >> 3, v = i & 7;
      *reinterpret_cast<uint4*>(&xs[r][8 * v]) = xv[u];
      if (r < R) *reinterpret_cast<uint4*>(&as[r][8 * v]) = av[u];
    }
    __syncthreads();
    if (k0 + kTileK < ke) load(k0 + kTileK);
    if (warp * 16 < nt_tok) {
#pragma unroll
      for (int kk = 0; kk < kTileK; kk += 16) {
        uint32_t a[4];
        a[0] = *reinterpret_cast<const uint32_t*>(&xs[warp * 16 + g][kk + 2 * q]);
        a[1] = *reinterpret_cast<const uint32_t*>(&xs[warp * 16 + g + 8][kk + 2 * q]);
        a[2] = *reinterpret_cast<const uint32_t*>(&xs[warp * 16 + g][kk + 8 + 2 * q]);
        a[3] = *reinterpret_cast<const uint32_t*>(&xs[warp * 16 + g + 8][kk + 8 + 2 * q]);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (j < nt) {
            const int n = 8 * j + g;
            uint32_t b[2] = {0u, 0u};
            if (n < R) {
              b[0] = *reinterpret_cast<const uint32_t*>(&as[n][kk + 2 * q]);
              b[1] = *reinterpret_cast<const uint32_t*>(&as[n][kk + 8 + 2 * q]);
            }
            mma_bf16_m16n8k16(c[j], a, b);
          }
        }
      }
    }
    __syncthreads();
  }
  const int r0 = warp * 16 + g, r1 = r0 + 8;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int col = 8 * j + 2 * q;
    if (j < nt && col < R) {
      if (r0 < nt_tok) {
        atomicAdd(&V[(int64_t)ts[r0] * ldv + col], c[j][0]);
        atomicAdd(&V[(int64_t)ts[r0] * ldv + col + 1], c[j][1]);
      }
      if (r1 < nt_tok) {
        atomicAdd(&V[(int64_t)ts[r1] * ldv + col], c[j][2]);
        atomicAdd(&V[(int64_t)ts[r1] * ldv + col + 1], c[j][3]);
      }
    }
  }
}

constexpr int kShrinkThreads = 256;
constexpr int kShrinkChunk = 512;   // K elements per CTA (16 per lane)
constexpr int kShrinkTok = 16;      // tokens staged in shared memory at a time

// shrink for short segments (decode): CTA = (segment, 512-wide K chunk); each warp holds rows of
// A in registers (16-byte loads) and streams the segment's tokens from shared memory; fp32 atomics
// combine the K chunks (V zeroed first).
__global__ void __launch_bounds__(kShrinkThreads) lora_shrink_seg_kernel(
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

// expand: Y[t, n] += scale[slot] * sum_r B[slot, n, r] * V[t, roff(n) + r]; CTA = one 64-token tile
// x 256 output columns (one per thread, its 16 B values in registers), the tile's V rows staged in
// shared memory.
__global__ void __launch_bounds__(kExpandThreads) lora_expand_kernel(
    __nv_bfloat16* __restrict__ Y, int64_t ldy, const float* __restrict__ V, int ldv,
    const __nv_bfloat16* __restrict__ B, int N, int rank, int n1, int n2, const float* __restrict__ scales,
    const int* __restrict__ seg_ptr, const int* __restrict__ tok_idx, const int* __restrict__ seg_slot,
    const int2* __restrict__ tiles) {
  __shared__ float vs[kLoraTile][64];
  __shared__ int ts[kLoraTile];
  const int2 tile = tiles[blockIdx.x];
  const int seg = tile.x, p0 = tile.y;
  const int p1 = min(p0 + kLoraTile, seg_ptr[seg + 1]), nt = p1 - p0;
  const int n = blockIdx.y * kExpandThreads + threadIdx.x;
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
  for (int i = threadIdx.x; i < nt; i += kExpandThreads) ts[i] = tok_idx[p0 + i];
  __syncthreads();
  for (int i = threadIdx.x; i < nt * ldv; i += kExpandThreads) {
    const int tt = i / ldv, r = i % ldv;
    vs[tt][r] = V[(int64_t)ts[tt] * ldv + r];
  }
  __syncthreads();
  if (n >= N) return;
  for (int t0 = 0; t0 < nt; t0 += 8) {  // 8 tokens per round: their Y loads overlap
    float old[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) old[u] = t0 + u < nt ? __bfloat162float(Y[(int64_t)ts[t0 + u] * ldy + n]) : 0.f;
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      if (t0 + u < nt) {
        float y = 0.f;
#pragma unroll
        for (int r = 0; r < 16; ++r) y = fmaf(b[r], vs[t0 + u][roff + r], y);
        Y[(int64_t)ts[t0 + u] * ldy + n] = __float2bfloat16(old[u] + sc * y);
      }
    }
  }
}

}  // namespace

namespace gollek {

void launch_lora_shrink(float* V, int ldv, const void* x, int64_t ldx, const void* A, int R, int K,
                        const int* seg_ptr, const int* tok_idx, const int* seg_slot, const int* tiles, int num_tiles,
                        int num_segs, int max_seg, cudaStream_t s) {
  throw_if(R > 64 || R % 2 != 0, "lora shrink: at most 64 rank rows (modules x rank), an even count");
  throw_if(K % 64 != 0 || ldx % 8 != 0, "lora shrink: K a multiple of 64, 16-byte aligned rows");
  if (num_tiles == 0) return;
  auto* xb = reinterpret_cast<const __nv_bfloat16*>(x);
  auto* ab = reinterpret_cast<const __nv_bfloat16*>(A);
  if (max_seg <= kShrinkTok) {  // short segments: wide A loads per (segment, K chunk)
    dim3 grid(num_segs, (K + kShrinkChunk - 1) / kShrinkChunk);
    lora_shrink_seg_kernel<<<grid, kShrinkThreads, 0, s>>>(V, ldv, xb, ldx, ab, R, K, seg_ptr, tok_idx, seg_slot);
  } else {
    // enough CTAs to fill the GPU: split K further when there are few tiles
    const int ksplit = std::max(1, std::min(K / kTileK, (2 * 148 + num_tiles - 1) / num_tiles));
    lora_shrink_kernel<<<dim3(num_tiles, ksplit), 128, 0, s>>>(V, ldv, xb, ldx, ab, R, K, seg_ptr, tok_idx, seg_slot,
                                                               reinterpret_cast<const int2*>(tiles));
  }
  check_launch("lora_shrink");
}

void launch_lora_expand(void* Y, int64_t ldy, const float* V, int ldv, const void* B, int N, int rank, int n1,
                        int n2, const float* scales, const int* seg_ptr, const int* tok_idx, const int* seg_slot,
                        const int* tiles, int num_tiles, cudaStream_t s) {
  throw_if(rank > 16, "lora expand: rank must be <= 16");
  throw_if(ldv > 64, "lora expand: at most 64 rank columns");
  if (num_tiles == 0) return;
  dim3 grid(num_tiles, (N + kExpandThreads - 1) / kExpandThreads);
  lora_expand_kernel<<<grid, kExpandThreads, 0, s>>>(reinterpret_cast<__nv_bfloat16*>(Y), ldy, V, ldv,
                                                     reinterpret_cast<const __nv_bfloat16*>(B), N, rank, n1, n2,
                                                     scales, seg_ptr, tok_idx, seg_slot,
                                                     reinterpret_cast<const int2*>(tiles));
  check_launch("lora_expand");
}

}  // namespace gollek
