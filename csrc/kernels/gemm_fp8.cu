// K6: block-scaled FP8 GEMM on tcgen05 (sm_100a).
//
//   C[M, N'] = epilogue( sum_kb  (A_kb · B_kb^T) * sa[m, kb] * sb[n / 128, kb] )
//   A e4m3 [M, K] with per-token-group scales sa [M, K/128] (1 x 128 groups, fp32)
//   B e4m3 [N, K] with block scales sb [N/128, K/128]      (128 x 128 blocks, fp32)
//
// One pipeline stage = one 128-deep K block = one scale block (128 fp8 = one 128-byte swizzled
// row per operand row). The MMA warp issues 4 x tcgen05.mma kind::f8f6f4 (K = 32 each) into a
// fresh TMEM partial (two partial buffers alternate); eight epilogue warps read the partial
// (two warps per TMEM lane quarter, each owning half of the 128 columns), multiply by the row's
// activation scale times the tile's weight-block scale and accumulate in fp32 registers; after
// the tile's last K block they apply the epilogue (none / SwiGLU) and store bf16.
// Split-K (decode-sized M): each CTA covers a K range and writes scaled fp32 partial sums that the
// reduce kernel of gemm.cu combines (and applies the epilogue to).
//
// Reference op: gollek_blackwell_matmul_fp8 (kernel/blackwell/gollek-kernel-blackwell/…/binding/
// BlackwellBinding.java:66,344-350); scale layout as DeepSeek-style FP8 serving. All waits bounded.
#include "../common/common.cuh"
#include "../common/tma_host.h"
#include "launchers.h"

#include <algorithm>

using namespace gollek;

namespace {

constexpr int kBM = 128, kBN = 128, kBK = 128;  // BK in elements = bytes (fp8)
constexpr int kStages = 6;
constexpr int kABytes = kBM * kBK, kBBytes = kBN * kBK, kStageBytes = kABytes + kBBytes;
constexpr int kThreads = 320;  // warp 0 TMA, warp 1 MMA, warps 2..9 epilogue
constexpr int kSmem = 1024 + kStages * kStageBytes + 512;
constexpr uint64_t kWait = 2000000000ull;

GOLLEK_DEVICE uint64_t gt() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
GOLLEK_DEVICE bool waitb(uint64_t* bar, uint32_t parity, uint32_t* status, volatile int* abort_flag) {
  for (int i = 0; i < 256; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = gt();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (gt() - t0 > kWait) {
      report_status(status, kStatusMbarTimeout);
      *abort_flag = 1;
      return false;
    }
  }
}
GOLLEK_DEVICE void drainb(uint64_t* bar, uint32_t parity) {
  const uint64_t t0 = gt();
  while (!mbar_try_wait(bar, parity))
    if (gt() - t0 > kWait) break;
}
// Bounded wait until a shared counter reaches `target` (false on timeout or abort).
GOLLEK_DEVICE bool spin_ge(volatile int* p, int target, volatile int* abort_flag, uint32_t* status) {
  const uint64_t t0 = gt();
  while (*p < target) {
    if (*abort_flag) return false;
    if (gt() - t0 > kWait) {
      report_status(status, kStatusMbarTimeout);
      *abort_flag = 1;
      return false;
    }
  }
  return true;
}

template <int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_fp8_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    __nv_bfloat16* __restrict__ C, int64_t ldc, const float* __restrict__ sa,
                    const float* __restrict__ sb, int M, int N, int K, int group_m, int splits,
                    float* __restrict__ partial, uint32_t* status, int* __restrict__ cnt, int epi) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint8_t* sA = smem;
  uint8_t* sB = smem + kStages * kABytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);
  uint64_t* empty = full + kStages;
  uint64_t* pfull = empty + kStages;  // [2]
  uint64_t* pempty = pfull + 2;       // [2]
  uint64_t* done_bar = pempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* consumed = abort_flag + 1;
  volatile int* fx_last = consumed + 1;    // split-K fixup: this CTA finishes the tile
  volatile int* fx_arrive = fx_last + 1;   // epilogue warps done with their partial rows
  volatile int* fx_gen = fx_arrive + 1;    // fixups decided

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_m = (M + kBM - 1) / kBM, num_n = (N + kBN - 1) / kBN;
  const int num_tiles = num_m * num_n;
  const int num_units = num_tiles * splits;
  const int num_kb = (K + kBK - 1) / kBK;
  const int kb_per = (num_kb + splits - 1) / splits;
  const int ksc = num_kb;  // scale row stride (K/128 blocks)
  constexpr uint32_t idesc = make_idesc_e4m3(kBM, kBN);

  auto unit_coords = [&](int u, int& m0, int& n0, int& kb0, int& kb1) {
    const int ks = u / num_tiles, tile = u % num_tiles;
    const int gsz = group_m * num_n;
    const int g = tile / gsz, r = tile % gsz;
    const int first_m = g * group_m;
    const int gm = min(num_m - first_m, group_m);
    m0 = (first_m + r % gm) * kBM;
    n0 = (r / gm) * kBN;
    kb0 = ks * kb_per;
    kb1 = min(num_kb, kb0 + kb_per);
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&pfull[a], 1);
      mbar_init(&pempty[a], 8);
    }
    mbar_init(done_bar, 1);
    *abort_flag = 0;
    *consumed = 0;
    *fx_arrive = 0;
    *fx_gen = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 2 * kBN);
    tmem_relinquish();
  }
  tcgen05_fence_before();
  __syncthreads();
  tcgen05_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (elect_one()) {
      int stage = 0, issued = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x) {
        int m0, n0, kb0, kb1;
        unit_coords(u, m0, n0, kb0, kb1);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!waitb(&empty[stage], phase ^ 1, status, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], kStageBytes);
          tma_load_2d(sA + stage * kABytes, &tmA, kb * kBK, m0, &full[stage]);
          tma_load_2d(sB + stage * kBBytes, &tmB, kb * kBK, n0, &full[stage]);
          ++issued;
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok)
        for (int i = max(*consumed, issued - kStages); i < issued; ++i) drainb(&full[i % kStages], (i / kStages) & 1);
    }
  } else if (warp == 1) {
    if (elect_one()) {
      int stage = 0, used = 0, kbc = 0;  // kbc: global K-block counter (selects the partial buffer)
      uint32_t phase = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x) {
        int m0, n0, kb0, kb1;
        unit_coords(u, m0, n0, kb0, kb1);
        for (int kb = kb0; kb < kb1; ++kb, ++kbc) {
          const int pb = kbc & 1;
          if (!waitb(&pempty[pb], ((kbc >> 1) & 1) ^ 1, status, abort_flag) ||
              !waitb(&full[stage], phase, status, abort_flag)) {
            ok = false;
            break;
          }
          tcgen05_fence_after();
          const uint64_t a_desc = make_smem_desc_sw128(smem_u32(sA + stage * kABytes));
          const uint64_t b_desc = make_smem_desc_sw128(smem_u32(sB + stage * kBBytes));
#pragma unroll
          for (int k = 0; k < kBK / 32; ++k)
            umma_f8_ss(tmem_base + pb * kBN, a_desc + 2 * k, b_desc + 2 * k, idesc, k > 0 ? 1u : 0u);
          umma_commit(&empty[stage]);
          umma_commit(&pfull[pb]);
          *consumed = ++used;
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok) {
        umma_commit(done_bar);
        drainb(done_bar, 0);
      }
    }
  } else {
    // epilogue warps 2..9: lane quarter (warp & 3), column half (warp - 2) / 4
    const int lg = warp & 3, half = (warp - 2) >> 2;
    constexpr int kCols = kBN / 2;
    int kbc = 0;
    int fx_seq = 0;  // split units this CTA has finished (the same sequence in all 8 epilogue warps)
    for (int u = blockIdx.x; u < num_units; u += gridDim.x) {
      int m0, n0, kb0, kb1;
      unit_coords(u, m0, n0, kb0, kb1);
      const int row = m0 + lg * 32 + lane;
      const int nb = n0 / 128;
      float acc[kCols];
#pragma unroll
      for (int c = 0; c < kCols; ++c) acc[c] = 0.f;
      bool ok = true;
      for (int kb = kb0; kb < kb1; ++kb, ++kbc) {
        const int pb = kbc & 1;
        const float s = (row < M ? sa[(int64_t)row * ksc + kb] : 0.f) * sb[(int64_t)nb * ksc + kb];
        if (!waitb(&pfull[pb], (kbc >> 1) & 1, status, abort_flag)) {
          ok = false;
          break;
        }
        tcgen05_fence_after();
        const uint32_t tb = tmem_base + ((uint32_t)(lg * 32) << 16) + pb * kBN + half * kCols;
#pragma unroll
        for (int c = 0; c < kCols; c += 32) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(tb + c, r);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 32; ++e) acc[c + e] = fmaf(__uint_as_float(r[e]), s, acc[c + e]);
        }
        tcgen05_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&pempty[pb]);
      }
      if (!ok) break;
      const int col0 = n0 + half * kCols;
      if (splits > 1) {
        if (row < M) {
          float* prow = partial + ((int64_t)(u / num_tiles) * M + row) * N + col0;
#pragma unroll
          for (int c = 0; c < kCols; c += 4)
            if (col0 + c + 4 <= N) *reinterpret_cast<float4*>(prow + c) = make_float4(acc[c], acc[c + 1], acc[c + 2], acc[c + 3]);
        }
        if (cnt != nullptr) {
          // the tile's last unit to finish sums the split partials and writes the output (no
          // reduce kernel); the 8 epilogue warps meet through shared counters with bounded waits
          const int tile = u % num_tiles;
          __threadfence();
          __syncwarp();
          if (lane == 0) atomicAdd((int*)fx_arrive, 1);
          bool last = false;
          if (lane == 0) {
            if (warp == 2) {
              if (spin_ge(fx_arrive, 8 * (fx_seq + 1), abort_flag, status)) {
                __threadfence();
                *fx_last = atomicAdd(&cnt[tile], 1) == splits - 1;
              } else {
                *fx_last = 0;
              }
              __threadfence_block();
              *fx_gen = fx_seq + 1;
            }
            last = spin_ge(fx_gen, fx_seq + 1, abort_flag, status) && *fx_last;
          }
          last = __shfl_sync(0xffffffffu, last, 0);
          ++fx_seq;
          if (last) {
            __threadfence();
            // all 256 epilogue threads share the tile's (row, 8-column group) items; each item's
            // split partials are loaded 4 splits at a time with every load in flight
            const int64_t sstride = (int64_t)M * N;
            const int rows_valid = min(kBM, M - m0);
            const bool glu = epi == kEpiSwiglu;
            const int groups = glu ? 8 : 16;  // 8-column outputs per tile row
            const int et = threadIdx.x - 64;  // 0..255
            for (int it = et; it < rows_valid * groups; it += 256) {
              const int r = m0 + it / groups, g8 = (it % groups) * 8;
              const float* base = partial + (int64_t)r * N + n0 + g8;  // gate (SwiGLU) or plain columns
              float a[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
              float b[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
              for (int sp0 = 0; sp0 < splits; sp0 += 4) {
                float4 va[4][2], vb[4][2];
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                  if (sp0 + q < splits) {
                    const float4* pa = reinterpret_cast<const float4*>(base + (sp0 + q) * sstride);
                    va[q][0] = __ldcg(pa);
                    va[q][1] = __ldcg(pa + 1);
                    if (glu) {
                      vb[q][0] = __ldcg(pa + 16);  // the up columns: 64 further
                      vb[q][1] = __ldcg(pa + 17);
                    }
                  }
                }
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                  if (sp0 + q < splits) {
                    a[0] += va[q][0].x; a[1] += va[q][0].y; a[2] += va[q][0].z; a[3] += va[q][0].w;
                    a[4] += va[q][1].x; a[5] += va[q][1].y; a[6] += va[q][1].z; a[7] += va[q][1].w;
                    if (glu) {
                      b[0] += vb[q][0].x; b[1] += vb[q][0].y; b[2] += vb[q][0].z; b[3] += vb[q][0].w;
                      b[4] += vb[q][1].x; b[5] += vb[q][1].y; b[6] += vb[q][1].z; b[7] += vb[q][1].w;
                    }
                  }
                }
              }
              if (glu) {
#pragma unroll
                for (int e = 0; e < 8; ++e) a[e] = silu(a[e]) * b[e];
                *reinterpret_cast<uint4*>(C + (int64_t)r * ldc + n0 / 2 + g8) = float_to_bf16x8(a);
              } else {
                *reinterpret_cast<uint4*>(C + (int64_t)r * ldc + n0 + g8) = float_to_bf16x8(a);
              }
            }
            if (warp == 2 && lane == 0) cnt[tile] = 0;  // ready for the next launch
          }
        }
      } else if (row < M) {  // (SwiGLU always runs split-K: the reduce pairs gate and up columns)
#pragma unroll
        for (int c = 0; c < kCols; c += 8) {
          if (col0 + c + 8 <= N)
            *reinterpret_cast<uint4*>(C + (int64_t)row * ldc + col0 + c) = float_to_bf16x8(&acc[c]);
        }
      }
    }
  }
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tcgen05_fence_after();
    tmem_dealloc(tmem_base, 2 * kBN);
  }
}

// K7: per-token-group (1 x 128) activation quantisation: one warp per (row, group), 4 values per lane.
__global__ void act_quant_fp8_kernel(uint8_t* __restrict__ q, float* __restrict__ scale,
                                     const __nv_bfloat16* __restrict__ x, int64_t ldx, int M, int K) {
  const int64_t wid = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int groups = K / 128;
  if (wid >= (int64_t)M * groups) return;
  const int row = wid / groups, g = wid % groups;
  const __nv_bfloat16* src = x + (int64_t)row * ldx + g * 128 + lane * 4;
  const uint2 u = *reinterpret_cast<const uint2*>(src);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
  float2 a = __bfloat1622float2(h[0]), b = __bfloat1622float2(h[1]);
  float amax = fmaxf(fmaxf(fabsf(a.x), fabsf(a.y)), fmaxf(fabsf(b.x), fabsf(b.y)));
  amax = warp_max(amax);
  const float sc = fmaxf(amax, 1e-10f) / 448.f;
  const float inv = 1.f / sc;
  uint32_t packed = 0;
  const float v[4] = {a.x * inv, a.y * inv, b.x * inv, b.y * inv};
#pragma unroll
  for (int e = 0; e < 4; ++e)
    packed |= (uint32_t)__nv_cvt_float_to_fp8(v[e], __NV_SATFINITE, __NV_E4M3) << (8 * e);
  *reinterpret_cast<uint32_t*>(q + (int64_t)row * K + g * 128 + lane * 4) = packed;
  if (lane == 0) scale[(int64_t)row * groups + g] = sc;
}

// 128 x 128 weight-block quantisation: one CTA (256 threads) per block.
__global__ void weight_quant_fp8_kernel(uint8_t* __restrict__ q, float* __restrict__ scale,
                                        const __nv_bfloat16* __restrict__ w, int N, int K) {
  const int nb = blockIdx.y, kb = blockIdx.x;
  __shared__ float red[8];
  float amax = 0.f;
  for (int i = threadIdx.x; i < 128 * 16; i += blockDim.x) {  // 16 groups of 8 per row
    const int r = i / 16, c = (i % 16) * 8;
    const int n = nb * 128 + r;
    if (n < N) {
      float f[8];
      bf16x8_to_float(*reinterpret_cast<const uint4*>(w + (int64_t)n * K + kb * 128 + c), f);
#pragma unroll
      for (int e = 0; e < 8; ++e) amax = fmaxf(amax, fabsf(f[e]));
    }
  }
  amax = warp_max(amax);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < 8 ? red[threadIdx.x] : 0.f;
    t = warp_max(t);
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  const float sc = fmaxf(red[0], 1e-10f) / 448.f;
  const float inv = 1.f / sc;
  for (int i = threadIdx.x; i < 128 * 16; i += blockDim.x) {
    const int r = i / 16, c = (i % 16) * 8;
    const int n = nb * 128 + r;
    if (n < N) {
      float f[8];
      bf16x8_to_float(*reinterpret_cast<const uint4*>(w + (int64_t)n * K + kb * 128 + c), f);
      uint2 out;
      uint32_t* o = reinterpret_cast<uint32_t*>(&out);
      o[0] = o[1] = 0;
#pragma unroll
      for (int e = 0; e < 8; ++e)
        o[e >> 2] |= (uint32_t)__nv_cvt_float_to_fp8(f[e] * inv, __NV_SATFINITE, __NV_E4M3) << (8 * (e & 3));
      *reinterpret_cast<uint2*>(q + (int64_t)n * K + kb * 128 + c) = out;
    }
  }
  if (threadIdx.x == 0) scale[(int64_t)nb * (K / 128) + kb] = sc;
}

}  // namespace

namespace gollek {

void launch_act_quant_fp8(void* q, float* scale, const void* x, int64_t ldx, int M, int K, cudaStream_t s) {
  throw_if(K % 128 != 0, "fp8 activation quant: K must be a multiple of 128");
  throw_if(ldx % 4 != 0, "fp8 activation quant: row pitch must be a multiple of 4 elements");
  if (M == 0) return;
  const int64_t warps = (int64_t)M * (K / 128);
  act_quant_fp8_kernel<<<(unsigned)((warps * 32 + 255) / 256), 256, 0, s>>>(
      reinterpret_cast<uint8_t*>(q), scale, reinterpret_cast<const __nv_bfloat16*>(x), ldx, M, K);
  check_launch("act_quant_fp8");
}

void launch_weight_quant_fp8(void* q, float* scale, const void* w, int N, int K, cudaStream_t s) {
  throw_if(K % 128 != 0, "fp8 weight quant: K must be a multiple of 128");
  dim3 grid(K / 128, (N + 127) / 128);
  weight_quant_fp8_kernel<<<grid, 256, 0, s>>>(reinterpret_cast<uint8_t*>(q), scale,
                                                reinterpret_cast<const __nv_bfloat16*>(w), N, K);
  check_launch("weight_quant_fp8");
}

void splitk_reduce(void* out, int64_t ldc, const float* partial, const void* residual, int64_t ldr, int M, int N,
                   int splits, int epi, cudaStream_t s);

int gemm_fp8_splits(int M, int N, int K, int epi);

void launch_gemm_fp8(void* out, int64_t ldc, const void* a, int64_t lda, const float* sa, const void* b, int64_t ldb,
                     const float* sb, int M, int N, int K, int epi, int splits, float* partial, uint32_t* status,
                     cudaStream_t s, int* tile_cnt) {
  throw_if(K % 128 != 0, "fp8 gemm: K must be a multiple of 128 (one scale block)");
  throw_if(N % 128 != 0, "fp8 gemm: N must be a multiple of 128");
  throw_if(lda % 16 != 0 || ldb % 16 != 0, "fp8 gemm: operand row pitch must be a multiple of 16 bytes");
  if (M == 0) return;
  const int num_m = (M + kBM - 1) / kBM, num_n = N / kBN;
  const int tiles = num_m * num_n;
  const int num_kb = K / kBK;
  if (splits <= 0) splits = gemm_fp8_splits(M, N, K, epi);
  if (epi == kEpiSwiglu && splits == 1) splits = 2;  // SwiGLU is applied by the reduce pass
  throw_if(splits > 1 && partial == nullptr, "fp8 gemm: split-K needs an fp32 workspace");
  CUtensorMap ta = make_tmap_2d(a, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, M, K, lda, kBM, kBK, CU_TENSOR_MAP_SWIZZLE_128B);
  CUtensorMap tb = make_tmap_2d(b, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, N, K, ldb, kBN, kBK, CU_TENSOR_MAP_SWIZZLE_128B);
  const int64_t a_tile_bytes = (int64_t)kBM * K;
  const int group_m = (int)std::max<int64_t>(1, std::min<int64_t>(num_m, (32ll << 20) / a_tile_bytes));
  const int grid = std::min(tiles * splits, gemm_grid_sms());
  auto kern = gemm_fp8_kernel<kEpiNone>;
  GOLLEK_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem));
  int* cnt = splits > 1 ? tile_cnt : nullptr;  // zeroed [tiles] counters: the kernel finishes split tiles
  kern<<<grid, kThreads, kSmem, s>>>(ta, tb, reinterpret_cast<__nv_bfloat16*>(out), ldc, sa, sb, M, N, K, group_m,
                                     splits, partial, status, cnt, epi);
  check_launch("gemm_fp8");
  if (splits > 1 && cnt == nullptr) splitk_reduce(out, ldc, partial, nullptr, 0, M, N, splits, epi, s);
}

// Split-K factor for decode-sized M: as many K splits as fit the SMs in ONE wave (tiles x splits <=
// SMs; a second wave of a few units would double the kernel time), at least 4 K blocks per split.
int gemm_fp8_splits(int M, int N, int K, int epi) {
  const int tiles = ((M + kBM - 1) / kBM) * (N / kBN);
  int splits = 1;
  const int sms = gemm_grid_sms();
  if (tiles < sms) splits = std::max(1, std::min({sms / tiles, (K / kBK) / 4, 16}));
  if (epi == kEpiSwiglu && splits == 1) splits = 2;
  return splits;
}

}  // namespace gollek
