// K9b: GGUF Q4_K weights in a dequant-fused tcgen05 GEMM (sm_100a).
//
//   C[M, N'] = epilogue( A[M, K] · dequant(W)[N, K]^T )   A bf16, W ggml Q4_K blocks, fp32 accumulate
//
// The weight never exists in bf16 in global memory: its 144-byte super-blocks (256 weights: fp16 d,
// dmin, twelve bytes of 6-bit sub-block scales / mins, 128 bytes of nibbles) stream by TMA (a
// 128-row x 144-byte box per super-block) into shared memory, and converter warps decode each
// 64-deep K slice into the 128-byte-swizzled bf16 B tile the tensor cores read. One CTA per SM:
//   warp 0       TMA producer of the A tiles (128 x 64 bf16, SW128)
//   warp 1       MMA issuer: tcgen05.mma M=128, N=128, K=16 into a double-buffered TMEM accumulator
//   warp 2       TMA producer of the raw super-blocks (128 x 144 B, four in flight)
//   warps 3..10  converters: two threads per weight row, each decodes 32 of the slice's 64 weights
//                (w = d * scale * q - dmin * min, the ggml formula, in fp32, rounded once to bf16)
//                and stores them with the swizzle; fence.proxy.async publishes them to the MMA
//   warps 11..14 epilogue: tcgen05.ld, SwiGLU / plain bf16 store, or fp32 split-K partials
// So HBM sees 0.5625 bytes per weight (plus the activations) instead of the 2 of a bf16 weight, at
// any token count; split-K fills the SMs for decode-sized M (the reduce pass of gemm.cu applies the
// epilogue). Reference: the Q4_K layout and decode of ggml (k_quants), which the reference decodes
// only on the CPU (runner/gguf/gollek-gguf-loader/…/gguf/quant/Dequantizer.java).
// Every mbarrier wait is bounded; on timeout the CTA records a status bit and drains before exit.
#include "../common/common.cuh"
#include "../common/tma_host.h"
#include "launchers.h"

#include <algorithm>

using namespace gollek;

namespace {

constexpr int kBM = 128, kBN = 128, kBK = 64, kSB = 256;  // kBK: one 64-weight nibble group of a super-block
constexpr int kRawBytes = kBN * 144;                       // one super-block of 128 weight rows
constexpr int kABytes = kBM * kBK * 2, kBBytes = kBN * kBK * 2;
constexpr int kAStages = 4, kBStages = 3, kRStages = 4;
constexpr int kConvWarps = 8, kEpiWarps = 4;
constexpr int kConv0 = 3;  // first converter warp (0: A producer, 1: MMA, 2: raw producer)
constexpr int kThreads = 32 * (3 + kConvWarps + kEpiWarps);
constexpr int kSmem = 1024 + kAStages * kABytes + kBStages * kBBytes + kRStages * kRawBytes + 256;
constexpr uint64_t kWaitNs = 2000000000ull;

GOLLEK_DEVICE uint64_t gtime() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
GOLLEK_DEVICE bool waitq(uint64_t* bar, uint32_t parity, uint32_t* status, volatile int* abort_flag) {
  for (int i = 0; i < 256; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = gtime();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (gtime() - t0 > kWaitNs) {
      report_status(status, kStatusMbarTimeout);
      *abort_flag = 1;
      return false;
    }
  }
}
GOLLEK_DEVICE void drainq(uint64_t* bar, uint32_t parity) {
  const uint64_t t0 = gtime();
  while (!mbar_try_wait(bar, parity))
    if (gtime() - t0 > kWaitNs) break;
}

GOLLEK_DEVICE float half_to_float_bits(uint32_t bits) {
  __half h;
  *reinterpret_cast<uint16_t*>(&h) = (uint16_t)bits;
  return __half2float(h);
}
GOLLEK_DEVICE uint32_t scale_byte(const uint4& hdr, int i) {  // byte i of the 12 packed scale bytes
  const uint32_t w = i < 4 ? hdr.y : (i < 8 ? hdr.z : hdr.w);
  return (w >> (8 * (i & 3))) & 0xFF;
}
// 6-bit scale and min of sub-block j (0..7) of a super-block header
GOLLEK_DEVICE void q4k_scale_min(const uint4& hdr, int j, float& a, float& b) {
  const float d = half_to_float_bits(hdr.x & 0xFFFF), dmin = half_to_float_bits(hdr.x >> 16);
  uint32_t sv, mv;
  if (j < 4) {
    sv = scale_byte(hdr, j) & 63;
    mv = scale_byte(hdr, j + 4) & 63;
  } else {
    sv = (scale_byte(hdr, j + 4) & 0xF) | ((scale_byte(hdr, j - 4) >> 6) << 4);
    mv = (scale_byte(hdr, j + 4) >> 4) | ((scale_byte(hdr, j) >> 6) << 4);
  }
  a = d * (float)sv;
  b = dmin * (float)mv;
}

template <int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_q4k_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW,
                    __nv_bfloat16* __restrict__ C, int64_t ldc, int M, int N, int K, int splits,
                    float* __restrict__ partial, uint32_t* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint8_t* sA = smem;
  uint8_t* sB = sA + kAStages * kABytes;
  uint8_t* sR = sB + kBStages * kBBytes;
  uint64_t* a_full = reinterpret_cast<uint64_t*>(sR + kRStages * kRawBytes);
  uint64_t* a_empty = a_full + kAStages;
  uint64_t* b_full = a_empty + kAStages;
  uint64_t* b_empty = b_full + kBStages;
  uint64_t* r_full = b_empty + kBStages;
  uint64_t* r_empty = r_full + kRStages;
  uint64_t* tfull = r_empty + kRStages;  // [2]
  uint64_t* tempty = tfull + 2;          // [2]
  uint64_t* done_bar = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_m = (M + kBM - 1) / kBM, num_n = N / kBN;
  const int num_tiles = num_m * num_n;
  const int num_units = num_tiles * splits;
  const int nsb = K / kSB;
  const int sb_per = (nsb + splits - 1) / splits;
  auto unit_coords = [&](int u, int& m0, int& n0, int& sb0, int& sb1) {
    const int ks = u / num_tiles, tile = u % num_tiles;
    m0 = (tile % num_m) * kBM;  // M-tiles adjacent: CTAs of one wave share each weight tile in L2
    n0 = (tile / num_m) * kBN;
    sb0 = ks * sb_per;
    sb1 = min(nsb, sb0 + sb_per);
  };
  constexpr uint32_t idesc = make_idesc_bf16(kBM, kBN);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kAStages; ++s) {
      mbar_init(&a_full[s], 1);
      mbar_init(&a_empty[s], 1);
    }
    for (int s = 0; s < kBStages; ++s) {
      mbar_init(&b_full[s], kConvWarps);
      mbar_init(&b_empty[s], 1);
    }
    for (int s = 0; s < kRStages; ++s) {
      mbar_init(&r_full[s], 1);
      mbar_init(&r_empty[s], kConvWarps);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], kEpiWarps);
    }
    mbar_init(done_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmW);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 2 * kBN);
    tmem_relinquish();
  }
  tcgen05_fence_before();
  __syncthreads();
  tcgen05_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 2) {
    // ---------------------------------------------------------------- raw super-block producer
    if (elect_one()) {
      int rs = 0, r_issued = 0;
      uint32_t rph = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x) {
        int m0, n0, sb0, sb1;
        unit_coords(u, m0, n0, sb0, sb1);
        for (int sb = sb0; sb < sb1; ++sb) {
          if (!waitq(&r_empty[rs], rph ^ 1, status, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&r_full[rs], kRawBytes);
          tma_load_2d(sR + rs * kRawBytes, &tmW, sb * 144, n0, &r_full[rs]);
          ++r_issued;
          if (++rs == kRStages) {
            rs = 0;
            rph ^= 1;
          }
        }
      }
      if (!ok)  // wait (bounded) for our own copies in flight before the CTA may exit
        for (int i = max(0, r_issued - kRStages); i < r_issued; ++i) drainq(&r_full[i % kRStages], (i / kRStages) & 1);
    }
  } else if (warp == 0) {
    // ---------------------------------------------------------------- A tile producer
    if (elect_one()) {
      int as = 0;
      uint32_t aph = 0;
      bool ok = true;
      int a_issued = 0;
      for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x) {
        int m0, n0, sb0, sb1;
        unit_coords(u, m0, n0, sb0, sb1);
        for (int sb = sb0; sb < sb1 && ok; ++sb) {
          for (int g = 0; g < kSB / kBK; ++g) {
            if (!waitq(&a_empty[as], aph ^ 1, status, abort_flag)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&a_full[as], kABytes);
            tma_load_2d(sA + as * kABytes, &tmA, sb * kSB + g * kBK, m0, &a_full[as]);
            ++a_issued;
            if (++as == kAStages) {
              as = 0;
              aph ^= 1;
            }
          }
        }
      }
      if (!ok)  // wait (bounded) for our own copies in flight before the CTA may exit
        for (int i = max(0, a_issued - kAStages); i < a_issued; ++i) drainq(&a_full[i % kAStages], (i / kAStages) & 1);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (elect_one()) {
      int as = 0, bs = 0, local = 0;
      uint32_t aph = 0, bph = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x, ++local) {
        int m0, n0, sb0, sb1;
        unit_coords(u, m0, n0, sb0, sb1);
        const int acc = local & 1;
        if (!waitq(&tempty[acc], ((local >> 1) & 1) ^ 1, status, abort_flag)) {
          ok = false;
          break;
        }
        tcgen05_fence_after();
        const uint32_t d_tmem = tmem_base + acc * kBN;
        const int nkb = (sb1 - sb0) * (kSB / kBK);
        for (int kb = 0; kb < nkb; ++kb) {
          if (!waitq(&a_full[as], aph, status, abort_flag) || !waitq(&b_full[bs], bph, status, abort_flag)) {
            ok = false;
            break;
          }
          tcgen05_fence_after();
          const uint64_t a_desc = make_smem_desc_sw128(smem_u32(sA + as * kABytes));
          const uint64_t b_desc = make_smem_desc_sw128(smem_u32(sB + bs * kBBytes));
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k)
            umma_f16_ss(d_tmem, a_desc + 2 * k, b_desc + 2 * k, idesc, (kb > 0 || k > 0) ? 1u : 0u);
          umma_commit(&a_empty[as]);
          umma_commit(&b_empty[bs]);
          if (++as == kAStages) {
            as = 0;
            aph ^= 1;
          }
          if (++bs == kBStages) {
            bs = 0;
            bph ^= 1;
          }
        }
        if (!ok) break;
        umma_commit(&tfull[acc]);
      }
      if (!ok) {
        umma_commit(done_bar);
        drainq(done_bar, 0);
      }
    }
  } else if (warp < kConv0 + kConvWarps) {
    // ---------------------------------------------------------------- converters
    // thread ct: weight row ct / 2 of the tile, half ct % 2 of each 64-weight slice (16-byte chunks
    // {2h, 2h+1} from the low nibbles, {4+2h, 5+2h} from the high nibbles)
    const int ct = threadIdx.x - 32 * kConv0;
    const int row = ct >> 1, h = ct & 1;
    int bs = 0, rs = 0;
    uint32_t bph = 0, rph = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x) {
      int m0, n0, sb0, sb1;
      unit_coords(u, m0, n0, sb0, sb1);
      for (int sb = sb0; sb < sb1 && ok; ++sb) {
        if (!waitq(&r_full[rs], rph, status, abort_flag)) {
          ok = false;
          break;
        }
        const uint8_t* raw = sR + rs * kRawBytes + row * 144;
        const uint4 hdr = *reinterpret_cast<const uint4*>(raw);
        float sa[8], sm[8];  // the super-block's eight sub-block scales and mins, decoded once
#pragma unroll
        for (int j = 0; j < 8; ++j) q4k_scale_min(hdr, j, sa[j], sm[j]);
#pragma unroll
        for (int g = 0; g < kSB / kBK; ++g) {
          if (!waitq(&b_empty[bs], bph ^ 1, status, abort_flag)) {
            ok = false;
            break;
          }
          // the 16 nibble bytes [16h, 16h + 16) of group g: 8 weights x 2 chunks low, 2 chunks high
          const uint4 q = *reinterpret_cast<const uint4*>(raw + 16 + 32 * g + 16 * h);
          const float alo = sa[2 * g], blo = sm[2 * g], ahi = sa[2 * g + 1], bhi = sm[2 * g + 1];
          const uint32_t w[4] = {q.x, q.y, q.z, q.w};
          uint8_t* brow = sB + bs * kBBytes + row * 128;
#pragma unroll
          for (int hi = 0; hi < 2; ++hi) {
            const float a = hi ? ahi : alo, b = hi ? bhi : blo;
#pragma unroll
            for (int cc = 0; cc < 2; ++cc) {  // chunk 2h + cc (+ 4 for the high nibbles)
              uint32_t o[4];
#pragma unroll
              for (int e2 = 0; e2 < 4; ++e2) {
                const uint32_t word = w[2 * cc + (e2 >> 1)];
                const int sh = 16 * (e2 & 1) + 4 * hi;
                const float v0 = a * (float)((word >> sh) & 0xF) - b;
                const float v1 = a * (float)((word >> (sh + 8)) & 0xF) - b;
                o[e2] = pack_bf16x2(v0, v1);
              }
              const int chunk = 4 * hi + 2 * h + cc;
              *reinterpret_cast<uint4*>(brow + ((chunk ^ (row & 7)) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
            }
          }
          fence_proxy_async_smem();  // generic-proxy stores -> visible to the tensor cores
          __syncwarp();
          if (lane == 0) mbar_arrive(&b_full[bs]);
          if (++bs == kBStages) {
            bs = 0;
            bph ^= 1;
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&r_empty[rs]);
        if (++rs == kRStages) {
          rs = 0;
          rph ^= 1;
        }
      }
    }
  } else {
    // ---------------------------------------------------------------- epilogue
    const int lg = warp & 3;  // TMEM lane quarter this warp may access
    int local = 0;
    for (int u = blockIdx.x; u < num_units; u += gridDim.x, ++local) {
      int m0, n0, sb0, sb1;
      unit_coords(u, m0, n0, sb0, sb1);
      const int acc = local & 1;
      if (!waitq(&tfull[acc], (local >> 1) & 1, status, abort_flag)) break;
      tcgen05_fence_after();
      const int row = m0 + lg * 32 + lane;
      const uint32_t tbase = tmem_base + ((uint32_t)(lg * 32) << 16) + acc * kBN;
      if (splits > 1) {
        float* prow = partial + ((int64_t)(u / num_tiles) * M + row) * N;
#pragma unroll 1
        for (int c = 0; c < kBN; c += 32) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(tbase + c, r);
          tmem_ld_wait();
          if (row < M) {
#pragma unroll
            for (int j = 0; j < 8; ++j)
              *reinterpret_cast<uint4*>(prow + n0 + c + 4 * j) = make_uint4(r[4 * j], r[4 * j + 1], r[4 * j + 2], r[4 * j + 3]);
          }
        }
      } else if constexpr (EPI == kEpiSwiglu) {
        // gate columns n0 + [0, 64), up n0 + [64, 128) -> outputs n0 / 2 + [0, 64)
#pragma unroll 1
        for (int c = 0; c < 64; c += 32) {
          uint32_t g[32], v[32];
          tmem_ld_32x32b_x32(tbase + c, g);
          tmem_ld_32x32b_x32(tbase + 64 + c, v);
          tmem_ld_wait();
          if (row < M) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              float o[8];
#pragma unroll
              for (int e = 0; e < 8; ++e)
                o[e] = silu(__uint_as_float(g[8 * j + e])) * __uint_as_float(v[8 * j + e]);
              *reinterpret_cast<uint4*>(C + (int64_t)row * ldc + n0 / 2 + c + 8 * j) = float_to_bf16x8(o);
            }
          }
        }
      } else {
#pragma unroll 1
        for (int c = 0; c < kBN; c += 32) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(tbase + c, r);
          tmem_ld_wait();
          if (row < M) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              float o[8];
#pragma unroll
              for (int e = 0; e < 8; ++e) o[e] = __uint_as_float(r[8 * j + e]);
              *reinterpret_cast<uint4*>(C + (int64_t)row * ldc + n0 + c + 8 * j) = float_to_bf16x8(o);
            }
          }
        }
      }
      tcgen05_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
    }
  }
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tcgen05_fence_after();
    tmem_dealloc(tmem_base, 2 * kBN);
  }
}

}  // namespace

namespace gollek {

int gemm_q4k_splits(int M, int N, int K) {
  const int tiles = ((M + kBM - 1) / kBM) * (N / kBN);
  const int sms = gemm_grid_sms();
  if (tiles >= sms) return 1;
  return std::max(1, std::min(sms / tiles, (K / kSB) / 2));  // >= 2 super-blocks per split
}

void launch_gemm_q4k(void* out, int64_t ldc, const void* a, int64_t lda, const void* w, int M, int N, int K, int epi,
                     int splits, float* partial, uint32_t* status, cudaStream_t s) {
  throw_if(K % kSB != 0, "q4k gemm: K must be a multiple of 256");
  throw_if(N % kBN != 0, "q4k gemm: N must be a multiple of 128");
  throw_if(epi != kEpiNone && epi != kEpiSwiglu, "q4k gemm: plain or SwiGLU epilogue");
  throw_if(lda % 8 != 0 || ldc % 8 != 0, "q4k gemm: rows must keep 16-byte alignment");
  if (M == 0) return;
  if (splits <= 0) splits = gemm_q4k_splits(M, N, K);
  throw_if(splits > 1 && partial == nullptr, "q4k gemm: split-K needs an fp32 workspace");
  const uint64_t row_bytes = (uint64_t)(K / kSB) * 144;
  CUtensorMap ta = make_tmap_2d(a, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, M, K, lda, kBM, kBK, CU_TENSOR_MAP_SWIZZLE_128B);
  CUtensorMap tw = make_tmap_2d(w, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, N, row_bytes, row_bytes, kBN, 144,
                                CU_TENSOR_MAP_SWIZZLE_NONE);
  const int units = ((M + kBM - 1) / kBM) * (N / kBN) * splits;
  const int grid = std::min(units, gemm_grid_sms());
  if (epi == kEpiSwiglu && splits == 1) {
    GOLLEK_CUDA_CHECK(cudaFuncSetAttribute(gemm_q4k_kernel<kEpiSwiglu>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem));
    gemm_q4k_kernel<kEpiSwiglu><<<grid, kThreads, kSmem, s>>>(ta, tw, reinterpret_cast<__nv_bfloat16*>(out), ldc, M, N,
                                                             K, splits, partial, status);
  } else {
    GOLLEK_CUDA_CHECK(cudaFuncSetAttribute(gemm_q4k_kernel<kEpiNone>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem));
    gemm_q4k_kernel<kEpiNone><<<grid, kThreads, kSmem, s>>>(ta, tw, reinterpret_cast<__nv_bfloat16*>(out), ldc, M, N, K,
                                                           splits, partial, status);
  }
  check_launch("gemm_q4k");
  if (splits > 1) splitk_reduce(out, ldc, partial, nullptr, 0, M, N, splits, epi, s);
}

}  // namespace gollek
