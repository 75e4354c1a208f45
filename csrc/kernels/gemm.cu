// K5/K8: bf16 GEMM on the 5th-generation tensor cores (tcgen05 + TMEM + TMA), sm_100a.
//
//   C[M, N'] = epilogue( A[M, K] · B[N, K]^T )      A, B bf16 K-major (nn.Linear layout), fp32 accumulate
//
// Persistent, warp-specialised CTA (192 threads, one CTA per SM):
//   warp 0      TMA producer: one elected lane streams 128x64 A tiles and BNx64 B tiles
//               (128-byte swizzle) into a STAGES-deep shared-memory ring (mbarrier tx counts).
//   warp 1      MMA issuer: one elected lane issues tcgen05.mma (M=128, N=BN, K=16) into a
//               double-buffered TMEM accumulator (2 x BN fp32 columns) and releases smem
//               stages / publishes finished accumulators with tcgen05.commit.
//   warps 2..5  epilogue: tcgen05.ld 32 columns at a time from the TMEM lane quarter the warp
//               may access, apply the fused epilogue, store bf16 to global. Runs concurrently
//               with the next tile's main loop (the other TMEM buffer).
// Fused epilogues: none, +residual (o_proj / down_proj residual add), SwiGLU
// (gate/up rows interleaved in groups of 64 so one tile holds matching gate and up columns;
// output width N/2).
//
// Reference ops replaced: gollek_cuda_matmul / gollek_blackwell_matmul
// (kernel/cuda/gollek-kernel-cuda/…/cuda/binding/CudaBinding.java:59,282-288) and silu_ffn
// (…/CudaBinding.java:64,390-395), CPU math CudaCpuFallback.java:61-117,261-290.
//
// Every mbarrier wait is bounded (globaltimer deadline); on timeout the CTA records a status bit,
// stops issuing, drains its own in-flight copies/MMAs (bounded) and frees its TMEM before returning.
#include "../comm/push.h"
#include "../common/common.cuh"
#include "../common/tma_host.h"
#include "launchers.h"

#include <algorithm>

using namespace gollek;

namespace {

template <int BN>
struct GemmCfg {
  static constexpr int BM = 128, BK = 64;
  static constexpr int STAGES = (BN == 256) ? 4 : (BN == 128 ? 6 : 8);
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr int SMEM = 1024 + STAGES * STAGE_BYTES + 256;
};

GOLLEK_DEVICE uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

constexpr uint64_t kWaitNs = 2000000000ull;  // 2 s: no legitimate wait inside one GEMM comes close

// Bounded, abortable mbarrier wait. Returns false on timeout (status recorded) or abort.
GOLLEK_DEVICE bool wait_bar(uint64_t* bar, uint32_t parity, uint32_t* status, volatile int* abort_flag) {
  for (int i = 0; i < 256; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (globaltimer() - t0 > kWaitNs) {
      report_status(status, kStatusMbarTimeout);
      *abort_flag = 1;
      return false;
    }
  }
}
// Drain wait used only on the abort path (no abort check, still bounded).
GOLLEK_DEVICE void drain_bar(uint64_t* bar, uint32_t parity) {
  const uint64_t t0 = globaltimer();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer() - t0 > kWaitNs) break;
  }
}

template <int BN, int EPI>
__global__ void __launch_bounds__(192, 1)
    gemm_bf16_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmBt,
                     __nv_bfloat16* __restrict__ C, int64_t ldc, const __nv_bfloat16* __restrict__ R, int64_t ldr,
                     int M, int N, int K, int group_m, int splits, float* __restrict__ partial,
                     uint32_t* status, const int* __restrict__ tile_group, const int* __restrict__ num_m_dev,
                     const PushArgs push, int full_tiles, int bnt, const RopeArgs rope) {
  using Cfg = GemmCfg<BN>;
  constexpr int STAGES = Cfg::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * Cfg::A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * Cfg::STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;   // [2]
  uint64_t* tempty = tfull + 2;       // [2]
  uint64_t* done_bar = tempty + 2;    // [1] abort-path drain of the MMA pipe
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* consumed = abort_flag + 1;  // k-blocks consumed by the MMA warp (abort drain)

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Grouped mode (MoE experts): A rows are grouped per expert, each group padded to BM rows;
  // tile_group[m-tile] names the expert whose B rows [g*N, g*N+N) multiply that M tile, and the
  // number of valid M tiles is read from device memory (no host round trip).
  const int num_m = tile_group ? min(*num_m_dev, (M + Cfg::BM - 1) / Cfg::BM) : (M + Cfg::BM - 1) / Cfg::BM;
  const int num_n = (N + BN - 1) / BN;
  const int num_tiles = num_m * num_n;
  // Tail re-tiling (bnt > 0): the first full_tiles tiles (whole waves of the grid) are BN wide; each
  // remaining tile is cut into BN / bnt tiles bnt wide, so the last wave is a short one of narrow
  // tiles instead of a mostly idle one of wide tiles. Each unit is a whole output tile (no split-K).
  const int sub = bnt > 0 ? BN / bnt : 1;
  const int num_units = bnt > 0 ? full_tiles + (num_tiles - full_tiles) * sub : num_tiles * splits;
  const int num_kb = (K + Cfg::BK - 1) / Cfg::BK;
  const int kb_per = (num_kb + splits - 1) / splits;
  // work unit -> (m0, n0, k-block range, tile width). Units are split-major so CTAs running at the
  // same time share a K slice of A; tiles follow a grouped raster (group_m M-tiles swept across all
  // N tiles) so a slab of A stays resident in L2 while B streams.
  auto unit_coords = [&](int u, int& m0, int& n0, int& kb0, int& kb1, int& bnu) {
    int ks, tile, part = 0;
    bnu = BN;
    if (bnt > 0 && u >= full_tiles) {
      ks = 0;
      tile = full_tiles + (u - full_tiles) / sub;
      part = (u - full_tiles) % sub;
      bnu = bnt;
    } else {
      ks = u / num_tiles;
      tile = u % num_tiles;
    }
    const int gsz = group_m * num_n;
    const int g = tile / gsz, r = tile % gsz;
    const int first_m = g * group_m;
    const int gm = min(num_m - first_m, group_m);
    m0 = (first_m + r % gm) * Cfg::BM;
    n0 = (r / gm) * BN + part * bnu;
    kb0 = ks * kb_per;
    kb1 = min(num_kb, kb0 + kb_per);
  };
  constexpr uint32_t idesc = make_idesc_bf16(Cfg::BM, BN);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 4);
    }
    mbar_init(done_bar, 1);
    *abort_flag = 0;
    *consumed = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  tcgen05_fence_before();
  __syncthreads();
  tcgen05_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x) {
        int m0, n0, kb0, kb1, bnu;
        unit_coords(u, m0, n0, kb0, kb1, bnu);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!wait_bar(&empty[stage], phase ^ 1, status, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], Cfg::A_BYTES + bnu * Cfg::BK * 2);
          tma_load_2d(sA + stage * Cfg::A_BYTES, &tmA, kb * Cfg::BK, m0, &full[stage]);
          tma_load_2d(sB + stage * Cfg::B_BYTES, bnu == BN ? &tmB : &tmBt, kb * Cfg::BK,
                      tile_group ? n0 + tile_group[m0 / Cfg::BM] * N : n0, &full[stage]);
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok) {
        // wait (bounded) for our own loads still in flight before the CTA may exit
        for (int i = max(*consumed, issued - STAGES); i < issued; ++i)
          drain_bar(&full[i % STAGES], (i / STAGES) & 1);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      int used = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x, ++local) {
        int m0, n0, kb0, kb1, bnu;
        unit_coords(u, m0, n0, kb0, kb1, bnu);
        const uint32_t id = bnu == BN ? idesc : (bnu == 128 ? make_idesc_bf16(Cfg::BM, 128) : make_idesc_bf16(Cfg::BM, 64));
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!wait_bar(&tempty[acc], acc_phase ^ 1, status, abort_flag)) {
          ok = false;
          break;
        }
        tcgen05_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!wait_bar(&full[stage], phase, status, abort_flag)) {
            ok = false;
            break;
          }
          tcgen05_fence_after();
          const uint64_t a_desc = make_smem_desc_sw128(smem_u32(sA + stage * Cfg::A_BYTES));
          const uint64_t b_desc = make_smem_desc_sw128(smem_u32(sB + stage * Cfg::B_BYTES));
#pragma unroll
          for (int k = 0; k < Cfg::BK / 16; ++k) {
            // +32 bytes along K inside the 128-byte swizzled row = +2 in the encoded address
            umma_f16_ss(d_tmem, a_desc + 2 * k, b_desc + 2 * k, id, (kb > kb0 || k > 0) ? 1u : 0u);
          }
          umma_commit(&empty[stage]);
          *consumed = ++used;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit(&tfull[acc]);
      }
      if (!ok) {
        umma_commit(done_bar);
        drain_bar(done_bar, 0);
      }
    }
  } else {
    // ------------------------------------------------------------------ epilogue (warps 2..5)
    const int lg = warp & 3;  // TMEM lane quarter this warp may access
    int local = 0;
    // push epilogue: the epoch the consumer of this call will wait for (it increments on completion)
    uint32_t push_epoch = 0;
    if constexpr (EPI == kEpiPush)
      push_epoch = *reinterpret_cast<volatile const uint32_t*>(
                       &reinterpret_cast<const SymmHeader*>(push.bases[push.rank])->epoch) + 1;
    for (int u = blockIdx.x; u < num_units; u += gridDim.x, ++local) {
      int m0, n0, kb0, kb1, bnu;
      unit_coords(u, m0, n0, kb0, kb1, bnu);
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!wait_bar(&tfull[acc], acc_phase, status, abort_flag)) break;
      tcgen05_fence_after();
      const int row = m0 + lg * 32 + lane;
      const uint32_t tbase = tmem_base + ((uint32_t)(lg * 32) << 16) + acc * BN;
      if (splits > 1) {
        // split-K: raw fp32 partial sums; the reduce kernel applies the epilogue
        float* prow = partial + ((int64_t)(u / num_tiles) * M + row) * N;
#pragma unroll 1
        for (int c = 0; c < bnu; c += 32) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(tbase + c, r);
          tmem_ld_wait();
          const int col = n0 + c;
          if (row < M) {
#pragma unroll
            for (int j = 0; j < 8; ++j)
              if (col + 4 * j + 4 <= N)
                *reinterpret_cast<uint4*>(prow + col + 4 * j) =
                    make_uint4(r[4 * j], r[4 * j + 1], r[4 * j + 2], r[4 * j + 3]);
          }
        }
      } else if constexpr (EPI == kEpiSwiglu || EPI == kEpiGeglu) {
        const int out_n = N / 2;
#pragma unroll 1
        for (int p = 0; p < bnu / 128; ++p) {
#pragma unroll 1
          for (int h = 0; h < 64; h += 32) {
            uint32_t g[32], u[32];
            tmem_ld_32x32b_x32(tbase + p * 128 + h, g);
            tmem_ld_32x32b_x32(tbase + p * 128 + 64 + h, u);
            tmem_ld_wait();
            const int col = n0 / 2 + p * 64 + h;
            if (row < M) {
              __nv_bfloat16* dst = C + (int64_t)row * ldc + col;
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                if (col + 8 * j + 8 <= out_n) {
                  float v[8];
#pragma unroll
                  for (int e = 0; e < 8; ++e) {
                    const float gv = __uint_as_float(g[8 * j + e]);
                    v[e] = (EPI == kEpiSwiglu ? silu(gv) : gelu_tanh(gv)) * __uint_as_float(u[8 * j + e]);
                  }
                  *reinterpret_cast<uint4*>(dst + 8 * j) = float_to_bf16x8(v);
                }
              }
            }
          }
        }
      } else if constexpr (EPI == kEpiRope) {
        // head_dim-128 heads: q (rotated) -> q_out, k (rotated) / v -> the row's paged cache slot.
        // The fp32 accumulator is rotated directly (one rounding, at the store).
        const bool live = row < M;
        int pos = live ? rope.positions[row] : 0;
        pos = pos < 0 ? 0 : (pos >= rope.max_pos ? rope.max_pos - 1 : pos);
        const float* cs = rope.cos_sin + (int64_t)pos * 128;
        int slot = live && rope.slots != nullptr ? rope.slots[row] : -1;
        if (slot >= 0 && (slot / rope.block_size >= rope.num_blocks)) slot = -1;  // beyond the pool: not written
        auto* qo = reinterpret_cast<__nv_bfloat16*>(rope.q_out);
        auto* kc = reinterpret_cast<__nv_bfloat16*>(rope.cache);
#pragma unroll 1
        for (int hb = 0; hb < bnu; hb += 128) {
          const int head = (n0 + hb) >> 7;
          __nv_bfloat16* dst = nullptr;
          if (head < rope.H) {
            dst = qo + ((int64_t)row * rope.H + head) * 128;
          } else if (slot >= 0) {
            const int which = head < rope.H + rope.Hk ? 0 : 1, kh = head - rope.H - which * rope.Hk;
            const int64_t blk = slot / rope.block_size, off = slot % rope.block_size;
            dst = kc + (((blk * 2 + which) * rope.Hk + kh) * rope.block_size + off) * 128;
          }
          const bool rotate = head < rope.H + rope.Hk;
#pragma unroll 1
          for (int c = 0; c < 64; c += 32) {
            uint32_t x1[32], x2[32];
            tmem_ld_32x32b_x32(tbase + hb + c, x1);
            tmem_ld_32x32b_x32(tbase + hb + 64 + c, x2);
            tmem_ld_wait();
            if (!live || dst == nullptr) continue;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              float o1[8], o2[8];
              if (rotate) {
                const float4* cp = reinterpret_cast<const float4*>(cs + c + 8 * j);
                const float4* sp = reinterpret_cast<const float4*>(cs + 64 + c + 8 * j);
                const float4 c0 = __ldg(cp), c1 = __ldg(cp + 1), s0 = __ldg(sp), s1 = __ldg(sp + 1);
                const float cv[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
                const float sv[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                  const float a = __uint_as_float(x1[8 * j + e]), b = __uint_as_float(x2[8 * j + e]);
                  o1[e] = a * cv[e] - b * sv[e];
                  o2[e] = b * cv[e] + a * sv[e];
                }
              } else {
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                  o1[e] = __uint_as_float(x1[8 * j + e]);
                  o2[e] = __uint_as_float(x2[8 * j + e]);
                }
              }
              *reinterpret_cast<uint4*>(dst + c + 8 * j) = float_to_bf16x8(o1);
              *reinterpret_cast<uint4*>(dst + 64 + c + 8 * j) = float_to_bf16x8(o2);
            }
          }
        }
      } else {
#pragma unroll 1
        for (int c = 0; c < bnu; c += 32) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(tbase + c, r);
          tmem_ld_wait();
          const int col = n0 + c;
          __nv_bfloat16* dst = C + (int64_t)row * ldc + col;
          bool store_row = row < M;
          if constexpr (EPI == kEpiScatter) {  // per-row destination (0: padding row, skipped)
            const uint64_t rp = store_row ? reinterpret_cast<const uint64_t*>(C)[row] : 0ull;
            store_row = rp != 0ull;
            dst = reinterpret_cast<__nv_bfloat16*>(rp) + col;
          }
          if (store_row) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              if (col + 8 * j + 8 <= N) {
                float v[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) v[e] = __uint_as_float(r[8 * j + e]);
                if constexpr (EPI == kEpiResidual) {
                  float rr[8];
                  bf16x8_to_float(*reinterpret_cast<const uint4*>(R + (int64_t)row * ldr + col + 8 * j), rr);
#pragma unroll
                  for (int e = 0; e < 8; ++e) v[e] += rr[e];
                }
                const uint4 packed = float_to_bf16x8(v);
                *reinterpret_cast<uint4*>(dst + 8 * j) = packed;
                if constexpr (EPI == kEpiPush) {
                  // the same bytes into this rank's slot of every peer's inbox (NVLink stores)
                  const int64_t off = ((int64_t)push.rank * push.slot_elems + (int64_t)row * N + col + 8 * j) * 2;
                  for (int p = 0; p < push.world; ++p) {
                    if (p == push.rank) continue;
                    *reinterpret_cast<uint4*>(push.bases[p] + push.inbox_off + off) = packed;
                  }
                }
              }
            }
          }
        }
        if constexpr (EPI == kEpiPush) {
          // publish this warp's 32 rows of the tile: every lane's stores ordered before the flags
          __threadfence_system();
          __syncwarp();
          if (lane == 0) {
            const int grp = (m0 >> 7) * 4 + lg;
            const int64_t fi = ((int64_t)push.rank * push.g_max + grp) * push.nt_max + n0 / BN;
            for (int p = 0; p < push.world; ++p)
              st_release_sys(reinterpret_cast<uint32_t*>(push.bases[p] + push.flags_off) + fi, push_epoch);
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
    tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}

// Split-K reduction: out = epilogue(sum_s partial[s]) for one 8-column group per thread.
template <int EPI>
__global__ void splitk_reduce_kernel(__nv_bfloat16* __restrict__ C, int64_t ldc, const float* __restrict__ partial,
                                     const __nv_bfloat16* __restrict__ R, int64_t ldr, int M, int N, int splits) {
  const int out_n = (EPI == kEpiSwiglu || EPI == kEpiGeglu) ? N / 2 : N;
  const int groups = out_n / 8;
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (int64_t)M * groups) return;
  const int row = idx / groups, col = (idx % groups) * 8;
  float v[8];
  if constexpr (EPI == kEpiSwiglu || EPI == kEpiGeglu) {
    const int gc = (col / 64) * 128 + col % 64;  // gate column of the interleaved weight rows
    float g[8] = {0}, u[8] = {0};
    for (int s = 0; s < splits; ++s) {
      const float* p = partial + ((int64_t)s * M + row) * N;
      const float4 g0 = *reinterpret_cast<const float4*>(p + gc), g1 = *reinterpret_cast<const float4*>(p + gc + 4);
      const float4 u0 = *reinterpret_cast<const float4*>(p + gc + 64), u1 = *reinterpret_cast<const float4*>(p + gc + 68);
      g[0] += g0.x; g[1] += g0.y; g[2] += g0.z; g[3] += g0.w; g[4] += g1.x; g[5] += g1.y; g[6] += g1.z; g[7] += g1.w;
      u[0] += u0.x; u[1] += u0.y; u[2] += u0.z; u[3] += u0.w; u[4] += u1.x; u[5] += u1.y; u[6] += u1.z; u[7] += u1.w;
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = (EPI == kEpiSwiglu ? silu(g[e]) : gelu_tanh(g[e])) * u[e];
  } else {
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = 0.f;
    for (int s = 0; s < splits; ++s) {
      const float* p = partial + ((int64_t)s * M + row) * N + col;
      const float4 a = *reinterpret_cast<const float4*>(p), b = *reinterpret_cast<const float4*>(p + 4);
      v[0] += a.x; v[1] += a.y; v[2] += a.z; v[3] += a.w; v[4] += b.x; v[5] += b.y; v[6] += b.z; v[7] += b.w;
    }
    if constexpr (EPI == kEpiResidual) {
      float rr[8];
      bf16x8_to_float(*reinterpret_cast<const uint4*>(R + (int64_t)row * ldr + col), rr);
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] += rr[e];
    }
  }
  *reinterpret_cast<uint4*>(C + (int64_t)row * ldc + col) = float_to_bf16x8(v);
}

template <int BN, int EPI>
void launch_gemm_t(void* out, int64_t ldc, const void* a, int64_t lda, const void* b, int64_t ldb, const void* res,
                   int64_t ldr, int M, int N, int K, int splits, float* partial, uint32_t* status, int grid_limit,
                   cudaStream_t s, const int* tile_group = nullptr, const int* num_m_dev = nullptr, int groups = 1,
                   bool reduce = true, const PushArgs* push = nullptr, const RopeArgs* rope = nullptr) {
  using Cfg = GemmCfg<BN>;
  CUtensorMap ta = make_tmap_2d(a, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, M, K, lda, Cfg::BM, Cfg::BK,
                                CU_TENSOR_MAP_SWIZZLE_128B);
  CUtensorMap tb = make_tmap_2d(b, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (uint64_t)N * groups, K, ldb, BN, Cfg::BK,
                                CU_TENSOR_MAP_SWIZZLE_128B);
  auto kern = gemm_bf16_kernel<BN, EPI>;
  GOLLEK_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM));
  const int num_m = (M + Cfg::BM - 1) / Cfg::BM;
  const int tiles = num_m * ((N + BN - 1) / BN);
  // grouped raster: a ~32 MB slab of A (group_m M-tiles) stays L2-resident while B streams
  const int64_t a_tile_bytes = (int64_t)Cfg::BM * K * 2;
  const int group_m = (int)std::max<int64_t>(1, std::min<int64_t>(num_m, (32ll << 20) / a_tile_bytes));
  int grid = std::min(tiles * splits, gemm_grid_sms());
  if (grid_limit > 0) grid = std::min(grid, grid_limit);
  // tail re-tiling: plain GEMMs only (no split-K, no grouped / push mode, whole output tiles)
  int full_tiles = 0, bnt = 0;
  if (splits == 1 && tile_group == nullptr && push == nullptr && N % BN == 0)
    gemm_retile_plan(tiles, grid, BN, epi_wide(EPI), full_tiles, bnt);
  CUtensorMap tbt = bnt > 0 ? make_tmap_2d(b, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (uint64_t)N * groups, K, ldb, bnt,
                                           Cfg::BK, CU_TENSOR_MAP_SWIZZLE_128B)
                            : tb;
  if (bnt > 0) grid = std::min(full_tiles + (tiles - full_tiles) * (BN / bnt), std::max(grid, 1));
  kern<<<grid, 192, Cfg::SMEM, s>>>(ta, tb, tbt, reinterpret_cast<__nv_bfloat16*>(out), ldc,
                                     reinterpret_cast<const __nv_bfloat16*>(res), ldr, M, N, K, group_m, splits,
                                     partial, status, tile_group, num_m_dev, push ? *push : PushArgs{}, full_tiles,
                                     bnt, rope ? *rope : RopeArgs{});
  check_launch("gemm_bf16");
  if (splits > 1 && reduce) {
    const int out_n = (EPI == kEpiSwiglu || EPI == kEpiGeglu) ? N / 2 : N;
    const int64_t threads = (int64_t)M * (out_n / 8);
    splitk_reduce_kernel<EPI><<<(unsigned)((threads + 255) / 256), 256, 0, s>>>(
        reinterpret_cast<__nv_bfloat16*>(out), ldc, partial, reinterpret_cast<const __nv_bfloat16*>(res), ldr, M, N,
        splits);
    check_launch("gemm_bf16 split-K reduce");
  }
}

}  // namespace

namespace gollek {

int device_num_sms() { return num_sms(); }

void splitk_reduce(void* out, int64_t ldc, const float* partial, const void* residual, int64_t ldr, int M, int N,
                   int splits, int epi, cudaStream_t s) {
  const int out_n = epi_gated(epi) ? N / 2 : N;
  const int64_t threads = (int64_t)M * (out_n / 8);
  const unsigned grid = (unsigned)((threads + 255) / 256);
  auto* o = reinterpret_cast<__nv_bfloat16*>(out);
  auto* r = reinterpret_cast<const __nv_bfloat16*>(residual);
  if (epi == kEpiSwiglu)
    splitk_reduce_kernel<kEpiSwiglu><<<grid, 256, 0, s>>>(o, ldc, partial, r, ldr, M, N, splits);
  else if (epi == kEpiGeglu)
    splitk_reduce_kernel<kEpiGeglu><<<grid, 256, 0, s>>>(o, ldc, partial, r, ldr, M, N, splits);
  else if (epi == kEpiResidual)
    splitk_reduce_kernel<kEpiResidual><<<grid, 256, 0, s>>>(o, ldc, partial, r, ldr, M, N, splits);
  else
    splitk_reduce_kernel<kEpiNone><<<grid, 256, 0, s>>>(o, ldc, partial, r, ldr, M, N, splits);
  check_launch("split-K reduce");
}

// Relative time of one 128-row output tile of width bn (same K) against a 256-wide one: measured
// 1.14x lower per-FLOP throughput of 128-wide tiles at M = 4352 gives 0.57; 64-wide tiles reload the
// same A tile for a quarter of the MMA work.
static double tile_time(int bn) { return bn >= 256 ? 1.0 : (bn == 128 ? 0.57 : 0.36); }

void gemm_retile_plan(int tiles, int grid, int bn, bool gated, int& full_tiles, int& bnt) {
  full_tiles = 0;
  bnt = 0;
  if (grid <= 0 || tiles <= grid) return;  // one partial wave: nothing to rebalance against
  const int full = (tiles / grid) * grid, tail = tiles - full;
  if (tail == 0) return;
  double best = tile_time(bn);  // the tail as one more wave of bn-wide tiles
  for (int t : {128, 64}) {
    if (t >= bn || (gated && t < 128)) continue;  // gated epilogues need a gate/up pair (128 columns)
    const int units = tail * (bn / t);
    const double c = (double)((units + grid - 1) / grid) * tile_time(t);
    if (c < 0.9 * best) {
      best = c;
      bnt = t;
    }
  }
  if (bnt > 0) full_tiles = full;
}

// Output-tile waves x tile time for a bn-wide persistent GEMM, with the tail re-tiling.
static double gemm_cost(int tiles, int sms, int bn, bool gated) {
  int full, bnt;
  gemm_retile_plan(tiles, sms, bn, gated, full, bnt);
  if (bnt == 0) return (double)((tiles + sms - 1) / sms) * tile_time(bn);
  const int units = (tiles - full) * (bn / bnt);
  return (double)(full / sms) * tile_time(bn) + (double)((units + sms - 1) / sms) * tile_time(bnt);
}

int gemm_pick_bn(int M, int N, int epi) {
  const int num_m = (M + 127) / 128;
  const int sms = num_sms();
  if (num_m >= 4) {
    // Compute-bound: the persistent grid runs ceil(tiles / SMs) rounds of tiles, so pick the width
    // with the fewest rounds x tile time. A 128-wide tile takes ~0.57 of a 256-wide one (measured
    // 1.14x lower per-FLOP throughput at M = 4352), which makes 128 win when 256-wide tiles leave a
    // mostly idle last round (e.g. M = 1344, N = 4096: 176 tiles on 148 SMs).
    auto cost = [&](int bn) { return gemm_cost(num_m * ((N + bn - 1) / bn), sms, bn, epi_wide(epi)); };
    return cost(128) < cost(256) ? 128 : 256;
  }
  if (epi_wide(epi)) return (num_m * ((N + 255) / 256) >= sms) ? 256 : 128;
  if (num_m * ((N + 255) / 256) >= sms) return 256;
  if (num_m * ((N + 127) / 128) >= sms / 2) return 128;
  return 64;
}

// Tile width and split-K factor for one GEMM.
//
// Decode-sized M (one or two 128-row tiles) with a narrow output (o_proj / down_proj, N = 4096):
// without a split the GEMM has too few output tiles to occupy the GPU (64 tiles of 64 columns on 148
// SMs), and each CTA streams its weight slice plus the whole activation from L2 alone. 128-wide
// tiles split along K into s = floor(SMs / tiles) parts (one wave, fp32 partials summed with the
// epilogue by a reduce pass) let every SM stream 1/s of the K range. Measured on B200 (M = 64 / 128 /
// 256): o_proj 4096 x 4096 0.0179 / 0.0191 / 0.0199 -> 0.0129 / 0.0144 / 0.0165 ms, down_proj
// 4096 x 14336 0.0462 / 0.0477 / 0.0491 -> 0.0276 / 0.0298 / 0.0375 ms. The qkv output (6144 wide,
// K = 4096) lost with a split (M = 128: 0.0168 -> 0.0187 ms: the fp32 partials cost more than the
// idle SMs), so outputs wider than 4096 split only for K >= 8192; gate/up (gated) and RoPE
// epilogues never split.
void gemm_plan(int M, int N, int K, int epi, int& bn, int& splits) {
  const int num_m = (M + 127) / 128;
  const int sms = num_sms();
  splits = 1;
  if (bn == 0) {
    bn = gemm_pick_bn(M, N, epi);
    if ((epi == kEpiNone || epi == kEpiResidual) && num_m <= 2 && N % 128 == 0) {
      const int tiles = num_m * (N / 128);
      const int s = std::min(8, sms / std::max(1, tiles));
      if (2 * tiles <= sms && s >= 2 && K / s >= 1024 && (N <= 4096 || K >= 8192)) {
        bn = 128;
        splits = s;
      }
    }
  }
  if (epi_wide(epi) && bn < 128) bn = 128;
}

int gemm_splits(int M, int N, int K, int epi) {
  int bn = 0, sp = 1;
  gemm_plan(M, N, K, epi, bn, sp);
  return sp;
}

void launch_gemm_bf16(void* out, int64_t ldc, const void* a, int64_t lda, const void* b, int64_t ldb,
                      const void* residual, int64_t ldr, int M, int N, int K, int epi, int bn, int splits,
                      float* partial, uint32_t* status, int grid_limit, cudaStream_t s) {
  throw_if(K % 8 != 0, "gemm: K must be a multiple of 8");
  throw_if(ldc % 8 != 0, "gemm: output row pitch must keep 16-byte alignment");
  if (M == 0) return;
  if (epi_gated(epi)) throw_if(N % 128 != 0, "gemm swiglu/geglu: N must be a multiple of 128");
  else throw_if(N % 8 != 0, "gemm: N must be a multiple of 8");
  if (epi == kEpiResidual) throw_if(residual == nullptr || ldr % 8 != 0, "gemm residual: bf16 residual required");
  if (bn == 0) {
    int sp = 1;
    gemm_plan(M, N, K, epi, bn, sp);
    if (splits <= 0) splits = sp;
  }
  if (splits <= 0) splits = 1;
  if (epi_wide(epi) && bn < 128) bn = 128;
  throw_if(splits > 1 && partial == nullptr, "gemm: split-K needs an fp32 workspace");
#define GOLLEK_GEMM_CASE(BNV, EPIV) \
  if (bn == BNV && epi == EPIV)     \
    return launch_gemm_t<BNV, EPIV>(out, ldc, a, lda, b, ldb, residual, ldr, M, N, K, splits, partial, status, \
                                    grid_limit, s);
  GOLLEK_GEMM_CASE(256, kEpiNone)
  GOLLEK_GEMM_CASE(128, kEpiNone)
  GOLLEK_GEMM_CASE(64, kEpiNone)
  GOLLEK_GEMM_CASE(256, kEpiResidual)
  GOLLEK_GEMM_CASE(128, kEpiResidual)
  GOLLEK_GEMM_CASE(64, kEpiResidual)
  GOLLEK_GEMM_CASE(256, kEpiSwiglu)
  GOLLEK_GEMM_CASE(128, kEpiSwiglu)
  GOLLEK_GEMM_CASE(256, kEpiGeglu)
  GOLLEK_GEMM_CASE(128, kEpiGeglu)
#undef GOLLEK_GEMM_CASE
  throw_if(true, "gemm: unsupported tile width " + std::to_string(bn) + " / epilogue " + std::to_string(epi));
}

void launch_gemm_rope_kv(const void* a, int64_t lda, const void* b, int64_t ldb, int M, int K, const RopeArgs& rope,
                         cudaStream_t s) {
  throw_if(K % 8 != 0, "qkv gemm: K must be a multiple of 8");
  throw_if(rope.H <= 0 || rope.Hk <= 0 || rope.positions == nullptr || rope.cos_sin == nullptr || rope.q_out == nullptr,
           "qkv gemm + rope: arguments");
  throw_if(rope.max_pos <= 0 || (rope.cache != nullptr && (rope.slots == nullptr || rope.block_size <= 0)),
           "qkv gemm + rope: cache arguments");
  if (M == 0) return;
  const int N = (rope.H + 2 * rope.Hk) * 128;
  int bn = 0, splits = 1;
  gemm_plan(M, N, K, kEpiRope, bn, splits);
  // heads are 128 wide: 128- or 256-wide tiles hold whole heads (the re-tiled tail too)
  if (bn == 256)
    return launch_gemm_t<256, kEpiRope>(rope.q_out, N, a, lda, b, ldb, nullptr, 0, M, N, K, 1, nullptr, nullptr, 0, s,
                                        nullptr, nullptr, 1, true, nullptr, &rope);
  return launch_gemm_t<128, kEpiRope>(rope.q_out, N, a, lda, b, ldb, nullptr, 0, M, N, K, 1, nullptr, nullptr, 0, s,
                                      nullptr, nullptr, 1, true, nullptr, &rope);
}

void launch_gemm_push(void* out, const void* a, int64_t lda, const void* b, int64_t ldb, int M, int N, int K, int bn,
                      const std::vector<uint64_t>& bases, int rank, int64_t inbox_off, int64_t slot_elems,
                      int64_t flags_off, int g_max, int nt_max, uint32_t* status, cudaStream_t s) {
  throw_if(K % 8 != 0 || N % 8 != 0, "push gemm: N and K must be multiples of 8");
  throw_if(bases.empty() || bases.size() > 8 || rank < 0 || rank >= (int)bases.size(), "push gemm: 1..8 ranks");
  throw_if((M + 31) / 32 > g_max || (N + bn - 1) / bn > nt_max, "push gemm: flag array too small for this call");
  throw_if(inbox_off % 16 != 0 || (slot_elems * 2) % 16 != 0, "push gemm: inbox must keep 16-byte alignment");
  if (M == 0) return;
  PushArgs p{};
  for (size_t i = 0; i < bases.size(); ++i) p.bases[i] = reinterpret_cast<uint8_t*>(bases[i]);
  p.inbox_off = inbox_off;
  p.slot_elems = slot_elems;
  p.flags_off = flags_off;
  p.world = (int)bases.size();
  p.rank = rank;
  p.g_max = g_max;
  p.nt_max = nt_max;
#define GOLLEK_PUSH_CASE(BNV) \
  if (bn == BNV)              \
    return launch_gemm_t<BNV, kEpiPush>(out, N, a, lda, b, ldb, nullptr, 0, M, N, K, 1, nullptr, status, 0, s, \
                                        nullptr, nullptr, 1, true, &p);
  GOLLEK_PUSH_CASE(256)
  GOLLEK_PUSH_CASE(128)
  GOLLEK_PUSH_CASE(64)
#undef GOLLEK_PUSH_CASE
  throw_if(true, "push gemm: unsupported tile width " + std::to_string(bn));
}

void launch_gemm_grouped(void* out, int64_t ldc, const void* a, int64_t lda, const void* b, int64_t ldb, int M_cap,
                         int N, int K, int groups, int epi, int bn, const int* tile_group, const int* num_m_dev,
                         int splits, float* partial, uint32_t* status, cudaStream_t s) {
  throw_if(K % 8 != 0, "grouped gemm: K must be a multiple of 8");
  throw_if(ldc % 8 != 0, "grouped gemm: output row pitch must keep 16-byte alignment");
  throw_if(M_cap % 128 != 0, "grouped gemm: row capacity must be a multiple of 128");
  throw_if(tile_group == nullptr || num_m_dev == nullptr, "grouped gemm: tile map required");
  throw_if(epi == kEpiResidual, "grouped gemm: residual epilogue not supported");
  if (M_cap == 0) return;
  if (epi == kEpiSwiglu) throw_if(N % 128 != 0, "grouped gemm swiglu: N must be a multiple of 128");
  else throw_if(N % 8 != 0, "grouped gemm: N must be a multiple of 8");
  if (bn == 0) {
    // typical live M tiles: one per expert at decode, capacity/128 when every expert is full
    const int m_tiles = std::max(groups, std::min(M_cap / 128, groups * 2));
    bn = (m_tiles * ((N + 255) / 256) >= num_sms() || epi == kEpiSwiglu) ? 256 : 128;
  }
  if (epi_wide(epi) && bn < 128) bn = 128;
  if (splits < 1) splits = 1;
  // split-K partials [splits, M_cap, N] are left for the caller to reduce (no reduce pass here)
  throw_if(splits > 1 && (partial == nullptr || epi != kEpiNone), "grouped gemm: split-K needs fp32 partials, no epilogue");
  throw_if(epi == kEpiScatter && splits > 1, "grouped gemm: the scatter epilogue has no split-K");
#define GOLLEK_GG_CASE(BNV, EPIV) \
  if (bn == BNV && epi == EPIV)   \
    return launch_gemm_t<BNV, EPIV>(out, ldc, a, lda, b, ldb, nullptr, 0, M_cap, N, K, splits, partial, status, 0, s, \
                                    tile_group, num_m_dev, groups, /*reduce=*/false);
  GOLLEK_GG_CASE(256, kEpiNone)
  GOLLEK_GG_CASE(128, kEpiNone)
  GOLLEK_GG_CASE(64, kEpiNone)
  GOLLEK_GG_CASE(256, kEpiSwiglu)
  GOLLEK_GG_CASE(128, kEpiSwiglu)
  GOLLEK_GG_CASE(256, kEpiScatter)
  GOLLEK_GG_CASE(128, kEpiScatter)
  GOLLEK_GG_CASE(64, kEpiScatter)
#undef GOLLEK_GG_CASE
  throw_if(true, "grouped gemm: unsupported tile width " + std::to_string(bn));
}

}  // namespace gollek
