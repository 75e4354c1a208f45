// K4 on tcgen05: paged, varlen, causal prefill attention, head_dim 128 (sm_100a).
//
// One CTA = 128 query rows of one sequence x one query head. 6 warps:
//   warp 0   TMA: Q tile once (2 boxes of 64 dims), then per 128-key KV tile the 8 paged blocks of
//            K and of V (box 64 dims x 16 tokens, 128-byte swizzle) into a 2-stage ring.
//   warp 1   MMA (one thread): S_j = Q K_j^T into one of two TMEM S buffers, and O += P_{j-1} V_{j-1}
//            into the TMEM O accumulator, interleaved (S_{j+1} is computed while the softmax warps
//            work on S_j). P is an smem A operand (K-major, swizzled); V is an MN-major B operand.
//   warps 2-5 softmax, one query row per thread (= TMEM lane): online softmax in the log2 domain,
//            causal / length mask, rescale of O in TMEM when the row max moves, P (bf16) to smem,
//            final O / l to global.
// All mbarrier waits are bounded; on timeout the CTA records a status bit and drains.
//
// Replaces the reference's FA2/FA3/FA4 bindings (kernel/cuda/gollek-kernel-cuda/…/CudaBinding.java:61-62,
// core/optimization/gollek-plugin-fa4/…/FlashAttention4Binding.java:15-46) with paged-KV semantics of
// runner/safetensor/gollek-safetensor-engine/…/attention/PagedAttentionVectorAPI.java:20-127.
#include "../common/common.cuh"
#include "../common/tma_host.h"
#include "launchers.h"

using namespace gollek;

namespace {

constexpr int kTQ = 128, kTK = 128, kD = 128, kBS = 16;
constexpr int kQBytes = kTQ * kD * 2;    // 32 KB (two 16 KB boxes)
constexpr int kKVTile = kTK * kD * 2;    // 32 KB per K (or V) tile
constexpr int kStages = 2;
constexpr int kPBytes = kTQ * kTK * 2;   // 32 KB
constexpr int kThreads = 192;
constexpr int kSmem = 1024 + kQBytes + kStages * 2 * kKVTile + kPBytes + 256;
constexpr uint64_t kWait = 2000000000ull;

GOLLEK_DEVICE uint64_t gtime() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
GOLLEK_DEVICE bool waitq(uint64_t* bar, uint32_t parity, uint32_t* status, volatile int* abort_flag) {
  for (int i = 0; i < 128; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = gtime();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (gtime() - t0 > kWait) {
      report_status(status, kStatusMbarTimeout);
      *abort_flag = 1;
      return false;
    }
  }
}
GOLLEK_DEVICE void drainq(uint64_t* bar, uint32_t parity) {
  const uint64_t t0 = gtime();
  while (!mbar_try_wait(bar, parity))
    if (gtime() - t0 > kWait) break;
}

GOLLEK_DEVICE void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]),
      "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]),
      "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

// MN-major, 128-byte-swizzled operand descriptor: atoms of 64 elements along MN (LBO apart),
// 8-row groups along K 1024 bytes apart.
GOLLEK_DEVICE uint64_t make_desc_mn_sw128(uint32_t addr, uint32_t lbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((addr & 0x3FFFF) >> 4);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

__global__ void __launch_bounds__(kThreads, 1)
    prefill_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmKV,
                      __nv_bfloat16* __restrict__ out, int64_t out_stride, const int* __restrict__ block_tables,
                      int bt_stride, const int* __restrict__ seq_lens, const int* __restrict__ query_start,
                      const int* __restrict__ tiles, int H, int Hk, float scale_log2, uint32_t* status, int window,
                      float softcap_log2) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint8_t* sQ = smem;
  uint8_t* sKV = sQ + kQBytes;                 // stage s: K at + s*2*tile, V at + s*2*tile + tile
  uint8_t* sP = sKV + kStages * 2 * kKVTile;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + kPBytes);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;                // [2]
  uint64_t* kv_empty = bars + 3;               // [2]
  uint64_t* s_full = bars + 5;                 // [2]
  uint64_t* s_free = bars + 7;                 // [2]
  uint64_t* p_full = bars + 9;
  uint64_t* pv_done = bars + 10;
  uint64_t* done_bar = bars + 11;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 12);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = tiles[2 * blockIdx.x], q_off = tiles[2 * blockIdx.x + 1];
  const int h = blockIdx.y, kh = h / (H / Hk);
  const int qs = query_start[b], qlen = query_start[b + 1] - qs;
  const int L = seq_lens[b];
  const int ctx0 = L - qlen;
  const int rows = min(kTQ, qlen - q_off);
  const int kv_end = min(L, ctx0 + q_off + rows);
  // KV tiles [j0, j0 + nt): with a sliding window the first query row sees keys >= its position - window + 1
  const int j0 = window > 0 ? max(0, ctx0 + q_off - window + 1) / kTK : 0;
  const int nt = (kv_end + kTK - 1) / kTK - j0;
  const int* bt = block_tables + (int64_t)b * bt_stride;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 4);
    }
    mbar_init(p_full, 4);
    mbar_init(pv_done, 1);
    mbar_init(done_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tcgen05_fence_before();
  __syncthreads();
  tcgen05_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS = tmem;            // S buffers at columns 0 and 128
  const uint32_t tO = tmem + 256;      // O accumulator at columns 256..383

  if (warp == 0) {
    if (elect_one()) {
      prefetch_tmap(&tmQ);
      prefetch_tmap(&tmKV);
      mbar_arrive_expect_tx(q_full, kQBytes);
      const int qrow = qs + q_off;
      tma_load_2d(sQ, &tmQ, h * kD, qrow, q_full);
      tma_load_2d(sQ + kQBytes / 2, &tmQ, h * kD + 64, qrow, q_full);
      int issued = 0;
      bool ok = true;
      for (int j = 0; j < nt; ++j) {
        const int st = j & 1;
        if (!waitq(&kv_empty[st], ((j >> 1) & 1) ^ 1, status, abort_flag)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&kv_full[st], 2 * kKVTile);
        uint8_t* dk = sKV + st * 2 * kKVTile;
        uint8_t* dv = dk + kKVTile;
        for (int blk = 0; blk < kTK / kBS; ++blk) {
          const int kb = ((j0 + j) * kTK) / kBS + blk;
          const int pb = (kb * kBS < kv_end) ? bt[kb] : bt[0];
          const int rk = ((pb * 2 + 0) * Hk + kh) * kBS, rv = ((pb * 2 + 1) * Hk + kh) * kBS;
          tma_load_2d(dk + blk * 2048, &tmKV, 0, rk, &kv_full[st]);
          tma_load_2d(dk + kKVTile / 2 + blk * 2048, &tmKV, 64, rk, &kv_full[st]);
          tma_load_2d(dv + blk * 2048, &tmKV, 0, rv, &kv_full[st]);
          tma_load_2d(dv + kKVTile / 2 + blk * 2048, &tmKV, 64, rv, &kv_full[st]);
        }
        ++issued;
      }
      if (!ok) {
        drainq(q_full, 0);
        for (int j = max(0, issued - 2); j < issued; ++j) drainq(&kv_full[j & 1], (j >> 1) & 1);
      }
    }
  } else if (warp == 1) {
    if (elect_one()) {
      constexpr uint32_t idesc_s = make_idesc_bf16(kTQ, kTK);                      // Q K^T, both K-major
      constexpr uint32_t idesc_o = make_idesc_bf16(kTQ, kD) | (1u << 16);          // P V, V MN-major
      bool ok = waitq(q_full, 0, status, abort_flag);
      const uint32_t q_addr = smem_u32(sQ), p_addr = smem_u32(sP);
      auto issue_pv = [&](int jp) {
        const int st = jp & 1;
        const uint32_t v_addr = smem_u32(sKV + st * 2 * kKVTile + kKVTile);
#pragma unroll
        for (int ks = 0; ks < kTK / 16; ++ks) {
          const uint64_t a = make_smem_desc_sw128(p_addr + (ks >> 2) * (kPBytes / 2) + (ks & 3) * 32);
          const uint64_t bd = make_desc_mn_sw128(v_addr + ks * 2048, kKVTile / 2);
          umma_f16_ss(tO, a, bd, idesc_o, (jp > 0 || ks > 0) ? 1u : 0u);
        }
        umma_commit(pv_done);
        umma_commit(&kv_empty[st]);
      };
      for (int j = 0; j < nt && ok; ++j) {
        const int st = j & 1;
        if (!waitq(&kv_full[st], (j >> 1) & 1, status, abort_flag) ||
            !waitq(&s_free[st], ((j >> 1) & 1) ^ 1, status, abort_flag)) {
          ok = false;
          break;
        }
        tcgen05_fence_after();
        const uint32_t k_addr = smem_u32(sKV + st * 2 * kKVTile);
#pragma unroll
        for (int ks = 0; ks < kD / 16; ++ks) {
          const uint64_t a = make_smem_desc_sw128(q_addr + (ks >> 2) * (kQBytes / 2) + (ks & 3) * 32);
          const uint64_t bd = make_smem_desc_sw128(k_addr + (ks >> 2) * (kKVTile / 2) + (ks & 3) * 32);
          umma_f16_ss(tS + st * kTK, a, bd, idesc_s, ks > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[st]);
        if (j >= 1) {
          if (!waitq(p_full, (j - 1) & 1, status, abort_flag)) {
            ok = false;
            break;
          }
          tcgen05_fence_after();
          issue_pv(j - 1);
        }
      }
      if (ok && nt > 0) {
        if (waitq(p_full, (nt - 1) & 1, status, abort_flag)) {
          tcgen05_fence_after();
          issue_pv(nt - 1);
        } else {
          ok = false;
        }
      }
      if (!ok) {
        umma_commit(done_bar);
        drainq(done_bar, 0);
      }
    }
  } else {
    // softmax warps 2..5: TMEM lane quarter = warp & 3; row r of the tile = lane quarter * 32 + lane
    const int lg = warp & 3;
    const int r = lg * 32 + lane;
    const int qpos = ctx0 + q_off + r;
    const uint32_t lane_off = (uint32_t)(lg * 32) << 16;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < nt; ++j) {
      const int st = j & 1;
      if (!waitq(&s_full[st], (j >> 1) & 1, status, abort_flag)) {
        ok = false;
        break;
      }
      tcgen05_fence_after();
      float s[kTK];
#pragma unroll
      for (int c = 0; c < kTK; c += 32) {
        uint32_t u[32];
        tmem_ld_32x32b_x32(tS + st * kTK + lane_off + c, u);
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 32; ++e) s[c + e] = __uint_as_float(u[e]);
      }
      tcgen05_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_free[st]);
      float mx = -INFINITY;
      const int k0 = (j0 + j) * kTK;
      if (softcap_log2 > 0.f) {  // uniform branch: soft-capped scores (Gemma-2)
        const float inv_cap = 1.f / softcap_log2;
#pragma unroll
        for (int c = 0; c < kTK; ++c) s[c] = softcap_log2 * tanh_approx(s[c] * scale_log2 * inv_cap);
      } else {
#pragma unroll
        for (int c = 0; c < kTK; ++c) s[c] *= scale_log2;
      }
      // visible keys of this row: [klo, khi] (causal, sequence end, sliding window)
      const int khi = min(qpos, kv_end - 1) - k0;
      const int klo = (window > 0 ? qpos - window + 1 : 0) - k0;
#pragma unroll
      for (int c = 0; c < kTK; ++c) {
        const float v = (c > khi || c < klo) ? -INFINITY : s[c];
        s[c] = v;
        mx = fmaxf(mx, v);
      }
      const float mnew = fmaxf(m, mx);
      const float ms = mnew == -INFINITY ? 0.f : mnew;
      const float corr = exp2f(m - ms);
      m = mnew;
      float psum = 0.f;
      uint32_t pk[kTK / 2];
#pragma unroll
      for (int c = 0; c < kTK; c += 2) {
        const float p0 = exp2f(s[c] - ms), p1 = exp2f(s[c + 1] - ms);
        psum += p0 + p1;
        pk[c >> 1] = pack_bf16x2(p0, p1);
      }
      l = l * corr + psum;
      if (j >= 1) {  // PV of the previous tile must finish before O is rescaled and P overwritten
        if (!waitq(pv_done, (j - 1) & 1, status, abort_flag)) {
          ok = false;
          break;
        }
        tcgen05_fence_after();
        if (__any_sync(0xffffffffu, corr != 1.f)) {
#pragma unroll
          for (int c = 0; c < kD; c += 32) {
            uint32_t u[32];
            tmem_ld_32x32b_x32(tO + lane_off + c, u);
            tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 32; ++e) u[e] = __float_as_uint(__uint_as_float(u[e]) * corr);
            tmem_st_32x32b_x32(tO + lane_off + c, u);
          }
          tmem_st_wait();
        }
      }
      // P row -> shared memory, K-major swizzled: chunk c (8 keys) of row r in slab c / 8
#pragma unroll
      for (int c = 0; c < kTK / 8; ++c) {
        uint8_t* dst = sP + (c >> 3) * (kPBytes / 2) + r * 128 + (((c & 7) ^ (r & 7)) << 4);
        *reinterpret_cast<uint4*>(dst) = make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
      }
      fence_proxy_async_smem();
      tcgen05_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
    }
    if (ok && nt > 0 && waitq(pv_done, (nt - 1) & 1, status, abort_flag)) {
      tcgen05_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      __nv_bfloat16* dst = out + (int64_t)(qs + q_off + r) * out_stride + h * kD;
#pragma unroll
      for (int c = 0; c < kD; c += 32) {
        uint32_t u[32];
        tmem_ld_32x32b_x32(tO + lane_off + c, u);
        tmem_ld_wait();
        if (r < rows) {
#pragma unroll
          for (int e = 0; e < 32; e += 8) {
            float f[8];
#pragma unroll
            for (int x = 0; x < 8; ++x) f[x] = __uint_as_float(u[e + x]) * inv;
            *reinterpret_cast<uint4*>(dst + c + e) = float_to_bf16x8(f);
          }
        }
      }
    }
  }
  tcgen05_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tcgen05_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace

namespace gollek {

void launch_paged_prefill_tc(void* out, int64_t out_stride, const void* q, int64_t q_rows, int64_t q_stride,
                             const void* cache, int num_blocks, const int* block_tables, int bt_stride,
                             const int* seq_lens, const int* query_start, const int* tiles, int ntiles, int H,
                             int Hk, float scale, int window, float softcap, cudaStream_t s) {
  throw_if(H % Hk != 0, "H must be a multiple of Hk");
  throw_if(q_stride % 8 != 0, "prefill: q row pitch must keep 16-byte alignment");
  if (ntiles == 0) return;
  const uint64_t kv_rows = (uint64_t)num_blocks * 2 * Hk * kBS;
  CUtensorMap tq = make_tmap_2d(q, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, q_rows, (uint64_t)H * kD, q_stride, kTQ, 64,
                                CU_TENSOR_MAP_SWIZZLE_128B);
  CUtensorMap tkv = make_tmap_2d(cache, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, kv_rows, kD, kD, kBS, 64,
                                 CU_TENSOR_MAP_SWIZZLE_128B);
  GOLLEK_CUDA_CHECK(cudaFuncSetAttribute(prefill_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem));
  dim3 grid(ntiles, H);
  prefill_tc_kernel<<<grid, kThreads, kSmem, s>>>(tq, tkv, reinterpret_cast<__nv_bfloat16*>(out), out_stride,
                                                  block_tables, bt_stride, seq_lens, query_start, tiles, H, Hk,
                                                  scale * 1.4426950408889634f, nullptr, window,
                                                  softcap > 0.f ? softcap * 1.4426950408889634f : 0.f);
  check_launch("paged_prefill_attention (tcgen05)");
}

}  // namespace gollek
