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

#include <cstdlib>

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
                      float softcap_log2, int num_blocks) {
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
          const int pb = checked_index((kb * kBS < kv_end) ? bt[kb] : bt[0], num_blocks, status);
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

// ---------------------------------------------------------------------------------------------
// Two-tile prefill kernel (the serving default for head_dim 128).
//
// One CTA = one work item = two 128-row query tiles ("slots") that read the same KV tiles: two query
// heads of one GQA group over the same rows (group size even), or two consecutive row tiles of one
// head. Head pairs share each K/V tile between two heads and are the host's default where the group
// size allows. The grid is one CTA per item, heaviest items first.
// 10 warps:
//   warps 0-3  softmax of slot 0, warps 4-7 softmax of slot 1 (one query row per thread = TMEM lane)
//   warp 8     TMA: both Q tiles once, then K and V of each 128-key tile (16-token paged boxes) into a
//              2-stage ring with separate K / V barriers (S can start before V lands)
//   warp 9     MMA (one thread): per KV tile j the tensor pipe runs PV0(j-1), S0(j), PV1(j-1), S1(j),
//              so slot 1's softmax overlaps PV0/S0 and slot 0's overlaps PV1/S1
// TMEM (512 columns): S0 | S1 | O0 | O1. P (bf16) is written back over the first 64 columns of its
// S buffer and is the TMEM A operand of the PV MMA; tcgen05.mma ops of one thread run in issue
// order, so PV_i(j-1) has read P_i before S_i(j) overwrites it.
// Online softmax in the log2 domain keeps a running max that is only raised when a tile's max exceeds
// it by more than 8 (P <= 2^8 stays exact enough in bf16), so O is rescaled in TMEM only on those
// rare tiles; s_full_i(j) is committed after PV_i(j-1) was issued, so O_i is quiescent while the
// softmax of tile j runs. Tiles that need no mask (below the causal diagonal, inside the sequence
// and the window) skip the mask, and EMU > 0 evaluates a share of the exponentials with a cubic
// on the FMA pipe instead of MUFU (EMU 1: every 4th column, 2: every 2nd).
// ---------------------------------------------------------------------------------------------
constexpr int kFaThreads = 320;
constexpr int fa_smem(int hd) { return 1024 + 2 * kTQ * hd * 2 + kStages * 2 * kTK * hd * 2 + 256; }

GOLLEK_DEVICE float ex2_mufu(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// 2^x on the FMA pipe: x = n + f with n = round(x) (the 1.5 * 2^23 shifter), |f| <= 1/2, 2^f by a
// cubic fitted to 2^f on [-1/2, 1/2] (relative error 7.5e-5, below bf16's 2^-8), 2^n added to the
// exponent field. x is clamped to -125 so the result stays a normal float.
GOLLEK_DEVICE float ex2_poly(float x) {
  x = fmaxf(x, -125.f);
  const float t = x + 12582912.f;
  const float f = x - (t - 12582912.f);
  const float p = fmaf(fmaf(fmaf(0.05517150089144707f, f, 0.24261096119880676f), f, 0.6932609677314758f), f,
                       0.9999280571937561f);
  return __int_as_float(__float_as_int(p) + (__float_as_int(t) << 23));
}

GOLLEK_DEVICE void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                               uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

struct FaSlot {
  int h, q_off, rows, kv_end, a, b;  // KV tiles [a, b)
};

struct FaItem {
  int b, qs, ctx0, kh, jlo, jhi, kv_end;
  const int* bt;
  FaSlot sl[2];
};

// Item of round r0 / gridDim.x for this CTA: rounds alternate direction over the heaviest-first list
// (CTA c takes the c-th item of even rounds and the c-th from the end of odd ones), which evens out
// the per-CTA totals a plain round-robin skews towards the low CTAs. -1: none left.
GOLLEK_DEVICE int fa_snake(int r0, int nwork) {
  const int round = r0 / (int)gridDim.x;
  const int w = r0 + ((round & 1) ? (int)gridDim.x - 1 - (int)blockIdx.x : (int)blockIdx.x);
  return w < nwork ? w : -1;
}

// Work item w of the list: its sequence, slots (heads / row tiles) and KV tile range.
GOLLEK_DEVICE FaItem fa_item(const int4* __restrict__ work, int w, const int* __restrict__ seq_lens,
                             const int* __restrict__ query_start, const int* __restrict__ block_tables,
                             int bt_stride, int H, int Hk, int window) {
  FaItem it;
  const int4 wk = work[w];
  it.b = wk.x;
  const int pair_heads = wk.w >> 16, hbase = wk.w & 0xffff;
  it.qs = query_start[it.b];
  const int qlen = query_start[it.b + 1] - it.qs;
  const int L = seq_lens[it.b];
  it.ctx0 = L - qlen;
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    FaSlot& t = it.sl[i];
    t.h = pair_heads ? hbase + i : hbase;
    t.q_off = pair_heads ? wk.y : (i == 0 ? wk.y : wk.z);
    const bool valid = t.q_off >= 0 && t.q_off < qlen;
    t.rows = valid ? min(kTQ, qlen - t.q_off) : 0;
    t.kv_end = valid ? min(L, it.ctx0 + t.q_off + t.rows) : 0;
    t.a = (valid && window > 0) ? max(0, it.ctx0 + t.q_off - window + 1) / kTK : 0;
    t.b = valid ? (t.kv_end + kTK - 1) / kTK : 0;
    if (t.b <= t.a) t.a = t.b = 0;
  }
  it.kh = it.sl[0].h / (H / Hk);
  const bool v0 = it.sl[0].b > it.sl[0].a, v1 = it.sl[1].b > it.sl[1].a;
  it.jlo = (v0 && v1) ? min(it.sl[0].a, it.sl[1].a) : (v0 ? it.sl[0].a : it.sl[1].a);
  it.jhi = max(it.sl[0].b, it.sl[1].b);
  it.kv_end = max(it.sl[0].kv_end, it.sl[1].kv_end);
  it.bt = block_tables + (int64_t)it.b * bt_stride;
  return it;
}

// Persistent: each CTA runs one item per round of gridDim.x items (fa_snake order; the list is sorted
// heaviest first). Across
// items the KV ring, the S / P barriers and the Q buffer keep running counters, so the next item's Q
// and first KV tiles load, and its first S MMAs run, while the softmax warps still normalise and store
// the previous item's O: q_empty (committed after an item's last S MMA) frees the Q buffer, o_free[i]
// (the slot's four softmax warps, after reading O_i) lets the next item's first PV overwrite O_i.
template <int EMU, int HD>
__global__ void __launch_bounds__(kFaThreads, 1)
    prefill_fa_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmKV,
                      __nv_bfloat16* __restrict__ out, int64_t out_stride, const int* __restrict__ block_tables,
                      int bt_stride, const int* __restrict__ seq_lens, const int* __restrict__ query_start,
                      const int4* __restrict__ work, int nwork, int H, int Hk, float scale_log2,
                      uint32_t* status, int window, float softcap_log2, int num_blocks) {
  // head size HD (64 or 128): Q / K / V tiles are HD / 64 boxes of 64 dims (128-byte swizzle), each
  // box 128 rows x 128 bytes
  constexpr int QB = kTQ * HD * 2, KVT = kTK * HD * 2, NBOX = HD / 64;
  constexpr int BOXQ = kTQ * 64 * 2, BOXK = kTK * 64 * 2;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint8_t* sQ = smem;                          // slot i at + i * QB
  uint8_t* sKV = sQ + 2 * QB;             // stage s: K at + s*2*tile, V at + s*2*tile + tile
  uint64_t* bars = reinterpret_cast<uint64_t*>(sKV + kStages * 2 * KVT);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;                 // [2]
  uint64_t* v_full = bars + 3;                 // [2]
  uint64_t* kv_empty = bars + 5;               // [2]
  uint64_t* s_full = bars + 7;                 // [slot]
  uint64_t* p_full = bars + 9;                 // [slot]
  uint64_t* o_done = bars + 11;                // [slot]
  uint64_t* done_bar = bars + 13;
  uint64_t* q_empty = bars + 14;
  uint64_t* o_free = bars + 15;                // [slot]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 17);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 4);
      mbar_init(&o_done[i], 1);
      mbar_init(&o_free[i], 4);
    }
    mbar_init(done_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 9) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tcgen05_fence_before();
  __syncthreads();
  tcgen05_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 8) {
    if (elect_one()) {
      prefetch_tmap(&tmQ);
      prefetch_tmap(&tmKV);
      int g = 0, nq = 0;  // KV tiles and Q loads issued so far
      bool ok = true;
      for (int r0 = 0; r0 < nwork && ok; r0 += gridDim.x) {
        const int w = fa_snake(r0, nwork);
        if (w < 0) continue;
        const FaItem it = fa_item(work, w, seq_lens, query_start, block_tables, bt_stride, H, Hk, window);
        if (it.jhi <= it.jlo) continue;
        // the previous item's S MMAs have read its Q tiles
        if (nq > 0 && !waitq(q_empty, (nq - 1) & 1, status, abort_flag)) {
          ok = false;
          break;
        }
        const bool v0 = it.sl[0].b > it.sl[0].a, v1 = it.sl[1].b > it.sl[1].a;
        mbar_arrive_expect_tx(q_full, ((v0 ? 1 : 0) + (v1 ? 1 : 0)) * QB);
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          if (it.sl[i].b > it.sl[i].a) {
            const int qrow = it.qs + it.sl[i].q_off;
#pragma unroll
            for (int bx = 0; bx < NBOX; ++bx)
              tma_load_2d(sQ + i * QB + bx * BOXQ, &tmQ, it.sl[i].h * HD + 64 * bx, qrow, q_full);
          }
        }
        ++nq;
        for (int j = it.jlo; j < it.jhi; ++j, ++g) {
          const int st = g & 1;
          if (!waitq(&kv_empty[st], ((g >> 1) & 1) ^ 1, status, abort_flag)) {
            ok = false;
            break;
          }
          uint8_t* dk = sKV + st * 2 * KVT;
          uint8_t* dv = dk + KVT;
          mbar_arrive_expect_tx(&k_full[st], KVT);
          for (int blk = 0; blk < kTK / kBS; ++blk) {
            const int kb = (j * kTK) / kBS + blk;
            const int pb = checked_index((kb * kBS < it.kv_end) ? it.bt[kb] : it.bt[0], num_blocks, status);
            const int rk = ((pb * 2 + 0) * Hk + it.kh) * kBS;
#pragma unroll
            for (int bx = 0; bx < NBOX; ++bx) tma_load_2d(dk + bx * BOXK + blk * 2048, &tmKV, 64 * bx, rk, &k_full[st]);
          }
          mbar_arrive_expect_tx(&v_full[st], KVT);
          for (int blk = 0; blk < kTK / kBS; ++blk) {
            const int kb = (j * kTK) / kBS + blk;
            const int pb = checked_index((kb * kBS < it.kv_end) ? it.bt[kb] : it.bt[0], num_blocks, status);
            const int rv = ((pb * 2 + 1) * Hk + it.kh) * kBS;
#pragma unroll
            for (int bx = 0; bx < NBOX; ++bx) tma_load_2d(dv + bx * BOXK + blk * 2048, &tmKV, 64 * bx, rv, &v_full[st]);
          }
        }
      }
      if (!ok) {  // copies still in flight land before the CTA leaves
        if (nq > 0) drainq(q_full, (nq - 1) & 1);
        for (int x = max(0, g - 2); x < g; ++x) {
          drainq(&k_full[x & 1], (x >> 1) & 1);
          drainq(&v_full[x & 1], (x >> 1) & 1);
        }
      }
    }
  } else if (warp == 9) {
    if (elect_one()) {
      constexpr uint32_t idesc_s = make_idesc_bf16(kTQ, kTK);              // Q K^T, both K-major
      constexpr uint32_t idesc_o = make_idesc_bf16(kTQ, HD) | (1u << 16);  // P (TMEM) V, V MN-major
      int g = 0, nq = 0;
      int np[2] = {0, 0};  // P tiles consumed per slot
      int no[2] = {0, 0};  // items finished per slot (O handed to the epilogue)
      bool ok = true;
      for (int r0 = 0; r0 < nwork && ok; r0 += gridDim.x) {
        const int w = fa_snake(r0, nwork);
        if (w < 0) continue;
        const FaItem it = fa_item(work, w, seq_lens, query_start, block_tables, bt_stride, H, Hk, window);
        if (it.jhi <= it.jlo) continue;
        if (!waitq(q_full, nq & 1, status, abort_flag)) {
          ok = false;
          break;
        }
        for (int j = it.jlo; j <= it.jhi && ok; ++j) {
          const int gi = g + (j - it.jlo);
          const bool prev = j > it.jlo, cur = j < it.jhi;
          if (prev && !waitq(&v_full[(gi - 1) & 1], ((gi - 1) >> 1) & 1, status, abort_flag)) {
            ok = false;
            break;
          }
          bool k_ready = false;
          tcgen05_fence_after();
#pragma unroll
          for (int i = 0; i < 2; ++i) {
            const FaSlot& t = it.sl[i];
            const uint32_t tS = tmem + i * kTK, tO = tmem + 256 + i * HD;
            if (prev && j - 1 >= t.a && j - 1 < t.b) {
              if (!waitq(&p_full[i], np[i] & 1, status, abort_flag)) {
                ok = false;
                break;
              }
              ++np[i];
              // the first PV of an item overwrites O_i: the previous item's epilogue must have read it
              if (j - 1 == t.a && no[i] > 0 && !waitq(&o_free[i], (no[i] - 1) & 1, status, abort_flag)) {
                ok = false;
                break;
              }
              tcgen05_fence_after();
              const uint32_t v_addr = smem_u32(sKV + ((gi - 1) & 1) * 2 * KVT + KVT);
#pragma unroll
              for (int ks = 0; ks < kTK / 16; ++ks)
                umma_f16_ts(tO, tS + ks * 8, make_desc_mn_sw128(v_addr + ks * 2048, BOXK), idesc_o,
                            (j - 1 > t.a || ks > 0) ? 1u : 0u);
              if (j == t.b) {
                umma_commit(&o_done[i]);
                ++no[i];
              }
            }
            if (cur && j >= t.a && j < t.b) {
              if (!k_ready) {
                if (!waitq(&k_full[gi & 1], (gi >> 1) & 1, status, abort_flag)) {
                  ok = false;
                  break;
                }
                tcgen05_fence_after();
                k_ready = true;
              }
              const uint32_t q_addr = smem_u32(sQ + i * QB);
              const uint32_t k_addr = smem_u32(sKV + (gi & 1) * 2 * KVT);
#pragma unroll
              for (int ks = 0; ks < HD / 16; ++ks) {
                const uint64_t a = make_smem_desc_sw128(q_addr + (ks >> 2) * (BOXQ) + (ks & 3) * 32);
                const uint64_t bd = make_smem_desc_sw128(k_addr + (ks >> 2) * (BOXK) + (ks & 3) * 32);
                umma_f16_ss(tS, a, bd, idesc_s, ks > 0 ? 1u : 0u);
              }
              umma_commit(&s_full[i]);
            }
          }
          if (prev && ok) umma_commit(&kv_empty[(gi - 1) & 1]);
          if (j == it.jhi - 1 && ok) umma_commit(q_empty);  // the item's last S MMAs read Q
        }
        g += it.jhi - it.jlo;
        ++nq;
      }
      if (!ok) {
        umma_commit(done_bar);
        drainq(done_bar, 0);
      }
    }
  } else {
    // softmax: slot i = warp / 4, TMEM lane quarter = warp & 3, query row r = quarter * 32 + lane.
    // Two passes over S in TMEM, 32 columns at a time (row max, then P): S is re-read instead of
    // held in registers, which keeps the unrolled code small (instruction-cache bound otherwise).
    const int i = warp >> 2, lg = warp & 3;
    const int r = lg * 32 + lane;
    const uint32_t lane_off = (uint32_t)(lg * 32) << 16;
    const uint32_t tS = tmem + i * kTK + lane_off, tO = tmem + 256 + i * HD + lane_off;
    const bool capped = softcap_log2 > 0.f;
    const float inv_cap = capped ? 1.f / softcap_log2 : 0.f;
    bool ok = true;
    int ns = 0, no = 0;  // S tiles and items of this slot so far
    for (int r0 = 0; r0 < nwork && ok; r0 += gridDim.x) {
        const int w = fa_snake(r0, nwork);
        if (w < 0) continue;
      const FaItem it = fa_item(work, w, seq_lens, query_start, block_tables, bt_stride, H, Hk, window);
      const FaSlot t = i == 0 ? it.sl[0] : it.sl[1];
      if (it.jhi <= it.jlo || t.b <= t.a) continue;
      const int ctx0 = it.ctx0;
      const int qpos = ctx0 + t.q_off + r;
      const int qmin = ctx0 + t.q_off + lg * 32, qmax = qmin + 31;
      float m = -INFINITY, l = 0.f;
      int n = 0;
      for (int j = t.a; j < t.b; ++j, ++n) {
        if (!waitq(&s_full[i], ns & 1, status, abort_flag)) {
          ok = false;
          break;
        }
        ++ns;
        tcgen05_fence_after();
        const int k0 = j * kTK;
        // visible keys of row qpos: [qpos - window + 1, min(qpos, kv_end - 1)] - k0
        const bool need_mask = (k0 + kTK - 1 > qmin) || (k0 + kTK > t.kv_end) ||
                               (window > 0 && k0 < qmax - window + 1);
        const int khi = min(qpos, t.kv_end - 1) - k0;
        const int klo = (window > 0 ? qpos - window + 1 : 0) - k0;
        // pass 1: the four 32-column loads in flight at once, row max over 8 independent chains
        float mx;
        {
          uint32_t u[kTK];
#pragma unroll
          for (int c = 0; c < kTK; c += 32) tmem_ld_32x32b_x32(tS + c, u + c);
          tmem_ld_wait();
          float m8[8];
#pragma unroll
          for (int x = 0; x < 8; ++x) m8[x] = -INFINITY;
          if (need_mask) {
#pragma unroll
            for (int c = 0; c < kTK; ++c)
              m8[c & 7] = fmaxf(m8[c & 7], (c <= khi && c >= klo) ? __uint_as_float(u[c]) : -INFINITY);
          } else {
#pragma unroll
            for (int c = 0; c < kTK; ++c) m8[c & 7] = fmaxf(m8[c & 7], __uint_as_float(u[c]));
          }
          mx = fmaxf(fmaxf(fmaxf(m8[0], m8[1]), fmaxf(m8[2], m8[3])), fmaxf(fmaxf(m8[4], m8[5]), fmaxf(m8[6], m8[7])));
        }
        // running max in the scaled log2 domain (soft cap is monotonic: cap the raw max)
        const float mnew = mx == -INFINITY ? -INFINITY
                           : capped        ? softcap_log2 * tanh_approx(mx * scale_log2 * inv_cap)
                                           : mx * scale_log2;
        float corr = 1.f;
        if (n == 0) {
          m = mnew;
        } else if (mnew > m + 8.f) {
          corr = exp2f(m - mnew);
          m = mnew;
        }
        const float ms = m == -INFINITY ? 0.f : m;
        const int mode = capped ? 3 : need_mask ? 2 : (EMU > 0 ? 1 : 0);
        // pass 2: S re-read 32 columns at a time, the next chunk's load overlapping this chunk's math
        float ps[4] = {0.f, 0.f, 0.f, 0.f};
        auto p_chunk = [&](const uint32_t* u, int c0) {
          uint32_t pk[16];
          if (mode == 1) {  // full tile: a share of the exponentials on the FMA pipe
#pragma unroll
            for (int e = 0; e < 32; e += 2) {
              const float p0 = ex2_mufu(fmaf(__uint_as_float(u[e]), scale_log2, -ms));
              const float x1 = fmaf(__uint_as_float(u[e + 1]), scale_log2, -ms);
              const float p1 = (EMU == 2 || (e & 3) == 2) ? ex2_poly(x1) : ex2_mufu(x1);
              ps[(e >> 1) & 3] += p0 + p1;
              pk[e >> 1] = pack_bf16x2(p0, p1);
            }
          } else if (mode == 0) {
#pragma unroll
            for (int e = 0; e < 32; e += 2) {
              const float p0 = ex2_mufu(fmaf(__uint_as_float(u[e]), scale_log2, -ms));
              const float p1 = ex2_mufu(fmaf(__uint_as_float(u[e + 1]), scale_log2, -ms));
              ps[(e >> 1) & 3] += p0 + p1;
              pk[e >> 1] = pack_bf16x2(p0, p1);
            }
          } else {  // masked and / or soft-capped
#pragma unroll
            for (int e = 0; e < 32; e += 2) {
              float p[2];
#pragma unroll
              for (int x = 0; x < 2; ++x) {
                const int c = c0 + e + x;
                float v = __uint_as_float(u[e + x]);
                v = capped ? softcap_log2 * tanh_approx(v * scale_log2 * inv_cap) : v * scale_log2;
                p[x] = (c <= khi && c >= klo) ? ex2_mufu(v - ms) : 0.f;
              }
              ps[(e >> 1) & 3] += p[0] + p[1];
              pk[e >> 1] = pack_bf16x2(p[0], p[1]);
            }
          }
          tmem_st_32x32b_x16(tS + (c0 >> 1), pk);
        };
        {
          uint32_t ua[32], ub[32];
          tmem_ld_32x32b_x32(tS, ua);
          tmem_ld_wait();
#pragma unroll 1
          for (int c0 = 0; c0 < kTK; c0 += 64) {
            tmem_ld_32x32b_x32(tS + c0 + 32, ub);
            p_chunk(ua, c0);
            tmem_ld_wait();
            if (c0 + 64 < kTK) tmem_ld_32x32b_x32(tS + c0 + 64, ua);
            p_chunk(ub, c0 + 32);
            tmem_ld_wait();
          }
        }
        const float psum = (ps[0] + ps[1]) + (ps[2] + ps[3]);
        l = l * corr + psum;
        if (__any_sync(0xffffffffu, corr != 1.f)) {  // O_i is quiescent: PV_i(j-1) completed before S_i(j)
#pragma unroll 1
          for (int c = 0; c < HD; c += 32) {
            uint32_t u[32];
            tmem_ld_32x32b_x32(tO + c, u);
            tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 32; ++e) u[e] = __float_as_uint(__uint_as_float(u[e]) * corr);
            tmem_st_32x32b_x32(tO + c, u);
          }
        }
        tmem_st_wait();
        tcgen05_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[i]);
      }
      if (!ok || !waitq(&o_done[i], no & 1, status, abort_flag)) {
        ok = false;
        break;
      }
      ++no;
      tcgen05_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      __nv_bfloat16* dst = out + (int64_t)(it.qs + t.q_off + r) * out_stride + t.h * HD;
      uint32_t u[HD];
#pragma unroll
      for (int c = 0; c < HD; c += 32) tmem_ld_32x32b_x32(tO + c, u + c);
      tmem_ld_wait();
      // O_i is in registers: the next item's first PV may overwrite it
      tcgen05_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&o_free[i]);
      if (r < t.rows) {
#pragma unroll
        for (int e = 0; e < HD; e += 8) {
          float f[8];
#pragma unroll
          for (int x = 0; x < 8; ++x) f[x] = __uint_as_float(u[e + x]) * inv;
          *reinterpret_cast<uint4*>(dst + e) = float_to_bf16x8(f);
        }
      }
    }
  }
  tcgen05_fence_before();
  __syncthreads();
  if (warp == 9) {
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
                                                  scale * 1.4426950408889634f, bounds_status(), window,
                                                  softcap > 0.f ? softcap * 1.4426950408889634f : 0.f, num_blocks);
  check_launch("paged_prefill_attention (tcgen05)");
}


void launch_paged_prefill_fa(void* out, int64_t out_stride, const void* q, int64_t q_rows, int64_t q_stride,
                             const void* cache, int num_blocks, const int* block_tables, int bt_stride,
                             const int* seq_lens, const int* query_start, const int* work, int nwork, int H, int Hk,
                             float scale, int window, float softcap, int emu, cudaStream_t s, int head_dim) {
  throw_if(H % Hk != 0, "H must be a multiple of Hk");
  throw_if(q_stride % 8 != 0, "prefill: q row pitch must keep 16-byte alignment");
  throw_if(head_dim != 64 && head_dim != 128, "two-tile tcgen05 prefill: head_dim 64 or 128");
  if (nwork == 0) return;
  const uint64_t kv_rows = (uint64_t)num_blocks * 2 * Hk * kBS;
  CUtensorMap tq = make_tmap_2d(q, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, q_rows, (uint64_t)H * head_dim, q_stride, kTQ,
                                64, CU_TENSOR_MAP_SWIZZLE_128B);
  CUtensorMap tkv = make_tmap_2d(cache, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, kv_rows, head_dim, head_dim, kBS, 64,
                                 CU_TENSOR_MAP_SWIZZLE_128B);
  // one CTA per SM looping over the items; GOLLEK_PREFILL_PERSISTENT=0: one CTA per item
  const char* pe = getenv("GOLLEK_PREFILL_PERSISTENT");
  dim3 grid((pe && pe[0] == '0') ? nwork : std::min(nwork, num_sms()));
  const float sl2 = scale * 1.4426950408889634f, cap = softcap > 0.f ? softcap * 1.4426950408889634f : 0.f;
  auto* o = reinterpret_cast<__nv_bfloat16*>(out);
  auto* w4 = reinterpret_cast<const int4*>(work);
#define GOLLEK_FA_LAUNCH(E, HDV)                                                                                   \
  do {                                                                                                             \
    GOLLEK_CUDA_CHECK(cudaFuncSetAttribute(prefill_fa_kernel<E, HDV>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                                           fa_smem(HDV)));                                                         \
    prefill_fa_kernel<E, HDV><<<grid, kFaThreads, fa_smem(HDV), s>>>(tq, tkv, o, out_stride, block_tables,         \
                                                                     bt_stride, seq_lens, query_start, w4, nwork,  \
                                                                     H, Hk, sl2, bounds_status(), window, cap,     \
                                                                     num_blocks);                                  \
  } while (0)
  if (head_dim == 64) {
    if (emu == 2)
      GOLLEK_FA_LAUNCH(2, 64);
    else if (emu == 1)
      GOLLEK_FA_LAUNCH(1, 64);
    else
      GOLLEK_FA_LAUNCH(0, 64);
  } else {
    if (emu == 2)
      GOLLEK_FA_LAUNCH(2, 128);
    else if (emu == 1)
      GOLLEK_FA_LAUNCH(1, 128);
    else
      GOLLEK_FA_LAUNCH(0, 128);
  }
#undef GOLLEK_FA_LAUNCH
  check_launch("paged_prefill_attention (tcgen05, two-tile)");
}

}  // namespace gollek
