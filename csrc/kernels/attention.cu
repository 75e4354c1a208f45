// Paged attention over the block table (sm_100a).
//
//   K3 paged_decode_attention : one query token per sequence, GQA-packed (all G query heads
//       that share a KV head are served by one CTA, so each KV byte is read from HBM once),
//       flash-decoding split-KV with an fp32 combine pass when the batch is too small to fill
//       148 SMs. KV tiles are streamed with fully coalesced 16-byte loads (512 B per warp
//       instruction = two cache rows of one paged block).
//   K4 paged_prefill_attention : varlen causal attention of new query tokens over the paged
//       KV (prefix + chunk), FlashAttention-2 style tiling on the warp-level tensor-core path
//       (mma.sync m16n8k16 bf16 -> fp32), cp.async double-buffered K/V tiles gathered from
//       the block table into XOR-swizzled shared memory.
//
// Reference semantics: core/optimization/gollek-plugin-paged-attention/…/PagedAttentionCpuFallback.java:37-124
// (decode), runner/safetensor/gollek-safetensor-engine/…/attention/PagedAttentionVectorAPI.java:20-127
// (online softmax over blocks, GQA, causal). KV layout per layer: [blocks, 2, Hk, block_size, D].
#include "../common/common.cuh"
#include "launchers.h"

using namespace gollek;

namespace {

constexpr float kLog2e = 1.4426950408889634f;

// =============================================================================================
// K3: decode
// =============================================================================================
// Lane layout inside a warp for one paged block of BS tokens x D dims (bf16):
//   CH  = D / 8 16-byte chunks per token row, TPI = 32 / CH tokens per warp instruction,
//   NI  = BS / TPI instructions per block. Lane l owns chunk c = l % CH of tokens
//   t = i * TPI + l / CH (i = 0..NI-1), so every warp load reads TPI*D*2 = 512 contiguous bytes.
template <int D, int G, int BS>
struct DecodeCfg {
  static constexpr int CH = D / 8;
  static constexpr int TPI = 32 / CH;
  static constexpr int NI = BS / TPI;
  static_assert(32 % CH == 0 && BS % TPI == 0, "unsupported head_dim / block_size");
};

constexpr int kDecodeWarps = 4;

template <int D, int G, int BS>
__global__ void __launch_bounds__(kDecodeWarps * 32) paged_decode_kernel(
    __nv_bfloat16* __restrict__ out,            // [B, H, D]          (num_splits == 1)
    float* __restrict__ part_o,                 // [B, H, S, D]       (num_splits > 1)
    float* __restrict__ part_ml,                // [B, H, S, 2]
    const __nv_bfloat16* __restrict__ q,        // [B, H, D] rows at q_stride
    const __nv_bfloat16* __restrict__ cache,    // [NB, 2, Hk, BS, D]
    const int* __restrict__ block_tables, int bt_stride, const int* __restrict__ seq_lens, int Hk,
    int num_splits, float scale_log2, int64_t q_stride) {
  using C = DecodeCfg<D, G, BS>;
  const int b = blockIdx.x, kh = blockIdx.y, split = blockIdx.z;
  const int H = Hk * G;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c = lane % C::CH, tsub = lane / C::CH;
  const int L = seq_lens[b];
  const int nblocks = (L + BS - 1) / BS;
  const int per = (nblocks + num_splits - 1) / num_splits;
  const int blk_begin = split * per;
  const int blk_end = min(nblocks, blk_begin + per);

  // query chunk for this lane, pre-scaled into the log2 domain
  float qv[G][8];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const uint4 u = *reinterpret_cast<const uint4*>(q + (int64_t)b * q_stride + (kh * G + g) * D + c * 8);
    bf16x8_to_float(u, qv[g]);
#pragma unroll
    for (int e = 0; e < 8; ++e) qv[g][e] *= scale_log2;
  }
  float m[G], l[G], acc[G][8];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[g][e] = 0.f;
  }
  const int* bt = block_tables + (int64_t)b * bt_stride;
  const int64_t head_stride = (int64_t)BS * D;           // one (block, kv, head) tile
  for (int blk = blk_begin + warp; blk < blk_end; blk += kDecodeWarps) {
    const int64_t pb = bt[blk];
    const __nv_bfloat16* kbase = cache + ((pb * 2 + 0) * Hk + kh) * head_stride;
    const __nv_bfloat16* vbase = cache + ((pb * 2 + 1) * Hk + kh) * head_stride;
    uint4 kr[C::NI], vr[C::NI];
#pragma unroll
    for (int i = 0; i < C::NI; ++i) {
      const int t = i * C::TPI + tsub;
      kr[i] = __ldg(reinterpret_cast<const uint4*>(kbase + t * D + c * 8));
    }
#pragma unroll
    for (int i = 0; i < C::NI; ++i) {
      const int t = i * C::TPI + tsub;
      vr[i] = __ldg(reinterpret_cast<const uint4*>(vbase + t * D + c * 8));
    }
    // scores s[g][i] for token i*TPI + tsub
    float s[G][C::NI];
#pragma unroll
    for (int i = 0; i < C::NI; ++i) {
      float kf[8];
      bf16x8_to_float(kr[i], kf);
#pragma unroll
      for (int g = 0; g < G; ++g) {
        float d0 = 0.f;
#pragma unroll
        for (int e = 0; e < 8; ++e) d0 = fmaf(qv[g][e], kf[e], d0);
        s[g][i] = d0;
      }
    }
    // reduce over the CH lanes that hold one token row
#pragma unroll
    for (int o = C::CH / 2; o > 0; o >>= 1) {
#pragma unroll
      for (int g = 0; g < G; ++g)
#pragma unroll
        for (int i = 0; i < C::NI; ++i) s[g][i] += __shfl_xor_sync(0xffffffffu, s[g][i], o);
    }
    const int tok0 = blk * BS;
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float bm = -INFINITY;
#pragma unroll
      for (int i = 0; i < C::NI; ++i) {
        const bool valid = tok0 + i * C::TPI + tsub < L;
        s[g][i] = valid ? s[g][i] : -INFINITY;
        bm = fmaxf(bm, s[g][i]);
      }
#pragma unroll
      for (int o = 16; o >= C::CH; o >>= 1) bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, o));
      const float mn = fmaxf(m[g], bm);
      const float corr = exp2f(m[g] - mn);  // m = -inf initially -> 0
      m[g] = mn;
      l[g] *= corr;
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[g][e] *= corr;
#pragma unroll
      for (int i = 0; i < C::NI; ++i) {
        const float p = exp2f(s[g][i] - mn);  // masked tokens: exp2(-inf) = 0
        s[g][i] = p;
        l[g] += p;
      }
    }
#pragma unroll
    for (int i = 0; i < C::NI; ++i) {
      float vf[8];
      bf16x8_to_float(vr[i], vf);
      const bool valid = tok0 + i * C::TPI + tsub < L;
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float p = valid ? s[g][i] : 0.f;
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[g][e] = fmaf(p, valid ? vf[e] : 0.f, acc[g][e]);
      }
    }
  }
  // combine the lanes holding different token subsets (same chunk c)
#pragma unroll
  for (int g = 0; g < G; ++g) {
#pragma unroll
    for (int o = 16; o >= C::CH; o >>= 1) {
      l[g] += __shfl_xor_sync(0xffffffffu, l[g], o);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[g][e] += __shfl_xor_sync(0xffffffffu, acc[g][e], o);
    }
  }
  // cross-warp merge through shared memory
  __shared__ float sm_m[kDecodeWarps][G], sm_l[kDecodeWarps][G];
  __shared__ __align__(16) float sm_o[kDecodeWarps][G][D];
  if (lane < C::CH) {
#pragma unroll
    for (int g = 0; g < G; ++g) {
#pragma unroll
      for (int e = 0; e < 8; ++e) sm_o[warp][g][c * 8 + e] = acc[g][e];
    }
  }
  if (lane == 0) {
#pragma unroll
    for (int g = 0; g < G; ++g) {
      sm_m[warp][g] = m[g];
      sm_l[warp][g] = l[g];
    }
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < G * D; idx += blockDim.x) {
    const int g = idx / D, d = idx % D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kDecodeWarps; ++w) M = fmaxf(M, sm_m[w][g]);
    float Lsum = 0.f, O = 0.f;
#pragma unroll
    for (int w = 0; w < kDecodeWarps; ++w) {
      const float f = (sm_m[w][g] == -INFINITY) ? 0.f : exp2f(sm_m[w][g] - M);
      Lsum += sm_l[w][g] * f;
      O += sm_o[w][g][d] * f;
    }
    const int h = kh * G + g;
    if (num_splits == 1) {
      out[((int64_t)b * H + h) * D + d] = __float2bfloat16(Lsum > 0.f ? O / Lsum : 0.f);
    } else {
      const int64_t pi = ((int64_t)b * H + h) * num_splits + split;
      part_o[pi * D + d] = O;
      if (d == 0) {
        part_ml[pi * 2 + 0] = M;
        part_ml[pi * 2 + 1] = Lsum;
      }
    }
  }
}

// Combine split-KV partials: out = sum_s o_s 2^(m_s - M) / sum_s l_s 2^(m_s - M).
template <int D>
__global__ void decode_combine_kernel(__nv_bfloat16* __restrict__ out, const float* __restrict__ part_o,
                                      const float* __restrict__ part_ml, int num_splits) {
  const int bh = blockIdx.x;  // b * H + h
  const int d = threadIdx.x;
  const float* ml = part_ml + (int64_t)bh * num_splits * 2;
  float M = -INFINITY;
  for (int s = 0; s < num_splits; ++s) M = fmaxf(M, ml[2 * s]);
  float Lsum = 0.f, O = 0.f;
  for (int s = 0; s < num_splits; ++s) {
    const float ms = ml[2 * s];
    const float f = (ms == -INFINITY) ? 0.f : exp2f(ms - M);
    Lsum += ml[2 * s + 1] * f;
    if (d < D) O += part_o[((int64_t)bh * num_splits + s) * D + d] * f;
  }
  if (d < D) out[(int64_t)bh * D + d] = __float2bfloat16(Lsum > 0.f ? O / Lsum : 0.f);
}

// =============================================================================================
// K4: prefill (varlen, causal, paged KV), mma.sync m16n8k16
// =============================================================================================
constexpr int kPfBM = 64;   // query rows per CTA (4 warps x 16)
constexpr int kPfBN = 64;   // keys per iteration
constexpr int kPfThreads = 128;

GOLLEK_DEVICE void cp_async16(void* smem, const void* gmem, bool valid) {
  const uint32_t s = smem_u32(smem);
  const int n = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(s), "l"(gmem), "r"(n) : "memory");
}
GOLLEK_DEVICE void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
GOLLEK_DEVICE void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

GOLLEK_DEVICE void ldmatrix_x4(uint32_t* r, const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
GOLLEK_DEVICE void ldmatrix_x4_trans(uint32_t* r, const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
GOLLEK_DEVICE void mma_bf16_16816(float* d, const uint32_t* a, const uint32_t* b) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

// Swizzled offset (in elements) of 16-byte chunk `ch` of row `r` in a [rows][D] bf16 tile.
template <int D>
GOLLEK_DEVICE int swz(int r, int ch) {
  constexpr int CH = D / 8;
  return r * D + ((ch ^ (r & 7)) & (CH - 1)) * 8;
}

template <int D>
__global__ void __launch_bounds__(kPfThreads) paged_prefill_kernel(
    __nv_bfloat16* __restrict__ out, int64_t out_stride,      // [T, H*D]
    const __nv_bfloat16* __restrict__ q, int64_t q_stride,    // [T, H*D]
    const __nv_bfloat16* __restrict__ cache,                  // [NB, 2, Hk, BS, D]
    const int* __restrict__ block_tables, int bt_stride, const int* __restrict__ seq_lens,
    const int* __restrict__ query_start, const int* __restrict__ tiles,  // tiles[i] = (b, q_off)
    int H, int Hk, int BS, float scale_log2) {
  static_assert(D % 16 == 0 && D >= 32 && D <= 128, "head_dim");
  constexpr int KSTEPS = D / 16;  // k-steps over head dim for QK^T
  constexpr int DT = D / 8;       // n8 tiles over head dim for PV
  extern __shared__ __align__(128) uint8_t smem_raw[];
  __nv_bfloat16* sQ = reinterpret_cast<__nv_bfloat16*>(smem_raw);
  __nv_bfloat16* sK = sQ + kPfBM * D;        // 2 stages
  __nv_bfloat16* sV = sK + 2 * kPfBN * D;    // 2 stages

  const int b = tiles[2 * blockIdx.x], q_off = tiles[2 * blockIdx.x + 1];
  const int h = blockIdx.y;
  const int kh = h / (H / Hk);
  const int qs = query_start[b], qlen = query_start[b + 1] - qs;
  const int L = seq_lens[b];
  const int ctx0 = L - qlen;  // absolute position of query 0
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int rows = min(kPfBM, qlen - q_off);

  // ---- load Q tile
  for (int i = tid; i < kPfBM * (D / 8); i += kPfThreads) {
    const int r = i / (D / 8), ch = i % (D / 8);
    const bool v = r < rows;
    const __nv_bfloat16* src = q + (int64_t)(qs + q_off + (v ? r : 0)) * q_stride + h * D + ch * 8;
    cp_async16(sQ + swz<D>(r, ch), src, v);
  }
  const int last_q_pos = ctx0 + q_off + rows - 1;
  const int kv_end = min(L, last_q_pos + 1);
  const int n_tiles = (kv_end + kPfBN - 1) / kPfBN;
  const int* bt = block_tables + (int64_t)b * bt_stride;
  const int64_t head_stride = (int64_t)BS * D;

  auto load_kv = [&](int tile, int stage) {
    __nv_bfloat16* dK = sK + stage * kPfBN * D;
    __nv_bfloat16* dV = sV + stage * kPfBN * D;
    for (int i = tid; i < kPfBN * (D / 8); i += kPfThreads) {
      const int r = i / (D / 8), ch = i % (D / 8);
      const int kpos = tile * kPfBN + r;
      const bool v = kpos < kv_end;
      const int64_t pb = v ? bt[kpos / BS] : 0;
      const int off = kpos % BS;
      const __nv_bfloat16* ks = cache + ((pb * 2 + 0) * Hk + kh) * head_stride + off * D + ch * 8;
      const __nv_bfloat16* vs = cache + ((pb * 2 + 1) * Hk + kh) * head_stride + off * D + ch * 8;
      cp_async16(dK + swz<D>(r, ch), ks, v);
      cp_async16(dV + swz<D>(r, ch), vs, v);
    }
  };
  if (n_tiles > 0) load_kv(0, 0);
  cp_async_commit();

  // ---- per-warp state: 16 query rows
  float o[DT][4];
#pragma unroll
  for (int j = 0; j < DT; ++j)
#pragma unroll
    for (int e = 0; e < 4; ++e) o[j][e] = 0.f;
  float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};
  uint32_t qf[KSTEPS][4];
  const int r_lo = warp * 16 + (lane >> 2);  // rows held by this thread: r_lo, r_lo + 8
  const int qpos_lo = ctx0 + q_off + r_lo, qpos_hi = qpos_lo + 8;

  for (int t = 0; t < n_tiles; ++t) {
    if (t + 1 < n_tiles) load_kv(t + 1, (t + 1) & 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    if (t == 0) {
#pragma unroll
      for (int ks = 0; ks < KSTEPS; ++ks) {
        const int mi = lane >> 3, rr = lane & 7;
        const int row = warp * 16 + (mi & 1) * 8 + rr;
        const int ch = ks * 2 + (mi >> 1);
        ldmatrix_x4(qf[ks], sQ + swz<D>(row, ch));
      }
    }
    const __nv_bfloat16* cK = sK + (t & 1) * kPfBN * D;
    const __nv_bfloat16* cV = sV + (t & 1) * kPfBN * D;
    // S = Q K^T : 16 x 64 per warp (8 n-tiles)
    float s[kPfBN / 8][4];
#pragma unroll
    for (int j = 0; j < kPfBN / 8; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) s[j][e] = 0.f;
#pragma unroll
    for (int ks = 0; ks < KSTEPS; ++ks) {
#pragma unroll
      for (int jp = 0; jp < kPfBN / 16; ++jp) {
        uint32_t bfr[4];
        const int mi = lane >> 3, rr = lane & 7;
        const int key = jp * 16 + (mi >> 1) * 8 + rr;
        const int ch = ks * 2 + (mi & 1);
        ldmatrix_x4(bfr, cK + swz<D>(key, ch));
        mma_bf16_16816(s[2 * jp], qf[ks], bfr);
        mma_bf16_16816(s[2 * jp + 1], qf[ks], bfr + 2);
      }
    }
    // mask + online softmax (log2 domain)
    const int kbase = t * kPfBN;
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int j = 0; j < kPfBN / 8; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int kp = kbase + j * 8 + 2 * (lane & 3) + (e & 1);
        const int qp = (e < 2) ? qpos_lo : qpos_hi;
        float v = s[j][e] * scale_log2;
        v = (kp > qp || kp >= kv_end) ? -INFINITY : v;
        s[j][e] = v;
        mx[e >> 1] = fmaxf(mx[e >> 1], v);
      }
    }
#pragma unroll
    for (int hrow = 0; hrow < 2; ++hrow) {
      mx[hrow] = fmaxf(mx[hrow], __shfl_xor_sync(0xffffffffu, mx[hrow], 1));
      mx[hrow] = fmaxf(mx[hrow], __shfl_xor_sync(0xffffffffu, mx[hrow], 2));
    }
    float corr[2], mnew[2];
#pragma unroll
    for (int hrow = 0; hrow < 2; ++hrow) {
      mnew[hrow] = fmaxf(mrow[hrow], mx[hrow]);
      const float ms = mnew[hrow] == -INFINITY ? 0.f : mnew[hrow];
      corr[hrow] = exp2f(mrow[hrow] - ms);
      mrow[hrow] = mnew[hrow];
      mnew[hrow] = ms;
      lrow[hrow] *= corr[hrow];
    }
#pragma unroll
    for (int j = 0; j < DT; ++j) {
      o[j][0] *= corr[0];
      o[j][1] *= corr[0];
      o[j][2] *= corr[1];
      o[j][3] *= corr[1];
    }
    uint32_t pf[kPfBN / 16][4];
#pragma unroll
    for (int j = 0; j < kPfBN / 8; ++j) {
      const float p0 = exp2f(s[j][0] - mnew[0]), p1 = exp2f(s[j][1] - mnew[0]);
      const float p2 = exp2f(s[j][2] - mnew[1]), p3 = exp2f(s[j][3] - mnew[1]);
      lrow[0] += p0 + p1;
      lrow[1] += p2 + p3;
      pf[j >> 1][(j & 1) * 2 + 0] = pack_bf16x2(p0, p1);
      pf[j >> 1][(j & 1) * 2 + 1] = pack_bf16x2(p2, p3);
    }
    // O += P V
#pragma unroll
    for (int kk = 0; kk < kPfBN / 16; ++kk) {
#pragma unroll
      for (int jd = 0; jd < DT / 2; ++jd) {
        uint32_t bfr[4];
        const int mi = lane >> 3, rr = lane & 7;
        const int key = kk * 16 + (mi & 1) * 8 + rr;
        const int ch = jd * 2 + (mi >> 1);
        ldmatrix_x4_trans(bfr, cV + swz<D>(key, ch));
        mma_bf16_16816(o[2 * jd], pf[kk], bfr);
        mma_bf16_16816(o[2 * jd + 1], pf[kk], bfr + 2);
      }
    }
    __syncthreads();  // stage (t&1) may be overwritten by the next prefetch
  }
  cp_async_wait<0>();
  // finalize
#pragma unroll
  for (int hrow = 0; hrow < 2; ++hrow) {
    lrow[hrow] += __shfl_xor_sync(0xffffffffu, lrow[hrow], 1);
    lrow[hrow] += __shfl_xor_sync(0xffffffffu, lrow[hrow], 2);
  }
  const float inv0 = lrow[0] > 0.f ? 1.f / lrow[0] : 0.f;
  const float inv1 = lrow[1] > 0.f ? 1.f / lrow[1] : 0.f;
#pragma unroll
  for (int j = 0; j < DT; ++j) {
    const int d = j * 8 + 2 * (lane & 3);
    if (r_lo < rows) {
      __nv_bfloat16* dst = out + (int64_t)(qs + q_off + r_lo) * out_stride + h * D + d;
      *reinterpret_cast<uint32_t*>(dst) = pack_bf16x2(o[j][0] * inv0, o[j][1] * inv0);
    }
    if (r_lo + 8 < rows) {
      __nv_bfloat16* dst = out + (int64_t)(qs + q_off + r_lo + 8) * out_stride + h * D + d;
      *reinterpret_cast<uint32_t*>(dst) = pack_bf16x2(o[j][2] * inv1, o[j][3] * inv1);
    }
  }
}

template <int D, int G>
void launch_decode_t(void* out, const void* q, int64_t q_stride, const void* cache, const int* bt, int bt_stride,
                     const int* lens, int B, int Hk, int num_splits, float scale_log2, float* po, float* pml,
                     cudaStream_t s) {
  dim3 grid(B, Hk, num_splits);
  paged_decode_kernel<D, G, 16><<<grid, kDecodeWarps * 32, 0, s>>>(
      reinterpret_cast<__nv_bfloat16*>(out), po, pml, reinterpret_cast<const __nv_bfloat16*>(q),
      reinterpret_cast<const __nv_bfloat16*>(cache), bt, bt_stride, lens, Hk, num_splits, scale_log2, q_stride);
  check_launch("paged_decode_attention");
  if (num_splits > 1) {
    decode_combine_kernel<D><<<B * Hk * G, D, 0, s>>>(reinterpret_cast<__nv_bfloat16*>(out), po, pml, num_splits);
    check_launch("paged_decode_attention combine");
  }
}

}  // namespace

namespace gollek {

void launch_paged_decode(void* out, const void* q, int64_t q_stride, const void* cache, const int* block_tables,
                         int bt_stride, const int* seq_lens, int B, int H, int Hk, int D, int block_size,
                         int num_splits, float scale, float* part_o, float* part_ml, cudaStream_t s) {
  throw_if(block_size != 16, "decode attention is built for block_size 16");
  throw_if(H % Hk != 0, "H must be a multiple of Hk");
  throw_if(num_splits > 1 && (part_o == nullptr || part_ml == nullptr), "split-KV decode needs a workspace");
  if (B == 0) return;
  const int G = H / Hk;
  const float sl = scale * kLog2e;
#define GOLLEK_DECODE_CASE(DD, GG)                                                                            \
  if (D == DD && G == GG)                                                                                     \
    return launch_decode_t<DD, GG>(out, q, q_stride, cache, block_tables, bt_stride, seq_lens, B, Hk, num_splits, \
                                   sl, part_o, part_ml, s);
  GOLLEK_DECODE_CASE(128, 1)
  GOLLEK_DECODE_CASE(128, 2)
  GOLLEK_DECODE_CASE(128, 4)
  GOLLEK_DECODE_CASE(128, 8)
  GOLLEK_DECODE_CASE(64, 1)
  GOLLEK_DECODE_CASE(64, 4)
  GOLLEK_DECODE_CASE(64, 8)
  GOLLEK_DECODE_CASE(32, 1)
  GOLLEK_DECODE_CASE(32, 2)
  GOLLEK_DECODE_CASE(32, 4)
  GOLLEK_DECODE_CASE(32, 8)
#undef GOLLEK_DECODE_CASE
  throw_if(true, "decode attention: unsupported head_dim/group " + std::to_string(D) + "/" + std::to_string(G));
}

void launch_paged_prefill(void* out, int64_t out_stride, const void* q, int64_t q_stride, const void* cache,
                          const int* block_tables, int bt_stride, const int* seq_lens, const int* query_start,
                          const int* tiles, int ntiles, int H, int Hk, int D, int block_size, float scale,
                          cudaStream_t s) {
  throw_if(H % Hk != 0, "H must be a multiple of Hk");
  if (ntiles == 0) return;
  const float sl = scale * kLog2e;
  dim3 grid(ntiles, H);
#define GOLLEK_PREFILL_CASE(DD)                                                                               \
  if (D == DD) {                                                                                            \
    const size_t smem = (size_t)(kPfBM + 4 * kPfBN) * DD * 2;                                              \
    auto kern = paged_prefill_kernel<DD>;                                                                   \
    GOLLEK_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));  \
    kern<<<grid, kPfThreads, smem, s>>>(reinterpret_cast<__nv_bfloat16*>(out), out_stride,                  \
                                        reinterpret_cast<const __nv_bfloat16*>(q), q_stride,                \
                                        reinterpret_cast<const __nv_bfloat16*>(cache), block_tables,        \
                                        bt_stride, seq_lens, query_start, tiles, H, Hk, block_size, sl);    \
    check_launch("paged_prefill_attention");                                                                \
    return;                                                                                                 \
  }
  GOLLEK_PREFILL_CASE(128)
  GOLLEK_PREFILL_CASE(64)
  GOLLEK_PREFILL_CASE(32)
#undef GOLLEK_PREFILL_CASE
  throw_if(true, "prefill attention: unsupported head_dim " + std::to_string(D));
}

}  // namespace gollek
