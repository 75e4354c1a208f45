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
#include "../common/tma_host.h"
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
constexpr int kDecodeStages = 3;  // per-warp ring depth (blocks in flight per warp)

// Bounded wait for the per-warp ring barriers (no legitimate wait comes near the limit).
GOLLEK_DEVICE bool ring_wait(uint64_t* bar, uint32_t parity, uint32_t* status) {
  for (uint32_t i = 0; i < (1u << 24); ++i)
    if (mbar_try_wait(bar, parity)) return true;
  report_status(status, kStatusMbarTimeout);
  return false;
}

// Each warp owns a kDecodeStages-deep shared-memory ring; its lane 0 streams the warp's paged
// blocks (K tile and V tile, BS*D bf16 each, contiguous in the cache) with cp.async.bulk and the
// whole warp consumes them. Warps take blocks blk_begin + warp, + 4, ... of this CTA's split.
template <int D, int G, int BS>
__global__ void __launch_bounds__(kDecodeWarps * 32) paged_decode_kernel(
    __nv_bfloat16* __restrict__ out,            // [B, H, D]          (num_splits == 1)
    float* __restrict__ part_o,                 // [B, H, S, D]       (num_splits > 1)
    float* __restrict__ part_ml,                // [B, H, S, 2]
    const __nv_bfloat16* __restrict__ q,        // [B, H, D] rows at q_stride
    const __nv_bfloat16* __restrict__ cache,    // [NB, 2, Hk, BS, D]
    const int* __restrict__ block_tables, int bt_stride, const int* __restrict__ seq_lens, int Hk,
    int num_splits, float scale_log2, int64_t q_stride, uint32_t* status, int window, float softcap_log2,
    int num_blocks) {
  using C = DecodeCfg<D, G, BS>;
  constexpr int TILE = BS * D;                         // elements of one K (or V) tile
  constexpr uint32_t TILE_BYTES = TILE * 2;
  extern __shared__ __align__(128) uint8_t dsmem[];
  const int b = blockIdx.x, kh = blockIdx.y, split = blockIdx.z;
  const int H = Hk * G;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c = lane % C::CH, tsub = lane / C::CH;
  __nv_bfloat16* ring = reinterpret_cast<__nv_bfloat16*>(dsmem) + (size_t)warp * kDecodeStages * 2 * TILE;
  uint64_t* bars = reinterpret_cast<uint64_t*>(dsmem + (size_t)kDecodeWarps * kDecodeStages * 2 * TILE_BYTES) +
                   warp * kDecodeStages;
  float* sm_o = reinterpret_cast<float*>(bars - warp * kDecodeStages + kDecodeWarps * kDecodeStages);
  float* sm_m = sm_o + kDecodeWarps * G * D;
  float* sm_l = sm_m + kDecodeWarps * G;

  const int L = seq_lens[b];
  const int nblocks = (L + BS - 1) / BS;
  // sliding window: the query at position L-1 sees keys [L - window, L); earlier blocks are skipped
  const int kv_lo = window > 0 ? max(0, L - window) : 0;
  const int blk_lo = kv_lo / BS;
  const int per = (nblocks - blk_lo + num_splits - 1) / num_splits;
  const int blk_begin = blk_lo + split * per;
  const int blk_end = min(nblocks, blk_begin + per);
  const int nmine = blk_begin + warp < blk_end ? (blk_end - blk_begin - warp + kDecodeWarps - 1) / kDecodeWarps : 0;
  const int* bt = block_tables + (int64_t)b * bt_stride;

  if (lane == 0) {
    for (int st = 0; st < kDecodeStages; ++st) mbar_init(&bars[st], 1);
    fence_mbar_init();
  }
  __syncwarp();
  auto issue = [&](int j) {  // lane 0 only
    const int st = j % kDecodeStages;
    const int64_t pb = checked_index(bt[blk_begin + warp + kDecodeWarps * j], num_blocks, status);
    const __nv_bfloat16* kb = cache + ((pb * 2 + 0) * Hk + kh) * (int64_t)TILE;
    const __nv_bfloat16* vb = cache + ((pb * 2 + 1) * Hk + kh) * (int64_t)TILE;
    mbar_arrive_expect_tx(&bars[st], 2 * TILE_BYTES);
    bulk_g2s(ring + st * 2 * TILE, kb, TILE_BYTES, &bars[st]);
    bulk_g2s(ring + st * 2 * TILE + TILE, vb, TILE_BYTES, &bars[st]);
  };
  int issued = 0;
  if (lane == 0) {
    for (; issued < min(kDecodeStages, nmine); ++issued) issue(issued);
  }

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
  bool ok = true;
  int j = 0;
  for (; j < nmine; ++j) {
    const int st = j % kDecodeStages;
    if (!ring_wait(&bars[st], (j / kDecodeStages) & 1, status)) {
      ok = false;
      break;
    }
    const __nv_bfloat16* kt = ring + st * 2 * TILE;
    const __nv_bfloat16* vt = kt + TILE;
    const int tok0 = (blk_begin + warp + kDecodeWarps * j) * BS;
    uint4 kr[C::NI];
#pragma unroll
    for (int i = 0; i < C::NI; ++i)
      kr[i] = *reinterpret_cast<const uint4*>(kt + (i * C::TPI + tsub) * D + c * 8);
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
#pragma unroll
    for (int o = C::CH / 2; o > 0; o >>= 1) {
#pragma unroll
      for (int g = 0; g < G; ++g)
#pragma unroll
        for (int i = 0; i < C::NI; ++i) s[g][i] += __shfl_xor_sync(0xffffffffu, s[g][i], o);
    }
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float bm = -INFINITY;
#pragma unroll
      for (int i = 0; i < C::NI; ++i) {
        const int tk = tok0 + i * C::TPI + tsub;
        const bool valid = tk < L && tk >= kv_lo;
        float v = s[g][i];
        if (softcap_log2 > 0.f) v = softcap_log2 * tanh_approx(v * (1.f / softcap_log2));
        s[g][i] = valid ? v : -INFINITY;
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
      bf16x8_to_float(*reinterpret_cast<const uint4*>(vt + (i * C::TPI + tsub) * D + c * 8), vf);
      const bool valid = tok0 + i * C::TPI + tsub < L && tok0 + i * C::TPI + tsub >= kv_lo;
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float p = valid ? s[g][i] : 0.f;
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[g][e] = fmaf(p, valid ? vf[e] : 0.f, acc[g][e]);
      }
    }
    __syncwarp();  // every lane has read stage st before it is refilled
    if (lane == 0 && issued < nmine) {
      fence_proxy_async_smem();
      issue(issued);
      ++issued;
    }
  }
  if (!ok && lane == 0) {
    // bounded drain of our own copies still in flight before the CTA may exit
    for (int jj = j; jj < issued; ++jj) ring_wait(&bars[jj % kDecodeStages], (jj / kDecodeStages) & 1, nullptr);
  }
  __syncwarp();
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
  if (lane < C::CH) {
#pragma unroll
    for (int g = 0; g < G; ++g) {
#pragma unroll
      for (int e = 0; e < 8; ++e) sm_o[(warp * G + g) * D + c * 8 + e] = acc[g][e];
    }
  }
  if (lane == 0) {
#pragma unroll
    for (int g = 0; g < G; ++g) {
      sm_m[warp * G + g] = m[g];
      sm_l[warp * G + g] = l[g];
    }
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < G * D; idx += blockDim.x) {
    const int g = idx / D, d = idx % D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kDecodeWarps; ++w) M = fmaxf(M, sm_m[w * G + g]);
    float Lsum = 0.f, O = 0.f;
#pragma unroll
    for (int w = 0; w < kDecodeWarps; ++w) {
      const float mw = sm_m[w * G + g];
      const float f = (mw == -INFINITY) ? 0.f : exp2f(mw - M);
      Lsum += sm_l[w * G + g] * f;
      O += sm_o[(w * G + g) * D + d] * f;
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

template <int D, int G, int BS>
constexpr size_t decode_smem_bytes() {
  return (size_t)kDecodeWarps * kDecodeStages * 2 * BS * D * 2 + kDecodeWarps * kDecodeStages * 8 +
         (size_t)kDecodeWarps * G * D * 4 + 2 * kDecodeWarps * G * 4;
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

GOLLEK_DEVICE void mma_f16_16816(float* d, const uint32_t* a, const uint32_t* b) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

GOLLEK_DEVICE uint32_t pack_f16x2(float a, float b) {
  const __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// four e4m3 values (one 32-bit word, element 0 in the low byte) -> two f16x2 words (exact: every
// e4m3 value is an f16 value)
GOLLEK_DEVICE void e4m3x4_to_f16x4(uint32_t w, uint32_t& lo, uint32_t& hi) {
  asm("{\n\t.reg .b16 l, h;\n\tmov.b32 {l, h}, %2;\n\tcvt.rn.f16x2.e4m3x2 %0, l;\n\tcvt.rn.f16x2.e4m3x2 %1, h;\n\t}"
      : "=r"(lo), "=r"(hi)
      : "r"(w));
}

GOLLEK_DEVICE uint32_t bf16x2_to_f16x2(uint32_t v) {
  const __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(&v);
  const float2 f = __bfloat1622float2(b);
  return pack_f16x2(f.x, f.y);
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
    int H, int Hk, int BS, float scale_log2, int window, float softcap_log2, int num_blocks, uint32_t* bounds) {
  static_assert(D % 16 == 0 && D >= 32 && D <= 256, "head_dim");
  // head_dim 256: the O accumulator alone takes 128 registers per thread, so Q fragments are
  // re-read from shared memory for every key tile instead of being held in registers
  constexpr bool kQRegs = D <= 128;
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
  // sliding window: the first query row sees keys >= ctx0 + q_off - window + 1; earlier tiles skipped
  const int t_lo = window > 0 ? max(0, ctx0 + q_off - window + 1) / kPfBN : 0;
  const int* bt = block_tables + (int64_t)b * bt_stride;
  const int64_t head_stride = (int64_t)BS * D;

  auto load_kv = [&](int tile, int stage) {
    __nv_bfloat16* dK = sK + stage * kPfBN * D;
    __nv_bfloat16* dV = sV + stage * kPfBN * D;
    for (int i = tid; i < kPfBN * (D / 8); i += kPfThreads) {
      const int r = i / (D / 8), ch = i % (D / 8);
      const int kpos = tile * kPfBN + r;
      const bool v = kpos < kv_end;
      const int64_t pb = v ? checked_index(bt[kpos / BS], num_blocks, bounds) : 0;
      const int off = kpos % BS;
      const __nv_bfloat16* ks = cache + ((pb * 2 + 0) * Hk + kh) * head_stride + off * D + ch * 8;
      const __nv_bfloat16* vs = cache + ((pb * 2 + 1) * Hk + kh) * head_stride + off * D + ch * 8;
      cp_async16(dK + swz<D>(r, ch), ks, v);
      cp_async16(dV + swz<D>(r, ch), vs, v);
    }
  };
  if (n_tiles > t_lo) load_kv(t_lo, t_lo & 1);
  cp_async_commit();

  // ---- per-warp state: 16 query rows
  float o[DT][4];
#pragma unroll
  for (int j = 0; j < DT; ++j)
#pragma unroll
    for (int e = 0; e < 4; ++e) o[j][e] = 0.f;
  float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};
  uint32_t qf[kQRegs ? KSTEPS : 1][4];
  const int r_lo = warp * 16 + (lane >> 2);  // rows held by this thread: r_lo, r_lo + 8
  const int qpos_lo = ctx0 + q_off + r_lo, qpos_hi = qpos_lo + 8;
  auto load_qf = [&](uint32_t* dst, int ks) {
    const int mi = lane >> 3, rr = lane & 7;
    const int row = warp * 16 + (mi & 1) * 8 + rr;
    const int ch = ks * 2 + (mi >> 1);
    ldmatrix_x4(dst, sQ + swz<D>(row, ch));
  };

  for (int t = t_lo; t < n_tiles; ++t) {
    if (t + 1 < n_tiles) load_kv(t + 1, (t + 1) & 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    if constexpr (kQRegs) {
      if (t == t_lo) {
#pragma unroll
        for (int ks = 0; ks < KSTEPS; ++ks) load_qf(qf[ks], ks);
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
      const uint32_t* qk;
      uint32_t qtmp[4];
      if constexpr (kQRegs) {
        qk = qf[ks];
      } else {
        load_qf(qtmp, ks);
        qk = qtmp;
      }
#pragma unroll
      for (int jp = 0; jp < kPfBN / 16; ++jp) {
        uint32_t bfr[4];
        const int mi = lane >> 3, rr = lane & 7;
        const int key = jp * 16 + (mi >> 1) * 8 + rr;
        const int ch = ks * 2 + (mi & 1);
        ldmatrix_x4(bfr, cK + swz<D>(key, ch));
        mma_bf16_16816(s[2 * jp], qk, bfr);
        mma_bf16_16816(s[2 * jp + 1], qk, bfr + 2);
      }
    }
    // mask + online softmax (log2 domain)
    const int kbase = t * kPfBN;
    float mx[2] = {-INFINITY, -INFINITY};
    if (softcap_log2 > 0.f) {  // uniform branch: soft-capped scores (Gemma-2)
      const float inv_cap = 1.f / softcap_log2;
#pragma unroll
      for (int j = 0; j < kPfBN / 8; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) s[j][e] = softcap_log2 * tanh_approx(s[j][e] * scale_log2 * inv_cap);
    } else {
#pragma unroll
      for (int j = 0; j < kPfBN / 8; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) s[j][e] *= scale_log2;
    }
    // visible keys per row: [lo, hi] (causal, sequence end, sliding window), relative to kbase
    const int hi0 = min(qpos_lo, kv_end - 1) - kbase, hi1 = min(qpos_hi, kv_end - 1) - kbase;
    const int lo0 = (window > 0 ? qpos_lo - window + 1 : 0) - kbase;
    const int lo1 = (window > 0 ? qpos_hi - window + 1 : 0) - kbase;
#pragma unroll
    for (int j = 0; j < kPfBN / 8; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int kp = j * 8 + 2 * (lane & 3) + (e & 1);
        const bool vis = (e < 2) ? (kp <= hi0 && kp >= lo0) : (kp <= hi1 && kp >= lo1);
        const float v = vis ? s[j][e] : -INFINITY;
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

// =============================================================================================
// K3 (tensor-core variant, head_dim 128): the G query heads of one KV group form the M = 16 rows
// of mma.sync m16n8k16 (rows >= G are zero), the 16 tokens of a paged block are N, so one block
// costs 32 MMAs per warp instead of ~1000 CUDA-core instructions. K/V tiles arrive by 2-D TMA
// (box 64 dims x 16 tokens, 128-byte swizzle, two boxes per tile) into a per-warp 3-stage ring;
// ldmatrix reads them conflict-free.
// =============================================================================================
constexpr int kTcStages = 3;
constexpr int kTcTileBytes = 16 * 128 * 2;            // one K (or V) tile of a paged block
constexpr int kTcStageBytes = 2 * kTcTileBytes;       // K + V
// fp8 KV cache (e4m3, a fp32 scale per token and head): the ring holds fp8 tiles (one 16 x 128
// byte TMA box each, 128-byte swizzle) and every lane converts its MMA fragments straight from
// them (cvt e4m3x2 -> f16x2, exact) for f16 MMAs, with no staging copy. Two fixed permutations
// make each lane's fragment bytes contiguous, so a fragment group is one 16-byte shared load:
//  * QK^T sums over dims, so any dim order shared by Q and K gives the same scores: logical
//    k-step s = 4q + u, lane column c, offsets {0,1,8,9} + 2c read physical dims
//    64q + 16c + 4u + {0,1,2,3} (Q is gathered in that order once, in registers);
//  * P V: logical output column 8 jn + r (n-tile jn, lane row r) is physical dim 16 r + jn, so a
//    lane reads bytes [16r, 16r + 16) of its four token rows and byte-permutes token pairs; the
//    output partials are written back through the same map.
// Scores are multiplied by the key scales, probabilities by the value scales (the softmax sum
// uses the unscaled ones).
constexpr int kTcFp8TileBytes = 16 * 128;

GOLLEK_DEVICE uint32_t sw128_off(int row, int chunk16) {  // byte offset inside a [rows][128 dims] bf16 tile
  const int box = chunk16 >> 3, cc = chunk16 & 7;
  return box * 2048 + row * 128 + ((cc ^ (row & 7)) << 4);
}

template <int G, bool FP8>
__global__ void __launch_bounds__(kDecodeWarps * 32, FP8 ? 4 : 1) paged_decode_tc_kernel(
    const __grid_constant__ CUtensorMap tmap,      // cache rows [NB*2*Hk*16, 128] bf16 (fp8: 128 bytes)
    __nv_bfloat16* __restrict__ out, float* __restrict__ part_o, float* __restrict__ part_ml,
    const __nv_bfloat16* __restrict__ q, const int* __restrict__ block_tables, int bt_stride,
    const int* __restrict__ seq_lens, int Hk, int num_splits, float scale_log2, int64_t q_stride,
    uint32_t* status, int window, float softcap_log2, const float* __restrict__ kv_scales, int num_blocks) {
  static_assert(G >= 1 && G <= 16, "GQA group must fit the 16 MMA rows");
  constexpr int D = 128, BS = 16;
  constexpr int kStage = FP8 ? 2 * kTcFp8TileBytes : kTcStageBytes;
  extern __shared__ uint8_t dsm_raw[];
  uint8_t* dsm = dsm_raw + ((1024 - (smem_u32(dsm_raw) & 1023)) & 1023);
  const int b = blockIdx.x, kh = blockIdx.y, split = blockIdx.z;
  const int H = Hk * G;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint8_t* ring = dsm + warp * kTcStages * kStage;
  // fp8: the stage's 16 key and 16 value scales arrive by bulk copy on the tiles' barrier
  constexpr int kScaleBytes = FP8 ? 2 * BS * 4 : 0;
  float* sring = reinterpret_cast<float*>(dsm + kDecodeWarps * kTcStages * kStage) + warp * kTcStages * (kScaleBytes / 4);
  constexpr int kAfter = kDecodeWarps * kTcStages * (kStage + kScaleBytes);
  uint64_t* bars = reinterpret_cast<uint64_t*>(dsm + kAfter) + warp * kTcStages;
  // a warp's output partials [G, D] fp32 go into its own ring once its loads are consumed
  static_assert(G * D * 4 <= kTcStages * kStage, "partials must fit a warp's ring");
  auto sm_o = [&](int w) { return reinterpret_cast<float*>(dsm + w * kTcStages * kStage); };
  float* sm_m = reinterpret_cast<float*>(dsm + kAfter + kDecodeWarps * kTcStages * 8);
  float* sm_l = sm_m + kDecodeWarps * G;

  const int L = seq_lens[b];
  const int nblocks = (L + BS - 1) / BS;
  // sliding window: the query at position L-1 sees keys [L - window, L); earlier blocks are skipped
  const int kv_lo = window > 0 ? max(0, L - window) : 0;
  const int blk_lo = kv_lo / BS;
  const int per = (nblocks - blk_lo + num_splits - 1) / num_splits;
  const int blk_begin = blk_lo + split * per;
  const int blk_end = min(nblocks, blk_begin + per);
  const int nmine = blk_begin + warp < blk_end ? (blk_end - blk_begin - warp + kDecodeWarps - 1) / kDecodeWarps : 0;
  const int* bt = block_tables + (int64_t)b * bt_stride;

  if (lane == 0) {
    prefetch_tmap(&tmap);
    for (int st = 0; st < kTcStages; ++st) mbar_init(&bars[st], 1);
    fence_mbar_init();
  }
  __syncwarp();
  auto issue = [&](int j) {  // lane 0 only
    const int st = j % kTcStages;
    const int pb = checked_index(bt[blk_begin + warp + kDecodeWarps * j], num_blocks, status);
    const int rk = ((pb * 2 + 0) * Hk + kh) * BS, rv = ((pb * 2 + 1) * Hk + kh) * BS;
    uint8_t* dst = ring + st * kStage;
    mbar_arrive_expect_tx(&bars[st], kStage + kScaleBytes);
    if constexpr (FP8) {
      tma_load_2d(dst, &tmap, 0, rk, &bars[st]);
      tma_load_2d(dst + kTcFp8TileBytes, &tmap, 0, rv, &bars[st]);
      float* sd = sring + st * (kScaleBytes / 4);
      bulk_g2s(sd, kv_scales + rk, BS * 4, &bars[st]);           // rows rk .. rk + 15: this block's key scales
      bulk_g2s(sd + BS, kv_scales + rv, BS * 4, &bars[st]);      // and value scales
    } else {
      tma_load_2d(dst, &tmap, 0, rk, &bars[st]);
      tma_load_2d(dst + 2048, &tmap, 64, rk, &bars[st]);
      tma_load_2d(dst + kTcTileBytes, &tmap, 0, rv, &bars[st]);
      tma_load_2d(dst + kTcTileBytes + 2048, &tmap, 64, rv, &bars[st]);
    }
  };
  int issued = 0;
  if (lane == 0)
    for (; issued < min(kTcStages, nmine); ++issued) issue(issued);

  // Q as the A operand: rows = heads of this group (zero beyond G), K = 128 dims (8 k-steps)
  const int r = lane >> 2, cq = (lane & 3) * 2;
  uint32_t qf[8][4];
#pragma unroll
  for (int ks = 0; ks < 8; ++ks) {
    // element offsets of the lane's two k-pairs: logical (2c, 2c + 8), or physical under the fp8 map
    const int d0 = FP8 ? 64 * (ks >> 2) + 16 * (lane & 3) + 4 * (ks & 3) : ks * 16 + cq;
    const int d1 = FP8 ? d0 + 2 : d0 + 8;
    const __nv_bfloat16* q0 = q + (int64_t)b * q_stride + (int64_t)(kh * G) * D;
    qf[ks][0] = r < G ? *reinterpret_cast<const uint32_t*>(q0 + r * D + d0) : 0u;
    qf[ks][1] = r + 8 < G ? *reinterpret_cast<const uint32_t*>(q0 + (r + 8) * D + d0) : 0u;
    qf[ks][2] = r < G ? *reinterpret_cast<const uint32_t*>(q0 + r * D + d1) : 0u;
    qf[ks][3] = r + 8 < G ? *reinterpret_cast<const uint32_t*>(q0 + (r + 8) * D + d1) : 0u;
    if constexpr (FP8) {
#pragma unroll
      for (int e = 0; e < 4; ++e) qf[ks][e] = bf16x2_to_f16x2(qf[ks][e]);
    }
  }
  float o[16][4];
#pragma unroll
  for (int jn = 0; jn < 16; ++jn)
#pragma unroll
    for (int e = 0; e < 4; ++e) o[jn][e] = 0.f;
  float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};
  const int mi = lane >> 3, rr = lane & 7;
  bool ok = true;
  int j = 0;
  for (; j < nmine; ++j) {
    const int st = j % kTcStages;
    if (!ring_wait(&bars[st], (j / kTcStages) & 1, status)) {
      ok = false;
      break;
    }
    uint32_t kt = smem_u32(ring + st * kStage);
    uint32_t vt = kt + kTcTileBytes;
    float ksc[2][2], vsc[2][2];  // fp8: key / value scales of this lane's 4 token columns
    if constexpr (FP8) {
      const float* kp = sring + st * (kScaleBytes / 4);
      const float* vp = kp + BS;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          ksc[nt][e] = kp[nt * 8 + cq + e];
          vsc[nt][e] = vp[nt * 8 + cq + e];
        }
    }
    // S = Q K^T : 16 x 16 (two n-tiles of 8 tokens)
    float sc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    if constexpr (FP8) {
      // lane (r, c) of n-tile nt reads token row 8 nt + r, 16-byte chunks c and 4 + c (the two dim
      // halves); odd rows load the halves in the other order, so a quarter-warp reads 8 distinct
      // 16-byte bank groups
      const uint8_t* ktile = ring + st * kStage;
      const int c = lane & 3, par = r & 1;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        const int row = nt * 8 + r;
        const uint8_t* rowp = ktile + row * 128;
        const uint4 wa = *reinterpret_cast<const uint4*>(rowp + (((4 * par + c) ^ (row & 7)) << 4));
        const uint4 wb = *reinterpret_cast<const uint4*>(rowp + (((4 * (par ^ 1) + c) ^ (row & 7)) << 4));
        const uint4 h0 = par ? wb : wa, h1 = par ? wa : wb;
        const uint32_t wd[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
        float sc_odd[4] = {0.f, 0.f, 0.f, 0.f};  // two accumulation chains of 4 MMAs, not one of 8
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
          uint32_t bfr[2];
          e4m3x4_to_f16x4(wd[ks], bfr[0], bfr[1]);
          mma_f16_16816((ks & 1) ? sc_odd : sc[nt], qf[ks], bfr);
        }
#pragma unroll
        for (int e = 0; e < 4; ++e) sc[nt][e] += sc_odd[e];
      }
    } else {
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        uint32_t bfr[4];
        const int tok = (mi >> 1) * 8 + rr, ch = 2 * ks + (mi & 1);
        asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                     : "=r"(bfr[0]), "=r"(bfr[1]), "=r"(bfr[2]), "=r"(bfr[3])
                     : "r"(kt + sw128_off(tok, ch)));
        mma_bf16_16816(sc[0], qf[ks], bfr);
        mma_bf16_16816(sc[1], qf[ks], bfr + 2);
      }
    }
    if constexpr (FP8) {
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) sc[nt][e] *= ksc[nt][e & 1];
    }
    const int tok0 = (blk_begin + warp + kDecodeWarps * j) * BS;
    float mx[2] = {-INFINITY, -INFINITY};
    if (softcap_log2 > 0.f) {  // uniform branch: soft-capped scores (Gemma-2)
      const float inv_cap = 1.f / softcap_log2;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) sc[nt][e] = softcap_log2 * tanh_approx(sc[nt][e] * scale_log2 * inv_cap);
    } else {
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) sc[nt][e] *= scale_log2;
    }
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int t = tok0 + nt * 8 + cq + (e & 1);
        const float v = (t < L && t >= kv_lo) ? sc[nt][e] : -INFINITY;
        sc[nt][e] = v;
        mx[e >> 1] = fmaxf(mx[e >> 1], v);
      }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 1));
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 2));
    }
    float mnew[2], corr[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      mnew[h] = fmaxf(mrow[h], mx[h]);
      const float ms = mnew[h] == -INFINITY ? 0.f : mnew[h];
      corr[h] = exp2f(mrow[h] - ms);
      mrow[h] = mnew[h];
      mnew[h] = ms;
      lrow[h] *= corr[h];
    }
#pragma unroll
    for (int jn = 0; jn < 16; ++jn) {
      o[jn][0] *= corr[0];
      o[jn][1] *= corr[0];
      o[jn][2] *= corr[1];
      o[jn][3] *= corr[1];
    }
    uint32_t pf[4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      const float p0 = exp2f(sc[nt][0] - mnew[0]), p1 = exp2f(sc[nt][1] - mnew[0]);
      const float p2 = exp2f(sc[nt][2] - mnew[1]), p3 = exp2f(sc[nt][3] - mnew[1]);
      lrow[0] += p0 + p1;
      lrow[1] += p2 + p3;
      if constexpr (FP8) {
        pf[nt * 2 + 0] = pack_f16x2(p0 * vsc[nt][0], p1 * vsc[nt][1]);
        pf[nt * 2 + 1] = pack_f16x2(p2 * vsc[nt][0], p3 * vsc[nt][1]);
      } else {
        pf[nt * 2 + 0] = pack_bf16x2(p0, p1);
        pf[nt * 2 + 1] = pack_bf16x2(p2, p3);
      }
    }
    // O += P V : 16 x 128 (16 n-tiles of 8 dims), one k-step of 16 tokens
    if constexpr (FP8) {
      // lane (r, c): bytes [16r, 16r + 16) (physical dims 16r + jn) of token rows 2c, 2c+1, 2c+8,
      // 2c+9; byte j of a row pair -> the (k, k+1) f16x2 of n-tile jn = j
      const uint8_t* vtile = ring + st * kStage + kTcFp8TileBytes;
      const int c = lane & 3;
      auto ld = [&](int row) {
        return *reinterpret_cast<const uint4*>(vtile + row * 128 + ((r ^ (row & 7)) << 4));
      };
      const uint4 va = ld(2 * c), vb = ld(2 * c + 1), vc = ld(2 * c + 8), vd = ld(2 * c + 9);
      const uint32_t A[4] = {va.x, va.y, va.z, va.w}, Bv[4] = {vb.x, vb.y, vb.z, vb.w};
      const uint32_t C[4] = {vc.x, vc.y, vc.z, vc.w}, Dv[4] = {vd.x, vd.y, vd.z, vd.w};
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        uint32_t lo_ab, hi_ab, lo_cd, hi_cd;  // interleaved token pairs: [x0 y0 x1 y1], [x2 y2 x3 y3]
        asm("prmt.b32 %0, %1, %2, 0x5140;" : "=r"(lo_ab) : "r"(A[w]), "r"(Bv[w]));
        asm("prmt.b32 %0, %1, %2, 0x7362;" : "=r"(hi_ab) : "r"(A[w]), "r"(Bv[w]));
        asm("prmt.b32 %0, %1, %2, 0x5140;" : "=r"(lo_cd) : "r"(C[w]), "r"(Dv[w]));
        asm("prmt.b32 %0, %1, %2, 0x7362;" : "=r"(hi_cd) : "r"(C[w]), "r"(Dv[w]));
        uint32_t b01[2], b23[2], c01[2], c23[2];
        e4m3x4_to_f16x4(lo_ab, b01[0], b23[0]);  // n-tiles 4w, 4w+1: tokens (2c, 2c+1)
        e4m3x4_to_f16x4(lo_cd, b01[1], b23[1]);  //                   tokens (2c+8, 2c+9)
        e4m3x4_to_f16x4(hi_ab, c01[0], c23[0]);  // n-tiles 4w+2, 4w+3
        e4m3x4_to_f16x4(hi_cd, c01[1], c23[1]);
        mma_f16_16816(o[4 * w + 0], pf, b01);
        mma_f16_16816(o[4 * w + 1], pf, b23);
        mma_f16_16816(o[4 * w + 2], pf, c01);
        mma_f16_16816(o[4 * w + 3], pf, c23);
      }
    } else {
#pragma unroll
      for (int jd = 0; jd < 8; ++jd) {
        uint32_t bfr[4];
        const int tok = (mi & 1) * 8 + rr, ch = 2 * jd + (mi >> 1);
        asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                     : "=r"(bfr[0]), "=r"(bfr[1]), "=r"(bfr[2]), "=r"(bfr[3])
                     : "r"(vt + sw128_off(tok, ch)));
        mma_bf16_16816(o[2 * jd], pf, bfr);
        mma_bf16_16816(o[2 * jd + 1], pf, bfr + 2);
      }
    }
    __syncwarp();
    if (lane == 0 && issued < nmine) {
      fence_proxy_async_smem();
      issue(issued);
      ++issued;
    }
  }
  if (!ok && lane == 0)
    for (int jj = j; jj < issued; ++jj) ring_wait(&bars[jj % kTcStages], (jj / kTcStages) & 1, nullptr);
  __syncwarp();
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    lrow[h] += __shfl_xor_sync(0xffffffffu, lrow[h], 1);
    lrow[h] += __shfl_xor_sync(0xffffffffu, lrow[h], 2);
  }
  // per-warp partials to shared memory (rows r, r + 8 that are real heads)
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int g = r + 8 * h;
    if (g < G) {
#pragma unroll
      for (int jn = 0; jn < 16; ++jn) {
        // logical column 8 jn + cq (+1); the fp8 path's physical dim is 16 (cq (+1)) + jn
        const int d0 = FP8 ? 16 * cq + jn : jn * 8 + cq, d1 = FP8 ? d0 + 16 : d0 + 1;
        sm_o(warp)[g * D + d0] = o[jn][2 * h];
        sm_o(warp)[g * D + d1] = o[jn][2 * h + 1];
      }
      if ((lane & 3) == 0) {
        sm_m[warp * G + g] = mrow[h];
        sm_l[warp * G + g] = lrow[h];
      }
    }
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < G * D; idx += blockDim.x) {
    const int g = idx / D, d = idx % D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kDecodeWarps; ++w) M = fmaxf(M, sm_m[w * G + g]);
    float Lsum = 0.f, O = 0.f;
#pragma unroll
    for (int w = 0; w < kDecodeWarps; ++w) {
      const float mw = sm_m[w * G + g];
      const float f = (mw == -INFINITY) ? 0.f : exp2f(mw - M);
      Lsum += sm_l[w * G + g] * f;
      O += sm_o(w)[g * D + d] * f;
    }
    const int hq = kh * G + g;
    if (num_splits == 1) {
      out[((int64_t)b * H + hq) * D + d] = __float2bfloat16(Lsum > 0.f ? O / Lsum : 0.f);
    } else {
      const int64_t pi = ((int64_t)b * H + hq) * num_splits + split;
      part_o[pi * D + d] = O;
      if (d == 0) {
        part_ml[pi * 2 + 0] = M;
        part_ml[pi * 2 + 1] = Lsum;
      }
    }
  }
}

template <int G, bool FP8>
constexpr size_t decode_tc_smem_bytes() {
  constexpr size_t stage = FP8 ? 2 * kTcFp8TileBytes + 2 * 16 * 4 : kTcStageBytes;  // fp8: + the scales
  return 1024 + (size_t)kDecodeWarps * kTcStages * stage + kDecodeWarps * kTcStages * 8 + 2 * kDecodeWarps * G * 4;
}

template <int G, bool FP8>
void launch_decode_tc(void* out, const void* q, int64_t q_stride, const void* cache, int num_blocks, const int* bt,
                      int bt_stride, const int* lens, int B, int Hk, int num_splits, float scale_log2, float* po,
                      float* pml, int window, float softcap_log2, const float* kv_scales, cudaStream_t s) {
  const uint64_t rows = (uint64_t)num_blocks * 2 * Hk * 16;
  CUtensorMap tm = FP8 ? make_tmap_2d(cache, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, rows, 128, 128, 16, 128,
                                      CU_TENSOR_MAP_SWIZZLE_128B)
                       : make_tmap_2d(cache, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, rows, 128, 128, 16, 64,
                                      CU_TENSOR_MAP_SWIZZLE_128B);
  constexpr size_t smem = decode_tc_smem_bytes<G, FP8>();
  auto kern = paged_decode_tc_kernel<G, FP8>;
  GOLLEK_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  dim3 grid(B, Hk, num_splits);
  kern<<<grid, kDecodeWarps * 32, smem, s>>>(tm, reinterpret_cast<__nv_bfloat16*>(out), po, pml,
                                              reinterpret_cast<const __nv_bfloat16*>(q), bt, bt_stride, lens, Hk,
                                              num_splits, scale_log2, q_stride, bounds_status(), window,
                                              softcap_log2, kv_scales, num_blocks);
  check_launch("paged_decode_attention (tensor cores)");
  if (num_splits > 1) {
    decode_combine_kernel<128><<<B * Hk * G, 128, 0, s>>>(reinterpret_cast<__nv_bfloat16*>(out), po, pml,
                                                          num_splits);
    check_launch("paged_decode_attention combine");
  }
}

template <int D, int G>
void launch_decode_t(void* out, const void* q, int64_t q_stride, const void* cache, const int* bt, int bt_stride,
                     const int* lens, int B, int Hk, int num_splits, float scale_log2, float* po, float* pml,
                     int window, float softcap_log2, int num_blocks, cudaStream_t s) {
  dim3 grid(B, Hk, num_splits);
  constexpr size_t smem = decode_smem_bytes<D, G, 16>();
  auto kern = paged_decode_kernel<D, G, 16>;
  GOLLEK_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  kern<<<grid, kDecodeWarps * 32, smem, s>>>(
      reinterpret_cast<__nv_bfloat16*>(out), po, pml, reinterpret_cast<const __nv_bfloat16*>(q),
      reinterpret_cast<const __nv_bfloat16*>(cache), bt, bt_stride, lens, Hk, num_splits, scale_log2, q_stride,
      num_blocks > 0 ? bounds_status() : nullptr, window, softcap_log2, num_blocks);
  check_launch("paged_decode_attention");
  if (num_splits > 1) {
    decode_combine_kernel<D><<<B * Hk * G, D, 0, s>>>(reinterpret_cast<__nv_bfloat16*>(out), po, pml, num_splits);
    check_launch("paged_decode_attention combine");
  }
}

}  // namespace

namespace gollek {

void launch_paged_decode(void* out, const void* q, int64_t q_stride, const void* cache, int num_blocks,
                         const int* block_tables, int bt_stride, const int* seq_lens, int B, int H, int Hk, int D,
                         int block_size, int num_splits, float scale, float* part_o, float* part_ml,
                         int window, float softcap, cudaStream_t s, const float* kv_scales, bool tensor_cores) {
  throw_if(block_size != 16, "decode attention is built for block_size 16");
  throw_if(H % Hk != 0, "H must be a multiple of Hk");
  throw_if(num_splits > 1 && (part_o == nullptr || part_ml == nullptr), "split-KV decode needs a workspace");
  if (B == 0) return;
  const int G = H / Hk;
  const float sl = scale * kLog2e;
  const float cl = softcap > 0.f ? softcap * kLog2e : 0.f;
  if (kv_scales != nullptr) {  // fp8 e4m3 cache with per-token scales: tensor-core kernel, head_dim 128
    throw_if(D != 128 || num_blocks <= 0, "fp8 KV cache: decode attention is built for head_dim 128");
#define GOLLEK_DECODE_TC8(GG) \
  if (G == GG) return launch_decode_tc<GG, true>(out, q, q_stride, cache, num_blocks, block_tables, bt_stride, seq_lens, \
                                                 B, Hk, num_splits, sl, part_o, part_ml, window, cl, kv_scales, s);
    GOLLEK_DECODE_TC8(1)
    GOLLEK_DECODE_TC8(2)
    GOLLEK_DECODE_TC8(4)
    GOLLEK_DECODE_TC8(8)
    GOLLEK_DECODE_TC8(16)
#undef GOLLEK_DECODE_TC8
    throw_if(true, "fp8 KV cache: unsupported GQA group " + std::to_string(G));
  }
  if (D == 128 && num_blocks > 0 && tensor_cores) {
#define GOLLEK_DECODE_TC(GG) \
  if (G == GG) return launch_decode_tc<GG, false>(out, q, q_stride, cache, num_blocks, block_tables, bt_stride, seq_lens, \
                                                  B, Hk, num_splits, sl, part_o, part_ml, window, cl, nullptr, s);
    GOLLEK_DECODE_TC(1)
    GOLLEK_DECODE_TC(2)
    GOLLEK_DECODE_TC(4)
    GOLLEK_DECODE_TC(8)
    GOLLEK_DECODE_TC(16)
#undef GOLLEK_DECODE_TC
  }
#define GOLLEK_DECODE_CASE(DD, GG)                                                                            \
  if (D == DD && G == GG)                                                                                     \
    return launch_decode_t<DD, GG>(out, q, q_stride, cache, block_tables, bt_stride, seq_lens, B, Hk, num_splits, \
                                   sl, part_o, part_ml, window, cl, num_blocks, s);
  GOLLEK_DECODE_CASE(128, 1)
  GOLLEK_DECODE_CASE(128, 2)
  GOLLEK_DECODE_CASE(128, 4)
  GOLLEK_DECODE_CASE(128, 8)
  GOLLEK_DECODE_CASE(64, 1)
  GOLLEK_DECODE_CASE(64, 2)
  GOLLEK_DECODE_CASE(64, 4)
  GOLLEK_DECODE_CASE(64, 8)
  GOLLEK_DECODE_CASE(32, 1)
  GOLLEK_DECODE_CASE(32, 2)
  GOLLEK_DECODE_CASE(32, 4)
  GOLLEK_DECODE_CASE(32, 8)
  GOLLEK_DECODE_CASE(256, 1)
  GOLLEK_DECODE_CASE(256, 2)
  GOLLEK_DECODE_CASE(256, 4)
  GOLLEK_DECODE_CASE(256, 8)
#undef GOLLEK_DECODE_CASE
  throw_if(true, "decode attention: unsupported head_dim/group " + std::to_string(D) + "/" + std::to_string(G));
}

void launch_paged_prefill(void* out, int64_t out_stride, const void* q, int64_t q_stride, const void* cache,
                          const int* block_tables, int bt_stride, const int* seq_lens, const int* query_start,
                          const int* tiles, int ntiles, int H, int Hk, int D, int block_size, float scale,
                          int window, float softcap, cudaStream_t s, int num_blocks) {
  throw_if(H % Hk != 0, "H must be a multiple of Hk");
  if (ntiles == 0) return;
  const float sl = scale * kLog2e;
  const float cl = softcap > 0.f ? softcap * kLog2e : 0.f;
  dim3 grid(ntiles, H);
#define GOLLEK_PREFILL_CASE(DD)                                                                               \
  if (D == DD) {                                                                                            \
    const size_t smem = (size_t)(kPfBM + 4 * kPfBN) * DD * 2;                                              \
    auto kern = paged_prefill_kernel<DD>;                                                                   \
    GOLLEK_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));  \
    kern<<<grid, kPfThreads, smem, s>>>(reinterpret_cast<__nv_bfloat16*>(out), out_stride,                  \
                                        reinterpret_cast<const __nv_bfloat16*>(q), q_stride,                \
                                        reinterpret_cast<const __nv_bfloat16*>(cache), block_tables,        \
                                        bt_stride, seq_lens, query_start, tiles, H, Hk, block_size, sl,     \
                                        window, cl, num_blocks,                                             \
                                        num_blocks > 0 ? bounds_status() : nullptr);                        \
    check_launch("paged_prefill_attention");                                                                \
    return;                                                                                                 \
  }
  GOLLEK_PREFILL_CASE(256)
  GOLLEK_PREFILL_CASE(128)
  GOLLEK_PREFILL_CASE(64)
  GOLLEK_PREFILL_CASE(32)
#undef GOLLEK_PREFILL_CASE
  throw_if(true, "prefill attention: unsupported head_dim " + std::to_string(D));
}

}  // namespace gollek
