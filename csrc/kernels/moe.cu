// K12: MoE routing and token permutation, plus the expert combine (sm_100a).
//
//   moe_logits   (E >= 32) router logits x·Wrᵀ on tensor cores (mma m16n8k16, fp32 accumulation)
//   moe_route    router logits x·Wrᵀ (fp32 accumulate, E ≤ 256; read from moe_logits when it ran),
//                then one warp per token scores
//                and picks its top-k (k ≤ 8, ties to the lower expert id): softmax scores with
//                optional renormalisation of the k weights (Mixtral), or sigmoid scores whose
//                choice adds a per-expert correction bias, limited to the topk_group best of n_group
//                expert groups (group score = sum of its two best choice scores), weights = the
//                chosen sigmoid scores renormalised and times a scale (DeepSeek-V3); per-local-expert
//                token counts (atomics).
//   moe_plan     one thread: per-expert row offsets in the permuted buffer, each expert's rows
//                padded to the 128-row GEMM tile, the M-tile → expert map for the grouped GEMM
//                and the live M-tile count; re-zeroes the counters for the next call.
//   moe_gather   one warp per (token, choice) routed to a local expert: claims a row of its
//                expert's segment and copies the token's hidden vector there.
//   moe_combine  out[t] = Σ_j w[t,j] · Y[dest[t,j]] over the choices that were local (fp32 sum).
//
// The grouped expert GEMMs between gather and combine run on the tcgen05 GEMM (gemm.cu) in
// grouped mode. Nothing here synchronises with the host, so a MoE layer can be captured in a
// CUDA graph. Under expert parallelism each rank owns experts [e0, e0 + e_loc) of the replicated
// activations and ``out`` is its partial sum; the tensor-parallel all-reduce that follows adds the
// partials of all ranks.
//
// Reference behaviour: Mixtral routing in runner/safetensor/…/generation/moe/MoeForwardPass.java:39-128
// and the EP dispatch contract of core/optimization/gollek-plugin-elastic-ep/…/binding/ElasticEpBinding.java:19-45.
// The DeepSeek-V3 router (sigmoid, correction bias, group limit, routed scaling) follows the
// checkpoint's published routing rule; the reference serves those models through llama.cpp.
#include "../common/common.cuh"
#include "../common/tma_host.h"
#include "launchers.h"

#include <algorithm>

using namespace gollek;

namespace {

constexpr int kMaxE = 256;
constexpr int kMaxK = 8;
constexpr int kPerLane = kMaxE / 32;  // expert e = lane + 32 i is scored by lane (e & 31)

constexpr int kRouteTok = 4;  // tokens per routing CTA

// Router logits on tensor cores for many experts: logits[t, e] = x[t, :] . Wr[e, :] (bf16 operands,
// fp32 accumulation, fixed summation order per element). CTA = 64 tokens x 64 experts; per 64-wide
// K chunk both tiles are staged in shared memory with 16-byte loads (the next chunk prefetched into
// registers) and warp w multiplies its 16 tokens against the 64 experts with mma m16n8k16.
constexpr int kLgTile = 64, kLgK = 64, kLgPad = kLgK + 8;

__device__ __forceinline__ void mma_bf16_16816(float* d, const uint32_t* a, const uint32_t* b) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

__global__ void __launch_bounds__(128) moe_logits_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx,
                                                         const __nv_bfloat16* __restrict__ wr, int T, int H, int E,
                                                         float* __restrict__ logits, int kchunk) {
  // blockIdx.z: a K range of kchunk elements; its partial logits go to slab z of [splits, T, E]
  logits += (int64_t)blockIdx.z * T * E;
  const int kb = blockIdx.z * kchunk, ke = min(H, kb + kchunk);
  __shared__ __align__(16) __nv_bfloat16 xs[kLgTile][kLgPad];
  __shared__ __align__(16) __nv_bfloat16 ws[kLgTile][kLgPad];
  const int t0 = blockIdx.x * kLgTile, e0 = blockIdx.y * kLgTile;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, q = lane & 3;
  float c[8][4];
#pragma unroll
  for (int j = 0; j < 8; ++j) c[j][0] = c[j][1] = c[j][2] = c[j][3] = 0.f;
  uint4 xv[4], wv[4];
  auto load = [&](int k0) {
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int i = tid + 128 * u, r = i >> 3, v = i & 7;
      xv[u] = t0 + r < T ? *reinterpret_cast<const uint4*>(x + (int64_t)(t0 + r) * ldx + k0 + 8 * v)
                         : make_uint4(0, 0, 0, 0);
      wv[u] = e0 + r < E ? *reinterpret_cast<const uint4*>(wr + (int64_t)(e0 + r) * H + k0 + 8 * v)
                         : make_uint4(0, 0, 0, 0);
    }
  };
  if (kb < ke) load(kb);  // an empty trailing split writes zeros
  for (int k0 = kb; k0 < ke; k0 += kLgK) {
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int i = tid + 128 * u, r = i >> 3, v = i & 7;
      *reinterpret_cast<uint4*>(&xs[r][8 * v]) = xv[u];
      *reinterpret_cast<uint4*>(&ws[r][8 * v]) = wv[u];
    }
    __syncthreads();
    if (k0 + kLgK < ke) load(k0 + kLgK);
    if (t0 + warp * 16 < T) {
#pragma unroll
      for (int kk = 0; kk < kLgK; kk += 16) {
        uint32_t a[4];
        a[0] = *reinterpret_cast<const uint32_t*>(&xs[warp * 16 + g][kk + 2 * q]);
        a[1] = *reinterpret_cast<const uint32_t*>(&xs[warp * 16 + g + 8][kk + 2 * q]);
        a[2] = *reinterpret_cast<const uint32_t*>(&xs[warp * 16 + g][kk + 8 + 2 * q]);
        a[3] = *reinterpret_cast<const uint32_t*>(&xs[warp * 16 + g + 8][kk + 8 + 2 * q]);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          uint32_t b[2];
          b[0] = *reinterpret_cast<const uint32_t*>(&ws[8 * j + g][kk + 2 * q]);
          b[1] = *reinterpret_cast<const uint32_t*>(&ws[8 * j + g][kk + 8 + 2 * q]);
          mma_bf16_16816(c[j], a, b);
        }
      }
    }
    __syncthreads();
  }
  const int r0 = t0 + warp * 16 + g, r1 = r0 + 8;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int e = e0 + 8 * j + 2 * q;
    if (e < E) {  // E is even (checked by the launcher), so e + 1 < E too
      if (r0 < T) *reinterpret_cast<float2*>(logits + (int64_t)r0 * E + e) = make_float2(c[j][0], c[j][1]);
      if (r1 < T) *reinterpret_cast<float2*>(logits + (int64_t)r1 * E + e) = make_float2(c[j][2], c[j][3]);
    }
  }
}

// Routing: one CTA per 4 tokens. All 256 threads split the hidden dimension (8 elements each per
// 2048-wide stripe) and accumulate the 4 tokens x 8 experts of the current expert chunk, so the
// router weights are read once per CTA and every thread has many independent loads in flight;
// a shared-memory reduction gives the logits, then warp w < 4 does softmax / top-k for token w.
__global__ void __launch_bounds__(256) moe_route_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx,
                                                        const __nv_bfloat16* __restrict__ wr, int T, int H, int E,
                                                        int topk, int renorm, int e0, int e_loc, MoeRouting rt,
                                                        int* __restrict__ ids, float* __restrict__ wts,
                                                        int* __restrict__ counts) {
  __shared__ float s_part[8][kRouteTok * 8];
  __shared__ float s_logit[kRouteTok][kMaxE];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t0 = blockIdx.x * kRouteTok;
  const int ntok = min(kRouteTok, T - t0);
  if (rt.logits != nullptr) {  // logits computed by moe_logits_kernel: its K-split partials, added in order
    for (int i = threadIdx.x; i < ntok * E; i += blockDim.x) {
      float v = 0.f;
      for (int z = 0; z < rt.logit_splits; ++z) v += rt.logits[(int64_t)z * T * E + (int64_t)t0 * E + i];
      s_logit[i / E][i % E] = v;
    }
    __syncthreads();
  }
  for (int ec = 0; ec < (rt.logits != nullptr ? 0 : E); ec += 8) {
    float acc[kRouteTok][8];
#pragma unroll
    for (int a = 0; a < kRouteTok; ++a)
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[a][e] = 0.f;
    for (int h = threadIdx.x * 8; h < H; h += 2048) {
      uint4 wu[8];
#pragma unroll
      for (int e = 0; e < 8; ++e)
        wu[e] = (ec + e < E) ? *reinterpret_cast<const uint4*>(wr + (int64_t)(ec + e) * H + h) : make_uint4(0, 0, 0, 0);
      uint4 xu[kRouteTok];
#pragma unroll
      for (int a = 0; a < kRouteTok; ++a)
        xu[a] = a < ntok ? *reinterpret_cast<const uint4*>(x + (int64_t)(t0 + a) * ldx + h) : make_uint4(0, 0, 0, 0);
#pragma unroll
      for (int a = 0; a < kRouteTok; ++a) {
        float xv[8];
        bf16x8_to_float(xu[a], xv);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          float wv[8];
          bf16x8_to_float(wu[e], wv);
#pragma unroll
          for (int i = 0; i < 8; ++i) acc[a][e] = fmaf(xv[i], wv[i], acc[a][e]);
        }
      }
    }
#pragma unroll
    for (int a = 0; a < kRouteTok; ++a)
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float v = warp_sum(acc[a][e]);
        if (lane == 0) s_part[warp][a * 8 + e] = v;
      }
    __syncthreads();
    if (threadIdx.x < kRouteTok * 8) {
      float v = 0.f;
#pragma unroll
      for (int w = 0; w < 8; ++w) v += s_part[w][threadIdx.x];
      const int a = threadIdx.x >> 3, e = ec + (threadIdx.x & 7);
      if (e < E) s_logit[a][e] = v;
    }
    __syncthreads();
  }
  if (warp >= ntok) return;
  const int t = t0 + warp;
  float* lg = s_logit[warp];
  // p: the weight score of each owned expert; c: its choice score (-inf: absent or already taken)
  float p[kPerLane], c[kPerLane];
  if (rt.scoring == 0) {  // softmax over E
    float m = -INFINITY;
#pragma unroll
    for (int i = 0; i < kPerLane; ++i) m = fmaxf(m, lane + 32 * i < E ? lg[lane + 32 * i] : -INFINITY);
    m = warp_max(m);
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < kPerLane; ++i) {
      p[i] = lane + 32 * i < E ? __expf(lg[lane + 32 * i] - m) : 0.f;
      sum += p[i];
    }
    const float inv = 1.f / warp_sum(sum);
#pragma unroll
    for (int i = 0; i < kPerLane; ++i) {
      p[i] *= inv;
      c[i] = lane + 32 * i < E ? p[i] : -INFINITY;
    }
  } else {  // sigmoid; the choice adds the correction bias
#pragma unroll
    for (int i = 0; i < kPerLane; ++i) {
      const int e = lane + 32 * i;
      p[i] = e < E ? 1.f / (1.f + __expf(-lg[e])) : 0.f;
      c[i] = e < E ? p[i] + (rt.bias ? rt.bias[e] : 0.f) : -INFINITY;
    }
  }
  if (rt.n_group > 1) {
    // group score = sum of the two best choice scores of the group; keep the topk_group best groups
    // (ties to the lower group) and score every expert outside them 0
    __syncwarp();
#pragma unroll
    for (int i = 0; i < kPerLane; ++i)
      if (lane + 32 * i < E) lg[lane + 32 * i] = c[i];
    __syncwarp();
    const int gs = E / rt.n_group;
    float gscore = -INFINITY;
    if (lane < rt.n_group) {
      float b1 = -INFINITY, b2 = -INFINITY;
      for (int e = lane * gs; e < (lane + 1) * gs; ++e) {
        const float v = lg[e];
        if (v > b1) {
          b2 = b1;
          b1 = v;
        } else if (v > b2) {
          b2 = v;
        }
      }
      gscore = b1 + b2;
    }
    uint32_t keep = 0;
    for (int j = 0; j < rt.topk_group; ++j) {
      float bv = gscore;
      int bi = lane < rt.n_group ? lane : 1 << 30;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) {
          bv = ov;
          bi = oi;
        }
      }
      if (bi < 32) keep |= 1u << bi;
      if (bi == lane) gscore = -INFINITY;
    }
#pragma unroll
    for (int i = 0; i < kPerLane; ++i) {
      const int e = lane + 32 * i;
      if (e < E && !((keep >> (e / gs)) & 1u)) c[i] = 0.f;
    }
  }
  int sel_id[kMaxK];
  float sel_p[kMaxK];
  float psum = 0.f;
#pragma unroll
  for (int j = 0; j < kMaxK; ++j) {
    if (j >= topk) break;
    // lane-local best (lowest id on ties: the scan runs in increasing id), then the warp's best
    float bv = -INFINITY, bp = 0.f;
    int bi = 1 << 30;
#pragma unroll
    for (int i = 0; i < kPerLane; ++i) {
      if (lane + 32 * i < E && c[i] > bv) {
        bv = c[i];
        bp = p[i];
        bi = lane + 32 * i;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const float op = __shfl_xor_sync(0xffffffffu, bp, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bp = op;
        bi = oi;
      }
    }
    sel_id[j] = bi;
    sel_p[j] = bp;
    psum += bp;
#pragma unroll
    for (int i = 0; i < kPerLane; ++i)
      if (bi == lane + 32 * i) c[i] = -INFINITY;  // taken
  }
  if (lane == 0) {
    float scale = rt.scale;
    if (renorm) scale /= psum + (rt.scoring == 0 ? 0.f : 1e-20f);
    for (int j = 0; j < topk; ++j) {
      // routing runs over logical experts; ids (and the local counts) are physical slots
      const int phys = rt.expert_map ? rt.expert_map[sel_id[j]] : sel_id[j];
      ids[(int64_t)t * topk + j] = phys;
      wts[(int64_t)t * topk + j] = sel_p[j] * scale;
      const int le = phys - e0;
      if (le >= 0 && le < e_loc) atomicAdd(&counts[le], 1);
    }
  }
}

// ws layout (int32), fixed whatever e_loc is, so calls with different expert ranges can share it:
//   counts[256] | cursor[256] | offsets[257] | num_m[1] | tile_group[max_tiles]
// counts[0, e_loc) are zero between calls (route increments them, plan reads and re-zeroes them);
// plan zeroes cursor[0, e_loc) before gather claims rows with it.
constexpr int kWsCursor = kMaxE, kWsOffsets = 2 * kMaxE, kWsNumM = 3 * kMaxE + 1, kWsTiles = 3 * kMaxE + 2;

__global__ void moe_plan_kernel(int* __restrict__ ws, int e_loc, int max_tiles) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  int* counts = ws;
  int* cursor = ws + kWsCursor;
  int* offsets = ws + kWsOffsets;
  int* num_m = ws + kWsNumM;
  int* tile_group = ws + kWsTiles;
  int off = 0, mt = 0;
  for (int e = 0; e < e_loc; ++e) {
    const int c = counts[e];
    offsets[e] = off;
    const int nt = (c + 127) / 128;
    for (int i = 0; i < nt && mt < max_tiles; ++i) tile_group[mt++] = e;
    off += nt * 128;
    counts[e] = 0;
    cursor[e] = 0;
  }
  offsets[e_loc] = off;
  *num_m = mt;
}

__global__ void __launch_bounds__(256) moe_gather_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx,
                                                         const int* __restrict__ ids, int rows, int topk, int H,
                                                         int e0, int e_loc, int* __restrict__ ws,
                                                         int* __restrict__ dest, __nv_bfloat16* __restrict__ xp) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int idx = blockIdx.x * 8 + warp;
  if (idx >= rows) return;
  const int e = ids[idx] - e0;
  if (e < 0 || e >= e_loc) {
    if (lane == 0) dest[idx] = -1;
    return;
  }
  int* cursor = ws + kWsCursor;
  const int* offsets = ws + kWsOffsets;
  int pos = 0;
  if (lane == 0) pos = atomicAdd(&cursor[e], 1);
  pos = __shfl_sync(0xffffffffu, pos, 0);
  const int d = offsets[e] + pos;
  if (lane == 0) dest[idx] = d;
  const __nv_bfloat16* src = x + (int64_t)(idx / topk) * ldx;
  __nv_bfloat16* dst = xp + (int64_t)d * H;
  for (int h = lane * 8; h < H; h += 256)
    *reinterpret_cast<uint4*>(dst + h) = *reinterpret_cast<const uint4*>(src + h);
}

// yp: bf16 expert outputs [cap, H], or (splits > 1) the down GEMM's fp32 split-K partials
// [splits, cap, H], summed here instead of in a separate reduce pass.
__global__ void __launch_bounds__(256) moe_combine_kernel(__nv_bfloat16* __restrict__ out, int64_t ldo,
                                                          const __nv_bfloat16* __restrict__ yp, int64_t ldy,
                                                          const float* __restrict__ ypart, int splits, int64_t cap,
                                                          const int* __restrict__ dest, const float* __restrict__ wts,
                                                          int T, int topk, int H) {
  const int groups = H / 8;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)T * groups) return;
  const int t = (int)(i / groups), c = (int)(i % groups) * 8;
  float acc[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) acc[e] = 0.f;
  for (int j = 0; j < topk; ++j) {
    const int d = dest[(int64_t)t * topk + j];
    if (d < 0) continue;
    const float w = wts[(int64_t)t * topk + j];
    float y[8];
    if (splits > 1) {
#pragma unroll
      for (int e = 0; e < 8; ++e) y[e] = 0.f;
      for (int sp = 0; sp < splits; ++sp) {
        const float* p = ypart + ((int64_t)sp * cap + d) * H + c;
        const float4 a = *reinterpret_cast<const float4*>(p), b = *reinterpret_cast<const float4*>(p + 4);
        y[0] += a.x; y[1] += a.y; y[2] += a.z; y[3] += a.w; y[4] += b.x; y[5] += b.y; y[6] += b.z; y[7] += b.w;
      }
    } else {
      bf16x8_to_float(*reinterpret_cast<const uint4*>(yp + (int64_t)d * ldy + c), y);
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = fmaf(w, y[e], acc[e]);
  }
  *reinterpret_cast<uint4*>(out + (int64_t)t * ldo + c) = float_to_bf16x8(acc);
}

}  // namespace

namespace gollek {

int moe_capacity_rows(int T, int topk, int e_loc) {
  const int64_t rows = (int64_t)T * topk + 127ll * e_loc;
  return (int)((rows + 127) / 128 * 128);
}

// K splits of the tensor-core router: about four 64 x 64 tiles per SM, each split at least four
// 64-wide K chunks long.
int moe_logit_splits(int T, int E, int H) {
  const int tiles = ((T + kLgTile - 1) / kLgTile) * ((E + kLgTile - 1) / kLgTile);
  const int want = (4 * num_sms() + tiles - 1) / tiles;
  return std::max(1, std::min(want, H / kLgK / 4));
}

int moe_ws_ints(int T, int topk, int e_loc) { return kWsTiles + moe_capacity_rows(T, topk, e_loc) / 128; }

// Tile widths of the two grouped GEMMs and the down GEMM's split-K factor, from the expected live
// M tiles (a uniform router puts T*topk/E rows on each expert). Few tiles (decode, or one expert per
// rank under EP) would leave most SMs idle while the weights stream, so the down GEMM (K = F, long)
// is split over K and the combine kernel sums its fp32 partials.
void moe_plan_host(int T, int topk, int E, int e_loc, int H, int F, int& bn_gu, int& bn_dn, int& splits) {
  const int sms = num_sms();
  const int per_expert = (T * topk + E - 1) / E;
  const int m_live = std::max(1, std::min(moe_capacity_rows(T, topk, e_loc) / 128, e_loc * ((per_expert + 127) / 128)));
  bn_gu = (m_live * ((2 * F + 255) / 256) >= sms) ? 256 : 128;
  if (m_live * ((H + 255) / 256) >= sms) bn_dn = 256;
  else if (m_live * ((H + 127) / 128) >= sms / 2) bn_dn = 128;
  else bn_dn = 64;
  const int tiles = m_live * ((H + bn_dn - 1) / bn_dn);
  splits = 1;
  if (tiles < sms / 2) splits = std::max(1, std::min({(sms + tiles - 1) / tiles, F / 64 / 4, 8}));
}

void launch_moe_forward(void* out, int64_t ldo, const void* x, int64_t ldx, const void* wr, const void* w_gu,
                        const void* w_down, int* ws, int* ids, float* wts, int* dest, void* xp, void* hp, void* yp,
                        float* ypart, int T, int H, int F, int E, int topk, int renorm, int e0, int e_loc,
                        const MoeRouting& rt, uint32_t* status, cudaStream_t s) {
  throw_if(E > kMaxE || E < 1, "moe: at most 256 experts");
  throw_if(rt.scoring != 0 && rt.scoring != 1, "moe: scoring is 0 (softmax) or 1 (sigmoid)");
  throw_if(rt.n_group < 1 || rt.n_group > 32 || E % rt.n_group != 0 || (rt.n_group > 1 && E / rt.n_group < 2) ||
               rt.topk_group < 1 || rt.topk_group > rt.n_group,
           "moe: n_group must divide E (at most 32 groups of >= 2 experts), 1 <= topk_group <= n_group");
  throw_if(topk < 1 || topk > kMaxK || topk > E, "moe: top-k must be in [1, min(8, E)]");
  throw_if(H % 256 != 0, "moe: hidden size must be a multiple of 256");
  throw_if(F % 64 != 0, "moe: expert FFN width must be a multiple of 64");
  throw_if(ldx % 8 != 0 || ldo % 8 != 0, "moe: row pitches must keep 16-byte alignment");
  throw_if(e0 < 0 || e_loc < 1 || e0 + e_loc > E, "moe: bad local expert range");
  static_assert(kWsTiles == 3 * kMaxE + 2, "workspace layout");
  if (T == 0) return;
  const int cap = moe_capacity_rows(T, topk, e_loc);
  auto* xb = reinterpret_cast<const __nv_bfloat16*>(x);
  MoeRouting rr = rt;
  if (rt.logits != nullptr) {
    throw_if(E % 2 != 0, "moe: the tensor-core router needs an even expert count");
    rr.logit_splits = moe_logit_splits(T, E, H);
    const int kchunk = (H / kLgK + rr.logit_splits - 1) / rr.logit_splits * kLgK;
    moe_logits_kernel<<<dim3((T + kLgTile - 1) / kLgTile, (E + kLgTile - 1) / kLgTile, rr.logit_splits), 128, 0,
                        s>>>(xb, ldx, reinterpret_cast<const __nv_bfloat16*>(wr), T, H, E, rt.logits, kchunk);
    check_launch("moe_logits");
  }
  moe_route_kernel<<<(T + kRouteTok - 1) / kRouteTok, 256, 0, s>>>(xb, ldx, reinterpret_cast<const __nv_bfloat16*>(wr), T, H, E, topk,
                                               renorm, e0, e_loc, rr, ids, wts, ws);
  check_launch("moe_route");
  moe_plan_kernel<<<1, 32, 0, s>>>(ws, e_loc, cap / 128);
  check_launch("moe_plan");
  const int rows = T * topk;
  moe_gather_kernel<<<(rows + 7) / 8, 256, 0, s>>>(xb, ldx, ids, rows, topk, H, e0, e_loc, ws, dest,
                                                   reinterpret_cast<__nv_bfloat16*>(xp));
  check_launch("moe_gather");
  const int* num_m = ws + kWsNumM;
  const int* tile_group = ws + kWsTiles;
  int bn_gu, bn_dn, splits;
  moe_plan_host(T, topk, E, e_loc, H, F, bn_gu, bn_dn, splits);
  throw_if(splits > 1 && ypart == nullptr, "moe: split-K down projection needs the fp32 partial buffer");
  // gate/up (interleaved in groups of 64 per expert) with the SwiGLU epilogue: hp [cap, F]
  launch_gemm_grouped(hp, F, xp, H, w_gu, H, cap, 2 * F, H, e_loc, kEpiSwiglu, bn_gu, tile_group, num_m, 1,
                      nullptr, status, s);
  // down: yp [cap, H] (bf16), or fp32 partials [splits, cap, H] summed by the combine
  launch_gemm_grouped(yp, H, hp, F, w_down, F, cap, H, F, e_loc, kEpiNone, bn_dn, tile_group, num_m, splits,
                      ypart, status, s);
  const int64_t threads = (int64_t)T * (H / 8);
  moe_combine_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, s>>>(
      reinterpret_cast<__nv_bfloat16*>(out), ldo, reinterpret_cast<const __nv_bfloat16*>(yp), H, ypart, splits, cap,
      dest, wts, T, topk, H);
  check_launch("moe_combine");
}

// Routing only (expert-parallel all-to-all): physical expert ids and weights of every token; no
// local expert counting (e_loc = 0).
void launch_moe_route(const void* x, int64_t ldx, const void* wr, int T, int H, int E, int topk, int renorm,
                      const MoeRouting& rt, int* ids, float* wts, int* scratch, cudaStream_t s) {
  throw_if(E > kMaxE || E < 1, "moe route: at most 256 experts");
  throw_if(topk < 1 || topk > kMaxK || topk > E, "moe route: top-k must be in [1, min(8, E)]");
  throw_if(H % 256 != 0, "moe route: hidden size must be a multiple of 256");
  throw_if(rt.n_group < 1 || rt.n_group > 32 || E % rt.n_group != 0 || rt.topk_group < 1 ||
               rt.topk_group > rt.n_group,
           "moe route: bad group-limited routing parameters");
  if (T == 0) return;
  auto* xb = reinterpret_cast<const __nv_bfloat16*>(x);
  MoeRouting rr = rt;
  if (rt.logits != nullptr) {
    throw_if(E % 2 != 0, "moe: the tensor-core router needs an even expert count");
    rr.logit_splits = moe_logit_splits(T, E, H);
    const int kchunk = (H / kLgK + rr.logit_splits - 1) / rr.logit_splits * kLgK;
    moe_logits_kernel<<<dim3((T + kLgTile - 1) / kLgTile, (E + kLgTile - 1) / kLgTile, rr.logit_splits), 128, 0,
                        s>>>(xb, ldx, reinterpret_cast<const __nv_bfloat16*>(wr), T, H, E, rt.logits, kchunk);
    check_launch("moe_logits");
  }
  moe_route_kernel<<<(T + kRouteTok - 1) / kRouteTok, 256, 0, s>>>(
      xb, ldx, reinterpret_cast<const __nv_bfloat16*>(wr), T, H, E, topk, renorm, 0, 0, rr, ids, wts, scratch);
  check_launch("moe_route");
}

}  // namespace gollek
