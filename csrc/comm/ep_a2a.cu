// Expert-parallel all-to-all over NVLink peer memory (C3): token-sharded MoE layers.
//
// Each rank owns a chunk of the step's token rows (the sequence-parallel layout the NVLS
// collectives keep) and holds E_loc experts (global expert e lives on rank e / E_loc). One MoE
// layer is:
//   1. route        (moe.cu's router on the owned rows: physical expert ids + weights)
//   2. dispatch     ep_dispatch_kernel: every (token, choice) row is stored with 16-byte P2P
//                   stores into the expert owner's receive buffer, slot = a per-destination
//                   counter; the row's origin (token * k + choice) and local expert go along in a
//                   small meta record. The last CTA publishes the per-(destination, local expert)
//                   counts into each destination and raises that destination's dispatch flag.
//   3. compact      ep_compact_kernel (on the expert owner): waits for every source's flag,
//                   lays the received rows out as the grouped GEMM wants them (per local expert,
//                   each expert's rows padded to 128: sources in rank order, each source's rows
//                   in its slot order) and writes, for every grouped row, the address of its
//                   combine slot on the source rank (peer memory).
//   4. gate/up      grouped tcgen05 GEMM with the SwiGLU epilogue (local)
//   5. down         grouped tcgen05 GEMM whose epilogue stores each output row straight into its
//                   combine slot on the source rank (gemm.cu, scatter epilogue): the combine
//                   transfer overlaps the GEMM tile by tile
//   6. signal       ep_signal_kernel: the expert owner raises the combine flag of every source
//   7. combine      ep_combine_norm_kernel (on the source): waits for every owner's flag, sums
//                   the token's k expert rows with their routing weights (fp32, choice order),
//                   adds the residual, applies the next RMSNorm and stores the normalised row
//                   into every rank's x buffer (multimem.st through the NVSwitch), then a
//                   multicast counter barrier so no rank reads x before every row landed.
// Only k rows per owned token cross NVLink each way, instead of every token's hidden state
// (replicated activations) plus a full all-reduce.
//
// All waits are bounded (globaltimer); on timeout the status word records kStatusPeerTimeout and
// the kernel finishes (the host checks and raises). Peer memory is only touched with plain
// ld/st.global and the multicast address with multimem.st / multimem.red; no TMA or bulk copy
// touches another GPU's memory.
#include "../common/common.cuh"
#include "../kernels/launchers.h"
#include "push.h"

namespace gollek {

namespace {

constexpr int kEpThreads = 256;
constexpr int kEpMaxWorld = 8;
constexpr int kEpMaxLocal = 32;  // experts per rank

GOLLEK_DEVICE uint64_t ep_gtimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

GOLLEK_DEVICE bool ep_wait_geq(const uint32_t* flag, uint32_t target, uint64_t limit_ns) {
  if ((int32_t)(ld_acquire_sys(flag) - target) >= 0) return true;
  const uint64_t t0 = ep_gtimer();
  while ((int32_t)(ld_acquire_sys(flag) - target) < 0) {
    if (ep_gtimer() - t0 > limit_ns) return false;
  }
  return true;
}

GOLLEK_DEVICE void ep_mm_st_16(void* mc, const uint4& v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(mc), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}

GOLLEK_DEVICE void ep_mm_red_add_release(uint32_t* mc_flag, uint32_t v) {
  asm volatile("multimem.red.release.sys.global.add.u32 [%0], %1;" ::"l"(mc_flag), "r"(v) : "memory");
}

}  // namespace

struct EpArgs {
  uint8_t* bases[kEpMaxWorld];
  uint8_t* mc;          // multicast address of the region (0: not available)
  EpLayout lay;
  int rank, world, e_loc, k, H;
  uint64_t timeout_ns;
};

namespace {

GOLLEK_DEVICE SymmHeader* ep_hdr(uint8_t* b) { return reinterpret_cast<SymmHeader*>(b); }
GOLLEK_DEVICE uint32_t* ep_flag(const EpArgs& a, int rank, int which, int src) {
  return reinterpret_cast<uint32_t*>(a.bases[rank] + a.lay.flags_off) + which * kEpMaxWorld + src;
}
GOLLEK_DEVICE uint32_t ep_epoch(const EpArgs& a) {
  return *reinterpret_cast<volatile uint32_t*>(&ep_hdr(a.bases[a.rank])->ep_epoch) + 1;
}

// ws (local, int32): cnt[world * E_loc] (per destination and local expert) | arrive[1]; zero between calls
__global__ void __launch_bounds__(kEpThreads) ep_dispatch_kernel(EpArgs a, const __nv_bfloat16* __restrict__ x,
                                                                 int64_t ldx, const int* __restrict__ ids, int Tn,
                                                                 int* __restrict__ ws) {
  const uint32_t epoch = ep_epoch(a);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int* cnt = ws;
  int* arrive = ws + a.world * a.e_loc;
  const int rows = Tn * a.k;
  for (int idx = blockIdx.x * (kEpThreads / 32) + warp; idx < rows; idx += gridDim.x * (kEpThreads / 32)) {
    const int e = ids[idx];
    if (e < 0 || e >= a.world * a.e_loc) continue;  // not an expert id (uniform across the warp)
    const int dest = e / a.e_loc, le = e % a.e_loc;
    int slot_le = 0, slot = 0;
    if (lane == 0) {
      slot_le = atomicAdd(&cnt[dest * a.e_loc + le], 1);
      slot = atomicAdd(&cnt[a.world * a.e_loc + 1 + dest], 1);  // per-destination slot
    }
    slot_le = __shfl_sync(0xffffffffu, slot_le, 0);
    slot = __shfl_sync(0xffffffffu, slot, 0);
    if (slot >= a.lay.cap_src) continue;  // capacity is sized for the worst case; never taken
    const int64_t row = (int64_t)a.rank * a.lay.cap_src + slot;
    const __nv_bfloat16* src = x + (int64_t)(idx / a.k) * ldx;
    __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(a.bases[dest] + a.lay.recv_off) + row * a.H;
    for (int h = lane * 8; h < a.H; h += 256)
      *reinterpret_cast<uint4*>(dst + h) = *reinterpret_cast<const uint4*>(src + h);
    if (lane == 0)
      reinterpret_cast<int4*>(a.bases[dest] + a.lay.meta_off)[row] = make_int4(idx, le, slot_le, 0);
  }
  // last CTA: publish counts and raise the dispatch flags
  __shared__ int s_last;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    s_last = atomicAdd(arrive, 1) == (int)gridDim.x - 1;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence_system();
  for (int i = threadIdx.x; i < a.world * a.e_loc; i += blockDim.x) {
    const int dest = i / a.e_loc, le = i % a.e_loc;
    reinterpret_cast<int*>(a.bases[dest] + a.lay.counts_off)[a.rank * a.e_loc + le] =
        *reinterpret_cast<volatile int*>(&cnt[i]);
  }
  __syncthreads();
  if (threadIdx.x < a.world) {
    __threadfence_system();
    st_release_sys(ep_flag(a, threadIdx.x, 0, a.rank), epoch);
  }
  __syncthreads();
  // reset the local counters for the next call (this stream's next dispatch runs after this kernel)
  for (int i = threadIdx.x; i < a.world * a.e_loc + 1 + a.world; i += blockDim.x) ws[i] = 0;
}

// Grouped layout: local expert le's rows start at gstart[le] (multiple of 128); inside it source s's
// rows start at Σ_{s' < s} counts[s'][le]. Every CTA derives the offsets from the counts.
__global__ void __launch_bounds__(kEpThreads) ep_compact_kernel(EpArgs a, __nv_bfloat16* __restrict__ xg,
                                                                uint64_t* __restrict__ comb_ptr, int cap_dst,
                                                                int* __restrict__ tile_group,
                                                                int* __restrict__ num_m) {
  const uint32_t epoch = ep_epoch(a);
  __shared__ int s_cnt[kEpMaxWorld * kEpMaxLocal];
  __shared__ int s_srcbase[kEpMaxWorld * kEpMaxLocal];  // start of (source, expert) rows in the layout
  __shared__ int s_gstart[kEpMaxLocal + 1];             // start of each expert's (padded) rows
  __shared__ int s_gcount[kEpMaxLocal];                 // rows each expert received
  __shared__ int s_rows[kEpMaxWorld + 1];               // prefix of rows received per source
  SymmHeader* me = ep_hdr(a.bases[a.rank]);
  if (threadIdx.x < a.world && !ep_wait_geq(ep_flag(a, a.rank, 0, threadIdx.x), epoch, a.timeout_ns))
    atomicOr(&me->status, kStatusPeerTimeout);
  __syncthreads();
  const int* counts = reinterpret_cast<const int*>(a.bases[a.rank] + a.lay.counts_off);
  for (int i = threadIdx.x; i < a.world * a.e_loc; i += blockDim.x)
    s_cnt[i] = *reinterpret_cast<volatile const int*>(&counts[i]);
  __syncthreads();
  const int max_tiles = cap_dst / 128;
  if (threadIdx.x == 0) {
    int off = 0;
    for (int le = 0; le < a.e_loc; ++le) {
      int c = 0;
      for (int s = 0; s < a.world; ++s) {
        s_srcbase[s * a.e_loc + le] = off + c;
        c += s_cnt[s * a.e_loc + le];
      }
      s_gstart[le] = off;
      s_gcount[le] = c;
      const int nt = (c + 127) / 128;
      if (blockIdx.x == 0)
        for (int i = 0; i < nt && off / 128 + i < max_tiles; ++i) tile_group[off / 128 + i] = le;
      off += nt * 128;
    }
    s_gstart[a.e_loc] = off;
    if (blockIdx.x == 0) *num_m = min(off, cap_dst) / 128;
    s_rows[0] = 0;
    for (int s = 0; s < a.world; ++s) {
      int r = 0;
      for (int le = 0; le < a.e_loc; ++le) r += s_cnt[s * a.e_loc + le];
      s_rows[s + 1] = s_rows[s] + r;
    }
  }
  __syncthreads();
  // padding rows of each expert's last tile: no combine destination (the scatter epilogue skips
  // them); their stale inputs only reach outputs nobody stores. Every grouped row's pointer is
  // written exactly once: here (padding) or by the row copy below.
  for (int le = 0; le < a.e_loc; ++le) {
    const int p0 = s_gstart[le] + s_gcount[le], p1 = min(s_gstart[le + 1], cap_dst);
    for (int r = p0 + blockIdx.x * blockDim.x + threadIdx.x; r < p1; r += gridDim.x * blockDim.x) comb_ptr[r] = 0;
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int total = s_rows[a.world];
  const int4* meta = reinterpret_cast<const int4*>(a.bases[a.rank] + a.lay.meta_off);
  const __nv_bfloat16* recv = reinterpret_cast<const __nv_bfloat16*>(a.bases[a.rank] + a.lay.recv_off);
  for (int i = blockIdx.x * (kEpThreads / 32) + warp; i < total; i += gridDim.x * (kEpThreads / 32)) {
    int s = 0;
    while (s + 1 < a.world && s_rows[s + 1] <= i) ++s;
    const int slot = i - s_rows[s];
    const int64_t rrow = (int64_t)s * a.lay.cap_src + slot;
    const int4 m = meta[rrow];  // (token * k + choice, local expert, slot within it)
    const int g = s_srcbase[s * a.e_loc + m.y] + m.z;
    if (g >= cap_dst) continue;
    const __nv_bfloat16* src = recv + rrow * a.H;
    __nv_bfloat16* dst = xg + (int64_t)g * a.H;
    for (int h = lane * 8; h < a.H; h += 256)
      *reinterpret_cast<uint4*>(dst + h) = *reinterpret_cast<const uint4*>(src + h);
    if (lane == 0)
      comb_ptr[g] = reinterpret_cast<uint64_t>(a.bases[s] + a.lay.comb_off) + (uint64_t)m.x * a.H * 2;
  }
}

// After the down GEMM (its scatter epilogue wrote the rows into the sources' combine buffers):
// make those stores visible and raise every source's combine flag.
__global__ void ep_signal_kernel(EpArgs a) {
  const uint32_t epoch = ep_epoch(a);
  __threadfence_system();
  if (threadIdx.x < a.world) st_release_sys(ep_flag(a, threadIdx.x, 1, a.rank), epoch);
}

// VPL: 16-byte vectors per lane per row (H <= VPL * 256). One warp per owned token.
template <int VPL>
__global__ void __launch_bounds__(kEpThreads) ep_combine_norm_kernel(EpArgs a, int T, int r0, int Tn,
                                                                     const float* __restrict__ wts,
                                                                     __nv_bfloat16* __restrict__ residual,
                                                                     const __nv_bfloat16* __restrict__ w, float eps) {
  const uint32_t epoch = ep_epoch(a);
  SymmHeader* me = ep_hdr(a.bases[a.rank]);
  if (threadIdx.x < a.world && !ep_wait_geq(ep_flag(a, a.rank, 1, threadIdx.x), epoch, a.timeout_ns))
    atomicOr(&me->status, kStatusPeerTimeout);
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int nvec = a.H >> 3;
  const __nv_bfloat16* comb = reinterpret_cast<const __nv_bfloat16*>(a.bases[a.rank] + a.lay.comb_off);
  __nv_bfloat16* xmc = reinterpret_cast<__nv_bfloat16*>(a.mc + a.lay.x_off);
  const int warps = gridDim.x * (kEpThreads / 32);
  for (int t = blockIdx.x * (kEpThreads / 32) + (threadIdx.x >> 5); t < Tn; t += warps) {
    const int64_t row = (int64_t)(r0 + t) * a.H;
    float acc[VPL][8];
#pragma unroll
    for (int j = 0; j < VPL; ++j)
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[j][e] = 0.f;
    for (int c = 0; c < a.k; ++c) {
      const float wc = wts[(int64_t)t * a.k + c];
      const __nv_bfloat16* y = comb + ((int64_t)t * a.k + c) * a.H;
#pragma unroll
      for (int j = 0; j < VPL; ++j) {
        const int v = lane + 32 * j;
        if (v < nvec) {
          float f[8];
          bf16x8_to_float(*reinterpret_cast<const uint4*>(y + v * 8), f);
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[j][e] = fmaf(wc, f[e], acc[j][e]);
        }
      }
    }
    // moe output rounded to bf16 (as a stored activation), + residual, rounded: the new residual
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      const int v = lane + 32 * j;
      if (v < nvec) {
        float yv[8], rv[8];
        bf16x8_to_float(float_to_bf16x8(acc[j]), yv);
        bf16x8_to_float(*reinterpret_cast<const uint4*>(residual + row + v * 8), rv);
#pragma unroll
        for (int e = 0; e < 8; ++e) rv[e] += yv[e];
        const uint4 packed = float_to_bf16x8(rv);
        *reinterpret_cast<uint4*>(residual + row + v * 8) = packed;
        bf16x8_to_float(packed, acc[j]);
#pragma unroll
        for (int e = 0; e < 8; ++e) ss += acc[j][e] * acc[j][e];
      }
    }
    ss = warp_sum(ss);
    const float rs = rsqrtf(ss / (float)a.H + eps);
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      const int v = lane + 32 * j;
      if (v < nvec) {
        float wf[8];
        bf16x8_to_float(*reinterpret_cast<const uint4*>(w + v * 8), wf);
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[j][e] = acc[j][e] * rs * wf[e];
        ep_mm_st_16(xmc + row + v * 8, float_to_bf16x8(acc[j]));
      }
    }
  }
  // barrier: every rank's x rows landed before any rank goes on (multicast counter, like the NVLS
  // all-reduce's barrier C); the last CTA of this rank signals and waits, then records the epoch
  __shared__ int s_last;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    s_last = atomicAdd(&me->ep_arrive, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!s_last || threadIdx.x != 0) return;
  me->ep_arrive = 0;
  __threadfence_system();
  ep_mm_red_add_release(&ep_hdr(a.mc)->ep_done, 1u);
  if (!ep_wait_geq(&me->ep_done, epoch * (uint32_t)a.world, a.timeout_ns)) atomicOr(&me->status, kStatusPeerTimeout);
  *reinterpret_cast<volatile uint32_t*>(&me->ep_epoch) = epoch;
}

EpArgs make_ep_args(const std::vector<uint64_t>& bases, uint64_t mc, const EpLayout& lay, int rank, int e_loc,
                    int k, int H, double timeout_s) {
  throw_if(bases.empty() || bases.size() > kEpMaxWorld, "EP all-to-all: 1..8 ranks");
  throw_if(e_loc < 1 || e_loc > kEpMaxLocal, "EP all-to-all: 1..32 experts per rank");
  throw_if(H % 8 != 0 || H > 32 * 256, "EP all-to-all: hidden size must be a multiple of 8, <= 8192");
  throw_if(lay.recv_off % 16 || lay.comb_off % 16 || lay.meta_off % 16 || lay.x_off % 16,
           "EP all-to-all: buffers must be 16-byte aligned");
  EpArgs a{};
  for (size_t i = 0; i < bases.size(); ++i) a.bases[i] = reinterpret_cast<uint8_t*>(bases[i]);
  a.mc = reinterpret_cast<uint8_t*>(mc);
  a.lay = lay;
  a.rank = rank;
  a.world = (int)bases.size();
  a.e_loc = e_loc;
  a.k = k;
  a.H = H;
  a.timeout_ns = (uint64_t)(timeout_s * 1e9);
  return a;
}

}  // namespace

int ep_ws_ints(int world, int e_loc) { return world * e_loc + 1 + world; }

void launch_ep_dispatch(const std::vector<uint64_t>& bases, uint64_t mc, const EpLayout& lay, int rank, int e_loc,
                        int k, const void* x, int64_t ldx, int H, const int* ids, int Tn, int* ws, double timeout_s,
                        cudaStream_t s) {
  EpArgs a = make_ep_args(bases, mc, lay, rank, e_loc, k, H, timeout_s);
  throw_if((int64_t)Tn * k > lay.cap_src, "EP dispatch: more rows than a destination slot holds");
  const int rows = Tn * k;
  const int grid = std::max(1, std::min((rows + 7) / 8, 4 * device_num_sms()));
  ep_dispatch_kernel<<<grid, kEpThreads, 0, s>>>(a, reinterpret_cast<const __nv_bfloat16*>(x), ldx, ids, Tn, ws);
  check_launch("ep_dispatch");
}

void launch_ep_compact(const std::vector<uint64_t>& bases, uint64_t mc, const EpLayout& lay, int rank, int e_loc,
                       int k, int H, void* xg, uint64_t* comb_ptr, int cap_dst, int* tile_group, int* num_m,
                       double timeout_s, cudaStream_t s) {
  EpArgs a = make_ep_args(bases, mc, lay, rank, e_loc, k, H, timeout_s);
  throw_if(cap_dst % 128 != 0, "EP compact: grouped capacity must be a multiple of 128");
  const int grid = std::max(1, std::min(cap_dst / 8, 2 * device_num_sms()));
  ep_compact_kernel<<<grid, kEpThreads, 0, s>>>(a, reinterpret_cast<__nv_bfloat16*>(xg), comb_ptr, cap_dst,
                                                tile_group, num_m);
  check_launch("ep_compact");
}

void launch_ep_signal(const std::vector<uint64_t>& bases, uint64_t mc, const EpLayout& lay, int rank, int e_loc,
                      int k, int H, double timeout_s, cudaStream_t s) {
  EpArgs a = make_ep_args(bases, mc, lay, rank, e_loc, k, H, timeout_s);
  ep_signal_kernel<<<1, 32, 0, s>>>(a);
  check_launch("ep_signal");
}

void launch_ep_combine_norm(const std::vector<uint64_t>& bases, uint64_t mc, const EpLayout& lay, int rank,
                            int e_loc, int k, int H, int T, int r0, int Tn, const float* wts, void* residual,
                            const void* w, float eps, double timeout_s, cudaStream_t s) {
  EpArgs a = make_ep_args(bases, mc, lay, rank, e_loc, k, H, timeout_s);
  throw_if(mc == 0, "EP combine: needs the multicast address of the region");
  const int grid = std::max(1, std::min((Tn + 7) / 8, 8 * device_num_sms()));
  auto* res = reinterpret_cast<__nv_bfloat16*>(residual);
  auto* wp = reinterpret_cast<const __nv_bfloat16*>(w);
  const int nvec = H / 8;
  if (nvec <= 4 * 32)
    ep_combine_norm_kernel<4><<<grid, kEpThreads, 0, s>>>(a, T, r0, Tn, wts, res, wp, eps);
  else if (nvec <= 8 * 32)
    ep_combine_norm_kernel<8><<<grid, kEpThreads, 0, s>>>(a, T, r0, Tn, wts, res, wp, eps);
  else if (nvec <= 16 * 32)
    ep_combine_norm_kernel<16><<<grid, kEpThreads, 0, s>>>(a, T, r0, Tn, wts, res, wp, eps);
  else
    ep_combine_norm_kernel<32><<<grid, kEpThreads, 0, s>>>(a, T, r0, Tn, wts, res, wp, eps);
  check_launch("ep_combine_norm");
}

}  // namespace gollek
