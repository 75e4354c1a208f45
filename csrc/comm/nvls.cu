// Tensor-parallel collectives through NVLink SHARP (NVLS): the NVSwitch reduces and multicasts.
//
// The symmetric region of every rank is bound to one multicast object, so one virtual address
// (the multicast address, `mc`) names the same offset in every rank's region at once:
//   multimem.ld_reduce [mc + off]  → the switch reads `off` from every rank and returns the sum
//                                    (fp32 accumulation of the bf16 inputs);
//   multimem.st        [mc + off]  → the switch writes the value into every rank's region;
//   multimem.red.add   [mc + flag] → every rank's copy of a flag word is incremented (a one-
//                                    instruction signal to all ranks).
// None of these is a TMA or bulk copy: they are plain per-thread memory instructions on the
// multicast address, and no tensor map ever covers another GPU's memory.
//
// tp_nvls_ar_rmsnorm_kernel replaces "all-reduce → residual add → RMSNorm" after a row-parallel GEMM
// (o_proj / down_proj), whose partial [T, d] the GEMM wrote into this rank's partial buffer:
//   A) barrier: each rank adds 1 to every rank's `nv_a` (multimem.red) once its partial is
//      written; every CTA waits until its local `nv_a` reaches epoch * world.
//   two-shot (large T; sequence-parallel residual): rank r owns rows [r*c, (r+1)*c), c = ceil(T/N).
//      One warp per row: ld_reduce the row's partial sums, add the rank's residual rows (kept
//      only for the owned rows: the residual stream is sharded by rows across the TP ranks),
//      round, RMSNorm, and multimem.st the normalised row into every rank's x buffer. Then
//      C) barrier: the last CTA of each rank signals `nv_c` on all ranks and waits for all.
//      Traffic per rank and direction ≈ (1 + 1/N) · T · d · 2 bytes (a ring all-reduce moves
//      2(N-1)/N of it, and the residual is never all-gathered).
//   one-shot (decode-sized T): every rank ld_reduces all rows and normalises them locally (full
//      residual rows kept), so only barrier A is needed.
//   reduce-scatter: as two-shot, but the normalised owned rows stay local (the expert-parallel
//      all-to-all takes them from there); only barrier A.
// The partial buffers alternate by call parity: a rank reuses a buffer two calls later, after
// barrier A of the call in between proved every peer finished reading it.
//
// Every wait is bounded by a globaltimer deadline; on timeout the kernel records
// kStatusPeerTimeout in the header's status word and completes (the host checks and raises).
#include "../common/common.cuh"
#include "../kernels/launchers.h"
#include "push.h"

#include <cstddef>

namespace gollek {

namespace {

constexpr int kNvThreads = 256;

GOLLEK_DEVICE uint64_t nv_gtimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

GOLLEK_DEVICE bool nv_wait_geq(const uint32_t* flag, uint32_t target, uint64_t limit_ns) {
  if ((int32_t)(ld_acquire_sys(flag) - target) >= 0) return true;
  const uint64_t t0 = nv_gtimer();
  while ((int32_t)(ld_acquire_sys(flag) - target) < 0) {
    if (nv_gtimer() - t0 > limit_ns) return false;
  }
  return true;
}

// Sum over ranks of the 8 bf16 values at a multicast address (fp32 accumulation in the switch).
GOLLEK_DEVICE uint4 mm_ld_reduce_bf16x8(const void* mc) {
  uint4 r;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(mc)
               : "memory");
  return r;
}

// Store 16 bytes into every rank's copy of the multicast address.
GOLLEK_DEVICE void mm_st_16(void* mc, const uint4& v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(mc), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}

// Add `v` to every rank's copy of a flag word; release: this thread's earlier writes (and those
// ordered before it by a fence) are visible to whoever observes the increment.
GOLLEK_DEVICE void mm_red_add_release(uint32_t* mc_flag, uint32_t v) {
  asm volatile("multimem.red.release.sys.global.add.u32 [%0], %1;" ::"l"(mc_flag), "r"(v) : "memory");
}

struct NvlsArgs {
  uint8_t* uc;               // this rank's region (local address)
  uint8_t* mc;               // multicast address of the region (same offsets)
  int64_t partial_off[2];    // the two partial buffers (alternating by call parity)
  int64_t x_off;             // gathered normalised rows (two-shot output)
  int rank, world, T, d, parity, one_shot;
  int gather;                // two-shot: store x into every rank (1) or only locally (0)
  float eps;
  uint64_t timeout_ns;
};

GOLLEK_DEVICE SymmHeader* hdr(uint8_t* base) { return reinterpret_cast<SymmHeader*>(base); }

// Barrier A (all partials written). Returns the call's epoch.
GOLLEK_DEVICE uint32_t nv_enter(const NvlsArgs& a, uint32_t* s_epoch) {
  SymmHeader* me = hdr(a.uc);
  if (threadIdx.x == 0) *s_epoch = *reinterpret_cast<volatile uint32_t*>(&me->nv_epoch) + 1;
  __syncthreads();
  const uint32_t epoch = *s_epoch;
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    __threadfence_system();  // the partial (written by the previous kernel) before the signal
    mm_red_add_release(&hdr(a.mc)->nv_a, 1u);
  }
  if (threadIdx.x == 0 && !nv_wait_geq(&me->nv_a, epoch * (uint32_t)a.world, a.timeout_ns))
    atomicOr(&me->status, kStatusPeerTimeout);
  __syncthreads();
  return epoch;
}

// End of a call: the last CTA of this rank adds 1 to every rank's nv_c (after all of this rank's
// multicast stores) and, when `wait`, waits until every rank did the same; it then records the
// epoch. `s_last` is shared scratch.
GOLLEK_DEVICE void nv_leave(const NvlsArgs& a, uint32_t epoch, bool wait, int* s_last) {
  SymmHeader* me = hdr(a.uc);
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    const uint32_t prev = atomicAdd(&me->nv_arrive, 1u);
    *s_last = prev == gridDim.x - 1;
  }
  __syncthreads();
  if (!*s_last || threadIdx.x != 0) return;
  me->nv_arrive = 0;
  __threadfence_system();
  mm_red_add_release(&hdr(a.mc)->nv_c, 1u);
  if (wait && !nv_wait_geq(&me->nv_c, epoch * (uint32_t)a.world, a.timeout_ns))
    atomicOr(&me->status, kStatusPeerTimeout);
  *reinterpret_cast<volatile uint32_t*>(&me->nv_epoch) = epoch;
}

// VPL: 16-byte vectors per lane per row (d <= VPL * 256). One warp per row.
template <int VPL>
__global__ void __launch_bounds__(kNvThreads) tp_nvls_ar_rmsnorm_kernel(NvlsArgs a,
                                                                        __nv_bfloat16* __restrict__ residual,
                                                                        const __nv_bfloat16* __restrict__ w,
                                                                        __nv_bfloat16* __restrict__ x_local) {
  __shared__ uint32_t s_epoch;
  __shared__ int s_last;
  const uint32_t epoch = nv_enter(a, &s_epoch);
  const int lane = threadIdx.x & 31;
  const int nvec = a.d >> 3;
  int r0 = 0, r1 = a.T;
  if (!a.one_shot) {
    const int chunk = (a.T + a.world - 1) / a.world;
    r0 = min(a.T, a.rank * chunk);
    r1 = min(a.T, r0 + chunk);
  }
  const __nv_bfloat16* pmc = reinterpret_cast<const __nv_bfloat16*>(a.mc + a.partial_off[a.parity]);
  __nv_bfloat16* xmc = reinterpret_cast<__nv_bfloat16*>(a.mc + a.x_off);
  const int warps = gridDim.x * (kNvThreads / 32);
  // The next row's reductions are issued before this row is normalised, so a warp with several
  // rows pays the NVSwitch round trip once (the grid is at most one CTA per SM).
  int row = r0 + blockIdx.x * (kNvThreads / 32) + (threadIdx.x >> 5);
  uint4 p[VPL];
  if (row < r1) {
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      const int v = lane + 32 * j;
      if (v < nvec) p[j] = mm_ld_reduce_bf16x8(pmc + (int64_t)row * a.d + v * 8);
    }
  }
  for (; row < r1; row += warps) {
    const int64_t base = (int64_t)row * a.d;
    uint4 res[VPL];
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      const int v = lane + 32 * j;
      if (v < nvec) res[j] = *reinterpret_cast<const uint4*>(residual + base + v * 8);
    }
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      const int v = lane + 32 * j;
      if (v < nvec) {
        float f[8], g[8];
        bf16x8_to_float(p[j], f);
        bf16x8_to_float(res[j], g);
#pragma unroll
        for (int e = 0; e < 8; ++e) f[e] += g[e];
        res[j] = float_to_bf16x8(f);  // the new residual, rounded as stored
        *reinterpret_cast<uint4*>(residual + base + v * 8) = res[j];
        bf16x8_to_float(res[j], f);
#pragma unroll
        for (int e = 0; e < 8; ++e) ss += f[e] * f[e];
      }
    }
    ss = warp_sum(ss);
    const float rs = rsqrtf(ss / (float)a.d + a.eps);
    const int nxt = row + warps;  // prefetch: p[] is free once the new residual is in res[]
    if (nxt < r1) {
#pragma unroll
      for (int j = 0; j < VPL; ++j) {
        const int v = lane + 32 * j;
        if (v < nvec) p[j] = mm_ld_reduce_bf16x8(pmc + (int64_t)nxt * a.d + v * 8);
      }
    }
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      const int v = lane + 32 * j;
      if (v < nvec) {
        float f[8], wf[8];
        bf16x8_to_float(res[j], f);
        bf16x8_to_float(*reinterpret_cast<const uint4*>(w + v * 8), wf);
#pragma unroll
        for (int e = 0; e < 8; ++e) f[e] = f[e] * rs * wf[e];
        const uint4 o = float_to_bf16x8(f);
        if (a.one_shot || !a.gather)
          *reinterpret_cast<uint4*>(x_local + base + v * 8) = o;
        else
          mm_st_16(xmc + base + v * 8, o);
      }
    }
  }
  nv_leave(a, epoch, !a.one_shot && a.gather, &s_last);
}

// Plain sum all-reduce of the partial buffer. two-shot: rank r reduces its 1/N slice and stores
// the sum back into every rank's partial buffer (result read locally from the partial buffer);
// one-shot: every rank reduces everything into `out` (local).
__global__ void __launch_bounds__(kNvThreads) tp_nvls_allreduce_kernel(NvlsArgs a, int64_t nvec_total,
                                                                       __nv_bfloat16* __restrict__ out) {
  __shared__ uint32_t s_epoch;
  __shared__ int s_last;
  const uint32_t epoch = nv_enter(a, &s_epoch);
  int64_t v0 = 0, v1 = nvec_total;
  if (!a.one_shot) {
    const int64_t chunk = (nvec_total + a.world - 1) / a.world;
    v0 = min(nvec_total, (int64_t)a.rank * chunk);
    v1 = min(nvec_total, v0 + chunk);
  }
  __nv_bfloat16* pmc = reinterpret_cast<__nv_bfloat16*>(a.mc + a.partial_off[a.parity]);
  constexpr int kU = 4;  // vectors in flight per thread
  const int64_t stride = (int64_t)gridDim.x * kNvThreads;
  for (int64_t i0 = v0 + (int64_t)blockIdx.x * kNvThreads + threadIdx.x; i0 < v1; i0 += kU * stride) {
    uint4 r[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int64_t i = i0 + u * stride;
      if (i < v1) r[u] = mm_ld_reduce_bf16x8(pmc + i * 8);
    }
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int64_t i = i0 + u * stride;
      if (i < v1) {
        if (a.one_shot)
          *reinterpret_cast<uint4*>(out + i * 8) = r[u];
        else
          mm_st_16(pmc + i * 8, r[u]);
      }
    }
  }
  nv_leave(a, epoch, !a.one_shot, &s_last);
}

// All-gather of column shards (vocab-parallel logits): rank r's [B, v] shard is stored once through
// the multicast address into columns [r*v, (r+1)*v) of the [B, ld] buffer at `dst_off`, so the
// switch writes it into every rank's copy (each shard byte crosses NVLink once per rank instead of
// once per peer). Barrier A first (no rank overwrites a buffer a peer may still read), barrier C
// last (every rank's shard has landed before the caller reads the gathered rows).
__global__ void __launch_bounds__(kNvThreads) tp_nvls_gather_cols_kernel(NvlsArgs a,
                                                                         const __nv_bfloat16* __restrict__ src,
                                                                         int64_t src_stride, int B, int v,
                                                                         int64_t dst_off, int64_t ld) {
  __shared__ uint32_t s_epoch;
  __shared__ int s_last;
  const uint32_t epoch = nv_enter(a, &s_epoch);
  const int vv = v / 8;
  const int64_t total = (int64_t)B * vv;
  __nv_bfloat16* dmc = reinterpret_cast<__nv_bfloat16*>(a.mc + dst_off) + (int64_t)a.rank * v;
  constexpr int kU = 4;  // 16-byte vectors in flight per thread
  const int64_t stride = (int64_t)gridDim.x * kNvThreads;
  for (int64_t i0 = (int64_t)blockIdx.x * kNvThreads + threadIdx.x; i0 < total; i0 += kU * stride) {
    uint4 r[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int64_t i = i0 + u * stride;
      if (i < total) r[u] = *reinterpret_cast<const uint4*>(src + (i / vv) * src_stride + (i % vv) * 8);
    }
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int64_t i = i0 + u * stride;
      if (i < total) mm_st_16(dmc + (i / vv) * ld + (i % vv) * 8, r[u]);
    }
  }
  nv_leave(a, epoch, true, &s_last);
}

NvlsArgs make_nvls_args(uint64_t uc, uint64_t mc, int rank, int world, int64_t p0, int64_t p1, int64_t x_off,
                        int parity, bool one_shot, int T, int d, float eps, double timeout_s) {
  throw_if(world < 1 || world > 8, "NVLS collectives: 1..8 ranks");
  throw_if(uc % 256 != 0 || mc % 256 != 0, "NVLS collectives: region addresses must be 256-byte aligned");
  throw_if(p0 % 16 != 0 || p1 % 16 != 0 || x_off % 16 != 0, "NVLS collectives: buffer offsets must be 16-byte aligned");
  NvlsArgs a{};
  a.uc = reinterpret_cast<uint8_t*>(uc);
  a.mc = reinterpret_cast<uint8_t*>(mc);
  a.partial_off[0] = p0;
  a.partial_off[1] = p1;
  a.x_off = x_off;
  a.rank = rank;
  a.world = world;
  a.T = T;
  a.d = d;
  a.parity = parity & 1;
  a.one_shot = one_shot ? 1 : 0;
  a.gather = 1;
  a.eps = eps;
  a.timeout_ns = (uint64_t)(timeout_s * 1e9);
  return a;
}

}  // namespace

void launch_tp_nvls_ar_rmsnorm(uint64_t uc, uint64_t mc, int rank, int world, int64_t p0, int64_t p1, int64_t x_off,
                               int parity, int mode, void* residual, const void* w, void* x_local, int T, int d,
                               float eps, double timeout_s, int grid, cudaStream_t s) {
  throw_if(d % 8 != 0 || d > 32 * 256, "NVLS all-reduce + RMSNorm: hidden size must be a multiple of 8, <= 8192");
  throw_if(mode < 0 || mode > 2, "NVLS all-reduce + RMSNorm: mode 0 one-shot, 1 two-shot, 2 reduce-scatter");
  throw_if(mode != 1 && x_local == nullptr, "NVLS all-reduce + RMSNorm: this mode needs a local output");
  if (T == 0) return;
  NvlsArgs a = make_nvls_args(uc, mc, rank, world, p0, p1, x_off, parity, mode == 0, T, d, eps, timeout_s);
  a.gather = mode == 1 ? 1 : 0;
  auto* res = reinterpret_cast<__nv_bfloat16*>(residual);
  auto* wp = reinterpret_cast<const __nv_bfloat16*>(w);
  auto* xl = reinterpret_cast<__nv_bfloat16*>(x_local);
  const int nvec = d / 8;
  if (nvec <= 4 * 32)
    tp_nvls_ar_rmsnorm_kernel<4><<<grid, kNvThreads, 0, s>>>(a, res, wp, xl);
  else if (nvec <= 8 * 32)
    tp_nvls_ar_rmsnorm_kernel<8><<<grid, kNvThreads, 0, s>>>(a, res, wp, xl);
  else if (nvec <= 16 * 32)
    tp_nvls_ar_rmsnorm_kernel<16><<<grid, kNvThreads, 0, s>>>(a, res, wp, xl);
  else
    tp_nvls_ar_rmsnorm_kernel<32><<<grid, kNvThreads, 0, s>>>(a, res, wp, xl);
  check_launch("tp_nvls_allreduce_add_rmsnorm");
}

void launch_tp_nvls_allreduce(uint64_t uc, uint64_t mc, int rank, int world, int64_t p0, int64_t p1, int parity,
                              bool one_shot, void* out, int64_t numel, double timeout_s, int grid, cudaStream_t s) {
  throw_if(numel % 8 != 0, "NVLS all-reduce: element count must be a multiple of 8");
  throw_if(one_shot && out == nullptr, "NVLS all-reduce: one-shot needs a local output");
  if (numel == 0) return;
  NvlsArgs a = make_nvls_args(uc, mc, rank, world, p0, p1, 0, parity, one_shot, 0, 0, 0.f, timeout_s);
  tp_nvls_allreduce_kernel<<<grid, kNvThreads, 0, s>>>(a, numel / 8, reinterpret_cast<__nv_bfloat16*>(out));
  check_launch("tp_nvls_allreduce");
}

void launch_tp_nvls_gather_cols(uint64_t uc, uint64_t mc, int rank, int world, const void* src, int64_t src_stride,
                                int B, int v, int64_t dst_off, int64_t ld, double timeout_s, int grid, cudaStream_t s) {
  throw_if(v % 8 != 0 || src_stride % 8 != 0 || ld % 8 != 0 || dst_off % 16 != 0 ||
               reinterpret_cast<uintptr_t>(src) % 16 != 0,
           "NVLS column gather: shard width, strides and offsets must be whole 16-byte vectors");
  throw_if(ld < (int64_t)world * v, "NVLS column gather: destination row narrower than world * v");
  if (B == 0) return;
  NvlsArgs a = make_nvls_args(uc, mc, rank, world, 0, 0, 0, 0, false, 0, 0, 0.f, timeout_s);
  tp_nvls_gather_cols_kernel<<<grid, kNvThreads, 0, s>>>(a, reinterpret_cast<const __nv_bfloat16*>(src), src_stride,
                                                         B, v, dst_off, ld);
  check_launch("tp_nvls_gather_cols");
}

}  // namespace gollek
