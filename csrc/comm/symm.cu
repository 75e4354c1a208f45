// Symmetric device heap over CUDA IPC + fused tensor-parallel collectives over NVLink P2P (sm_100a).
//
// Heap: each rank cudaMalloc's one region of identical size; IPC handles are exchanged by the
// host (gloo) and every peer region is mapped with cudaIpcOpenMemHandle, so a kernel can load
// from / store to any rank's region through NVLink/NVSwitch. A small header at the start of
// each region holds the barrier flags, an arrive counter, the epoch and a status word.
//
// tp_allreduce_add_rmsnorm (C1/C4 in the design): for the row-parallel projections (o_proj,
// down_proj) each rank's GEMM writes its partial [T, d] directly into its own symmetric
// "partial" buffer (two of them, alternating per call). One persistent kernel then
//   A) start barrier: every rank is past its previous call (so no peer still reads a buffer
//      this call overwrites);
//   1) reduce-scatter by rows: rank r sums the N partials of its row chunk with P2P loads,
//      adds the residual rows, and writes the new residual rows to its "gather" buffer;
//   B) barrier: every rank finished phase 1 (last CTA to arrive signals all peers);
//   2) all-gather + RMSNorm: every rank reads each row from its owner's gather buffer (P2P),
//      stores it as the new residual and writes x = rmsnorm(residual) * w.
// (one_shot = true skips the scatter: every rank sums all N partials for all rows, one barrier;
// the latency-optimal choice for decode-sized T.)
//
// Flags carry a per-call epoch (monotonic), so nothing is reset between calls. All waits are
// bounded by a globaltimer deadline; on timeout a status bit is set and the kernel finishes
// without the missing data (the host checks the status word and raises). No multicast and no
// TMA on peer memory: plain ld/st.global over NVLink.
#include "../common/common.cuh"
#include "../kernels/launchers.h"
#include "push.h"

#include <vector>

namespace gollek {

constexpr int kArThreads = 512;

GOLLEK_DEVICE uint64_t gtimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Wait until flag >= target (wrap-safe), bounded by `limit_ns`.
GOLLEK_DEVICE bool wait_geq(const uint32_t* flag, uint32_t target, uint64_t limit_ns) {
  if ((int32_t)(ld_acquire_sys(flag) - target) >= 0) return true;
  const uint64_t t0 = gtimer();
  while ((int32_t)(ld_acquire_sys(flag) - target) < 0) {
    if (gtimer() - t0 > limit_ns) return false;
  }
  return true;
}

struct ArArgs {
  uint8_t* bases[8];          // every rank's region base (own included)
  int64_t partial_off[2];     // byte offsets of the two partial buffers in a region
  int64_t gather_off;         // byte offset of the gather buffer
  int rank, world;
  int T, d;
  int parity;                 // which partial buffer this call reads
  int one_shot;
  float eps;
  uint64_t timeout_ns;
};

constexpr int kMaxWorld = 8;

// acc += the 8-element bf16 vector at element offset `off` of buffer `buf_off` of every rank, in
// rank order; all world loads (NVLink for the peers) are issued before the first add.
GOLLEK_DEVICE void add_ranks(float* acc, const ArArgs& a, int64_t buf_off, int64_t off) {
  const int world = a.world;
  uint4 v[kMaxWorld];
#pragma unroll
  for (int p = 0; p < kMaxWorld; ++p)
    if (p < world)
      v[p] = *reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(a.bases[p] + buf_off) + off);
#pragma unroll
  for (int p = 0; p < kMaxWorld; ++p) {
    if (p < world) {
      float t[8];
      bf16x8_to_float(v[p], t);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] += t[e];
    }
  }
}

__global__ void __launch_bounds__(kArThreads) tp_ar_rmsnorm_kernel(ArArgs a, __nv_bfloat16* __restrict__ residual,
                                                                    const __nv_bfloat16* __restrict__ w,
                                                                    __nv_bfloat16* __restrict__ x_out) {
  SymmHeader* me = reinterpret_cast<SymmHeader*>(a.bases[a.rank]);
  __shared__ uint32_t s_epoch;
  __shared__ float red[4 * (kArThreads / 32)];
  __shared__ float red_rows[4];
  __shared__ int s_ok;
  if (threadIdx.x == 0) {
    s_epoch = *reinterpret_cast<volatile uint32_t*>(&me->epoch) + 1;
    s_ok = 1;
  }
  __syncthreads();
  const uint32_t epoch = s_epoch;
  // ---- barrier A
  if (blockIdx.x == 0 && threadIdx.x < a.world) {
    __threadfence_system();
    SymmHeader* peer = reinterpret_cast<SymmHeader*>(a.bases[threadIdx.x]);
    st_release_sys(&peer->flag_a[a.rank], epoch);
  }
  if (threadIdx.x < a.world) {
    if (!wait_geq(&me->flag_a[threadIdx.x], epoch, a.timeout_ns)) {
      atomicOr(&me->status, kStatusPeerTimeout);
      s_ok = 0;
    }
  }
  __syncthreads();
  const int nvec = a.d / 8;
  const int world = a.world;
  if (!a.one_shot) {
    // ---- phase 1: reduce my row chunk into my gather buffer
    const int chunk = (a.T + world - 1) / world;
    const int r0 = a.rank * chunk, r1 = min(a.T, r0 + chunk);
    __nv_bfloat16* gmine = reinterpret_cast<__nv_bfloat16*>(a.bases[a.rank] + a.gather_off);
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < (int64_t)(r1 - r0) * nvec;
         i += (int64_t)gridDim.x * blockDim.x) {
      const int row = r0 + (int)(i / nvec), v = (int)(i % nvec);
      const int64_t off = (int64_t)row * a.d + v * 8;
      float acc[8];
      bf16x8_to_float(*reinterpret_cast<const uint4*>(residual + off), acc);
      add_ranks(acc, a, a.partial_off[a.parity], off);
      *reinterpret_cast<uint4*>(gmine + off) = float_to_bf16x8(acc);
    }
    // ---- barrier B: last local CTA signals every peer
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence_system();
      const uint32_t prev = atomicAdd(&me->arrive, 1u);
      if (prev == gridDim.x - 1) {
        me->arrive = 0;
        for (int p = 0; p < world; ++p) {
          SymmHeader* peer = reinterpret_cast<SymmHeader*>(a.bases[p]);
          st_release_sys(&peer->flag_b[a.rank], epoch);
        }
      }
    }
    if (threadIdx.x < world) {
      if (!wait_geq(&me->flag_b[threadIdx.x], epoch, a.timeout_ns)) {
        atomicOr(&me->status, kStatusPeerTimeout);
        s_ok = 0;
      }
    }
    __syncthreads();
  }
  // ---- phase 2: gather rows (or reduce all rows, one-shot) + RMSNorm; with many rows per CTA, kRows
  // rows per iteration whose loads are all in flight before the first row's sum of squares is
  // reduced (one row per iteration otherwise: the most CTAs busy for decode-sized T)
  constexpr int kRows = 4;
  const int nr = a.T > kRows * (int)gridDim.x ? kRows : 1;
  const int chunk = (a.T + world - 1) / world;
  for (int row0 = blockIdx.x * nr; row0 < a.T; row0 += gridDim.x * nr) {
    // each thread owns up to 2 vectors of each row (d <= 8192)
    float vals[kRows][2][8];
    float ss[kRows];
#pragma unroll
    for (int j = 0; j < kRows; ++j) {
      ss[j] = 0.f;
      const int row = j < nr ? row0 + j : a.T;
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const int v = threadIdx.x + k * kArThreads;
        if (row < a.T && v < nvec) {
          const int64_t off = (int64_t)row * a.d + v * 8;
          if (a.one_shot) {
            bf16x8_to_float(*reinterpret_cast<const uint4*>(residual + off), vals[j][k]);
            add_ranks(vals[j][k], a, a.partial_off[a.parity], off);
          } else {
            const int owner = min(row / chunk, world - 1);
            const __nv_bfloat16* src = reinterpret_cast<const __nv_bfloat16*>(a.bases[owner] + a.gather_off);
            bf16x8_to_float(*reinterpret_cast<const uint4*>(src + off), vals[j][k]);
          }
        }
      }
    }
#pragma unroll
    for (int j = 0; j < kRows; ++j) {
      const int row = j < nr ? row0 + j : a.T;
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const int v = threadIdx.x + k * kArThreads;
        if (row < a.T && v < nvec) {
          const int64_t off = (int64_t)row * a.d + v * 8;
          uint4 packed = float_to_bf16x8(vals[j][k]);
          if (a.one_shot) bf16x8_to_float(packed, vals[j][k]);  // normalise the rounded residual
          *reinterpret_cast<uint4*>(residual + off) = packed;
#pragma unroll
          for (int e = 0; e < 8; ++e) ss[j] += vals[j][k][e] * vals[j][k][e];
        }
      }
      ss[j] = warp_sum(ss[j]);
    }
    if ((threadIdx.x & 31) == 0) {
#pragma unroll
      for (int j = 0; j < kRows; ++j) red[j * (kArThreads / 32) + (threadIdx.x >> 5)] = ss[j];
    }
    __syncthreads();
    if (threadIdx.x < 32) {
#pragma unroll
      for (int j = 0; j < kRows; ++j) {
        float t = threadIdx.x < kArThreads / 32 ? red[j * (kArThreads / 32) + threadIdx.x] : 0.f;
        t = warp_sum(t);
        if (threadIdx.x == 0) red_rows[j] = t;
      }
    }
    __syncthreads();
#pragma unroll
    for (int j = 0; j < kRows; ++j) {
      const int row = j < nr ? row0 + j : a.T;
      const float rs = rsqrtf(red_rows[j] / (float)a.d + a.eps);
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const int v = threadIdx.x + k * kArThreads;
        if (row < a.T && v < nvec) {
          float wf[8];
          bf16x8_to_float(*reinterpret_cast<const uint4*>(w + v * 8), wf);
#pragma unroll
          for (int e = 0; e < 8; ++e) vals[j][k][e] = vals[j][k][e] * rs * wf[e];
          *reinterpret_cast<uint4*>(x_out + (int64_t)row * a.d + v * 8) = float_to_bf16x8(vals[j][k]);
        }
      }
    }
    __syncthreads();
  }
  // ---- epilogue: the call is complete on this rank once every CTA got here; CTA 0 records it
  if (a.one_shot) {
    __syncthreads();
    if (threadIdx.x == 0) {
      const uint32_t prev = atomicAdd(&me->arrive, 1u);
      if (prev == gridDim.x - 1) {
        me->arrive = 0;
        me->epoch = epoch;
      }
    }
  } else if (blockIdx.x == 0 && threadIdx.x == 0) {
    me->epoch = epoch;  // every CTA read the epoch before barrier B completed
  }
}

// Consumer of the push path: the row-parallel GEMM of every rank already stored its partial
// tiles into this rank's inbox and raised per-(source, 32-row group, n-tile) flags. For each row:
// wait (bounded) for the flags of its group from every source, then residual + Σ_p inbox[p][row]
// in rank order (identical on every rank) → new residual, RMSNorm → x. All reads are local.
__global__ void __launch_bounds__(kArThreads) tp_push_ar_rmsnorm_kernel(PushArgs a, int nt, int T, int d, float eps,
                                                                         uint64_t timeout_ns,
                                                                         __nv_bfloat16* __restrict__ residual,
                                                                         const __nv_bfloat16* __restrict__ w,
                                                                         __nv_bfloat16* __restrict__ x_out) {
  SymmHeader* me = reinterpret_cast<SymmHeader*>(a.bases[a.rank]);
  const uint32_t* flags = reinterpret_cast<const uint32_t*>(a.bases[a.rank] + a.flags_off);
  const __nv_bfloat16* inbox = reinterpret_cast<const __nv_bfloat16*>(a.bases[a.rank] + a.inbox_off);
  __shared__ uint32_t s_epoch;
  __shared__ float red[kArThreads / 32];
  __shared__ int s_group;
  if (threadIdx.x == 0) {
    s_epoch = *reinterpret_cast<volatile uint32_t*>(&me->epoch) + 1;
    s_group = -1;
  }
  __syncthreads();
  const uint32_t epoch = s_epoch;
  const int nvec = d / 8;
  for (int row = blockIdx.x; row < T; row += gridDim.x) {
    const int g = row >> 5;
    if (g != s_group) {  // uniform across the CTA
      for (int i = threadIdx.x; i < a.world * nt; i += blockDim.x) {
        const int p = i / nt, t = i % nt;
        if (!wait_geq(flags + ((int64_t)p * a.g_max + g) * a.nt_max + t, epoch, timeout_ns))
          atomicOr(&me->status, kStatusPeerTimeout);
      }
      __syncthreads();
      if (threadIdx.x == 0) s_group = g;
    }
    const int64_t base = (int64_t)row * d;
    float ss = 0.f;
    float vals[2][8];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int v = threadIdx.x + k * kArThreads;
      if (v < nvec) {
        const int64_t off = base + v * 8;
        bf16x8_to_float(*reinterpret_cast<const uint4*>(residual + off), vals[k]);
        uint4 in[kMaxWorld];
#pragma unroll
        for (int p = 0; p < kMaxWorld; ++p)
          if (p < a.world) in[p] = *reinterpret_cast<const uint4*>(inbox + (int64_t)p * a.slot_elems + off);
#pragma unroll
        for (int p = 0; p < kMaxWorld; ++p) {
          if (p < a.world) {
            float t[8];
            bf16x8_to_float(in[p], t);
#pragma unroll
            for (int e = 0; e < 8; ++e) vals[k][e] += t[e];
          }
        }
        const uint4 packed = float_to_bf16x8(vals[k]);
        bf16x8_to_float(packed, vals[k]);
        *reinterpret_cast<uint4*>(residual + off) = packed;
#pragma unroll
        for (int e = 0; e < 8; ++e) ss += vals[k][e] * vals[k][e];
      }
    }
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x < 32) {
      float t = threadIdx.x < kArThreads / 32 ? red[threadIdx.x] : 0.f;
      t = warp_sum(t);
      if (threadIdx.x == 0) red[0] = t;
    }
    __syncthreads();
    const float rs = rsqrtf(red[0] / (float)d + eps);
    __syncthreads();
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int v = threadIdx.x + k * kArThreads;
      if (v < nvec) {
        float wf[8];
        bf16x8_to_float(*reinterpret_cast<const uint4*>(w + v * 8), wf);
#pragma unroll
        for (int e = 0; e < 8; ++e) vals[k][e] = vals[k][e] * rs * wf[e];
        *reinterpret_cast<uint4*>(x_out + base + v * 8) = float_to_bf16x8(vals[k]);
      }
    }
  }
  // the call is complete on this rank once every CTA got here
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint32_t prev = atomicAdd(&me->arrive, 1u);
    if (prev == gridDim.x - 1) {
      me->arrive = 0;
      me->epoch = epoch;
    }
  }
}

// C5: distributed greedy argmax of a vocab-parallel lm_head. CTA b takes row b of this rank's
// logit shard, finds its (max, lowest index) and stores the packed candidate — the float's
// order-preserving key in the high word, ~global index in the low word, so one unsigned max
// picks the larger logit and, among equal logits, the lower token id — into slot [rank][b] of
// every rank's candidate array (double-buffered by call parity). The last CTA to finish
// publishes flag_b[rank] = epoch to every peer, waits (bounded) for every peer's flag and
// reduces the W candidates of every row into `out`. Only B x W x 8 bytes cross NVLink instead of
// the B x V logits an all-gather would move.
GOLLEK_DEVICE uint32_t float_order_key(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__global__ void __launch_bounds__(kArThreads) tp_argmax_kernel(ArArgs a, const __nv_bfloat16* __restrict__ logits,
                                                               int64_t stride, int V, int64_t vocab_offset, int B,
                                                               int64_t cand_off, int cand_rows, int parity,
                                                               int64_t* __restrict__ out) {
  SymmHeader* me = reinterpret_cast<SymmHeader*>(a.bases[a.rank]);
  __shared__ uint32_t s_epoch;
  __shared__ unsigned long long s_best[kArThreads / 32];
  __shared__ int s_last;
  if (threadIdx.x == 0) s_epoch = *reinterpret_cast<volatile uint32_t*>(&me->epoch) + 1;
  __syncthreads();
  const uint32_t epoch = s_epoch;
  const int b = blockIdx.x;
  const __nv_bfloat16* row = logits + (int64_t)b * stride;
  unsigned long long best = 0ull;
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    const float f = __bfloat162float(row[i]);
    const unsigned long long key = ((unsigned long long)float_order_key(f) << 32) |
                                   (uint32_t)~(uint32_t)(vocab_offset + i);
    best = key > best ? key : best;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
    best = other > best ? other : best;
  }
  if ((threadIdx.x & 31) == 0) s_best[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < kArThreads / 32; ++w) best = s_best[w] > best ? s_best[w] : best;
    best = s_best[0] > best ? s_best[0] : best;
    const int64_t slot = ((int64_t)parity * a.world + a.rank) * cand_rows + b;
    for (int p = 0; p < a.world; ++p)
      reinterpret_cast<unsigned long long*>(a.bases[p] + cand_off)[slot] = best;
    __threadfence_system();
    const uint32_t prev = atomicAdd(&me->arrive, 1u);
    s_last = prev == gridDim.x - 1;
  }
  __syncthreads();
  if (!s_last) return;
  // last CTA: publish, wait for every peer, reduce every row
  if (threadIdx.x < a.world) {
    SymmHeader* peer = reinterpret_cast<SymmHeader*>(a.bases[threadIdx.x]);
    st_release_sys(&peer->flag_b[a.rank], epoch);
  }
  if (threadIdx.x < a.world && !wait_geq(&me->flag_b[threadIdx.x], epoch, a.timeout_ns))
    atomicOr(&me->status, kStatusPeerTimeout);
  __syncthreads();
  const unsigned long long* cand = reinterpret_cast<const unsigned long long*>(a.bases[a.rank] + cand_off);
  for (int r = threadIdx.x; r < B; r += blockDim.x) {
    unsigned long long m = 0ull;
    for (int p = 0; p < a.world; ++p) {
      const unsigned long long c = *reinterpret_cast<volatile const unsigned long long*>(
          &cand[((int64_t)parity * a.world + p) * cand_rows + r]);
      m = c > m ? c : m;
    }
    out[r] = (int64_t)(uint32_t)~(uint32_t)(m & 0xffffffffull);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    me->arrive = 0;
    me->epoch = epoch;
  }
}

// Plain all-reduce (sum) of the partial buffer into `out` (no residual / norm), one-shot.
__global__ void __launch_bounds__(kArThreads) tp_allreduce_kernel(ArArgs a, __nv_bfloat16* __restrict__ out,
                                                                  int64_t nvec_total) {
  SymmHeader* me = reinterpret_cast<SymmHeader*>(a.bases[a.rank]);
  __shared__ uint32_t s_epoch;
  if (threadIdx.x == 0) s_epoch = *reinterpret_cast<volatile uint32_t*>(&me->epoch) + 1;
  __syncthreads();
  const uint32_t epoch = s_epoch;
  if (blockIdx.x == 0 && threadIdx.x < a.world) {
    __threadfence_system();
    SymmHeader* peer = reinterpret_cast<SymmHeader*>(a.bases[threadIdx.x]);
    st_release_sys(&peer->flag_a[a.rank], epoch);
  }
  if (threadIdx.x < a.world && !wait_geq(&me->flag_a[threadIdx.x], epoch, a.timeout_ns))
    atomicOr(&me->status, kStatusPeerTimeout);
  __syncthreads();
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nvec_total;
       i += (int64_t)gridDim.x * blockDim.x) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    add_ranks(acc, a, a.partial_off[a.parity], i * 8);
    *reinterpret_cast<uint4*>(out + i * 8) = float_to_bf16x8(acc);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint32_t prev = atomicAdd(&me->arrive, 1u);
    if (prev == gridDim.x - 1) {
      me->arrive = 0;
      me->epoch = epoch;
    }
  }
}

// All-gather of column shards over P2P (vocab-parallel logits without NVLS): rank r stores its
// [B, v] shard into columns [r*v, (r+1)*v) of the [B, ld] buffer at `dst_off` of every rank
// (plain 16-byte stores over NVLink, 2-byte stores when the shard is not a whole number of
// vectors). Barrier A first (no rank overwrites a buffer a peer may still read); the last CTA
// then publishes flag_b and waits for every peer's, so the gathered rows are complete when the
// kernel ends.
__global__ void __launch_bounds__(kArThreads) tp_gather_cols_kernel(ArArgs a, const __nv_bfloat16* __restrict__ src,
                                                                    int64_t src_stride, int B, int v, int64_t dst_off,
                                                                    int64_t ld, int vec) {
  SymmHeader* me = reinterpret_cast<SymmHeader*>(a.bases[a.rank]);
  __shared__ uint32_t s_epoch;
  __shared__ int s_last;
  if (threadIdx.x == 0) s_epoch = *reinterpret_cast<volatile uint32_t*>(&me->epoch) + 1;
  __syncthreads();
  const uint32_t epoch = s_epoch;
  if (blockIdx.x == 0 && threadIdx.x < a.world) {
    SymmHeader* peer = reinterpret_cast<SymmHeader*>(a.bases[threadIdx.x]);
    st_release_sys(&peer->flag_a[a.rank], epoch);
  }
  if (threadIdx.x < a.world && !wait_geq(&me->flag_a[threadIdx.x], epoch, a.timeout_ns))
    atomicOr(&me->status, kStatusPeerTimeout);
  __syncthreads();
  const int64_t col0 = (int64_t)a.rank * v;
  const int64_t step = (int64_t)gridDim.x * blockDim.x;
  if (vec) {
    const int vv = v / 8;
    const int64_t total = (int64_t)B * vv;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += step) {
      const int64_t row = i / vv, c = (i % vv) * 8;
      const uint4 x = *reinterpret_cast<const uint4*>(src + row * src_stride + c);
#pragma unroll
      for (int p = 0; p < kMaxWorld; ++p)
        if (p < a.world)
          *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(a.bases[p] + dst_off) + row * ld + col0 + c) = x;
    }
  } else {
    const int64_t total = (int64_t)B * v;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += step) {
      const int64_t row = i / v, c = i % v;
      const __nv_bfloat16 x = src[row * src_stride + c];
      for (int p = 0; p < a.world; ++p)
        reinterpret_cast<__nv_bfloat16*>(a.bases[p] + dst_off)[row * ld + col0 + c] = x;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    const uint32_t prev = atomicAdd(&me->arrive, 1u);
    s_last = prev == gridDim.x - 1;
  }
  __syncthreads();
  if (!s_last) return;
  if (threadIdx.x < a.world) {
    SymmHeader* peer = reinterpret_cast<SymmHeader*>(a.bases[threadIdx.x]);
    st_release_sys(&peer->flag_b[a.rank], epoch);
  }
  if (threadIdx.x < a.world && !wait_geq(&me->flag_b[threadIdx.x], epoch, a.timeout_ns))
    atomicOr(&me->status, kStatusPeerTimeout);
  __syncthreads();
  if (threadIdx.x == 0) {
    me->arrive = 0;
    me->epoch = epoch;
  }
}

// ------------------------------------------------------------------------------- host side
void* symm_alloc(size_t bytes) {
  void* p = nullptr;
  GOLLEK_CUDA_CHECK(cudaMalloc(&p, bytes));
  GOLLEK_CUDA_CHECK(cudaMemset(p, 0, bytes));
  return p;
}

void symm_free(void* p) { cudaFree(p); }

std::vector<uint8_t> symm_ipc_handle(void* p) {
  cudaIpcMemHandle_t h;
  GOLLEK_CUDA_CHECK(cudaIpcGetMemHandle(&h, p));
  const uint8_t* b = reinterpret_cast<const uint8_t*>(&h);
  return std::vector<uint8_t>(b, b + sizeof(h));
}

void* symm_open_peer(const std::vector<uint8_t>& handle) {
  throw_if(handle.size() != sizeof(cudaIpcMemHandle_t), "bad IPC handle size");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle.data(), sizeof(h));
  void* p = nullptr;
  GOLLEK_CUDA_CHECK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  return p;
}

void symm_close_peer(void* p) { cudaIpcCloseMemHandle(p); }

static ArArgs make_args(const std::vector<uint64_t>& bases, int rank, int64_t p0, int64_t p1, int64_t g, int T,
                        int d, int parity, bool one_shot, float eps, double timeout_s) {
  ArArgs a{};
  throw_if(bases.size() > 8 || bases.empty(), "tp collectives support 1..8 ranks");
  for (size_t i = 0; i < bases.size(); ++i) a.bases[i] = reinterpret_cast<uint8_t*>(bases[i]);
  a.partial_off[0] = p0;
  a.partial_off[1] = p1;
  a.gather_off = g;
  a.rank = rank;
  a.world = (int)bases.size();
  a.T = T;
  a.d = d;
  a.parity = parity;
  a.one_shot = one_shot ? 1 : 0;
  a.eps = eps;
  a.timeout_ns = (uint64_t)(timeout_s * 1e9);
  return a;
}

void launch_tp_ar_rmsnorm(const std::vector<uint64_t>& bases, int rank, int64_t p0, int64_t p1, int64_t g,
                          int parity, bool one_shot, void* residual, const void* w, void* x_out, int T, int d,
                          float eps, double timeout_s, int grid, cudaStream_t s) {
  throw_if(d % 8 != 0 || d > 16 * kArThreads, "tp all-reduce: hidden size must be a multiple of 8, <= 8192");
  if (T == 0) return;
  ArArgs a = make_args(bases, rank, p0, p1, g, T, d, parity, one_shot, eps, timeout_s);
  tp_ar_rmsnorm_kernel<<<grid, kArThreads, 0, s>>>(a, reinterpret_cast<__nv_bfloat16*>(residual),
                                                   reinterpret_cast<const __nv_bfloat16*>(w),
                                                   reinterpret_cast<__nv_bfloat16*>(x_out));
  check_launch("tp_allreduce_add_rmsnorm");
}

void launch_tp_allreduce(const std::vector<uint64_t>& bases, int rank, int64_t p0, int64_t p1, int parity, void* out,
                         int64_t numel, double timeout_s, int grid, cudaStream_t s) {
  throw_if(numel % 8 != 0, "tp all-reduce: element count must be a multiple of 8");
  if (numel == 0) return;
  ArArgs a = make_args(bases, rank, p0, p1, 0, 0, 0, parity, true, 0.f, timeout_s);
  tp_allreduce_kernel<<<grid, kArThreads, 0, s>>>(a, reinterpret_cast<__nv_bfloat16*>(out), numel / 8);
  check_launch("tp_allreduce");
}

void launch_tp_push_ar_rmsnorm(const std::vector<uint64_t>& bases, int rank, int64_t inbox_off, int64_t slot_elems,
                               int64_t flags_off, int g_max, int nt_max, int nt, void* residual, const void* w,
                               void* x_out, int T, int d, float eps, double timeout_s, int grid, cudaStream_t s) {
  throw_if(d % 8 != 0 || d > 16 * kArThreads, "tp push all-reduce: hidden size must be a multiple of 8, <= 8192");
  throw_if(bases.empty() || bases.size() > 8, "tp push all-reduce: 1..8 ranks");
  throw_if((T + 31) / 32 > g_max || nt > nt_max, "tp push all-reduce: flag array too small for this call");
  if (T == 0) return;
  PushArgs p{};
  for (size_t i = 0; i < bases.size(); ++i) p.bases[i] = reinterpret_cast<uint8_t*>(bases[i]);
  p.inbox_off = inbox_off;
  p.slot_elems = slot_elems;
  p.flags_off = flags_off;
  p.world = (int)bases.size();
  p.rank = rank;
  p.g_max = g_max;
  p.nt_max = nt_max;
  tp_push_ar_rmsnorm_kernel<<<grid, kArThreads, 0, s>>>(p, nt, T, d, eps, (uint64_t)(timeout_s * 1e9),
                                                        reinterpret_cast<__nv_bfloat16*>(residual),
                                                        reinterpret_cast<const __nv_bfloat16*>(w),
                                                        reinterpret_cast<__nv_bfloat16*>(x_out));
  check_launch("tp_push_allreduce_add_rmsnorm");
}

void launch_tp_argmax(const std::vector<uint64_t>& bases, int rank, const void* logits, int64_t stride, int B, int V,
                      int64_t vocab_offset, int64_t cand_off, int cand_rows, int parity, int64_t* out,
                      double timeout_s, cudaStream_t s) {
  throw_if(B > cand_rows, "tp argmax: more rows than candidate slots");
  throw_if(cand_off % 8 != 0, "tp argmax: candidate array must be 8-byte aligned");
  if (B == 0) return;
  ArArgs a = make_args(bases, rank, 0, 0, 0, 0, 0, 0, true, 0.f, timeout_s);
  tp_argmax_kernel<<<B, kArThreads, 0, s>>>(a, reinterpret_cast<const __nv_bfloat16*>(logits), stride, V,
                                            vocab_offset, B, cand_off, cand_rows, parity, out);
  check_launch("tp_argmax");
}

void launch_tp_gather_cols(const std::vector<uint64_t>& bases, int rank, const void* src, int64_t src_stride, int B,
                           int v, int64_t dst_off, int64_t ld, double timeout_s, int grid, cudaStream_t s) {
  throw_if(ld < (int64_t)bases.size() * v, "tp column gather: destination row narrower than world * v");
  throw_if(dst_off % 16 != 0, "tp column gather: destination offset must be 16-byte aligned");
  if (B == 0) return;
  ArArgs a = make_args(bases, rank, 0, 0, 0, 0, 0, 0, true, 0.f, timeout_s);
  const bool vec = v % 8 == 0 && src_stride % 8 == 0 && ld % 8 == 0 && reinterpret_cast<uintptr_t>(src) % 16 == 0;
  tp_gather_cols_kernel<<<grid, kArThreads, 0, s>>>(a, reinterpret_cast<const __nv_bfloat16*>(src), src_stride, B, v,
                                                    dst_off, ld, vec ? 1 : 0);
  check_launch("tp_gather_cols");
}

uint32_t symm_read_status(void* base) {
  uint32_t st = 0;
  GOLLEK_CUDA_CHECK(cudaMemcpy(&st, reinterpret_cast<uint8_t*>(base) + offsetof(SymmHeader, status), 4,
                               cudaMemcpyDeviceToHost));
  return st;
}

}  // namespace gollek
