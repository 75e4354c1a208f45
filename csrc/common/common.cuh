// Shared device helpers for the gollek_b200 sm_100a kernels.
//
// Everything here is written for sm_100a only: mbarrier / bulk-copy / TMA /
// tcgen05 wrappers are inline PTX. Every spin-wait is bounded: after
// GOLLEK_SPIN_LIMIT polls it records an error code in a device status word and
// returns false so the caller can drain and exit instead of hanging the GPU.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <stdexcept>
#include <string>

#define GOLLEK_DEVICE __device__ __forceinline__

#ifndef GOLLEK_SPIN_LIMIT
#define GOLLEK_SPIN_LIMIT (1u << 26)   // ~ tens of ms of polling before giving up
#endif

namespace gollek {

// ----------------------------------------------------------------------------
// Device status word: kernels OR an error code into it instead of trapping.
// ----------------------------------------------------------------------------
enum StatusCode : uint32_t {
  kStatusOk = 0,
  kStatusMbarTimeout = 1u << 0,     // an mbarrier wait ran out of polls
  kStatusPeerTimeout = 1u << 1,     // a cross-GPU flag wait ran out of polls
  kStatusBounds = 1u << 2,          // a bounds check failed (index recorded separately)
  kStatusBadArg = 1u << 3,
};

GOLLEK_DEVICE void report_status(uint32_t* status, uint32_t code) {
  if (status) atomicOr(status, code);
}

// Bounds checks of indices that kernels read from device memory (block-table entries, KV slots,
// token ids, gathered row indices). They are compiled in unless -DGOLLEK_BOUNDS_CHECK=0 and are
// active while the host has bound a status buffer (`bounds` != nullptr; a null pointer costs one
// uniform branch). An index outside [0, n) ORs kStatusBounds into bounds[0], records the first bad
// index in bounds[1] (sentinel 0xffffffff) and returns `safe` instead: a read then uses a valid
// index (a wrong result, never a fault), a write is skipped by its caller. Nothing traps.
#ifndef GOLLEK_BOUNDS_CHECK
#define GOLLEK_BOUNDS_CHECK 1
#endif
GOLLEK_DEVICE int checked_index(int i, int n, uint32_t* bounds, int safe = 0) {
#if GOLLEK_BOUNDS_CHECK
  if (bounds != nullptr && (i < 0 || i >= n)) {
    atomicOr(bounds, kStatusBounds);
    atomicCAS(bounds + 1, 0xffffffffu, (uint32_t)i);
    return safe;
  }
#endif
  return i;
}

// ----------------------------------------------------------------------------
// Small numeric helpers
// ----------------------------------------------------------------------------
// Hardware tanh (MUFU, one instruction, relative error ~2^-11): used for attention logit softcapping,
// whose result only feeds a bf16 probability.
GOLLEK_DEVICE float tanh_approx(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

GOLLEK_DEVICE float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
GOLLEK_DEVICE float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

struct __align__(16) bf16x8 { __nv_bfloat162 h[4]; };

GOLLEK_DEVICE void bf16x8_to_float(const uint4& u, float* f) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}
GOLLEK_DEVICE uint4 float_to_bf16x8(const float* f) {
  uint4 u;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
  return u;
}
GOLLEK_DEVICE uint32_t pack_bf16x2(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

GOLLEK_DEVICE float silu(float x) { return x / (1.0f + __expf(-x)); }
// GELU, tanh approximation (Hendrycks & Gimpel 2016): 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3)))
GOLLEK_DEVICE float gelu_tanh(float x) {
  const float u = 0.7978845608028654f * (x + 0.044715f * x * x * x);
  return 0.5f * x * (1.f + tanhf(u));
}

// ----------------------------------------------------------------------------
// Shared-memory address helpers
// ----------------------------------------------------------------------------
GOLLEK_DEVICE uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ----------------------------------------------------------------------------
// mbarrier (bounded waits)
// ----------------------------------------------------------------------------
GOLLEK_DEVICE void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
GOLLEK_DEVICE void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
GOLLEK_DEVICE void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
GOLLEK_DEVICE void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
GOLLEK_DEVICE bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Returns false (and records kStatusMbarTimeout) if the phase never completes.
GOLLEK_DEVICE bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t* status) {
  for (uint32_t i = 0; i < GOLLEK_SPIN_LIMIT; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
  }
  report_status(status, kStatusMbarTimeout);
  return false;
}

// ----------------------------------------------------------------------------
// Bulk async copies (TMA engine). No .multicast::cluster anywhere in this tree.
// ----------------------------------------------------------------------------
// Untiled bulk copy global -> shared; both addresses 16-byte aligned, bytes % 16 == 0.
GOLLEK_DEVICE void bulk_g2s(void* smem_dst, const void* gmem_src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// 2-D tiled TMA load (tensor map in param space). x is the innermost coordinate.
GOLLEK_DEVICE void tma_load_2d(void* smem_dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cta.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}
GOLLEK_DEVICE void tma_load_3d(void* smem_dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cta.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(
          smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}
GOLLEK_DEVICE void tma_store_2d(const CUtensorMap* map, const void* smem_src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(smem_src)), "r"(x), "r"(y)
               : "memory");
}
GOLLEK_DEVICE void tma_store_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
GOLLEK_DEVICE void tma_store_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
GOLLEK_DEVICE void tma_store_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
GOLLEK_DEVICE void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
GOLLEK_DEVICE void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// ----------------------------------------------------------------------------
// tcgen05 (5th-gen tensor core) wrappers, cta_group::1.
// ----------------------------------------------------------------------------
// Allocate ncols TMEM columns (power of two >= 32); whole warp executes. Address -> *dst (smem).
GOLLEK_DEVICE void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
GOLLEK_DEVICE void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
GOLLEK_DEVICE void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, kind::f16 (bf16/fp16 inputs, fp32 accumulate).
GOLLEK_DEVICE void umma_f16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                               uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// kind::f8f6f4 (e4m3 x e4m3 here), fp32 accumulate.
GOLLEK_DEVICE void umma_f8_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                              uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on an mbarrier once all previously issued tcgen05 ops of this thread complete.
GOLLEK_DEVICE void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}
GOLLEK_DEVICE void tcgen05_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
GOLLEK_DEVICE void tcgen05_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
GOLLEK_DEVICE void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 32 lanes x 32b, 16 consecutive columns per thread.
GOLLEK_DEVICE void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
// 32 lanes x 32b, 32 consecutive columns per thread.
GOLLEK_DEVICE void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
// Store 32 lanes x 32b, 16 columns per thread (used to stage P into TMEM).
GOLLEK_DEVICE void tmem_st_32x32b_x16(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
GOLLEK_DEVICE void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// UMMA shared-memory descriptor (sm100 "version 1"): K-major operand stored as rows of
// 128 bytes with the 128-byte swizzle, 8-row core groups 1024 bytes apart.
GOLLEK_DEVICE uint64_t make_smem_desc_sw128(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr & 0x3FFFF) >> 4);        // start address  [0,14)
  d |= (uint64_t)(16 >> 4) << 16;                     // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;                   // stride byte offset: 8 rows * 128 B
  d |= (uint64_t)1 << 46;                             // version = 1 (sm100)
  d |= (uint64_t)2 << 61;                             // layout: SWIZZLE_128B
  return d;
}

// Instruction descriptor for kind::f16: bf16 A/B (K-major), fp32 D, shape M x N.
__host__ __device__ constexpr uint32_t make_idesc_bf16(int M, int N) {
  return (1u << 4)                       // D format f32
         | (1u << 7)                     // A format bf16
         | (1u << 10)                    // B format bf16
         | ((uint32_t)(N >> 3) << 17)    // N >> 3
         | ((uint32_t)(M >> 4) << 24);   // M >> 4
}
// Instruction descriptor for kind::f8f6f4: e4m3 A/B (K-major), fp32 D.
__host__ __device__ constexpr uint32_t make_idesc_e4m3(int M, int N) {
  return (1u << 4) | (0u << 7) | (0u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

GOLLEK_DEVICE uint32_t elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .b32 %%rx;\n\t.reg .pred %%px;\n\t"
      "elect.sync %%rx|%%px, %1;\n\t"
      "@%%px mov.s32 %0, 1;\n\t}"
      : "+r"(pred)
      : "r"(0xffffffffu));
  return pred;
}

// ----------------------------------------------------------------------------
// Cross-GPU (system scope) flag helpers for the P2P collectives.
// ----------------------------------------------------------------------------
GOLLEK_DEVICE void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
GOLLEK_DEVICE uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
GOLLEK_DEVICE uint32_t ld_volatile_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.volatile.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// Wait until *flag >= target. Bounded; returns false and flags kStatusPeerTimeout on timeout.
GOLLEK_DEVICE bool wait_flag_geq(const uint32_t* flag, uint32_t target, uint32_t* status) {
  for (uint32_t i = 0; i < GOLLEK_SPIN_LIMIT; ++i) {
    if ((int32_t)(ld_acquire_sys(flag) - target) >= 0) return true;
  }
  report_status(status, kStatusPeerTimeout);
  return false;
}

}  // namespace gollek

#define GOLLEK_CUDA_CHECK(expr)                                                                   \
  do {                                                                                            \
    cudaError_t _e = (expr);                                                                      \
    if (_e != cudaSuccess)                                                                        \
      throw std::runtime_error(std::string("CUDA error: ") + cudaGetErrorString(_e) + " at " +   \
                               __FILE__ + ":" + std::to_string(__LINE__));                       \
  } while (0)
