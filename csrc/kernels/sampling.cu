// K11: batched token sampling (sm_100a), one CTA per row, no sort.
//
//   argmax            greedy fast path (ties -> lowest token id)
//   apply_penalties   repetition (HF divide/multiply) over every listed token, frequency (x count)
//                     and presence (if count > 0) over generated ones; (row, token, count) triples
//   sample            temperature -> top-k (radix select of the k-th largest logit) -> min-p
//                     (closed-form threshold) -> top-p (radix search of the probability-mass
//                     threshold among survivors) -> exponential race (Gumbel-max) with a
//                     counter-based hash RNG, so the draw is reproducible from (seed, step).
//
// Reference sampler order: runner/safetensor/gollek-safetensor-engine/…/generation/TokenSampler.java:62-208
// and the llama.cpp chain in runner/llamacpp/gollek-runner-llamacpp/…/LlamaHandles.java:174-203.
#include "../common/common.cuh"
#include "launchers.h"

using namespace gollek;

namespace {

constexpr int kSampThreads = 1024;

template <typename T>
GOLLEK_DEVICE float to_f(T v);
template <>
GOLLEK_DEVICE float to_f<float>(float v) { return v; }
template <>
GOLLEK_DEVICE float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

GOLLEK_DEVICE uint32_t ord_key(float f) {
  uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// 32-bit integer hash (xor-shift-multiply finaliser, constants 0x7feb352d / 0x846ca68b).
GOLLEK_DEVICE uint32_t hash32(uint32_t x) {
  x ^= x >> 16;
  x *= 0x7feb352du;
  x ^= x >> 15;
  x *= 0x846ca68bu;
  x ^= x >> 16;
  return x;
}

struct ArgMax {
  float v;
  int i;
};
GOLLEK_DEVICE ArgMax better(ArgMax a, ArgMax b) {
  if (b.v > a.v || (b.v == a.v && b.i < a.i)) return b;
  return a;
}
GOLLEK_DEVICE ArgMax warp_argmax(ArgMax a) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    ArgMax b;
    b.v = __shfl_xor_sync(0xffffffffu, a.v, o);
    b.i = __shfl_xor_sync(0xffffffffu, a.i, o);
    a = better(a, b);
  }
  return a;
}
GOLLEK_DEVICE ArgMax block_argmax(ArgMax a, ArgMax* sh) {
  a = warp_argmax(a);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) sh[w] = a;
  __syncthreads();
  if (w == 0) {
    ArgMax b = (l < (int)(blockDim.x >> 5)) ? sh[l] : ArgMax{-INFINITY, 0x7fffffff};
    b = warp_argmax(b);
    if (l == 0) sh[0] = b;
  }
  __syncthreads();
  ArgMax r = sh[0];
  __syncthreads();
  return r;
}
GOLLEK_DEVICE float block_sum(float v, float* sh) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) sh[w] = v;
  __syncthreads();
  if (w == 0) {
    float b = (l < (int)(blockDim.x >> 5)) ? sh[l] : 0.f;
    b = warp_sum(b);
    if (l == 0) sh[0] = b;
  }
  __syncthreads();
  float r = sh[0];
  __syncthreads();
  return r;
}

template <typename T>
__global__ void __launch_bounds__(kSampThreads) argmax_kernel(int64_t* __restrict__ out, const T* __restrict__ logits,
                                                              int V, int64_t stride) {
  __shared__ ArgMax sh[32];
  const T* row = logits + (int64_t)blockIdx.x * stride;
  ArgMax best{-INFINITY, 0x7fffffff};
  // 16-byte vector loads when the row is aligned (8 bf16 / 4 fp32 per load), two in flight
  constexpr int kVec = 16 / sizeof(T);
  const bool aligned = ((reinterpret_cast<uintptr_t>(row) & 15) == 0);
  const int nv = aligned ? V / kVec : 0;
  for (int v = threadIdx.x; v < nv; v += 2 * blockDim.x) {
    const int v2 = v + blockDim.x;
    const uint4 a = __ldg(reinterpret_cast<const uint4*>(row) + v);
    const uint4 b = v2 < nv ? __ldg(reinterpret_cast<const uint4*>(row) + v2) : a;
    const T* ea = reinterpret_cast<const T*>(&a);
    const T* eb = reinterpret_cast<const T*>(&b);
#pragma unroll
    for (int e = 0; e < kVec; ++e) best = better(best, ArgMax{to_f(ea[e]), v * kVec + e});
    if (v2 < nv) {
#pragma unroll
      for (int e = 0; e < kVec; ++e) best = better(best, ArgMax{to_f(eb[e]), v2 * kVec + e});
    }
  }
  for (int i = nv * kVec + threadIdx.x; i < V; i += blockDim.x) best = better(best, ArgMax{to_f(row[i]), i});
  best = block_argmax(best, sh);
  if (threadIdx.x == 0) out[blockIdx.x] = best.i == 0x7fffffff ? 0 : best.i;
}

// triples: [n, 3] int32 (row, token, count); logits updated in place (fp32).
__global__ void penalties_kernel(float* __restrict__ logits, int64_t stride, const int* __restrict__ triples, int n,
                                 const float* __restrict__ rep, const float* __restrict__ freq,
                                 const float* __restrict__ pres) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int r = triples[3 * i], tok = triples[3 * i + 1], cnt = triples[3 * i + 2];
  float* p = logits + (int64_t)r * stride + tok;
  float v = *p;
  const float rp = rep[r];
  v = v > 0.f ? v / rp : v * rp;
  v -= freq[r] * (float)cnt + (cnt > 0 ? pres[r] : 0.f);
  *p = v;
}

// Calls f(value, index) for every element of a row: 16-byte vector loads when the row is aligned.
template <typename T, typename F>
GOLLEK_DEVICE void for_each_elem(const T* row, int V, F&& f) {
  constexpr int kVec = 16 / sizeof(T);
  const bool aligned = (reinterpret_cast<uintptr_t>(row) & 15) == 0;
  const int nv = aligned ? V / kVec : 0;
  for (int v = threadIdx.x; v < nv; v += blockDim.x) {
    const uint4 a = __ldg(reinterpret_cast<const uint4*>(row) + v);
    const T* e = reinterpret_cast<const T*>(&a);
#pragma unroll
    for (int j = 0; j < kVec; ++j) f(to_f(e[j]), v * kVec + j);
  }
  for (int i = nv * kVec + threadIdx.x; i < V; i += blockDim.x) f(to_f(row[i]), i);
}

constexpr int kHistCopies = kSampThreads / 32;  // one radix histogram per warp (no atomic contention)

// Sum the per-warp histograms into copy 0.
template <typename H>
GOLLEK_DEVICE void hist_reduce(H* hist) {
  __syncthreads();
  for (int b = threadIdx.x; b < 256; b += blockDim.x) {
    H t = 0;
    for (int c = 0; c < kHistCopies; ++c) t += hist[c * 256 + b];
    hist[b] = t;
  }
  __syncthreads();
}

// Radix select: largest key K such that #{keys >= K} >= k (i.e. the k-th largest key).
template <typename T>
GOLLEK_DEVICE uint32_t radix_kth_largest(const T* row, int V, int k, uint32_t* hist, uint32_t* sh_u) {
  uint32_t prefix = 0, mask = 0;
  int remaining = k;
  uint32_t* mine = hist + (threadIdx.x >> 5) * 256;
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = threadIdx.x; i < 256 * kHistCopies; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    for_each_elem(row, V, [&](float x, int) {
      const uint32_t key = ord_key(x);
      if ((key & mask) == prefix) atomicAdd(&mine[(key >> shift) & 255u], 1u);
    });
    hist_reduce(hist);
    if (threadIdx.x == 0) {
      int cum = 0, bin = 0;
      for (bin = 255; bin >= 0; --bin) {
        if (cum + (int)hist[bin] >= remaining) break;
        cum += hist[bin];
      }
      if (bin < 0) bin = 0;
      sh_u[0] = (uint32_t)bin;
      sh_u[1] = (uint32_t)(remaining - cum);
    }
    __syncthreads();
    prefix |= sh_u[0] << shift;
    mask |= 255u << shift;
    remaining = (int)sh_u[1];
    __syncthreads();
  }
  return prefix;
}

// Radix search of the mass threshold: largest key K such that sum_{key >= K} w >= target,
// over elements with key >= floor_key, where w = exp2((x - m) * inv_t_log2).
template <typename T>
GOLLEK_DEVICE uint32_t radix_mass_threshold(const T* row, int V, uint32_t floor_key, float m, float inv_t_log2,
                                            float target, float* hist_f, uint32_t* sh_u, float* sh_f) {
  uint32_t prefix = 0, mask = 0;
  float above = 0.f;
  float* mine = hist_f + (threadIdx.x >> 5) * 256;
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = threadIdx.x; i < 256 * kHistCopies; i += blockDim.x) hist_f[i] = 0.f;
    __syncthreads();
    for_each_elem(row, V, [&](float x, int) {
      const uint32_t key = ord_key(x);
      if (key >= floor_key && (key & mask) == prefix) atomicAdd(&mine[(key >> shift) & 255u], exp2f((x - m) * inv_t_log2));
    });
    hist_reduce(hist_f);
    if (threadIdx.x == 0) {
      float cum = above;
      int bin;
      for (bin = 255; bin >= 0; --bin) {
        if (cum + hist_f[bin] >= target) break;
        cum += hist_f[bin];
      }
      if (bin < 0) bin = 0;
      sh_u[0] = (uint32_t)bin;
      sh_f[0] = cum;
    }
    __syncthreads();
    prefix |= sh_u[0] << shift;
    mask |= 255u << shift;
    above = sh_f[0];
    __syncthreads();
  }
  return prefix;
}

template <typename T>
__global__ void __launch_bounds__(kSampThreads) sample_kernel(int64_t* __restrict__ out, const T* __restrict__ logits,
                                                              int V, int64_t stride, const float* __restrict__ temps,
                                                              const int* __restrict__ top_ks,
                                                              const float* __restrict__ top_ps,
                                                              const float* __restrict__ min_ps,
                                                              const int64_t* __restrict__ seeds,
                                                              const int64_t* __restrict__ offsets) {
  __shared__ ArgMax sha[32];
  __shared__ float shf[33];
  __shared__ uint32_t hist[256 * kHistCopies];
  __shared__ uint32_t sh_u[2];
  const int b = blockIdx.x;
  const T* row = logits + (int64_t)b * stride;
  const float t = temps[b];
  // 1) max
  ArgMax best{-INFINITY, 0x7fffffff};
  for_each_elem(row, V, [&](float x, int i) { best = better(best, ArgMax{x, i}); });
  best = block_argmax(best, sha);
  if (t <= 0.f) {
    if (threadIdx.x == 0) out[b] = best.i == 0x7fffffff ? 0 : best.i;
    return;
  }
  const float m = best.v;
  const float inv_t_log2 = 1.4426950408889634f / t;
  uint32_t floor_key = 0;
  // 2) top-k
  const int k = top_ks[b];
  if (k > 0 && k < V) floor_key = max(floor_key, radix_kth_largest(row, V, k, hist, sh_u));
  // 3) min-p: p_i >= min_p * p_max  <=>  x_i >= m + t * ln(min_p)
  const float mp = min_ps[b];
  if (mp > 0.f) floor_key = max(floor_key, ord_key(m + t * __logf(mp)));
  // 4) top-p over the survivors (renormalised)
  const float tp = top_ps[b];
  if (tp < 1.f) {
    float z = 0.f;
    for_each_elem(row, V, [&](float x, int) {
      if (ord_key(x) >= floor_key) z += exp2f((x - m) * inv_t_log2);
    });
    z = block_sum(z, shf);
    floor_key = max(floor_key, radix_mass_threshold(row, V, floor_key, m, inv_t_log2, tp * z,
                                                    reinterpret_cast<float*>(hist), sh_u, shf));
  }
  // 5) exponential race among survivors: argmax x/t + Gumbel(u)
  const uint32_t seed_mix = hash32((uint32_t)seeds[b] ^ hash32((uint32_t)offsets[b] + 0x9E3779B9u));
  ArgMax pick{-INFINITY, 0x7fffffff};
  for_each_elem(row, V, [&](float x, int i) {
    if (ord_key(x) < floor_key) return;
    const uint32_t h = hash32(seed_mix ^ hash32((uint32_t)i));
    const float u = ((float)(h >> 8) + 0.5f) * (1.0f / 16777216.0f);
    const float g = -__logf(-__logf(u));
    pick = better(pick, ArgMax{(x - m) / t + g, i});
  });
  pick = block_argmax(pick, sha);
  if (threadIdx.x == 0) out[b] = pick.i == 0x7fffffff ? best.i : pick.i;
}

}  // namespace

namespace gollek {

void launch_argmax(int64_t* out, const void* logits, bool is_bf16, int B, int V, int64_t stride, cudaStream_t s) {
  if (B == 0) return;
  if (is_bf16)
    argmax_kernel<__nv_bfloat16><<<B, kSampThreads, 0, s>>>(out, reinterpret_cast<const __nv_bfloat16*>(logits), V,
                                                            stride);
  else
    argmax_kernel<float><<<B, kSampThreads, 0, s>>>(out, reinterpret_cast<const float*>(logits), V, stride);
  check_launch("argmax");
}

void launch_penalties(float* logits, int64_t stride, const int* triples, int n, const float* rep, const float* freq,
                      const float* pres, cudaStream_t s) {
  if (n == 0) return;
  penalties_kernel<<<(n + 255) / 256, 256, 0, s>>>(logits, stride, triples, n, rep, freq, pres);
  check_launch("apply_penalties");
}

void launch_sample(int64_t* out, const void* logits, bool is_bf16, int B, int V, int64_t stride, const float* temps,
                   const int* top_ks, const float* top_ps, const float* min_ps, const int64_t* seeds,
                   const int64_t* offsets, cudaStream_t s) {
  if (B == 0) return;
  if (is_bf16)
    sample_kernel<__nv_bfloat16><<<B, kSampThreads, 0, s>>>(out, reinterpret_cast<const __nv_bfloat16*>(logits), V,
                                                            stride, temps, top_ks, top_ps, min_ps, seeds, offsets);
  else
    sample_kernel<float><<<B, kSampThreads, 0, s>>>(out, reinterpret_cast<const float*>(logits), V, stride, temps,
                                                    top_ks, top_ps, min_ps, seeds, offsets);
  check_launch("sample");
}

}  // namespace gollek
