// Memory-bound fused elementwise kernels (sm_100a):
//   K1  rms_norm / fused_add_rms_norm   (+ residual add, one HBM pass)
//   K2  rope_kv_write                   (QKV split + NeoX RoPE + paged KV-cache scatter)
//   K13 embedding gather
//   silu_mul (SwiGLU on a [gate | up] activation, used by the MoE path)
//
// Reference math: RMSNorm kernel/cuda/gollek-kernel-cuda/…/cuda/binding/CudaCpuFallback.java:181-211,
// SiLU·up :261-290, RoPE runner/safetensor/gollek-safetensor-engine/…/attention/RopeFrequencyCache.java:49-107,
// paged KV write …/attention/FlashAttentionKernel.java:166-194.
#include <ATen/cuda/CUDAContext.h>
#include <torch/extension.h>

#include "../common/common.cuh"

using namespace gollek;

namespace {

constexpr int kNormThreads = 256;

template <int MAXV, bool ADD>
__global__ void __launch_bounds__(kNormThreads) rms_norm_kernel(__nv_bfloat16* __restrict__ out,
                                                                const __nv_bfloat16* __restrict__ x,
                                                                __nv_bfloat16* __restrict__ residual,
                                                                const __nv_bfloat16* __restrict__ w, int d,
                                                                int64_t x_stride, int64_t out_stride, float eps) {
  const int row = blockIdx.x;
  const int nvec = d >> 3;
  const uint4* xr = reinterpret_cast<const uint4*>(x + (int64_t)row * x_stride);
  uint4* rr = ADD ? reinterpret_cast<uint4*>(residual + (int64_t)row * d) : nullptr;
  float v[MAXV][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    int idx = threadIdx.x + i * kNormThreads;
    if (idx < nvec) {
      bf16x8_to_float(xr[idx], v[i]);
      if (ADD) {
        float r[8];
        bf16x8_to_float(rr[idx], r);
#pragma unroll
        for (int j = 0; j < 8; ++j) v[i][j] += r[j];
        uint4 packed = float_to_bf16x8(v[i]);
        rr[idx] = packed;
        bf16x8_to_float(packed, v[i]);  // normalise the rounded residual, like the oracle
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += v[i][j] * v[i][j];
    }
  }
  __shared__ float red[kNormThreads / 32];
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < kNormThreads / 32 ? red[threadIdx.x] : 0.f;
    t = warp_sum(t);
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  const float rs = rsqrtf(red[0] / (float)d + eps);
  const uint4* wr = reinterpret_cast<const uint4*>(w);
  uint4* orow = reinterpret_cast<uint4*>(out + (int64_t)row * out_stride);
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    int idx = threadIdx.x + i * kNormThreads;
    if (idx < nvec) {
      float wf[8];
      bf16x8_to_float(wr[idx], wf);
#pragma unroll
      for (int j = 0; j < 8; ++j) v[i][j] = v[i][j] * rs * wf[j];
      orow[idx] = float_to_bf16x8(v[i]);
    }
  }
}

template <bool ADD>
void launch_rms_norm(torch::Tensor out, torch::Tensor x, torch::Tensor* residual, torch::Tensor w, double eps) {
  const int T = x.size(0), d = x.size(1);
  TORCH_CHECK(d % 8 == 0 && d <= 8 * 4 * kNormThreads, "rms_norm: hidden size must be a multiple of 8, <= 8192");
  TORCH_CHECK(x.stride(1) == 1 && out.stride(1) == 1, "rms_norm: rows must be contiguous");
  TORCH_CHECK(x.stride(0) % 8 == 0 && out.stride(0) % 8 == 0, "rms_norm: row stride must keep 16-byte alignment");
  if (T == 0) return;
  auto stream = at::cuda::getCurrentCUDAStream();
  auto* o = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  auto* xp = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  auto* rp = residual ? reinterpret_cast<__nv_bfloat16*>(residual->data_ptr()) : nullptr;
  auto* wp = reinterpret_cast<const __nv_bfloat16*>(w.data_ptr());
  const int nvec = d / 8;
  if (nvec <= kNormThreads)
    rms_norm_kernel<1, ADD><<<T, kNormThreads, 0, stream>>>(o, xp, rp, wp, d, x.stride(0), out.stride(0), eps);
  else if (nvec <= 2 * kNormThreads)
    rms_norm_kernel<2, ADD><<<T, kNormThreads, 0, stream>>>(o, xp, rp, wp, d, x.stride(0), out.stride(0), eps);
  else
    rms_norm_kernel<4, ADD><<<T, kNormThreads, 0, stream>>>(o, xp, rp, wp, d, x.stride(0), out.stride(0), eps);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ---------------------------------------------------------------------------------------------
// K2: RoPE + paged KV write. One CTA per token.
// ---------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(128) rope_kv_write_kernel(
    __nv_bfloat16* __restrict__ q_out, const __nv_bfloat16* __restrict__ qkv, const int* __restrict__ positions,
    const float* __restrict__ cos_sin, __nv_bfloat16* __restrict__ cache, const int* __restrict__ slots, int H,
    int Hk, int D, int block_size, int64_t qkv_stride, int max_pos) {
  const int t = blockIdx.x;
  const int half = D >> 1;
  int pos = positions[t];
  pos = pos < 0 ? 0 : (pos >= max_pos ? max_pos - 1 : pos);
  const float* cs = cos_sin + (int64_t)pos * D;
  const __nv_bfloat16* row = qkv + (int64_t)t * qkv_stride;
  const int slot = slots ? slots[t] : -1;
  const int64_t blk = slot >= 0 ? slot / block_size : 0;
  const int off = slot >= 0 ? slot % block_size : 0;
  // rotate q and k heads: each thread handles two adjacent rotation pairs
  const int npairs2 = (H + Hk) * half / 2;
  for (int i = threadIdx.x; i < npairs2; i += blockDim.x) {
    const int p = 2 * i;
    const int h = p / half, j = p % half;
    const __nv_bfloat16* src = row + h * D;
    float2 x1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(src + j));
    float2 x2 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(src + j + half));
    float c0 = cs[j], c1 = cs[j + 1], s0 = cs[half + j], s1 = cs[half + j + 1];
    __nv_bfloat162 y1 = __floats2bfloat162_rn(x1.x * c0 - x2.x * s0, x1.y * c1 - x2.y * s1);
    __nv_bfloat162 y2 = __floats2bfloat162_rn(x2.x * c0 + x1.x * s0, x2.y * c1 + x1.y * s1);
    if (h < H) {
      __nv_bfloat16* dst = q_out + ((int64_t)t * H + h) * D;
      *reinterpret_cast<__nv_bfloat162*>(dst + j) = y1;
      *reinterpret_cast<__nv_bfloat162*>(dst + j + half) = y2;
    } else if (slot >= 0) {
      const int kh = h - H;
      __nv_bfloat16* dst = cache + (((blk * 2 + 0) * Hk + kh) * block_size + off) * (int64_t)D;
      *reinterpret_cast<__nv_bfloat162*>(dst + j) = y1;
      *reinterpret_cast<__nv_bfloat162*>(dst + j + half) = y2;
    }
  }
  if (slot >= 0) {
    const int nv = Hk * D / 8;
    const uint4* vsrc = reinterpret_cast<const uint4*>(row + (H + Hk) * D);
    for (int i = threadIdx.x; i < nv; i += blockDim.x) {
      const int kh = (i * 8) / D, dd = (i * 8) % D;
      __nv_bfloat16* dst = cache + (((blk * 2 + 1) * Hk + kh) * block_size + off) * (int64_t)D + dd;
      *reinterpret_cast<uint4*>(dst) = vsrc[i];
    }
  }
}

// ---------------------------------------------------------------------------------------------
// K13: embedding gather (vectorised 16-byte copies).
// ---------------------------------------------------------------------------------------------
__global__ void embedding_kernel(__nv_bfloat16* __restrict__ out, const int* __restrict__ ids,
                                 const __nv_bfloat16* __restrict__ table, int d, int vocab) {
  const int t = blockIdx.x;
  int id = ids[t];
  id = id < 0 ? 0 : (id >= vocab ? vocab - 1 : id);
  const uint4* src = reinterpret_cast<const uint4*>(table + (int64_t)id * d);
  uint4* dst = reinterpret_cast<uint4*>(out + (int64_t)t * d);
  for (int i = threadIdx.x; i < d / 8; i += blockDim.x) dst[i] = src[i];
}

__global__ void silu_mul_kernel(__nv_bfloat16* __restrict__ out, const __nv_bfloat16* __restrict__ x, int d) {
  const int t = blockIdx.y;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;  // vector index (8 elements)
  if (i * 8 >= d) return;
  const __nv_bfloat16* row = x + (int64_t)t * 2 * d;
  float g[8], u[8], o[8];
  bf16x8_to_float(*reinterpret_cast<const uint4*>(row + i * 8), g);
  bf16x8_to_float(*reinterpret_cast<const uint4*>(row + d + i * 8), u);
#pragma unroll
  for (int j = 0; j < 8; ++j) o[j] = silu(g[j]) * u[j];
  *reinterpret_cast<uint4*>(out + (int64_t)t * d + i * 8) = float_to_bf16x8(o);
}

void check_bf16_cuda(const torch::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK(t.scalar_type() == at::kBFloat16, name, " must be bfloat16");
}

}  // namespace

void rms_norm_out(torch::Tensor out, torch::Tensor x, torch::Tensor w, double eps) {
  check_bf16_cuda(x, "x");
  check_bf16_cuda(out, "out");
  check_bf16_cuda(w, "w");
  launch_rms_norm<false>(out, x, nullptr, w, eps);
}

void fused_add_rms_norm_out(torch::Tensor out, torch::Tensor x, torch::Tensor residual, torch::Tensor w,
                            double eps) {
  check_bf16_cuda(x, "x");
  check_bf16_cuda(residual, "residual");
  TORCH_CHECK(residual.is_contiguous(), "residual must be contiguous");
  launch_rms_norm<true>(out, x, &residual, w, eps);
}

void rope_kv_write_out(torch::Tensor q_out, torch::Tensor qkv, torch::Tensor positions, torch::Tensor cos_sin,
                       c10::optional<torch::Tensor> cache, c10::optional<torch::Tensor> slots, int64_t H,
                       int64_t Hk, int64_t D) {
  check_bf16_cuda(qkv, "qkv");
  TORCH_CHECK(qkv.stride(1) == 1 && qkv.size(1) == (H + 2 * Hk) * D, "qkv shape mismatch");
  TORCH_CHECK(positions.scalar_type() == at::kInt && cos_sin.scalar_type() == at::kFloat, "positions int32, cos_sin fp32");
  TORCH_CHECK(D % 16 == 0 && cos_sin.size(1) == D, "head_dim must be a multiple of 16 and match cos_sin");
  TORCH_CHECK(q_out.is_contiguous(), "q_out must be contiguous");
  const int T = qkv.size(0);
  if (T == 0) return;
  __nv_bfloat16* cp = nullptr;
  const int* sp = nullptr;
  int bs = 16;
  if (cache.has_value() && slots.has_value()) {
    check_bf16_cuda(*cache, "kv_cache");
    TORCH_CHECK(cache->dim() == 5 && cache->size(1) == 2 && cache->size(2) == Hk && cache->size(4) == D,
                "kv cache must be [blocks, 2, Hk, block_size, D]");
    TORCH_CHECK(cache->is_contiguous() && slots->scalar_type() == at::kInt, "cache contiguous, slots int32");
    cp = reinterpret_cast<__nv_bfloat16*>(cache->data_ptr());
    sp = slots->data_ptr<int>();
    bs = cache->size(3);
  }
  auto stream = at::cuda::getCurrentCUDAStream();
  rope_kv_write_kernel<<<T, 128, 0, stream>>>(
      reinterpret_cast<__nv_bfloat16*>(q_out.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr()),
      positions.data_ptr<int>(), cos_sin.data_ptr<float>(), cp, sp, H, Hk, D, bs, qkv.stride(0),
      (int)cos_sin.size(0));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void embedding_out(torch::Tensor out, torch::Tensor ids, torch::Tensor table) {
  check_bf16_cuda(table, "table");
  TORCH_CHECK(ids.scalar_type() == at::kInt && table.is_contiguous() && out.is_contiguous(), "embedding args");
  const int T = ids.size(0), d = table.size(1);
  TORCH_CHECK(d % 8 == 0, "embedding dim must be a multiple of 8");
  if (T == 0) return;
  embedding_kernel<<<T, 128, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), ids.data_ptr<int>(),
      reinterpret_cast<const __nv_bfloat16*>(table.data_ptr()), d, (int)table.size(0));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void silu_mul_out(torch::Tensor out, torch::Tensor x) {
  check_bf16_cuda(x, "x");
  TORCH_CHECK(x.is_contiguous() && out.is_contiguous(), "silu_mul: contiguous tensors");
  const int T = x.size(0), d = x.size(1) / 2;
  TORCH_CHECK(d % 8 == 0, "silu_mul: width must be a multiple of 16");
  if (T == 0) return;
  dim3 grid((d / 8 + 127) / 128, T);
  silu_mul_kernel<<<grid, 128, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), d);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
