// K14: gated delta rule (Gated DeltaNet) layers of hybrid GDN / attention models (sm_100a).
//
// Per head, with state S in R^{dk x dv} (fp32, carried across chunks and steps):
//   alpha_t = exp(-exp(A_log) * softplus(a_t + dt_bias))     decay in (0, 1)
//   beta_t  = sigmoid(b_t)                                   write strength
//   S'  = alpha_t * S_{t-1}
//   u   = beta_t * (v_t - S'^T k_t)                          delta-rule correction (dv)
//   S_t = S' + k_t u^T
//   o_t = S_t^T q_t
// with q, k = L2-normalised silu(projection) (q also scaled by dk^-1/2) and v = silu(projection)
// (Yang, Kautz, Hatamizadeh, "Gated Delta Networks", ICLR 2025). Column j of S only depends on
// column j and on the shared k, q, alpha, beta, so the value dimension splits across warps with no
// reduction: one CTA is one head of one sequence, its 8 warps own 16 value columns each, two lanes
// per column with 64 state rows each in registers (one shuffle joins their partial dot products).
// The CTA stages 16 tokens at a time (q, k normalised and v activated once per chunk in shared
// memory); the scan over the chunk is 3 x 64 FMAs per lane per token with broadcast shared-memory
// reads.
// Decode (one token per sequence) and varlen prefill chunks are the same launch; `reset` starts a
// sequence from the zero state (first chunk) instead of reading its slot.
//
//   gdn_gated_norm  y = RMSNorm_head(o) * w * silu(g)   (one warp per token and head)
//
// Reference: core/optimization/gollek-plugin-hybrid-attn/…/hybridattn/binding/GdnBinding.java:18-58
// (gdn_layer_forward, gdn_gate_project; the kernels ship only as an absent .so).
#include "../common/common.cuh"
#include "launchers.h"

using namespace gollek;

namespace {

constexpr int kGdnD = 128;     // dk = dv
constexpr int kGdnChunk = 16;  // tokens staged per chunk
constexpr int kGdnThreads = 256;  // 8 warps x 16 value columns = one head per CTA

struct GdnArgs {
  const __nv_bfloat16* proj;  // [T, ldp]: q | k | v | g (Hg*D each) | a | b (Hg each)
  int64_t ldp;
  __nv_bfloat16* out;         // [T, Hg, D] raw o
  float* state;               // [slots, Hg, dk, dv] (this layer)
  int64_t state_slot_stride;  // elements between slots
  const int* slots;           // [n]
  const int* reset;           // [n]
  const int* query_start;     // [n + 1]
  const float* a_log;         // [Hg]
  const float* dt_bias;       // [Hg]
  int Hg;
  float q_scale;
};

GOLLEK_DEVICE float silu_f(float x) { return x / (1.f + __expf(-x)); }

__global__ void __launch_bounds__(kGdnThreads, 2) gdn_scan_kernel(const GdnArgs p) {
  __shared__ __align__(16) float qs[kGdnChunk][kGdnD];
  __shared__ __align__(16) float ks[kGdnChunk][kGdnD];
  __shared__ __align__(16) float vs[kGdnChunk][kGdnD];
  __shared__ __align__(16) __nv_bfloat16 raw[kGdnChunk][3 * kGdnD];  // q | k | v of the head
  __shared__ float al[kGdnChunk], be[kGdnChunk];
  const int b = blockIdx.x, h = blockIdx.y, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // warp w owns value columns [16 w, 16 w + 16); lanes l and l + 16 share column col, rows
  // [64 half, 64 half + 64) each, partial dot products joined with one shuffle
  const int col = warp * 16 + (lane & 15), half = lane >> 4;
  constexpr int R = kGdnD / 2;
  const int r0 = half * R;
  const int t0 = p.query_start[b], t1 = p.query_start[b + 1];
  if (t1 <= t0) return;
  const int HD = p.Hg * kGdnD;
  float* S = p.state + (int64_t)p.slots[b] * p.state_slot_stride + (int64_t)h * kGdnD * kGdnD + col;
  float s[R];
  if (p.reset[b]) {
#pragma unroll
    for (int i = 0; i < R; ++i) s[i] = 0.f;
  } else {
#pragma unroll
    for (int i = 0; i < R; ++i) s[i] = S[(int64_t)(r0 + i) * kGdnD];
  }
  const float A = __expf(p.a_log[h]), dtb = p.dt_bias[h];
  constexpr int kVec = 3 * kGdnD / 8;  // 16-byte vectors per staged token
  for (int c0 = t0; c0 < t1; c0 += kGdnChunk) {
    const int nc = min(kGdnChunk, t1 - c0);
    __syncthreads();  // the previous chunk's staged rows are no longer read
    // raw q, k, v rows of the head for the whole chunk: independent 16-byte loads by the CTA
    for (int idx = tid; idx < nc * kVec; idx += kGdnThreads) {
      const int tt = idx / kVec, vi = idx % kVec, part = vi / 16;
      const __nv_bfloat16* row = p.proj + (int64_t)(c0 + tt) * p.ldp + part * HD + h * kGdnD + 8 * (vi % 16);
      *reinterpret_cast<uint4*>(&raw[tt][8 * vi]) = *reinterpret_cast<const uint4*>(row);
    }
    if (tid < nc) {
      const __nv_bfloat16* row = p.proj + (int64_t)(c0 + tid) * p.ldp + 4 * HD;
      const float a = __bfloat162float(row[h]) + dtb, bb = __bfloat162float(row[p.Hg + h]);
      const float sp = a > 20.f ? a : log1pf(__expf(a));
      al[tid] = __expf(-A * sp);
      be[tid] = 1.f / (1.f + __expf(-bb));
    }
    __syncthreads();
    // silu + L2 norm of q and k, silu of v: warp w takes tokens w, w + 8, ...
    for (int tt = warp; tt < nc; tt += kGdnThreads / 32) {
      float q4[4], k4[4], v4[4], sq = 0.f, sk = 0.f;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        q4[e] = silu_f(__bfloat162float(raw[tt][4 * lane + e]));
        k4[e] = silu_f(__bfloat162float(raw[tt][kGdnD + 4 * lane + e]));
        v4[e] = silu_f(__bfloat162float(raw[tt][2 * kGdnD + 4 * lane + e]));
        sq = fmaf(q4[e], q4[e], sq);
        sk = fmaf(k4[e], k4[e], sk);
      }
      sq = warp_sum(sq);
      sk = warp_sum(sk);
      const float rq = rsqrtf(sq + 1e-6f) * p.q_scale, rk = rsqrtf(sk + 1e-6f);
      *reinterpret_cast<float4*>(&qs[tt][4 * lane]) = make_float4(q4[0] * rq, q4[1] * rq, q4[2] * rq, q4[3] * rq);
      *reinterpret_cast<float4*>(&ks[tt][4 * lane]) = make_float4(k4[0] * rk, k4[1] * rk, k4[2] * rk, k4[3] * rk);
      *reinterpret_cast<float4*>(&vs[tt][4 * lane]) = make_float4(v4[0], v4[1], v4[2], v4[3]);
    }
    __syncthreads();
    for (int tt = 0; tt < nc; ++tt) {
      const float alpha = al[tt], beta = be[tt];
      float kd[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int i = 0; i < R; i += 4) {
        const float4 k = *reinterpret_cast<const float4*>(&ks[tt][r0 + i]);
        kd[0] = fmaf(s[i], k.x, kd[0]);
        kd[1] = fmaf(s[i + 1], k.y, kd[1]);
        kd[2] = fmaf(s[i + 2], k.z, kd[2]);
        kd[3] = fmaf(s[i + 3], k.w, kd[3]);
      }
      float kS = (kd[0] + kd[1]) + (kd[2] + kd[3]);
      kS += __shfl_xor_sync(0xffffffffu, kS, 16);
      const float u = beta * (vs[tt][col] - alpha * kS);
      float od[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int i = 0; i < R; i += 4) {
        const float4 k = *reinterpret_cast<const float4*>(&ks[tt][r0 + i]);
        const float4 q = *reinterpret_cast<const float4*>(&qs[tt][r0 + i]);
        s[i] = fmaf(alpha, s[i], k.x * u);
        s[i + 1] = fmaf(alpha, s[i + 1], k.y * u);
        s[i + 2] = fmaf(alpha, s[i + 2], k.z * u);
        s[i + 3] = fmaf(alpha, s[i + 3], k.w * u);
        od[0] = fmaf(s[i], q.x, od[0]);
        od[1] = fmaf(s[i + 1], q.y, od[1]);
        od[2] = fmaf(s[i + 2], q.z, od[2]);
        od[3] = fmaf(s[i + 3], q.w, od[3]);
      }
      float o = (od[0] + od[1]) + (od[2] + od[3]);
      o += __shfl_xor_sync(0xffffffffu, o, 16);
      if (half == 0) p.out[((int64_t)(c0 + tt) * p.Hg + h) * kGdnD + col] = __float2bfloat16(o);
    }
  }
#pragma unroll
  for (int i = 0; i < R; ++i) S[(int64_t)(r0 + i) * kGdnD] = s[i];
}

// y[t, h*D + d] = o[t, h, d] * rsqrt(mean_d o^2 + eps) * w[d] * silu(g[t, h*D + d]); warp per (t, h)
__global__ void __launch_bounds__(256) gdn_gated_norm_kernel(__nv_bfloat16* __restrict__ y,
                                                             const __nv_bfloat16* __restrict__ o,
                                                             const __nv_bfloat16* __restrict__ g, int64_t ldg,
                                                             const __nv_bfloat16* __restrict__ w, int T, int Hg,
                                                             float eps) {
  const int warp = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (warp >= T * Hg) return;
  const int t = warp / Hg, h = warp % Hg;
  const __nv_bfloat16* orow = o + ((int64_t)t * Hg + h) * kGdnD;
  float v[4], ss = 0.f;
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    v[e] = __bfloat162float(orow[4 * lane + e]);
    ss = fmaf(v[e], v[e], ss);
  }
  const float r = rsqrtf(warp_sum(ss) / kGdnD + eps);
  const __nv_bfloat16* grow = g + (int64_t)t * ldg + h * kGdnD;
  __nv_bfloat16* yrow = y + (int64_t)t * Hg * kGdnD + h * kGdnD;
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const int d = 4 * lane + e;
    yrow[d] = __float2bfloat16(v[e] * r * __bfloat162float(w[d]) * silu_f(__bfloat162float(grow[d])));
  }
}

}  // namespace

namespace gollek {

void launch_gdn_scan(const void* proj, int64_t ldp, void* out, float* state, int64_t state_slot_stride,
                     const int* slots, const int* reset, const int* query_start, int n, const float* a_log,
                     const float* dt_bias, int Hg, int D, cudaStream_t s) {
  throw_if(D != kGdnD, "gdn: head_dim 128 only");
  throw_if(ldp % 8 != 0, "gdn: projection rows must keep 16-byte alignment");
  if (n == 0) return;
  GdnArgs a{reinterpret_cast<const __nv_bfloat16*>(proj), ldp, reinterpret_cast<__nv_bfloat16*>(out), state,
            state_slot_stride, slots, reset, query_start, a_log, dt_bias, Hg, 1.f / sqrtf((float)D)};
  gdn_scan_kernel<<<dim3(n, Hg), kGdnThreads, 0, s>>>(a);
  check_launch("gdn_scan");
}

void launch_gdn_gated_norm(void* y, const void* o, const void* g, int64_t ldg, const void* w, int T, int Hg, int D,
                           float eps, cudaStream_t s) {
  throw_if(D != kGdnD, "gdn: head_dim 128 only");
  const int64_t warps = (int64_t)T * Hg;
  if (warps == 0) return;
  gdn_gated_norm_kernel<<<(unsigned)((warps + 7) / 8), 256, 0, s>>>(
      reinterpret_cast<__nv_bfloat16*>(y), reinterpret_cast<const __nv_bfloat16*>(o),
      reinterpret_cast<const __nv_bfloat16*>(g), ldg, reinterpret_cast<const __nv_bfloat16*>(w), T, Hg, eps);
  check_launch("gdn_gated_norm");
}

}  // namespace gollek
