// Python bindings of the sm_100a kernels (module gollek_b200_C).
//
// All torch-tensor validation happens here (compiled by the host compiler); the .cu files
// only see raw pointers, strides and the current CUDA stream.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common/tma_host.h"
#include "kernels/launchers.h"

using namespace gollek;

namespace {

cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream(); }

void check_cuda(const torch::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
}
void check_bf16(const torch::Tensor& t, const char* name) {
  check_cuda(t, name);
  TORCH_CHECK(t.scalar_type() == at::kBFloat16, name, " must be bfloat16");
}
void check_i32(const torch::Tensor& t, const char* name) {
  check_cuda(t, name);
  TORCH_CHECK(t.scalar_type() == at::kInt, name, " must be int32");
}
void check_same_device(const torch::Tensor& a, const torch::Tensor& b) {
  TORCH_CHECK(a.device() == b.device(), "tensors on different devices");
}

void rms_norm_out(torch::Tensor out, torch::Tensor x, torch::Tensor w, double eps, bool center) {
  check_bf16(x, "x");
  check_bf16(out, "out");
  check_bf16(w, "w");
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1 && out.stride(1) == 1 && w.is_contiguous(), "rms_norm: row-major 2-D");
  TORCH_CHECK(out.sizes() == x.sizes() && w.numel() == x.size(1), "rms_norm: shape mismatch");
  launch_rms_norm(out.data_ptr(), x.data_ptr(), nullptr, w.data_ptr(), x.size(0), x.size(1), x.stride(0),
                  out.stride(0), (float)eps, cur_stream(), center);
}

void fused_add_rms_norm_out(torch::Tensor out, torch::Tensor x, torch::Tensor residual, torch::Tensor w,
                            double eps, bool center) {
  check_bf16(x, "x");
  check_bf16(out, "out");
  check_bf16(residual, "residual");
  check_bf16(w, "w");
  TORCH_CHECK(residual.is_contiguous() && residual.sizes() == x.sizes(), "residual must be contiguous [T, d]");
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1 && out.stride(1) == 1 && w.is_contiguous(), "rms_norm: row-major 2-D");
  TORCH_CHECK(out.sizes() == x.sizes() && w.numel() == x.size(1), "rms_norm: shape mismatch");
  launch_rms_norm(out.data_ptr(), x.data_ptr(), residual.data_ptr(), w.data_ptr(), x.size(0), x.size(1),
                  x.stride(0), out.stride(0), (float)eps, cur_stream(), center);
}

void rope_kv_write_out(torch::Tensor q_out, torch::Tensor qkv, torch::Tensor positions, torch::Tensor cos_sin,
                       c10::optional<torch::Tensor> cache, c10::optional<torch::Tensor> slots, int64_t H, int64_t Hk,
                       int64_t D, c10::optional<torch::Tensor> bias, c10::optional<torch::Tensor> q_norm,
                       c10::optional<torch::Tensor> k_norm, double norm_eps) {
  check_bf16(qkv, "qkv");
  check_bf16(q_out, "q_out");
  check_i32(positions, "positions");
  check_cuda(cos_sin, "cos_sin");
  TORCH_CHECK(cos_sin.scalar_type() == at::kFloat && cos_sin.is_contiguous() && cos_sin.size(1) <= D &&
                  cos_sin.size(1) % 4 == 0,
              "cos_sin must be fp32 [max_pos, rotary_dim <= head_dim]");
  TORCH_CHECK(qkv.dim() == 2 && qkv.stride(1) == 1 && qkv.size(1) == (H + 2 * Hk) * D, "qkv shape mismatch");
  TORCH_CHECK(qkv.stride(0) % 8 == 0, "qkv row pitch must keep 16-byte alignment");
  const int T = qkv.size(0);
  TORCH_CHECK(q_out.is_contiguous() && q_out.numel() == (int64_t)T * H * D, "q_out must be contiguous [T, H, D]");
  TORCH_CHECK(positions.numel() >= T, "positions too short");
  void* cp = nullptr;
  const int* sp = nullptr;
  int bs = 16;
  if (cache.has_value() && slots.has_value()) {
    check_bf16(*cache, "kv_cache");
    check_i32(*slots, "slots");
    TORCH_CHECK(cache->dim() == 5 && cache->size(1) == 2 && cache->size(2) == Hk && cache->size(4) == D,
                "kv cache must be [blocks, 2, Hk, block_size, D]");
    TORCH_CHECK(cache->is_contiguous() && slots->numel() >= T, "cache contiguous, enough slots");
    cp = cache->data_ptr();
    sp = slots->data_ptr<int>();
    bs = cache->size(3);
  }
  const void* bp = nullptr;
  const void* qn = nullptr;
  const void* kn = nullptr;
  if (bias.has_value()) {
    check_bf16(*bias, "bias");
    TORCH_CHECK(bias->is_contiguous() && bias->numel() == (int64_t)(H + 2 * Hk) * D, "qkv bias [(H + 2Hk) * D]");
    bp = bias->data_ptr();
  }
  if (q_norm.has_value() || k_norm.has_value()) {
    TORCH_CHECK(q_norm.has_value() && k_norm.has_value(), "QK-norm needs both q and k weights");
    check_bf16(*q_norm, "q_norm");
    check_bf16(*k_norm, "k_norm");
    TORCH_CHECK(q_norm->numel() == D && k_norm->numel() == D, "QK-norm weights are [head_dim]");
    qn = q_norm->data_ptr();
    kn = k_norm->data_ptr();
  }
  launch_rope_kv_write(q_out.data_ptr(), qkv.data_ptr(), positions.data_ptr<int>(), cos_sin.data_ptr<float>(), cp,
                       sp, T, H, Hk, D, bs, qkv.stride(0), (int)cos_sin.size(0), bp, qn, kn, (float)norm_eps,
                       (int)cos_sin.size(1), cur_stream(), cp ? (int)cache->size(0) : 0);
}

void embedding_out(torch::Tensor out, torch::Tensor ids, torch::Tensor table, double scale) {
  check_bf16(table, "table");
  check_bf16(out, "out");
  check_i32(ids, "ids");
  TORCH_CHECK(table.is_contiguous() && out.is_contiguous() && out.size(0) == ids.size(0) &&
                  out.size(1) == table.size(1),
              "embedding: shapes");
  launch_embedding(out.data_ptr(), ids.data_ptr<int>(), table.data_ptr(), ids.size(0), table.size(1), table.size(0),
                   (float)scale, cur_stream());
}

void silu_mul_out(torch::Tensor out, torch::Tensor x) {
  check_bf16(x, "x");
  check_bf16(out, "out");
  TORCH_CHECK(x.is_contiguous() && out.is_contiguous() && out.size(1) * 2 == x.size(1), "silu_mul: shapes");
  launch_silu_mul(out.data_ptr(), x.data_ptr(), x.size(0), x.size(1) / 2, cur_stream());
}

void paged_decode_attention_out(torch::Tensor out, torch::Tensor q, torch::Tensor cache, torch::Tensor block_tables,
                                torch::Tensor seq_lens, double scale, int64_t num_splits,
                                c10::optional<torch::Tensor> workspace, bool tensor_cores, int64_t window,
                                double softcap, c10::optional<torch::Tensor> kv_scales) {
  check_bf16(q, "q");
  check_bf16(out, "out");
  const float* scl = nullptr;
  if (kv_scales.has_value()) {  // fp8 e4m3 cache (uint8 storage) + fp32 per-token scales
    TORCH_CHECK(cache.scalar_type() == at::kByte && cache.is_cuda(), "fp8 kv_cache: uint8 storage on the device");
    TORCH_CHECK(kv_scales->scalar_type() == at::kFloat && kv_scales->is_contiguous() &&
                    kv_scales->numel() == cache.numel() / cache.size(4),
                "kv_scales must be fp32 [NB, 2, Hk, bs]");
    scl = kv_scales->data_ptr<float>();
  } else {
    check_bf16(cache, "kv_cache");
  }
  check_i32(block_tables, "block_tables");
  check_i32(seq_lens, "seq_lens");
  TORCH_CHECK(q.dim() == 3 && q.stride(2) == 1 && q.stride(1) == q.size(2), "q must be [B, H, D] with packed heads");
  TORCH_CHECK(out.is_contiguous() && out.sizes() == q.sizes(), "out must be contiguous like q");
  TORCH_CHECK(cache.is_contiguous() && cache.dim() == 5 && cache.size(4) == q.size(2), "cache [NB, 2, Hk, bs, D]");
  TORCH_CHECK(block_tables.stride(1) == 1 && block_tables.size(0) >= q.size(0) && seq_lens.numel() >= q.size(0),
              "block_tables [B, max_blocks] row-major");
  const int B = q.size(0), H = q.size(1), D = q.size(2);
  num_splits = std::max<int64_t>(1, num_splits);
  float* po = nullptr;
  float* pml = nullptr;
  if (num_splits > 1) {
    TORCH_CHECK(workspace.has_value() && workspace->is_cuda() && workspace->scalar_type() == at::kFloat &&
                    workspace->numel() >= (int64_t)B * H * num_splits * (D + 2),
                "decode attention: fp32 workspace too small for split-KV");
    po = workspace->data_ptr<float>();
    pml = po + (int64_t)B * H * num_splits * D;
  }
  launch_paged_decode(out.data_ptr(), q.data_ptr(), q.stride(0), cache.data_ptr(),
                      (int)cache.size(0), block_tables.data_ptr<int>(),
                      block_tables.stride(0), seq_lens.data_ptr<int>(), B, H, cache.size(2), D, cache.size(3),
                      (int)num_splits, (float)scale, po, pml, (int)window, (float)softcap, cur_stream(),
                      scl, tensor_cores);
}

void paged_prefill_attention_out(torch::Tensor out, torch::Tensor q, torch::Tensor cache, torch::Tensor block_tables,
                                 torch::Tensor seq_lens, torch::Tensor query_start, torch::Tensor tiles,
                                 double scale, bool tensor_cores, int64_t window, double softcap, int64_t emu) {
  check_bf16(q, "q");
  check_bf16(out, "out");
  check_bf16(cache, "kv_cache");
  check_i32(block_tables, "block_tables");
  check_i32(seq_lens, "seq_lens");
  check_i32(query_start, "query_start");
  check_i32(tiles, "tiles");
  TORCH_CHECK(q.dim() == 3 && q.stride(2) == 1 && q.stride(1) == q.size(2), "q must be [T, H, D]");
  TORCH_CHECK(out.dim() == 3 && out.stride(2) == 1 && out.stride(1) == out.size(2) && out.sizes() == q.sizes(),
              "out must be [T, H, D]");
  TORCH_CHECK(cache.is_contiguous() && cache.dim() == 5 && cache.size(4) == q.size(2), "cache [NB, 2, Hk, bs, D]");
  TORCH_CHECK(block_tables.stride(1) == 1 && tiles.is_contiguous() && query_start.is_contiguous(), "metadata layout");
  if (tensor_cores && (q.size(2) == 128 || q.size(2) == 64) && cache.size(3) == 16 && tiles.dim() == 2 &&
      tiles.size(1) == 4) {
    launch_paged_prefill_fa(out.data_ptr(), out.stride(0), q.data_ptr(), q.size(0), q.stride(0), cache.data_ptr(),
                            cache.size(0), block_tables.data_ptr<int>(), block_tables.stride(0),
                            seq_lens.data_ptr<int>(), query_start.data_ptr<int>(), tiles.data_ptr<int>(),
                            tiles.size(0), q.size(1), cache.size(2), (float)scale, (int)window, (float)softcap,
                            (int)emu, cur_stream(), (int)q.size(2));
    return;
  }
  if (tensor_cores && q.size(2) == 128 && cache.size(3) == 16) {
    launch_paged_prefill_tc(out.data_ptr(), out.stride(0), q.data_ptr(), q.size(0), q.stride(0), cache.data_ptr(),
                            cache.size(0), block_tables.data_ptr<int>(), block_tables.stride(0),
                            seq_lens.data_ptr<int>(), query_start.data_ptr<int>(), tiles.data_ptr<int>(),
                            tiles.size(0), q.size(1), cache.size(2), (float)scale, (int)window, (float)softcap,
                            cur_stream());
    return;
  }
  launch_paged_prefill(out.data_ptr(), out.stride(0), q.data_ptr(), q.stride(0), cache.data_ptr(),
                       block_tables.data_ptr<int>(), block_tables.stride(0), seq_lens.data_ptr<int>(),
                       query_start.data_ptr<int>(), tiles.data_ptr<int>(), tiles.size(0), q.size(1), cache.size(2),
                       q.size(2), cache.size(3), (float)scale, (int)window, (float)softcap, cur_stream(),
                       (int)cache.size(0));
}

void gemm_bf16_out(torch::Tensor out, torch::Tensor a, torch::Tensor b, c10::optional<torch::Tensor> residual,
                   int64_t epi, int64_t bn, c10::optional<torch::Tensor> status, int64_t grid_limit,
                   int64_t splits, c10::optional<torch::Tensor> workspace) {
  check_bf16(a, "a");
  check_bf16(b, "b");
  check_bf16(out, "out");
  check_same_device(a, b);
  TORCH_CHECK(a.dim() == 2 && b.dim() == 2 && a.size(1) == b.size(1), "gemm: shape mismatch");
  TORCH_CHECK(a.stride(1) == 1 && b.stride(1) == 1 && out.stride(1) == 1, "gemm: K-major operands, row-major out");
  const int M = a.size(0), N = b.size(0), K = a.size(1);
  TORCH_CHECK(out.size(0) == M, "gemm: out rows");
  if (epi_gated((int)epi)) {
    TORCH_CHECK(out.size(1) == N / 2, "gemm swiglu: out [M, N/2]");
  } else {
    TORCH_CHECK(out.size(1) == N, "gemm: out [M, N]");
  }
  const void* rp = nullptr;
  int64_t ldr = 0;
  if (epi == kEpiResidual) {
    TORCH_CHECK(residual.has_value(), "gemm residual: residual tensor required");
    check_bf16(*residual, "residual");
    TORCH_CHECK(residual->stride(1) == 1 && residual->size(0) == M && residual->size(1) == N, "residual [M, N]");
    rp = residual->data_ptr();
    ldr = residual->stride(0);
  }
  uint32_t* st = nullptr;
  if (status.has_value()) {
    check_cuda(*status, "status");
    st = reinterpret_cast<uint32_t*>(status->data_ptr());
  }
  int bn_i = (int)bn, sp = (int)splits;
  if (bn_i == 0) {
    int auto_sp = 1;
    gemm_plan(M, N, K, (int)epi, bn_i, auto_sp);
    if (sp <= 0) sp = auto_sp;
  }
  if (sp <= 0) sp = 1;
  float* part = nullptr;
  if (sp > 1) {
    TORCH_CHECK(workspace.has_value() && workspace->is_cuda() && workspace->scalar_type() == at::kFloat &&
                    workspace->numel() >= (int64_t)sp * M * N,
                "gemm: split-K ", sp, " needs an fp32 workspace of ", (int64_t)sp * M * N, " elements");
    part = workspace->data_ptr<float>();
  }
  launch_gemm_bf16(out.data_ptr(), out.stride(0), a.data_ptr(), a.stride(0), b.data_ptr(), b.stride(0), rp, ldr, M,
                   N, K, (int)epi, bn_i, sp, part, st, (int)grid_limit, cur_stream());
}

// MoE layer (K12 + grouped tcgen05 GEMMs). w_gu: [e_loc * 2F, H] gate/up rows interleaved in groups
// of 64 per expert; w_down: [e_loc * H, F]. ws: int32 [moe_ws_ints] zero-filled once at allocation
// (the plan kernel re-zeroes its counters after every use). ids/dest [T*topk] int32, wts fp32,
// xp/yp [cap, H] and hp [cap, F] bf16 scratch with cap = moe_capacity_rows(T, topk, e_loc).
void moe_forward_out(torch::Tensor out, torch::Tensor x, torch::Tensor router, torch::Tensor w_gu,
                     torch::Tensor w_down, torch::Tensor ws, torch::Tensor ids, torch::Tensor wts, torch::Tensor dest,
                     torch::Tensor xp, torch::Tensor hp, torch::Tensor yp, c10::optional<torch::Tensor> ypart,
                     int64_t topk, bool renorm, int64_t e0, int64_t e_loc, int64_t scoring,
                     c10::optional<torch::Tensor> score_bias, int64_t n_group, int64_t topk_group, double scale,
                     c10::optional<torch::Tensor> expert_map, c10::optional<torch::Tensor> logits) {
  for (auto* t : {&out, &x, &router, &w_gu, &w_down, &xp, &hp, &yp}) check_bf16(*t, "moe operand");
  MoeRouting rt;
  rt.scoring = (int)scoring;
  rt.n_group = (int)n_group;
  rt.topk_group = (int)topk_group;
  rt.scale = (float)scale;
  if (score_bias.has_value()) {
    TORCH_CHECK(score_bias->is_cuda() && score_bias->scalar_type() == at::kFloat && score_bias->is_contiguous() &&
                    score_bias->numel() == router.size(0),
                "moe: score correction bias must be fp32 [E] on the device");
    rt.bias = score_bias->data_ptr<float>();
  }
  if (expert_map.has_value()) {
    TORCH_CHECK(expert_map->is_cuda() && expert_map->scalar_type() == at::kInt && expert_map->is_contiguous() &&
                    expert_map->numel() == router.size(0),
                "moe: expert map must be int32 [E] on the device (logical expert -> physical slot)");
    rt.expert_map = expert_map->data_ptr<int>();
  }
  if (logits.has_value()) {
    TORCH_CHECK(logits->is_cuda() && logits->scalar_type() == at::kFloat && logits->is_contiguous() &&
                    logits->numel() >= (int64_t)moe_logit_splits(x.size(0), router.size(0), x.size(1)) *
                                           x.size(0) * router.size(0),
                "moe: router logits scratch must be fp32 [moe_logit_splits(T, E, H), T, E] on the device");
    rt.logits = logits->data_ptr<float>();
  }
  check_same_device(x, w_gu);
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1 && out.stride(1) == 1, "moe: x/out row-major [T, H]");
  const int T = x.size(0), H = x.size(1), E = router.size(0);
  TORCH_CHECK(router.dim() == 2 && router.size(1) == H && router.is_contiguous(), "moe: router [E, H]");
  TORCH_CHECK(w_down.dim() == 2 && w_down.size(0) == e_loc * H && w_down.is_contiguous(), "moe: w_down [e_loc*H, F]");
  const int F = w_down.size(1);
  TORCH_CHECK(w_gu.dim() == 2 && w_gu.size(0) == e_loc * 2 * F && w_gu.size(1) == H && w_gu.is_contiguous(),
              "moe: w_gu [e_loc*2F, H]");
  TORCH_CHECK(out.size(0) == T && out.size(1) == H, "moe: out [T, H]");
  const int cap = moe_capacity_rows(T, (int)topk, (int)e_loc);
  TORCH_CHECK(xp.is_contiguous() && xp.size(0) >= cap && xp.size(1) == H, "moe: xp [cap, H]");
  TORCH_CHECK(yp.is_contiguous() && yp.size(0) >= cap && yp.size(1) == H, "moe: yp [cap, H]");
  TORCH_CHECK(hp.is_contiguous() && hp.size(0) >= cap && hp.size(1) == F, "moe: hp [cap, F]");
  TORCH_CHECK(ws.scalar_type() == at::kInt && ws.is_cuda() && ws.numel() >= moe_ws_ints(T, (int)topk, (int)e_loc),
              "moe: int32 workspace too small");
  TORCH_CHECK(ids.scalar_type() == at::kInt && dest.scalar_type() == at::kInt && wts.scalar_type() == at::kFloat &&
                  ids.numel() >= (int64_t)T * topk && dest.numel() >= (int64_t)T * topk &&
                  wts.numel() >= (int64_t)T * topk,
              "moe: ids/dest int32 and wts fp32 of T*topk");
  int bn_gu, bn_dn, splits;
  moe_plan_host(T, (int)topk, E, (int)e_loc, H, F, bn_gu, bn_dn, splits);
  float* yq = nullptr;
  if (splits > 1) {
    TORCH_CHECK(ypart.has_value() && ypart->is_cuda() && ypart->scalar_type() == at::kFloat &&
                    ypart->numel() >= (int64_t)splits * cap * H,
                "moe: split-K down projection needs an fp32 buffer of ", (int64_t)splits * cap * H, " elements");
    yq = ypart->data_ptr<float>();
  }
  launch_moe_forward(out.data_ptr(), out.stride(0), x.data_ptr(), x.stride(0), router.data_ptr(), w_gu.data_ptr(),
                     w_down.data_ptr(), ws.data_ptr<int>(), ids.data_ptr<int>(), wts.data_ptr<float>(),
                     dest.data_ptr<int>(), xp.data_ptr(), hp.data_ptr(), yp.data_ptr(), yq, T, H, F, E, (int)topk,
                     renorm ? 1 : 0, (int)e0, (int)e_loc, rt, nullptr, cur_stream());
}

std::vector<int64_t> moe_plan_py(int64_t T, int64_t topk, int64_t E, int64_t e_loc, int64_t H, int64_t F) {
  int a, b, c;
  moe_plan_host((int)T, (int)topk, (int)E, (int)e_loc, (int)H, (int)F, a, b, c);
  return {a, b, c};
}

// cache [L, NB, 2, Hk, bs, D] bf16; packed [L, n, 2, Hk, bs, D] bf16; block_ids int32 [n] (device)
void gdn_scan_py(torch::Tensor proj, torch::Tensor out, torch::Tensor state, torch::Tensor slots,
                 torch::Tensor reset, torch::Tensor query_start, torch::Tensor a_log, torch::Tensor dt_bias,
                 int64_t Hg) {
  check_bf16(proj, "proj");
  check_bf16(out, "out");
  TORCH_CHECK(state.is_cuda() && state.scalar_type() == torch::kFloat32 && state.dim() == 4 &&
                  state.stride(3) == 1 && state.stride(2) == state.size(3) && state.stride(1) == state.size(2) * state.size(3),
              "state [slots, Hg, D, D] fp32 (slot stride free)");
  check_i32(slots, "slots");
  check_i32(reset, "reset");
  check_i32(query_start, "query_start");
  TORCH_CHECK(a_log.scalar_type() == torch::kFloat32 && dt_bias.scalar_type() == torch::kFloat32, "gates fp32");
  TORCH_CHECK(proj.stride(1) == 1 && out.is_contiguous(), "layouts");
  const int D = (int)state.size(3);
  TORCH_CHECK(proj.size(1) >= 4 * Hg * D + 2 * Hg && out.size(0) == proj.size(0), "proj / out shapes");
  launch_gdn_scan(proj.data_ptr(), proj.stride(0), out.data_ptr(), state.data_ptr<float>(), state.stride(0),
                  slots.data_ptr<int>(), reset.data_ptr<int>(), query_start.data_ptr<int>(), (int)slots.size(0),
                  a_log.data_ptr<float>(), dt_bias.data_ptr<float>(), (int)Hg, D, cur_stream());
}

void gdn_gated_norm_py(torch::Tensor y, torch::Tensor o, torch::Tensor g, torch::Tensor w, int64_t Hg, double eps) {
  check_bf16(y, "y");
  check_bf16(o, "o");
  check_bf16(g, "g");
  check_bf16(w, "w");
  TORCH_CHECK(g.stride(1) == 1 && o.is_contiguous() && y.is_contiguous(), "layouts");
  launch_gdn_gated_norm(y.data_ptr(), o.data_ptr(), g.data_ptr(), g.stride(0), w.data_ptr(), (int)o.size(0), (int)Hg,
                        (int)w.size(0), (float)eps, cur_stream());
}

torch::Tensor kv_key_norms_py(torch::Tensor cache, torch::Tensor block_ids) {
  check_bf16(cache, "kv_cache");
  check_i32(block_ids, "block_ids");
  TORCH_CHECK(cache.is_contiguous() && cache.dim() == 6 && cache.size(2) == 2, "cache [L, NB, 2, Hk, bs, D]");
  TORCH_CHECK(block_ids.is_contiguous() && block_ids.dim() == 1, "block_ids [n]");
  auto out = torch::empty({block_ids.size(0)}, cache.options().dtype(torch::kFloat32));
  launch_kv_key_norms(cache.data_ptr(), block_ids.data_ptr<int>(), out.data_ptr<float>(), (int)block_ids.size(0),
                      (int)cache.size(0), cache.size(1), (int)cache.size(3), (int)cache.size(4), (int)cache.size(5),
                      cur_stream());
  return out;
}

void kv_blocks_py(torch::Tensor cache, torch::Tensor packed, torch::Tensor block_ids, bool gather) {
  check_bf16(cache, "kv_cache");
  check_bf16(packed, "packed");
  check_i32(block_ids, "block_ids");
  check_same_device(cache, packed);
  TORCH_CHECK(cache.is_contiguous() && packed.is_contiguous() && cache.dim() == 6 && packed.dim() == 6,
              "kv transfer: contiguous [L, blocks, 2, Hk, bs, D] tensors");
  const int n = block_ids.numel();
  TORCH_CHECK(packed.size(0) == cache.size(0) && packed.size(1) == n, "kv transfer: packed [L, n, ...]");
  for (int d = 2; d < 6; ++d) TORCH_CHECK(packed.size(d) == cache.size(d), "kv transfer: block shape mismatch");
  const int64_t span = cache.numel() / (cache.size(0) * cache.size(1));
  launch_kv_blocks(cache.data_ptr(), packed.data_ptr(), block_ids.data_ptr<int>(), n, cache.size(0), cache.size(1),
                   span, gather, cur_stream());
}

// 4-bit weights: q uint8 [N, K/2], scale/zero bf16 [N, K/g] (zero absent for NF4)
static void check_int4(torch::Tensor q, torch::Tensor scale, c10::optional<torch::Tensor> zero, int64_t N,
                       int64_t K, int64_t g) {
  TORCH_CHECK(q.is_cuda() && q.scalar_type() == at::kByte && q.is_contiguous() && q.numel() == N * K / 2,
              "int4: q must be uint8 [N, K/2]");
  check_bf16(scale, "scale");
  TORCH_CHECK(scale.is_contiguous() && scale.numel() == N * (K / g), "int4: scale [N, K/g]");
  if (zero.has_value()) {
    check_bf16(*zero, "zero");
    TORCH_CHECK(zero->is_contiguous() && zero->numel() == N * (K / g), "int4: zero [N, K/g]");
  }
}

void int4_gemv_py(torch::Tensor out, torch::Tensor x, torch::Tensor q, torch::Tensor scale,
                  c10::optional<torch::Tensor> zero, int64_t N, int64_t K, int64_t g, bool lut, bool swiglu) {
  check_bf16(x, "x");
  check_bf16(out, "out");
  check_int4(q, scale, zero, N, K, g);
  TORCH_CHECK(x.dim() == 2 && x.size(1) == K && x.stride(1) == 1, "int4 gemv: x [M, K]");
  TORCH_CHECK(out.size(0) == x.size(0) && out.size(1) == (swiglu ? N / 2 : N) && out.stride(1) == 1, "int4 gemv: out");
  launch_int4_gemv(out.data_ptr(), out.stride(0), x.data_ptr(), x.stride(0), q.data_ptr(), scale.data_ptr(),
                   zero.has_value() ? zero->data_ptr() : nullptr, x.size(0), N, K, g, lut, swiglu, cur_stream());
}

void int4_dequant_py(torch::Tensor out, torch::Tensor q, torch::Tensor scale, c10::optional<torch::Tensor> zero,
                     int64_t N, int64_t K, int64_t g, bool lut) {
  check_bf16(out, "out");
  check_int4(q, scale, zero, N, K, g);
  TORCH_CHECK(out.is_contiguous() && out.numel() == N * K, "int4 dequant: out [N, K]");
  launch_int4_dequant(out.data_ptr(), q.data_ptr(), scale.data_ptr(), zero.has_value() ? zero->data_ptr() : nullptr,
                      N, K, g, lut, cur_stream());
}

std::vector<int64_t> gemm_plan_py(int64_t M, int64_t N, int64_t K, int64_t epi) {
  int bn = 0, sp = 1;
  gemm_plan((int)M, (int)N, (int)K, (int)epi, bn, sp);
  return {bn, sp};
}

std::vector<int64_t> gemm_retile_py(int64_t M, int64_t N, int64_t K, int64_t epi) {
  int bn = 0, sp = 1;
  gemm_plan((int)M, (int)N, (int)K, (int)epi, bn, sp);
  const int tiles = (int)((M + 127) / 128) * (int)((N + bn - 1) / bn);
  int full = 0, bnt = 0;
  if (sp == 1 && N % bn == 0) gemm_retile_plan(tiles, std::min(tiles, gemm_grid_sms()), bn, epi_gated((int)epi), full, bnt);
  return {bn, full, bnt};
}

void argmax_out(torch::Tensor out, torch::Tensor logits) {
  check_cuda(logits, "logits");
  TORCH_CHECK(logits.dim() == 2 && logits.stride(1) == 1, "argmax: [B, V] logits");
  TORCH_CHECK(out.scalar_type() == at::kLong && out.numel() >= logits.size(0), "argmax: int64 output");
  TORCH_CHECK(logits.scalar_type() == at::kFloat || logits.scalar_type() == at::kBFloat16, "argmax: fp32/bf16");
  launch_argmax(out.data_ptr<int64_t>(), logits.data_ptr(), logits.scalar_type() == at::kBFloat16, logits.size(0),
                logits.size(1), logits.stride(0), cur_stream());
}

void apply_penalties_(torch::Tensor logits, torch::Tensor triples, torch::Tensor rep, torch::Tensor freq,
                      torch::Tensor pres) {
  check_cuda(logits, "logits");
  TORCH_CHECK(logits.scalar_type() == at::kFloat && logits.stride(1) == 1, "penalties: fp32 logits");
  check_i32(triples, "triples");
  TORCH_CHECK(triples.is_contiguous() && (triples.numel() == 0 || triples.size(1) == 3), "triples [n, 3]");
  launch_penalties(logits.data_ptr<float>(), logits.stride(0), triples.data_ptr<int>(), triples.size(0),
                   rep.data_ptr<float>(), freq.data_ptr<float>(), pres.data_ptr<float>(), cur_stream());
}

void sample_out(torch::Tensor out, torch::Tensor logits, torch::Tensor temps, torch::Tensor top_ks,
                torch::Tensor top_ps, torch::Tensor min_ps, torch::Tensor seeds, torch::Tensor offsets) {
  check_cuda(logits, "logits");
  TORCH_CHECK(logits.dim() == 2 && logits.stride(1) == 1, "sample: [B, V] logits");
  TORCH_CHECK(logits.scalar_type() == at::kFloat || logits.scalar_type() == at::kBFloat16, "sample: fp32/bf16");
  TORCH_CHECK(temps.scalar_type() == at::kFloat && top_ps.scalar_type() == at::kFloat &&
                  min_ps.scalar_type() == at::kFloat && top_ks.scalar_type() == at::kInt &&
                  seeds.scalar_type() == at::kLong && offsets.scalar_type() == at::kLong &&
                  out.scalar_type() == at::kLong,
              "sample: parameter dtypes");
  launch_sample(out.data_ptr<int64_t>(), logits.data_ptr(), logits.scalar_type() == at::kBFloat16, logits.size(0),
                logits.size(1), logits.stride(0), temps.data_ptr<float>(), top_ks.data_ptr<int>(),
                top_ps.data_ptr<float>(), min_ps.data_ptr<float>(), seeds.data_ptr<int64_t>(),
                offsets.data_ptr<int64_t>(), cur_stream());
}

// ---------------------------------------------------------------- symmetric heap + TP collectives
torch::Tensor symm_alloc_tensor(int64_t bytes, int64_t device) {
  c10::cuda::CUDAGuard guard((c10::DeviceIndex)device);
  void* p = symm_alloc((size_t)bytes);
  return torch::from_blob(p, {bytes}, [](void* q) { symm_free(q); },
                          torch::TensorOptions().dtype(torch::kUInt8).device(torch::kCUDA, device));
}

pybind11::bytes symm_handle_py(torch::Tensor region) {
  auto h = symm_ipc_handle(region.data_ptr());
  return pybind11::bytes(reinterpret_cast<const char*>(h.data()), h.size());
}

uint64_t symm_open_py(pybind11::bytes handle) {
  std::string s = handle;
  std::vector<uint8_t> h(s.begin(), s.end());
  return reinterpret_cast<uint64_t>(symm_open_peer(h));
}

void symm_close_py(uint64_t p) { symm_close_peer(reinterpret_cast<void*>(p)); }

int64_t symm_status_py(torch::Tensor region) { return (int64_t)symm_read_status(region.data_ptr()); }

void tp_ar_rmsnorm_py(std::vector<uint64_t> bases, int64_t rank, int64_t p0, int64_t p1, int64_t g, int64_t parity,
                      bool one_shot, torch::Tensor residual, torch::Tensor w, torch::Tensor x_out, double eps,
                      double timeout_s, int64_t grid) {
  check_bf16(residual, "residual");
  check_bf16(w, "w");
  check_bf16(x_out, "x_out");
  TORCH_CHECK(residual.is_contiguous() && x_out.is_contiguous() && residual.sizes() == x_out.sizes(),
              "residual / x_out must be contiguous [T, d]");
  launch_tp_ar_rmsnorm(bases, (int)rank, p0, p1, g, (int)parity, one_shot, residual.data_ptr(), w.data_ptr(),
                       x_out.data_ptr(), residual.size(0), residual.size(1), (float)eps, timeout_s, (int)grid,
                       cur_stream());
}

// Row-parallel GEMM with the push epilogue: out = a · bᵀ ([T, N], this rank's inbox slot, a view of
// the symmetric region) plus the same tiles into every peer's inbox and per-tile ready flags.
void gemm_push_py(torch::Tensor out, torch::Tensor a, torch::Tensor b, int64_t bn, std::vector<uint64_t> bases,
                  int64_t rank, int64_t inbox_off, int64_t slot_elems, int64_t flags_off, int64_t g_max,
                  int64_t nt_max) {
  check_bf16(a, "a");
  check_bf16(b, "b");
  check_bf16(out, "out");
  TORCH_CHECK(a.dim() == 2 && b.dim() == 2 && a.size(1) == b.size(1) && a.stride(1) == 1 && b.stride(1) == 1,
              "push gemm: K-major operands");
  TORCH_CHECK(out.is_contiguous() && out.size(0) == a.size(0) && out.size(1) == b.size(0), "push gemm: out [T, N]");
  launch_gemm_push(out.data_ptr(), a.data_ptr(), a.stride(0), b.data_ptr(), b.stride(0), a.size(0), b.size(0),
                   a.size(1), (int)bn, bases, (int)rank, inbox_off, slot_elems, flags_off, (int)g_max, (int)nt_max,
                   nullptr, cur_stream());
}

void tp_push_ar_rmsnorm_py(std::vector<uint64_t> bases, int64_t rank, int64_t inbox_off, int64_t slot_elems,
                           int64_t flags_off, int64_t g_max, int64_t nt_max, int64_t nt, torch::Tensor residual,
                           torch::Tensor w, torch::Tensor x_out, double eps, double timeout_s, int64_t grid) {
  check_bf16(residual, "residual");
  check_bf16(w, "w");
  check_bf16(x_out, "x_out");
  TORCH_CHECK(residual.is_contiguous() && x_out.is_contiguous() && residual.sizes() == x_out.sizes(),
              "residual / x_out must be contiguous [T, d]");
  launch_tp_push_ar_rmsnorm(bases, (int)rank, inbox_off, slot_elems, flags_off, (int)g_max, (int)nt_max, (int)nt,
                            residual.data_ptr(), w.data_ptr(), x_out.data_ptr(), residual.size(0), residual.size(1),
                            (float)eps, timeout_s, (int)grid, cur_stream());
}

void tp_argmax_py(std::vector<uint64_t> bases, int64_t rank, torch::Tensor logits, int64_t vocab_offset,
                  int64_t cand_off, int64_t cand_rows, int64_t parity, torch::Tensor out, double timeout_s) {
  check_bf16(logits, "logits");
  TORCH_CHECK(logits.dim() == 2 && logits.stride(1) == 1, "tp argmax: logits [B, V_local] row-major");
  TORCH_CHECK(out.is_cuda() && out.scalar_type() == at::kLong && out.numel() >= logits.size(0), "tp argmax: out int64 [B]");
  launch_tp_argmax(bases, (int)rank, logits.data_ptr(), logits.stride(0), logits.size(0), logits.size(1), vocab_offset,
                   cand_off, (int)cand_rows, (int)parity, out.data_ptr<int64_t>(), timeout_s, cur_stream());
}

void tp_allreduce_py(std::vector<uint64_t> bases, int64_t rank, int64_t p0, int64_t p1, int64_t parity,
                     torch::Tensor out, double timeout_s, int64_t grid) {
  check_bf16(out, "out");
  TORCH_CHECK(out.is_contiguous(), "out must be contiguous");
  launch_tp_allreduce(bases, (int)rank, p0, p1, (int)parity, out.data_ptr(), out.numel(), timeout_s, (int)grid,
                      cur_stream());
}

// NVLS: `uc` / `mc` are this rank's local and multicast addresses of the symmetric region.
void tp_nvls_ar_rmsnorm_py(uint64_t uc, uint64_t mc, int64_t rank, int64_t world, int64_t p0, int64_t p1,
                           int64_t x_off, int64_t parity, int64_t mode, torch::Tensor residual, torch::Tensor w,
                           c10::optional<torch::Tensor> x_local, double eps, double timeout_s, int64_t grid) {
  check_bf16(residual, "residual");
  check_bf16(w, "w");
  TORCH_CHECK(residual.dim() == 2 && residual.is_contiguous(), "residual must be contiguous [T, d]");
  TORCH_CHECK(w.numel() == residual.size(1), "norm weight must have d elements");
  void* xl = nullptr;
  if (x_local.has_value()) {
    check_bf16(*x_local, "x_local");
    TORCH_CHECK(x_local->is_contiguous() && x_local->sizes() == residual.sizes(), "x_local must match residual");
    xl = x_local->data_ptr();
  }
  launch_tp_nvls_ar_rmsnorm(uc, mc, (int)rank, (int)world, p0, p1, x_off, (int)parity, (int)mode, residual.data_ptr(),
                            w.data_ptr(), xl, residual.size(0), residual.size(1), (float)eps, timeout_s, (int)grid,
                            cur_stream());
}

void tp_nvls_allreduce_py(uint64_t uc, uint64_t mc, int64_t rank, int64_t world, int64_t p0, int64_t p1,
                          int64_t parity, bool one_shot, int64_t numel, c10::optional<torch::Tensor> out,
                          double timeout_s, int64_t grid) {
  void* o = nullptr;
  if (out.has_value()) {
    check_bf16(*out, "out");
    TORCH_CHECK(out->is_contiguous() && out->numel() == numel, "out must be contiguous with numel elements");
    o = out->data_ptr();
  }
  launch_tp_nvls_allreduce(uc, mc, (int)rank, (int)world, p0, p1, (int)parity, one_shot, o, numel, timeout_s,
                           (int)grid, cur_stream());
}

// Column all-gather of a [B, v] bf16 shard into a [B, ld] buffer at byte offset dst_off of every
// rank's region; mc != 0 selects the NVLS multicast kernel.
void tp_gather_cols_py(std::vector<uint64_t> bases, uint64_t mc, int64_t rank, torch::Tensor src, int64_t dst_off,
                       int64_t ld, double timeout_s, int64_t grid) {
  check_bf16(src, "src");
  TORCH_CHECK(src.dim() == 2 && src.stride(1) == 1, "tp column gather: src [B, v] row-major");
  TORCH_CHECK(rank >= 0 && rank < (int64_t)bases.size(), "tp column gather: bad rank");
  if (mc != 0)
    launch_tp_nvls_gather_cols(bases[rank], mc, (int)rank, (int)bases.size(), src.data_ptr(), src.stride(0),
                               src.size(0), src.size(1), dst_off, ld, timeout_s, (int)grid, cur_stream());
  else
    launch_tp_gather_cols(bases, (int)rank, src.data_ptr(), src.stride(0), src.size(0), src.size(1), dst_off, ld,
                          timeout_s, (int)grid, cur_stream());
}

// ---------------------------------------------------------------- expert-parallel all-to-all (C3)
static EpLayout ep_layout_from(const std::vector<int64_t>& v) {
  TORCH_CHECK(v.size() == 8, "EP layout: [flags, counts, recv, meta, comb, x offsets, cap_src, cap_tok]");
  EpLayout l;
  l.flags_off = v[0];
  l.counts_off = v[1];
  l.recv_off = v[2];
  l.meta_off = v[3];
  l.comb_off = v[4];
  l.x_off = v[5];
  l.cap_src = (int)v[6];
  l.cap_tok = (int)v[7];
  return l;
}

void moe_route_py(torch::Tensor x, torch::Tensor router, int64_t topk, bool renorm, int64_t scoring,
                  c10::optional<torch::Tensor> score_bias, int64_t n_group, int64_t topk_group, double scale,
                  c10::optional<torch::Tensor> expert_map, c10::optional<torch::Tensor> logits, torch::Tensor ids,
                  torch::Tensor wts, torch::Tensor scratch) {
  check_bf16(x, "x");
  check_bf16(router, "router");
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1 && router.is_contiguous() && router.size(1) == x.size(1),
              "moe route: x [T, H] row-major, router [E, H]");
  TORCH_CHECK(ids.scalar_type() == at::kInt && wts.scalar_type() == at::kFloat && ids.numel() >= x.size(0) * topk &&
                  wts.numel() >= x.size(0) * topk,
              "moe route: ids int32 / wts fp32 [T * k]");
  MoeRouting rt;
  rt.scoring = (int)scoring;
  rt.n_group = (int)n_group;
  rt.topk_group = (int)topk_group;
  rt.scale = (float)scale;
  if (score_bias.has_value()) rt.bias = score_bias->data_ptr<float>();
  if (expert_map.has_value()) rt.expert_map = expert_map->data_ptr<int>();
  if (logits.has_value()) rt.logits = logits->data_ptr<float>();
  launch_moe_route(x.data_ptr(), x.stride(0), router.data_ptr(), x.size(0), x.size(1), router.size(0), (int)topk,
                   renorm ? 1 : 0, rt, ids.data_ptr<int>(), wts.data_ptr<float>(), scratch.data_ptr<int>(),
                   cur_stream());
}

void ep_dispatch_py(std::vector<uint64_t> bases, uint64_t mc, std::vector<int64_t> layout, int64_t rank, int64_t e_loc,
                    int64_t k, torch::Tensor x, torch::Tensor ids, torch::Tensor ws, double timeout_s) {
  check_bf16(x, "x");
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1, "EP dispatch: x [Tn, H] row-major");
  TORCH_CHECK(ids.scalar_type() == at::kInt && ids.is_contiguous() && ids.numel() >= x.size(0) * k, "EP dispatch: ids");
  TORCH_CHECK(ws.scalar_type() == at::kInt && ws.numel() >= ep_ws_ints((int)bases.size(), (int)e_loc), "EP dispatch: ws");
  launch_ep_dispatch(bases, mc, ep_layout_from(layout), (int)rank, (int)e_loc, (int)k, x.data_ptr(), x.stride(0),
                     x.size(1), ids.data_ptr<int>(), x.size(0), ws.data_ptr<int>(), timeout_s, cur_stream());
}

void ep_compact_py(std::vector<uint64_t> bases, uint64_t mc, std::vector<int64_t> layout, int64_t rank, int64_t e_loc,
                   int64_t k, torch::Tensor xg, torch::Tensor comb_ptr, torch::Tensor tile_group, torch::Tensor num_m,
                   double timeout_s) {
  check_bf16(xg, "xg");
  TORCH_CHECK(comb_ptr.scalar_type() == at::kLong && comb_ptr.numel() >= xg.size(0), "EP compact: comb_ptr int64 [cap]");
  TORCH_CHECK(tile_group.scalar_type() == at::kInt && tile_group.numel() >= xg.size(0) / 128 &&
                  num_m.scalar_type() == at::kInt,
              "EP compact: tile map int32");
  launch_ep_compact(bases, mc, ep_layout_from(layout), (int)rank, (int)e_loc, (int)k, xg.size(1), xg.data_ptr(),
                    reinterpret_cast<uint64_t*>(comb_ptr.data_ptr<int64_t>()), xg.size(0), tile_group.data_ptr<int>(),
                    num_m.data_ptr<int>(), timeout_s, cur_stream());
}

void ep_signal_py(std::vector<uint64_t> bases, uint64_t mc, std::vector<int64_t> layout, int64_t rank, int64_t e_loc,
                  int64_t k, int64_t H, double timeout_s) {
  launch_ep_signal(bases, mc, ep_layout_from(layout), (int)rank, (int)e_loc, (int)k, (int)H, timeout_s, cur_stream());
}

void ep_combine_norm_py(std::vector<uint64_t> bases, uint64_t mc, std::vector<int64_t> layout, int64_t rank,
                        int64_t e_loc, int64_t k, int64_t r0, int64_t Tn, torch::Tensor wts, torch::Tensor residual,
                        torch::Tensor w, double eps, double timeout_s) {
  check_bf16(residual, "residual");
  check_bf16(w, "w");
  TORCH_CHECK(residual.dim() == 2 && residual.is_contiguous() && r0 + Tn <= residual.size(0), "EP combine: residual");
  TORCH_CHECK(wts.scalar_type() == at::kFloat && wts.numel() >= Tn * k, "EP combine: wts fp32 [Tn * k]");
  launch_ep_combine_norm(bases, mc, ep_layout_from(layout), (int)rank, (int)e_loc, (int)k, residual.size(1),
                         residual.size(0), (int)r0, (int)Tn, wts.data_ptr<float>(), residual.data_ptr(), w.data_ptr(),
                         (float)eps, timeout_s, cur_stream());
}

// fp8 KV cache: step rows [T, 2, Hk, D] bf16 -> cache slots (uint8 e4m3 [NB, 2, Hk, bs, D]) + scales
void kv_quant_fp8_py(torch::Tensor kv, torch::Tensor slots, torch::Tensor cache, torch::Tensor scales) {
  check_bf16(kv, "kv");
  check_i32(slots, "slots");
  TORCH_CHECK(kv.dim() == 4 && kv.is_contiguous() && kv.size(1) == 2, "kv [T, 2, Hk, D]");
  TORCH_CHECK(cache.scalar_type() == at::kByte && cache.dim() == 5 && cache.is_contiguous() &&
                  cache.size(2) == kv.size(2) && cache.size(4) == kv.size(3),
              "fp8 cache uint8 [NB, 2, Hk, bs, D]");
  TORCH_CHECK(scales.scalar_type() == at::kFloat && scales.numel() == cache.numel() / cache.size(4), "scales fp32");
  TORCH_CHECK(slots.numel() >= kv.size(0), "one slot per token");
  launch_kv_quant_fp8(kv.data_ptr(), slots.data_ptr<int>(), cache.data_ptr(), scales.data_ptr<float>(), kv.size(0),
                      kv.size(2), kv.size(3), cache.size(3), cur_stream(), (int)cache.size(0));
}

void kv_dequant_blocks_py(torch::Tensor cache, torch::Tensor scales, torch::Tensor ids, torch::Tensor dst) {
  check_i32(ids, "ids");
  check_bf16(dst, "dst");
  TORCH_CHECK(cache.scalar_type() == at::kByte && cache.dim() == 5 && cache.is_contiguous(), "fp8 cache");
  TORCH_CHECK(scales.scalar_type() == at::kFloat && scales.numel() == cache.numel() / cache.size(4), "scales fp32");
  TORCH_CHECK(dst.is_contiguous() && dst.dim() == 5 && dst.size(0) >= ids.numel() && dst.size(1) == 2 &&
                  dst.size(2) == cache.size(2) && dst.size(3) == cache.size(3) && dst.size(4) == cache.size(4),
              "dst bf16 [n, 2, Hk, bs, D]");
  launch_kv_dequant_blocks(cache.data_ptr(), scales.data_ptr<float>(), ids.data_ptr<int>(), ids.numel(),
                           cache.size(0), cache.size(2), cache.size(4), cache.size(3), dst.data_ptr(), cur_stream());
}

// Grouped (per-expert) GEMM: out = a · b_g^T per M tile (tile_group names g); epi 0 none, 2 SwiGLU,
// 5 scatter (`out` is then the uint64 per-row destination table).
void gemm_grouped_py(torch::Tensor out, torch::Tensor a, torch::Tensor b, int64_t N, int64_t groups, int64_t epi,
                     torch::Tensor tile_group, torch::Tensor num_m) {
  check_bf16(a, "a");
  check_bf16(b, "b");
  TORCH_CHECK(a.dim() == 2 && a.stride(1) == 1 && b.dim() == 2 && b.stride(1) == 1 && a.size(1) == b.size(1),
              "grouped gemm: K-major operands");
  TORCH_CHECK(b.size(0) == N * groups, "grouped gemm: b [groups * N, K]");
  int64_t ldc = N;
  if (epi == kEpiScatter) {
    TORCH_CHECK(out.scalar_type() == at::kLong && out.numel() >= a.size(0), "grouped gemm scatter: int64 row table");
  } else {
    check_bf16(out, "out");
    ldc = out.stride(0);
    TORCH_CHECK(out.size(0) >= a.size(0), "grouped gemm: out rows");
  }
  launch_gemm_grouped(out.data_ptr(), ldc, a.data_ptr(), a.stride(0), b.data_ptr(), b.stride(0), a.size(0), (int)N,
                      a.size(1), (int)groups, (int)epi, 0, tile_group.data_ptr<int>(), num_m.data_ptr<int>(), 1,
                      nullptr, nullptr, cur_stream());
}

void lora_shrink_py(torch::Tensor V, torch::Tensor x, torch::Tensor A, torch::Tensor seg_ptr, torch::Tensor tok_idx,
                    torch::Tensor seg_slot, torch::Tensor tiles, int64_t max_seg) {
  check_cuda(V, "V");
  TORCH_CHECK(V.scalar_type() == at::kFloat && V.stride(1) == 1, "lora: V fp32 [T, R]");
  check_bf16(x, "x");
  check_bf16(A, "A");
  check_i32(seg_ptr, "seg_ptr");
  check_i32(tok_idx, "tok_idx");
  check_i32(seg_slot, "seg_slot");
  TORCH_CHECK(A.dim() == 3 && A.is_contiguous() && A.size(2) == x.size(1) && x.stride(1) == 1, "lora: A [slots, R, K]");
  TORCH_CHECK(V.size(1) >= A.size(1), "lora: V narrower than R");
  check_i32(tiles, "tiles");
  TORCH_CHECK(tiles.is_contiguous() && tiles.dim() == 2 && tiles.size(1) == 2, "lora: tiles [n, 2]");
  launch_lora_shrink(V.data_ptr<float>(), V.stride(0), x.data_ptr(), x.stride(0), A.data_ptr(), A.size(1), A.size(2),
                     seg_ptr.data_ptr<int>(), tok_idx.data_ptr<int>(), seg_slot.data_ptr<int>(), tiles.data_ptr<int>(),
                     tiles.size(0), seg_slot.numel(), (int)max_seg, cur_stream());
}

void lora_expand_py(torch::Tensor Y, torch::Tensor V, torch::Tensor B, int64_t n1, int64_t n2, torch::Tensor scales,
                    torch::Tensor seg_ptr, torch::Tensor tok_idx, torch::Tensor seg_slot, torch::Tensor tiles) {
  check_bf16(Y, "Y");
  check_cuda(V, "V");
  check_bf16(B, "B");
  TORCH_CHECK(V.scalar_type() == at::kFloat && V.is_contiguous(), "lora: V fp32 contiguous");
  TORCH_CHECK(B.dim() == 3 && B.is_contiguous() && B.size(1) == Y.size(1) && Y.stride(1) == 1, "lora: B [slots, N, r]");
  TORCH_CHECK(scales.scalar_type() == at::kFloat, "lora: fp32 scales");
  launch_lora_expand(Y.data_ptr(), Y.stride(0), V.data_ptr<float>(), V.size(1), B.data_ptr(), B.size(1), B.size(2),
                     (int)n1, (int)n2, scales.data_ptr<float>(), seg_ptr.data_ptr<int>(), tok_idx.data_ptr<int>(),
                     seg_slot.data_ptr<int>(), tiles.data_ptr<int>(), tiles.size(0), cur_stream());
}

void gguf_gemv_py(torch::Tensor y, torch::Tensor x, torch::Tensor W, int64_t qtype, int64_t N, int64_t K, bool swiglu) {
  check_bf16(y, "y");
  check_bf16(x, "x");
  check_cuda(W, "W");
  TORCH_CHECK(W.scalar_type() == at::kByte && W.is_contiguous(), "gguf: raw uint8 weight blocks");
  TORCH_CHECK(x.stride(1) == 1 && y.stride(1) == 1 && x.size(1) == K, "gguf gemv: shapes");
  TORCH_CHECK(x.stride(0) % 8 == 0, "gguf gemv: x row pitch must keep 16-byte alignment");
  launch_gguf_gemv(y.data_ptr(), y.stride(0), x.data_ptr(), x.stride(0), W.data_ptr(), (int)qtype, (int)N, (int)K,
                   x.size(0), swiglu, cur_stream());
}

void gguf_dequant_py(torch::Tensor out, torch::Tensor W, int64_t qtype) {
  check_bf16(out, "out");
  check_cuda(W, "W");
  TORCH_CHECK(W.scalar_type() == at::kByte && W.is_contiguous() && out.is_contiguous(), "gguf dequant: layout");
  launch_gguf_dequant(out.data_ptr(), W.data_ptr(), (int)qtype, out.numel(), cur_stream());
}

void embedding_q8_0_py(torch::Tensor out, torch::Tensor ids, torch::Tensor table, int64_t vocab) {
  check_bf16(out, "out");
  check_i32(ids, "ids");
  check_cuda(table, "table");
  TORCH_CHECK(out.is_contiguous(), "embedding: contiguous out");
  launch_embedding_q8_0(out.data_ptr(), ids.data_ptr<int>(), table.data_ptr(), ids.size(0), out.size(1), (int)vocab,
                        cur_stream());
}

void gemm_fp8_py(torch::Tensor out, torch::Tensor a, torch::Tensor sa, torch::Tensor b, torch::Tensor sb, int64_t epi,
                 int64_t splits, c10::optional<torch::Tensor> workspace, c10::optional<torch::Tensor> tile_cnt) {
  check_bf16(out, "out");
  check_cuda(a, "a");
  check_cuda(b, "b");
  TORCH_CHECK(a.scalar_type() == at::kFloat8_e4m3fn && b.scalar_type() == at::kFloat8_e4m3fn, "fp8: e4m3 operands");
  TORCH_CHECK(sa.scalar_type() == at::kFloat && sb.scalar_type() == at::kFloat && sa.is_contiguous() &&
                  sb.is_contiguous(),
              "fp8: fp32 contiguous scales");
  TORCH_CHECK(a.stride(1) == 1 && b.stride(1) == 1 && out.stride(1) == 1 && a.size(1) == b.size(1), "fp8: shapes");
  const int M = a.size(0), N = b.size(0), K = a.size(1);
  TORCH_CHECK(sa.numel() >= (int64_t)M * (K / 128) && sb.numel() >= (int64_t)((N + 127) / 128) * (K / 128),
              "fp8: scale tensors too small");
  TORCH_CHECK(out.size(0) == M && out.size(1) == (epi == kEpiSwiglu ? N / 2 : N), "fp8: out shape");
  int sp = (int)splits;
  if (sp <= 0) sp = gemm_fp8_splits(M, N, K, (int)epi);
  float* part = nullptr;
  if (sp > 1) {
    TORCH_CHECK(workspace.has_value() && workspace->scalar_type() == at::kFloat &&
                    workspace->numel() >= (int64_t)sp * M * N,
                "fp8 gemm: split-K ", sp, " needs an fp32 workspace of ", (int64_t)sp * M * N, " elements");
    part = workspace->data_ptr<float>();
  }
  int* cnt = nullptr;
  if (sp > 1 && tile_cnt.has_value()) {
    const int64_t tiles = (int64_t)((M + 127) / 128) * (N / 128);
    TORCH_CHECK(tile_cnt->is_cuda() && tile_cnt->scalar_type() == at::kInt && tile_cnt->numel() >= tiles,
                "fp8 gemm: ", tiles, " zeroed int32 tile counters expected");
    cnt = tile_cnt->data_ptr<int>();
  }
  launch_gemm_fp8(out.data_ptr(), out.stride(0), a.data_ptr(), a.stride(0), sa.data_ptr<float>(), b.data_ptr(),
                  b.stride(0), sb.data_ptr<float>(), M, N, K, (int)epi, sp, part, nullptr, cur_stream(), cnt);
}

void gemm_rope_kv_py(torch::Tensor q_out, torch::Tensor a, torch::Tensor w, torch::Tensor positions,
                     torch::Tensor cos_sin, c10::optional<torch::Tensor> cache, c10::optional<torch::Tensor> slots,
                     int64_t H, int64_t Hk) {
  check_bf16(a, "x");
  check_bf16(w, "w_qkv");
  check_bf16(q_out, "q_out");
  check_i32(positions, "positions");
  check_same_device(a, w);
  const int M = a.size(0), K = a.size(1);
  TORCH_CHECK(a.stride(1) == 1 && w.stride(1) == 1 && w.size(1) == K && w.size(0) == (H + 2 * Hk) * 128,
              "qkv gemm + rope: w [(H + 2 Hk) * 128, K]");
  TORCH_CHECK(q_out.is_contiguous() && q_out.numel() == (int64_t)M * H * 128, "qkv gemm + rope: q_out [T, H, 128]");
  TORCH_CHECK(cos_sin.scalar_type() == at::kFloat && cos_sin.is_contiguous() && cos_sin.size(1) == 128,
              "qkv gemm + rope: cos/sin table [max_pos, 128] fp32 (full rotary)");
  TORCH_CHECK(positions.numel() >= M, "qkv gemm + rope: one position per row");
  RopeArgs r;
  r.positions = positions.data_ptr<int>();
  r.cos_sin = cos_sin.data_ptr<float>();
  r.max_pos = (int)cos_sin.size(0);
  r.q_out = q_out.data_ptr();
  r.H = (int)H;
  r.Hk = (int)Hk;
  if (cache.has_value() && slots.has_value()) {
    check_bf16(*cache, "kv_cache");
    check_i32(*slots, "slots");
    TORCH_CHECK(cache->dim() == 5 && cache->size(1) == 2 && cache->size(2) == Hk && cache->size(4) == 128 &&
                    cache->is_contiguous() && slots->numel() >= M,
                "qkv gemm + rope: cache [blocks, 2, Hk, block_size, 128] bf16, one slot per row");
    r.cache = cache->data_ptr();
    r.slots = slots->data_ptr<int>();
    r.block_size = (int)cache->size(3);
    r.num_blocks = (int)cache->size(0);
  }
  launch_gemm_rope_kv(a.data_ptr(), a.stride(0), w.data_ptr(), w.stride(0), M, K, r, cur_stream());
}

void gemm_q4k_py(torch::Tensor out, torch::Tensor a, torch::Tensor w, int64_t N, int64_t K, int64_t epi,
                 int64_t splits, c10::optional<torch::Tensor> workspace) {
  check_bf16(a, "a");
  check_bf16(out, "out");
  check_cuda(w, "w");
  TORCH_CHECK(w.scalar_type() == at::kByte && w.is_contiguous() && w.numel() == N * (K / 256) * 144,
              "q4k gemm: raw Q4_K blocks [N, K/256 * 144] uint8");
  TORCH_CHECK(a.stride(1) == 1 && a.size(1) == K && out.stride(1) == 1, "q4k gemm: a [M, K], row-major out");
  const int M = a.size(0);
  TORCH_CHECK(out.size(0) == M && out.size(1) == (epi == kEpiSwiglu ? N / 2 : N), "q4k gemm: out shape");
  int sp = (int)splits;
  if (sp <= 0) sp = gemm_q4k_splits(M, (int)N, (int)K);
  float* part = nullptr;
  if (sp > 1) {
    TORCH_CHECK(workspace.has_value() && workspace->scalar_type() == at::kFloat && workspace->numel() >= (int64_t)sp * M * N,
                "q4k gemm: split-K ", sp, " needs an fp32 workspace of ", (int64_t)sp * M * N, " elements");
    part = workspace->data_ptr<float>();
  }
  launch_gemm_q4k(out.data_ptr(), out.stride(0), a.data_ptr(), a.stride(0), w.data_ptr(), M, (int)N, (int)K, (int)epi,
                  sp, part, nullptr, cur_stream());
}

void act_quant_fp8_py(torch::Tensor q, torch::Tensor scale, torch::Tensor x) {
  check_bf16(x, "x");
  TORCH_CHECK(q.scalar_type() == at::kFloat8_e4m3fn && q.is_contiguous() && scale.scalar_type() == at::kFloat,
              "act quant: e4m3 out, fp32 scales");
  TORCH_CHECK(x.stride(1) == 1, "act quant: row-major x");
  launch_act_quant_fp8(q.data_ptr(), scale.data_ptr<float>(), x.data_ptr(), x.stride(0), x.size(0), x.size(1),
                       cur_stream());
}

void weight_quant_fp8_py(torch::Tensor q, torch::Tensor scale, torch::Tensor w) {
  check_bf16(w, "w");
  TORCH_CHECK(w.is_contiguous() && q.is_contiguous() && q.scalar_type() == at::kFloat8_e4m3fn, "weight quant: layout");
  launch_weight_quant_fp8(q.data_ptr(), scale.data_ptr<float>(), w.data_ptr(), w.size(0), w.size(1), cur_stream());
}

int64_t gemm_fp8_splits_py(int64_t M, int64_t N, int64_t K, int64_t epi) {
  return gemm_fp8_splits((int)M, (int)N, (int)K, (int)epi);
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("gemm_fp8", &gemm_fp8_py, "block-scaled FP8 GEMM on tcgen05 (K6)", py::arg("out"), py::arg("a"),
        py::arg("sa"), py::arg("b"), py::arg("sb"), py::arg("epi"), py::arg("splits"), py::arg("workspace"),
        py::arg("tile_cnt") = py::none());
  m.def("gemm_fp8_splits", &gemm_fp8_splits_py);
  m.def("act_quant_fp8", &act_quant_fp8_py, "1x128 per-token-group FP8 quantisation (K7)");
  m.def("weight_quant_fp8", &weight_quant_fp8_py, "128x128 block FP8 weight quantisation");
  m.def("gguf_gemv", &gguf_gemv_py, "Q4_K / Q8_0 GEMV for up to 16 tokens (K9)");
  m.def("gguf_dequant", &gguf_dequant_py, "Q4_K / Q8_0 -> bf16 (K9)");
  m.def("embedding_q8_0", &embedding_q8_0_py, "embedding gather from a Q8_0 table (K9/K13)");
  m.def("lora_shrink", &lora_shrink_py, "multi-LoRA shrink V += x A^T per adapter segment (K10)");
  m.def("lora_expand", &lora_expand_py, "multi-LoRA expand Y += s V B^T per adapter segment (K10)");
  m.def("symm_alloc", &symm_alloc_tensor, "allocate a zeroed IPC-shareable device region (uint8 tensor)");
  m.def("symm_ipc_handle", &symm_handle_py);
  m.def("symm_open_peer", &symm_open_py);
  m.def("symm_close_peer", &symm_close_py);
  m.def("symm_status", &symm_status_py);
  m.def("tp_allreduce_add_rmsnorm", &tp_ar_rmsnorm_py, "fused TP all-reduce + residual add + RMSNorm over P2P");
  m.def("tp_allreduce", &tp_allreduce_py, "TP all-reduce over P2P");
  m.def("tp_nvls_allreduce_add_rmsnorm", &tp_nvls_ar_rmsnorm_py,
        "fused TP all-reduce + residual add + RMSNorm through NVLS multimem (sequence-parallel residual)");
  m.def("tp_nvls_allreduce", &tp_nvls_allreduce_py, "TP all-reduce through NVLS multimem");
  m.def("tp_gather_cols", &tp_gather_cols_py,
        "all-gather of vocab-parallel column shards (P2P stores, or NVLS multicast stores when mc != 0)");
  m.def("moe_route", &moe_route_py, "MoE routing only: physical expert ids and weights per token");
  m.def("ep_ws_ints", &ep_ws_ints);
  m.def("ep_dispatch", &ep_dispatch_py, "EP all-to-all dispatch: rows stored into the expert owners' buffers (P2P)");
  m.def("ep_compact", &ep_compact_py, "EP: received rows into the grouped-GEMM layout + combine destinations");
  m.def("ep_signal", &ep_signal_py, "EP: raise the combine flags of every source rank");
  m.def("ep_combine_norm", &ep_combine_norm_py,
        "EP combine: weighted sum of the returned rows + residual + RMSNorm, gathered via multimem.st");
  m.def("kv_quant_fp8", &kv_quant_fp8_py, "step K/V rows -> fp8 e4m3 cache slots + per-token scales");
  m.def("kv_dequant_blocks", &kv_dequant_blocks_py, "fp8 cache blocks -> bf16 blocks (prefill over an fp8 cache)");
  m.def("gemm_grouped", &gemm_grouped_py, "grouped tcgen05 GEMM (none / SwiGLU / scatter epilogue)");
  m.def(
      "set_bounds_status",
      [](c10::optional<torch::Tensor> st) {
        if (!st.has_value()) {
          bounds_status_slot() = nullptr;
          return;
        }
        TORCH_CHECK(st->is_cuda() && st->scalar_type() == at::kInt && st->numel() >= 2 && st->is_contiguous(),
                    "bounds status: int32 [2] on the GPU");
        bounds_status_slot() = reinterpret_cast<uint32_t*>(st->data_ptr<int>());
      },
      "bind (or, with None, unbind) the device status word of the kernels' bounds checks");
  m.def("set_gemm_sm_reserve", [](int64_t n) { gemm_sm_reserve() = (int)n; },
        "SMs the persistent GEMM grids leave free (for a collective running beside them)");
  m.def("tp_argmax", &tp_argmax_py, "distributed greedy argmax of vocab-parallel logits over P2P (C5)");
  m.def("gemm_push", &gemm_push_py, "row-parallel tcgen05 GEMM pushing its tiles to every rank's inbox (C1)");
  m.def("tp_push_allreduce_add_rmsnorm", &tp_push_ar_rmsnorm_py,
        "reduce pushed partials from local memory + residual + RMSNorm (C1 consumer)");
  m.doc() = "gollek_b200 sm_100a kernels";
  m.def("rms_norm", &rms_norm_out, "RMSNorm, or bias-free LayerNorm with center (K1)", py::arg("out"), py::arg("x"),
        py::arg("w"), py::arg("eps"), py::arg("center") = false);
  m.def("fused_add_rms_norm", &fused_add_rms_norm_out, "residual add + RMSNorm / LayerNorm (K1)", py::arg("out"),
        py::arg("x"), py::arg("residual"), py::arg("w"), py::arg("eps"), py::arg("center") = false);
  m.def("rope_kv_write", &rope_kv_write_out, "QKV split + RoPE + paged KV write (K2)");
  m.def("embedding", &embedding_out, "embedding gather (K13)");
  m.def("silu_mul", &silu_mul_out, "SwiGLU activation");
  m.def("paged_decode_attention", &paged_decode_attention_out, "paged decode attention (K3)");
  m.def("paged_prefill_attention", &paged_prefill_attention_out, "paged prefill attention (K4)");
  m.def("gemm_bf16", &gemm_bf16_out, "tcgen05 bf16 GEMM with fused epilogues (K5/K8)", py::arg("out"),
        py::arg("a"), py::arg("b"), py::arg("residual"), py::arg("epi"), py::arg("bn"), py::arg("status"),
        py::arg("grid_limit"), py::arg("splits"), py::arg("workspace"));
  m.def("gemm_pick_bn", &gemm_pick_bn, "tile width the GEMM would pick");
  m.def("gemm_plan", &gemm_plan_py, "(tile width, split-K factor) the GEMM picks for (M, N, K, epilogue)");
  m.def("gemm_rope_kv", &gemm_rope_kv_py,
        "QKV GEMM with the RoPE + paged KV-write epilogue (head_dim 128, full rotary, bf16 cache)");
  m.def("gemm_q4k", &gemm_q4k_py, "Q4_K weight dequantized inside a tcgen05 GEMM (plain / SwiGLU)");
  m.def("gemm_q4k_splits", [](int64_t M, int64_t N, int64_t K) { return gemm_q4k_splits((int)M, (int)N, (int)K); },
        "split-K factor of the fused Q4_K GEMM");
  m.def("gemm_retile", &gemm_retile_py, "(tile width, whole-wave tiles, narrow tail tile width or 0) of a GEMM");
  m.def("num_sms", &device_num_sms);
  m.def("moe_forward", &moe_forward_out, "MoE layer: route, permute, grouped tcgen05 expert GEMMs, combine (K12)",
        py::arg("out"), py::arg("x"), py::arg("router"), py::arg("w_gu"), py::arg("w_down"), py::arg("ws"),
        py::arg("ids"), py::arg("wts"), py::arg("dest"), py::arg("xp"), py::arg("hp"), py::arg("yp"),
        py::arg("ypart"), py::arg("topk"), py::arg("renorm"), py::arg("e0"), py::arg("e_loc"),
        py::arg("scoring") = 0, py::arg("score_bias") = py::none(), py::arg("n_group") = 1,
        py::arg("topk_group") = 1, py::arg("scale") = 1.0, py::arg("expert_map") = py::none(),
        py::arg("logits") = py::none());
  m.def("moe_capacity_rows", &moe_capacity_rows);
  m.def("int4_gemv", &int4_gemv_py, "4-bit group-quantized GEMV (GPTQ/AWQ/NF4), optional SwiGLU");
  m.def("int4_dequant", &int4_dequant_py, "4-bit group-quantized weights to bf16");
  m.def("kv_blocks", &kv_blocks_py, "gather (or scatter) one sequence's paged KV blocks, every layer");
  m.def("gdn_scan", &gdn_scan_py, "gated delta rule scan over varlen chunks (K14)");
  m.def("gdn_gated_norm", &gdn_gated_norm_py, "RMSNorm(o) * w * silu(g) per head");
  m.def("kv_key_norms", &kv_key_norms_py, "mean key L2 norm of each listed KV block (eviction scoring, K15)");
  m.def("moe_ws_ints", &moe_ws_ints);
  m.def("moe_logit_splits", &moe_logit_splits, "K splits of the tensor-core router logits for (T, E, H)");
  m.def("moe_plan", &moe_plan_py, "(gate/up tile width, down tile width, down split-K) for a MoE call");
  m.def("argmax", &argmax_out, "greedy argmax (K11)");
  m.def("apply_penalties", &apply_penalties_, "repetition/frequency/presence penalties (K11)");
  m.def("sample", &sample_out, "top-k/min-p/top-p sampling (K11)");
}
