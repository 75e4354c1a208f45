// Host launchers of the sm_100a kernels. The .cu files include only CUDA headers (fast nvcc
// builds); argument checking against torch tensors lives in csrc/bindings.cpp. Launchers throw
// std::runtime_error (surfaced as RuntimeError in Python) on invalid arguments or launch errors.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <stdexcept>
#include <string>
#include <vector>

#include "../comm/push.h"

namespace gollek {


inline void throw_if(bool bad, const std::string& msg) {
  if (bad) throw std::runtime_error(msg);
}
inline void check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

// ---- elementwise (K1, K2, K13)
void launch_rms_norm(void* out, const void* x, void* residual, const void* w, int T, int d, int64_t x_stride,
                     int64_t out_stride, float eps, cudaStream_t s,
                     bool center = false);
void launch_rope_kv_write(void* q_out, const void* qkv, const int* positions, const float* cos_sin, void* cache,
                          const int* slots, int T, int H, int Hk, int D, int block_size, int64_t qkv_stride,
                          int max_pos, const void* bias, const void* q_norm, const void* k_norm, float norm_eps,
                          int rot, cudaStream_t s, int num_blocks = 0);
void launch_embedding(void* out, const int* ids, const void* table, int T, int d, int vocab, float scale,
                      cudaStream_t s);
void launch_silu_mul(void* out, const void* x, int T, int d, cudaStream_t s);

// ---- attention (K3, K4)
// num_blocks > 0 enables the tensor-core path for head_dim 128 (needs the cache extent for its TMA map).
// Attention options: window > 0 restricts each query to the `window` most recent keys (sliding
// window, HF semantics kv > q - window); softcap > 0 applies softcap * tanh(score / softcap) to the
// scaled scores before the softmax (Gemma-2). 0 disables either.
// kv_scales != nullptr: the cache holds fp8 e4m3 values with one fp32 scale per (block, K/V, kv head,
// token) in kv_scales [NB, 2, Hk, 16] (head_dim 128, tensor-core kernel).
void launch_paged_decode(void* out, const void* q, int64_t q_stride, const void* cache, int num_blocks,
                         const int* block_tables, int bt_stride, const int* seq_lens, int B, int H, int Hk, int D,
                         int block_size, int num_splits, float scale, float* part_o, float* part_ml,
                         int window, float softcap, cudaStream_t s, const float* kv_scales = nullptr,
                         bool tensor_cores = true);
void launch_paged_prefill_tc(void* out, int64_t out_stride, const void* q, int64_t q_rows, int64_t q_stride,
                             const void* cache, int num_blocks, const int* block_tables, int bt_stride,
                             const int* seq_lens, const int* query_start, const int* tiles, int ntiles, int H,
                             int Hk, float scale, int window, float softcap, cudaStream_t s);
// Two-tile tcgen05 prefill (head_dim 64 or 128, block 16). work: one int4 per CTA (sequence, query offset of
// slot 0, query offset of slot 1 or -1, (pair << 16) | head): pair = 1 runs heads head and head + 1 (one
// GQA group, so the group size must be even) over the same query rows; pair = 0 runs two query tiles
// of one head. emu: share of exponentials on the FMA pipe (0 none, 1 a quarter, 2 half).
void launch_paged_prefill_fa(void* out, int64_t out_stride, const void* q, int64_t q_rows, int64_t q_stride,
                             const void* cache, int num_blocks, const int* block_tables, int bt_stride,
                             const int* seq_lens, const int* query_start, const int* work, int nwork, int H, int Hk,
                             float scale, int window, float softcap, int emu, cudaStream_t s, int head_dim = 128);
void launch_paged_prefill(void* out, int64_t out_stride, const void* q, int64_t q_stride, const void* cache,
                          const int* block_tables, int bt_stride, const int* seq_lens, const int* query_start,
                          const int* tiles, int ntiles, int H, int Hk, int D, int block_size, float scale,
                          int window, float softcap, cudaStream_t s, int num_blocks = 0);

// ---- GEMM (K5, K8)
// Gated epilogues (SwiGLU, GeGLU) read gate/up rows interleaved in groups of 64 and write N/2 columns.
// kEpiPush: plain output, also pushed to every tensor-parallel peer's inbox (GEMM → all-reduce).
// kEpiScatter: output row r is stored at the address in a per-row table (the `out` argument is a
// uint64 [M] table; 0 = skip the row); the destinations may be peer memory (NVLink stores)
// kEpiRope: the QKV projection's epilogue: head_dim-128 heads [q (H) | k (Hk) | v (Hk)] per row;
// NeoX RoPE of q and k heads (cos/sin of the row's position), q to q_out [T, H, 128], k / v into
// the paged bf16 cache at the row's slot (the RopeArgs below); no [T, (H + 2Hk) * 128] output.
enum GemmEpilogue : int { kEpiNone = 0, kEpiResidual = 1, kEpiSwiglu = 2, kEpiGeglu = 3, kEpiPush = 4, kEpiScatter = 5,
                          kEpiRope = 6 };
inline bool epi_gated(int epi) { return epi == kEpiSwiglu || epi == kEpiGeglu; }
// epilogues that need whole 128-column groups in a tile (gate/up pairs, head_dim-128 heads)
inline bool epi_wide(int epi) { return epi_gated(epi) || epi == kEpiRope; }
struct RopeArgs {
  const int* positions = nullptr;   // [T]
  const float* cos_sin = nullptr;   // [max_pos, 128]: 64 cos, then 64 sin
  int max_pos = 0;
  void* q_out = nullptr;            // bf16 [T, H, 128]
  void* cache = nullptr;            // bf16 [num_blocks, 2, Hk, block_size, 128]
  const int* slots = nullptr;       // [T] cache slot of each row (< 0: not written)
  int H = 0, Hk = 0, block_size = 16, num_blocks = 0;
};
// QKV GEMM with the RoPE + paged KV-write epilogue (head_dim 128, full rotary, bf16 cache).
void launch_gemm_rope_kv(const void* a, int64_t lda, const void* b, int64_t ldb, int M, int K, const RopeArgs& rope,
                         cudaStream_t s);
int gemm_pick_bn(int M, int N, int epi);
void gemm_plan(int M, int N, int K, int epi, int& bn, int& splits);
int gemm_splits(int M, int N, int K, int epi);
// Tail re-tiling of a persistent GEMM with `tiles` bn-wide output tiles on `grid` CTAs: full_tiles
// (whole waves) stay bn wide, the rest are cut bnt wide (0: no re-tiling).
void gemm_retile_plan(int tiles, int grid, int bn, bool gated, int& full_tiles, int& bnt);
// splits: 0 = automatic (with bn = 0), 1 = none; partial: fp32 [splits, M, N] workspace when splits > 1.
void launch_gemm_bf16(void* out, int64_t ldc, const void* a, int64_t lda, const void* b, int64_t ldb,
                      const void* residual, int64_t ldr, int M, int N, int K, int epi, int bn, int splits,
                      float* partial, uint32_t* status, int grid_limit, cudaStream_t s);

// Row-parallel GEMM fused with the all-reduce's data movement: C = A·Bᵀ written to `out` (this
// rank's inbox slot) and to the same slot of every peer's inbox, with per-tile ready flags
// (layout in csrc/comm/push.h). Followed by launch_tp_push_ar_rmsnorm.
void launch_gemm_push(void* out, const void* a, int64_t lda, const void* b, int64_t ldb, int M, int N, int K, int bn,
                      const std::vector<uint64_t>& bases, int rank, int64_t inbox_off, int64_t slot_elems,
                      int64_t flags_off, int g_max, int nt_max, uint32_t* status, cudaStream_t s);
// C5: greedy argmax over a vocab-parallel logits shard ([B, V] bf16 rows at `stride`, global
// token ids start at vocab_offset); candidates cross NVLink, every rank gets the global ids.
void launch_tp_argmax(const std::vector<uint64_t>& bases, int rank, const void* logits, int64_t stride, int B, int V,
                      int64_t vocab_offset, int64_t cand_off, int cand_rows, int parity, int64_t* out,
                      double timeout_s, cudaStream_t s);
void launch_tp_push_ar_rmsnorm(const std::vector<uint64_t>& bases, int rank, int64_t inbox_off, int64_t slot_elems,
                               int64_t flags_off, int g_max, int nt_max, int nt, void* residual, const void* w,
                               void* x_out, int T, int d, float eps, double timeout_s, int grid, cudaStream_t s);

// Grouped GEMM (MoE experts): A rows grouped per expert and padded to 128, tile_group[m-tile] =
// expert, live M-tile count in device memory; B = experts stacked [groups * N, K].
void launch_gemm_grouped(void* out, int64_t ldc, const void* a, int64_t lda, const void* b, int64_t ldb, int M_cap,
                         int N, int K, int groups, int epi, int bn, const int* tile_group, const int* num_m_dev,
                         int splits, float* partial, uint32_t* status, cudaStream_t s);

// ---- MoE (K12 routing / permutation / combine around two grouped GEMMs)
int moe_capacity_rows(int T, int topk, int e_loc);
int moe_ws_ints(int T, int topk, int e_loc);
void moe_plan_host(int T, int topk, int E, int e_loc, int H, int F, int& bn_gu, int& bn_dn, int& splits);
// Router options: scoring 0 = softmax (Mixtral), 1 = sigmoid with the per-expert fp32 correction
// ``bias`` added for the choice only, top-k limited to the topk_group best of n_group groups,
// weights times ``scale`` (DeepSeek-V3).
struct MoeRouting {
  int scoring = 0;
  const float* bias = nullptr;
  int n_group = 1;
  int topk_group = 1;
  float scale = 1.f;
  const int* expert_map = nullptr;  // logical expert -> physical slot (expert-parallel re-placement)
  float* logits = nullptr;          // fp32 [splits, T, E] scratch: when set, logits are computed on tensor cores first
  int logit_splits = 1;             // set by the launcher (moe_logit_splits)
};
int moe_logit_splits(int T, int E, int H);
void launch_moe_forward(void* out, int64_t ldo, const void* x, int64_t ldx, const void* wr, const void* w_gu,
                        const void* w_down, int* ws, int* ids, float* wts, int* dest, void* xp, void* hp, void* yp,
                        float* ypart, int T, int H, int F, int E, int topk, int renorm, int e0, int e_loc,
                        const MoeRouting& rt, uint32_t* status, cudaStream_t s);

// ---- KV block transfer (P/D disaggregation): packed [L, n, span] <-> cache [L, NB, span]
// K14 gated delta rule: proj [T, ldp] = q | k | v | g | a | b per token (Hg heads of D = 128);
// out [T, Hg, D] raw o; state [slots, Hg, D, D] fp32 of one layer (slot stride in elements).
void launch_gdn_scan(const void* proj, int64_t ldp, void* out, float* state, int64_t state_slot_stride,
                     const int* slots, const int* reset, const int* query_start, int n, const float* a_log,
                     const float* dt_bias, int Hg, int D, cudaStream_t s);
void launch_gdn_gated_norm(void* y, const void* o, const void* g, int64_t ldg, const void* w, int T, int Hg, int D,
                           float eps, cudaStream_t s);
// Mean key L2 norm per listed block (KV eviction scoring); cache [L, NB, 2, Hk, bs, D] bf16.
void launch_kv_key_norms(const void* cache, const int* block_ids, float* out, int n, int layers, int64_t num_blocks,
                         int Hk, int bs, int D, cudaStream_t s);
void launch_kv_blocks(void* cache, void* packed, const int* block_ids, int n, int layers, int64_t num_blocks,
                      int64_t span, bool gather, cudaStream_t s);

// ---- 4-bit group-quantized weights (GPTQ / AWQ / RTN int4, NF4), canonical row-major layout
void launch_int4_gemv(void* out, int64_t ldo, const void* x, int64_t ldx, const void* q, const void* scale,
                      const void* zero, int M, int N, int K, int g, bool lut, bool swiglu, cudaStream_t s);
void launch_int4_dequant(void* out, const void* q, const void* scale, const void* zero, int N, int K, int g, bool lut,
                         cudaStream_t s);

// ---- sampling (K11)
void launch_argmax(int64_t* out, const void* logits, bool is_bf16, int B, int V, int64_t stride, cudaStream_t s);
void launch_penalties(float* logits, int64_t stride, const int* triples, int n, const float* rep, const float* freq,
                      const float* pres, cudaStream_t s);
void launch_sample(int64_t* out, const void* logits, bool is_bf16, int B, int V, int64_t stride, const float* temps,
                   const int* top_ks, const float* top_ps, const float* min_ps, const int64_t* seeds,
                   const int64_t* offsets, cudaStream_t s);

int device_num_sms();

// ---- block-scaled FP8 (K6, K7)
void launch_gemm_fp8(void* out, int64_t ldc, const void* a, int64_t lda, const float* sa, const void* b, int64_t ldb,
                     const float* sb, int M, int N, int K, int epi, int splits, float* partial, uint32_t* status,
                     cudaStream_t s, int* tile_cnt = nullptr);
int gemm_fp8_splits(int M, int N, int K, int epi);
void launch_act_quant_fp8(void* q, float* scale, const void* x, int64_t ldx, int M, int K, cudaStream_t s);
void launch_weight_quant_fp8(void* q, float* scale, const void* w, int N, int K, cudaStream_t s);
// Q4_K weight (ggml super-blocks, [N rows] x [K / 256 x 144 bytes]) dequantized inside a tcgen05 GEMM
// (csrc/kernels/gemm_q4k.cu): plain or SwiGLU epilogue (gate/up rows interleaved in groups of 64),
// split-K partials reduced by splitk_reduce. splits <= 0: automatic.
int gemm_q4k_splits(int M, int N, int K);
void launch_gemm_q4k(void* out, int64_t ldc, const void* a, int64_t lda, const void* w, int M, int N, int K, int epi,
                     int splits, float* partial, uint32_t* status, cudaStream_t s);
void splitk_reduce(void* out, int64_t ldc, const float* partial, const void* residual, int64_t ldr, int M, int N,
                   int splits, int epi, cudaStream_t s);

// ---- GGUF quantized weights (K9); qtype = ggml type id (8 = Q8_0, 12 = Q4_K)
void launch_gguf_gemv(void* y, int64_t ldy, const void* x, int64_t ldx, const void* W, int qtype, int N, int K,
                      int M, bool swiglu, cudaStream_t s);
void launch_gguf_dequant(void* out, const void* W, int qtype, int64_t numel, cudaStream_t s);
void launch_embedding_q8_0(void* out, const int* ids, const void* table, int T, int d, int vocab, cudaStream_t s);

// ---- multi-LoRA (K10)
// tiles: int32 pairs (segment, first index into tok_idx) of 64-token tiles of the segments
// V must be zero: K chunks accumulate atomically
void launch_lora_shrink(float* V, int ldv, const void* x, int64_t ldx, const void* A, int R, int K,
                        const int* seg_ptr, const int* tok_idx, const int* seg_slot, const int* tiles, int num_tiles,
                        int num_segs, int max_seg, cudaStream_t s);
void launch_lora_expand(void* Y, int64_t ldy, const float* V, int ldv, const void* B, int N, int rank, int n1,
                        int n2, const float* scales, const int* seg_ptr, const int* tok_idx, const int* seg_slot,
                        const int* tiles, int num_tiles, cudaStream_t s);

// ---- symmetric heap + tensor-parallel collectives (csrc/comm/symm.cu)
void* symm_alloc(size_t bytes);
void symm_free(void* p);
std::vector<uint8_t> symm_ipc_handle(void* p);
void* symm_open_peer(const std::vector<uint8_t>& handle);
void symm_close_peer(void* p);
uint32_t symm_read_status(void* base);
void launch_tp_ar_rmsnorm(const std::vector<uint64_t>& bases, int rank, int64_t p0, int64_t p1, int64_t g,
                          int parity, bool one_shot, void* residual, const void* w, void* x_out, int T, int d,
                          float eps, double timeout_s, int grid, cudaStream_t s);
void launch_tp_allreduce(const std::vector<uint64_t>& bases, int rank, int64_t p0, int64_t p1, int parity, void* out,
                         int64_t numel, double timeout_s, int grid, cudaStream_t s);
// All-gather of [B, v] column shards into columns [rank*v, (rank+1)*v) of a [B, ld] buffer at
// `dst_off` in every rank's region (vocab-parallel logits); P2P stores, or NVLS multicast stores.
void launch_tp_gather_cols(const std::vector<uint64_t>& bases, int rank, const void* src, int64_t src_stride, int B,
                           int v, int64_t dst_off, int64_t ld, double timeout_s, int grid, cudaStream_t s);

// ---- expert-parallel all-to-all (csrc/comm/ep_a2a.cu); EpLayout in csrc/comm/push.h
int ep_ws_ints(int world, int e_loc);
void launch_ep_dispatch(const std::vector<uint64_t>& bases, uint64_t mc, const EpLayout& lay, int rank, int e_loc,
                        int k, const void* x, int64_t ldx, int H, const int* ids, int Tn, int* ws, double timeout_s,
                        cudaStream_t s);
void launch_ep_compact(const std::vector<uint64_t>& bases, uint64_t mc, const EpLayout& lay, int rank, int e_loc,
                       int k, int H, void* xg, uint64_t* comb_ptr, int cap_dst, int* tile_group, int* num_m,
                       double timeout_s, cudaStream_t s);
void launch_ep_signal(const std::vector<uint64_t>& bases, uint64_t mc, const EpLayout& lay, int rank, int e_loc,
                      int k, int H, double timeout_s, cudaStream_t s);
void launch_ep_combine_norm(const std::vector<uint64_t>& bases, uint64_t mc, const EpLayout& lay, int rank,
                            int e_loc, int k, int H, int T, int r0, int Tn, const float* wts, void* residual,
                            const void* w, float eps, double timeout_s, cudaStream_t s);
void launch_moe_route(const void* x, int64_t ldx, const void* wr, int T, int H, int E, int topk, int renorm,
                      const MoeRouting& rt, int* ids, float* wts, int* scratch, cudaStream_t s);

// ---- fp8 e4m3 paged KV cache (csrc/kernels/kv_fp8.cu)
void launch_kv_quant_fp8(const void* kv, const int* slots, void* cache, float* scales, int T, int Hk, int D,
                         int block_size, cudaStream_t s, int num_blocks = 0);
void launch_kv_dequant_blocks(const void* cache, const float* scales, const int* ids, int n, int num_blocks, int Hk,
                              int D, int block_size, void* dst, cudaStream_t s);

// ---- NVLS (multimem) collectives over a multicast-bound symmetric region (csrc/comm/nvls.cu)
// mode: 0 one-shot, 1 two-shot (x gathered into every rank's x buffer), 2 reduce-scatter (owned rows local)
void launch_tp_nvls_ar_rmsnorm(uint64_t uc, uint64_t mc, int rank, int world, int64_t p0, int64_t p1, int64_t x_off,
                               int parity, int mode, void* residual, const void* w, void* x_local, int T, int d,
                               float eps, double timeout_s, int grid, cudaStream_t s);
void launch_tp_nvls_allreduce(uint64_t uc, uint64_t mc, int rank, int world, int64_t p0, int64_t p1, int parity,
                              bool one_shot, void* out, int64_t numel, double timeout_s, int grid, cudaStream_t s);
void launch_tp_nvls_gather_cols(uint64_t uc, uint64_t mc, int rank, int world, const void* src, int64_t src_stride,
                                int B, int v, int64_t dst_off, int64_t ld, double timeout_s, int grid, cudaStream_t s);

}  // namespace gollek
