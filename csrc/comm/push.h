// Shared layout of the symmetric heap (csrc/comm/symm.cu) and the push-epilogue arguments the
// row-parallel GEMM uses to write its output tiles straight into every rank's inbox (gemm.cu).
#pragma once
#include <cstdint>

namespace gollek {

// Header at the start of every rank's region (peers write into it).
struct SymmHeader {
  uint32_t flag_a[16];   // flag_a[src] = epoch when rank src entered call `epoch`
  uint32_t flag_b[16];   // flag_b[src] = epoch when rank src finished phase 1
  uint32_t arrive;       // local CTA arrive counter for barrier B / call completion
  uint32_t epoch;        // last completed call
  uint32_t status;       // kStatus* bits
  // NVLS collectives (csrc/comm/nvls.cu): counters every rank increments on all ranks at once
  // through the multicast address, and this rank's count of completed NVLS calls
  uint32_t nv_a;         // += 1 per rank when its partial is written (barrier A)
  uint32_t nv_c;         // += 1 per rank when its multicast stores are done (barrier C)
  uint32_t nv_epoch;     // last completed NVLS call
  uint32_t nv_arrive;    // local CTA arrive counter of the NVLS kernels
  // expert-parallel all-to-all (csrc/comm/ep_a2a.cu)
  uint32_t ep_epoch;     // last completed MoE layer
  uint32_t ep_arrive;    // local CTA arrive counter of the combine kernel
  uint32_t ep_done;      // += 1 per rank (multicast) when its gathered rows are stored
  uint32_t pad[22];
};
static_assert(sizeof(SymmHeader) == 256, "header size");

// GEMM → all-reduce push path. Rank `rank`'s GEMM stores its [T, N] partial tile by tile into
// inbox slot `rank` of every rank (bases[p] + inbox_off + rank * slot_elems * 2 bytes), then
// raises flags[(rank * g_max + row_group) * nt_max + n_tile] = epoch in every rank's flag array
// (row_group = 32 output rows, the rows one epilogue warp owns). The consumer kernel waits for the
// flags of its rows from every source and reduces from local memory.
struct PushArgs {
  uint8_t* bases[8];
  int64_t inbox_off;     // byte offset of this call's inbox in every region
  int64_t slot_elems;    // elements per source slot (max_tokens * N)
  int64_t flags_off;     // byte offset of the uint32 flag array
  int world, rank, g_max, nt_max;
};

// Expert-parallel all-to-all region inside every rank's symmetric heap (csrc/comm/ep_a2a.cu);
// byte offsets from the region base.
struct EpLayout {
  int64_t flags_off;   // uint32 [2][8]: dispatch flags (by source), combine flags (by expert owner)
  int64_t counts_off;  // int32 [world][E_loc]: rows received from each source per local expert
  int64_t recv_off;    // bf16 [world][cap_src][H]: rows received from each source
  int64_t meta_off;    // int4 [world][cap_src]: (token * k + choice, local expert, slot within it, 0)
  int64_t comb_off;    // bf16 [cap_tok * k][H]: expert rows returned to this (source) rank
  int64_t x_off;       // bf16 [max_tokens][H]: gathered normalised rows (shared with the NVLS kernels)
  int cap_src;         // rows one source may send one destination
  int cap_tok;         // owned tokens per rank, at most
};

}  // namespace gollek
