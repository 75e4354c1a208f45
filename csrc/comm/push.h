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
  uint32_t pad[29];
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

}  // namespace gollek
