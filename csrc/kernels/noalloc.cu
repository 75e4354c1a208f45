// Allocation-free C entry point for split-KV paged decode attention.
//
// This entry point has no counterpart in the reference implementation; it exists for callers
// of this library that cannot allocate device memory themselves: hosts whose own memory manager
// owns the whole device budget and forbids allocations by libraries, and latency-critical serving
// loops that must never enter an allocator. Such a caller passes its inputs and its output buffer;
// the kernel's scratch (the split-KV partial results) lives in one fixed file-scope device array
// instead of a caller- or allocator-provided workspace. The C declarations are in noalloc.h.
//
// Call it from ordinary host code, not from inside a CUDA host callback or stream-ordered host
// function: it makes CUDA runtime calls (device query, symbol lookup, launch), which CUDA does not
// allow there.
//
// Contract:
//   * Scratch capacity: kNoAllocScratchBytes (8 MiB) per device. A call needs
//     B * H * num_splits * (head_dim + 2) * 4 bytes; larger requests return
//     GOLLEK_NOALLOC_ERR_SCRATCH without launching anything.
//   * The first call on a device looks up the array's device address (cudaGetSymbolAddress,
//     with that device current) and caches it. Make that first call outside any stream capture.
//   * The array is shared by every call on the device and keeps the previous call's contents.
//     Nothing in it needs to start at zero: each call writes every partial it later reads.
//     Calls whose kernels overlap on the GPU (different streams without ordering) race on the
//     array; serialise them (one stream, or events).
//   * No cudaMalloc / cudaFree / allocating library call is made, ever.
//   * Every loaded copy of this library holds the array on every GPU that uses it, until exit.
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

#include "launchers.h"
#include "noalloc.h"

namespace {

constexpr size_t kNoAllocScratchBytes = 8u << 20;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_decode_scratch[kNoAllocScratchBytes];

std::mutex g_mu;
void* g_scratch_addr[kMaxDevices] = {nullptr};

// Device address of the scratch array for the current device (looked up once per device).
cudaError_t scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_scratch_addr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_decode_scratch);
    if (e != cudaSuccess) return e;
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return cudaSuccess;
}

// head_dim / group pairs the decode kernels are built for (csrc/kernels/attention.cu)
bool decode_shape_supported(int head_dim, int group) {
  const bool g8 = group == 1 || group == 2 || group == 4 || group == 8;
  switch (head_dim) {
    case 32: case 64: case 256: return g8;
    case 128: return g8 || group == 16;
    default: return false;
  }
}

}  // namespace

// Split-KV paged decode attention without any allocation.
//   out          [B, H, head_dim] bf16 (written)
//   q            [B, H, head_dim] bf16, rows q_stride elements apart
//   cache        [num_blocks, 2, Hk, block_size, head_dim] bf16 (one layer's paged KV)
//   block_tables [B, bt_stride] int32, seq_lens [B] int32 (KV length per sequence)
// Returns GOLLEK_NOALLOC_OK or one of the error codes of noalloc.h; `stream` may be 0.
extern "C" __attribute__((visibility("default"))) int gollek_paged_decode_attention_noalloc(
    void* out, const void* q, int64_t q_stride, const void* cache, int num_blocks, const int* block_tables,
    int bt_stride, const int* seq_lens, int B, int H, int Hk, int head_dim, int block_size, int num_splits,
    float scale, cudaStream_t stream) {
  if (!out || !q || !cache || !block_tables || !seq_lens || B <= 0 || H <= 0 || Hk <= 0 || head_dim <= 0 ||
      num_splits <= 0 || num_blocks <= 0 || H % Hk != 0)
    return GOLLEK_NOALLOC_ERR_ARGS;
  if (block_size != 16 || !decode_shape_supported(head_dim, H / Hk)) return GOLLEK_NOALLOC_ERR_UNSUPPORTED;
  const size_t need = (size_t)B * H * num_splits * (head_dim + 2) * sizeof(float);
  if (need > kNoAllocScratchBytes) return GOLLEK_NOALLOC_ERR_SCRATCH;
  void* scratch = nullptr;
  if (scratch_address(&scratch) != cudaSuccess) return GOLLEK_NOALLOC_ERR_CUDA;
  float* part_o = static_cast<float*>(scratch);
  float* part_ml = part_o + (size_t)B * H * num_splits * head_dim;
  try {
    gollek::launch_paged_decode(out, q, q_stride, cache, num_blocks, block_tables, bt_stride,
                                seq_lens, B, H, Hk, head_dim, block_size, num_splits, scale,
                                num_splits > 1 ? part_o : nullptr, num_splits > 1 ? part_ml : nullptr,
                                /*window=*/0, /*softcap=*/0.f, stream);
  } catch (...) {  // the arguments were validated above: what remains is a failed launch
    return GOLLEK_NOALLOC_ERR_CUDA;
  }
  return GOLLEK_NOALLOC_OK;
}

// Capacity of the scratch array in bytes (for callers sizing their requests).
extern "C" __attribute__((visibility("default"))) size_t gollek_paged_decode_attention_noalloc_scratch_bytes() {
  return kNoAllocScratchBytes;
}
