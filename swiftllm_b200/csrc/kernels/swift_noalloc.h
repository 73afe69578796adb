// Allocation-free C entry point for split-KV paged decode attention.
//
// This entry point has no counterpart in the reference project: it is an
// addition of this library.
//
// Who it is for: callers that cannot allocate GPU memory while they run -
// for example code driven from inside another runtime's memory arena, a
// plugin host that forbids cudaMalloc/cudaFree on its hot path, or a C
// program that links this library without PyTorch (whose caching allocator
// the regular `paged_decode` binding relies on for its workspace). Such a
// caller passes only its inputs and outputs; the split-KV scratch lives in
// a fixed array inside this library.
//
// Scratch: a file-scope device array of SWIFT_NOALLOC_SCRATCH_BYTES (8 MiB)
// in attention_decode.cu. Every GPU that loads the library keeps it until the
// process exits. A call needs rows * Hq * splits * (head_dim + 2) * 4 bytes of
// it; larger requests are rejected with SWIFT_NOALLOC_ERR_TOO_LARGE. The
// kernels overwrite every scratch element they later read, so nothing has
// to be cleared between calls. All calls share the one array: calls whose
// work overlaps on the GPU (different streams, or different host threads on
// the same device) race on it and must be serialised by the caller.
//
// Failures inside the kernel: a bounded wait inside the kernel that runs out
// (a copy that never lands) makes it record a code in a second file-scope
// word and return without hanging; its output is then not valid. Read that
// word with swift_noalloc_status() after synchronising the stream: code 0
// means every call since the last clear completed normally.
//
// Set-up: the first call on each device looks up the array's device address
// (cudaGetSymbolAddress, with that device current) and sets the kernels'
// shared-memory limit; make that first call before any stream capture.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#define SWIFT_NOALLOC_SCRATCH_BYTES (8u << 20)

enum SwiftNoallocStatus {
  SWIFT_NOALLOC_OK = 0,
  SWIFT_NOALLOC_ERR_TOO_LARGE = 1,    // scratch need exceeds SWIFT_NOALLOC_SCRATCH_BYTES
  SWIFT_NOALLOC_ERR_UNSUPPORTED = 2,  // head_dim / block_size / GQA group not supported
  SWIFT_NOALLOC_ERR_CUDA = 3,         // a CUDA runtime call failed (see cudaGetLastError)
  SWIFT_NOALLOC_ERR_ARGS = 4,         // bad argument (null pointer, non-positive size,
                                      // pointer not 16-byte aligned, offset not a
                                      // multiple of 8 elements)
};

#ifdef __cplusplus
extern "C" {
#endif

// Same maths and layouts as swiftllm_b200._C.paged_decode with splits >= 1:
//   out, q     bf16 [rows, Hq, head_dim] (row-major, contiguous)
//   kv         bf16 paged pool [blocks, layers, 2, Hkv, block_size, head_dim]
//   blk_stride elements between blocks; layer_off = layer * (elements per
//              layer); kv_stride elements between the K and V halves
//   bt         int32 block table, row stride bt_stride; seq_lens int32 [rows]
//   window     sliding window in tokens (0: none)
// Launches on `stream`; returns a SwiftNoallocStatus.
int swift_paged_decode_noalloc(void* out, const void* q, const void* kv, int64_t blk_stride,
                               int64_t layer_off, int64_t kv_stride, int block_size, int head_dim,
                               const int32_t* bt, int64_t bt_stride, const int32_t* seq_lens,
                               int rows, int Hq, int Hkv, int splits, float scale, int window,
                               cudaStream_t stream);

// Status word of the allocation-free calls on the current device: *code = 0
// (no failure), 1 (a bounded wait inside a kernel gave up); *site = where.
// clear != 0 resets it. Waits for the device; returns a SwiftNoallocStatus.
int swift_noalloc_status(int* code, int* site, int clear);

#ifdef __cplusplus
}
#endif
