// Checkpoint parsers: safetensors and GGUF, memory-mapped.
//
// Parity:
//   crates/swiftllm-models/src/loaders/safetensors.rs (mmap, 8-byte header
//     length + JSON header, dtype table :44-138, :209-220)
//   crates/swiftllm-models/src/loaders/gguf.rs (GGUF v1-v3 header, typed
//     metadata, tensor infos, aligned data offset :181-258; type table :22-107)
// Fixes over the reference: GGUF arrays are read with their element type
// (the reference reads every array as u32, gguf.rs:449-458), the data offset
// honours `general.alignment`, and block-quantised tensors get their real
// byte size and a dequantiser (Q4_0, Q4_1, Q8_0, Q4_K, Q6_K, F16, BF16, F32).
// Tensors are returned as zero-copy views into the mapping; per-rank shard
// slicing happens on those views, so no full host copy is made.
#pragma once
#include <pybind11/pybind11.h>

void bind_loaders(pybind11::module_& m);
