// Shared-memory broadcast channel: the tensor-parallel control plane.
//
// Rank 0 (the engine) publishes one message per step (the packed batch
// metadata) and every worker rank reads it. One writer, up to 64 readers, a
// ring of fixed-size slots in a POSIX shared-memory segment; sequence numbers
// are std::atomic<uint64_t> (lock-free and address-free, so valid across
// processes). Every wait is bounded: a reader that sees no message before its
// deadline, or a writer whose slowest reader stopped acknowledging, raises a
// timeout error instead of hanging. Each side also stamps a heartbeat, and a
// stale peer heartbeat is reported as a dead peer.
//
// The reference declares broadcast / barrier collectives but implements none
// (crates/swiftllm-core/src/execution/tensor_parallel.rs:144-159).
#pragma once
#include <pybind11/pybind11.h>

void bind_shm_channel(pybind11::module_& m);
