// Tensor-parallel sum of the row-parallel GEMM outputs over NVLink peer memory.
//
// The reference declares TP all-reduce and returns NotImplemented
// (crates/swiftllm-core/src/execution/tensor_parallel.rs:115-141).
//
// Memory: one symmetric allocation per rank (same layout on every GPU, every
// rank holds the device addresses of all peers' copies, rendezvoused through
// torch.distributed._symmetric_memory):
//   [flags | in A | in B | red A | red B]
// The o_proj / down_proj GEMM epilogue stores its partial output directly in
// this rank's `in` buffer (A/B alternate by call so consecutive calls need no
// exit barrier), then this kernel runs a two-shot reduction:
//   phase 1  (reduce-scatter) block b sums, in fixed rank order and fp32, the
//            elements of this rank's 1/k slice that block b owns, loading
//            every peer's `in` over NVLink, and stores bf16 to its `red`;
//   phase 2  (all-gather) block b reads the elements that block b of each
//            peer produced in phase 1 from that peer's `red` into `out`.
// Each phase starts with a per-block barrier: block b stores the call epoch
// into every peer's flag slot for (phase, b, this rank) with st.release.sys
// and polls its own slots with ld.acquire.sys. Because every rank uses the
// same grid and the same element-to-block mapping, block b only ever waits
// for block b of its peers. Epochs live in device memory and advance inside
// the kernel, so CUDA-graph replays keep counting. Every poll is bounded by
// a %globaltimer deadline; on expiry the block records kErrPeerTimeout in the
// status word and returns (the host raises CommTimeoutError).
#include <algorithm>
#include <cstdlib>

#include "common.cuh"

namespace swift {

constexpr int kArMaxRanks = 8;
constexpr int kArBlocks = 64;
constexpr int kArThreads = 512;

struct ArPeers {
  uint64_t base[kArMaxRanks];  // byte address of each rank's symmetric allocation
};

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// flags: [2 phases][kArBlocks][kArMaxRanks] uint32 at offset 0 of each allocation.
__device__ __forceinline__ bool block_barrier(const ArPeers& P, int rank, int k, int phase,
                                              uint32_t epoch, int64_t timeout_ns, int* status) {
  __syncthreads();
  __shared__ int ok;
  if (threadIdx.x == 0) ok = 1;
  __syncthreads();
  const int t = threadIdx.x;
  if (t < k) {
    const int slot = (phase * kArBlocks + blockIdx.x) * kArMaxRanks;
    // announce: my arrival in peer t's slot [.., rank]
    uint32_t* remote = reinterpret_cast<uint32_t*>(P.base[t]) + slot + rank;
    __threadfence_system();
    st_release_sys(remote, epoch);
    // wait: peer t's arrival in my slot [.., t]
    const uint32_t* mine = reinterpret_cast<const uint32_t*>(P.base[rank]) + slot + t;
    const uint64_t deadline = globaltimer_ns() + static_cast<uint64_t>(timeout_ns);
    while (static_cast<int32_t>(ld_acquire_sys(mine) - epoch) < 0) {
      if (globaltimer_ns() > deadline) {
        set_status(status, kErrPeerTimeout, 200 + phase);
        atomicExch(&ok, 0);
        break;
      }
    }
  }
  __syncthreads();
  return ok != 0;
}

__global__ void __launch_bounds__(kArThreads)
    tp_allreduce_kernel(ArPeers P, int rank, int k, int64_t in_off, int64_t red_off,
                        __nv_bfloat16* __restrict__ out, int64_t n, uint32_t* __restrict__ epochs,
                        int64_t timeout_ns, int* status) {
  const uint32_t epoch = epochs[blockIdx.x] + 1;
  // slice boundaries in units of 8 elements (16-byte vectors)
  const int64_t nv = n / 8;
  auto slice_lo = [&](int r) { return nv * r / k; };
  if (!block_barrier(P, rank, k, 0, epoch, timeout_ns, status)) return;
  {
    const int64_t lo = slice_lo(rank), hi = slice_lo(rank + 1);
    uint4* red = reinterpret_cast<uint4*>(P.base[rank] + red_off);
    for (int64_t v = lo + blockIdx.x * int64_t(blockDim.x) + threadIdx.x; v < hi;
         v += int64_t(gridDim.x) * blockDim.x) {
      float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      for (int r = 0; r < k; ++r) {
        const uint4* src = reinterpret_cast<const uint4*>(P.base[r] + in_off) + v;
        uint4 x = __ldcg(src);
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&x);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float2 f = __bfloat1622float2(h[j]);
          acc[2 * j] += f.x;
          acc[2 * j + 1] += f.y;
        }
      }
      uint4 o;
      __nv_bfloat162* oh = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
      for (int j = 0; j < 4; ++j) oh[j] = __floats2bfloat162_rn(acc[2 * j], acc[2 * j + 1]);
      red[v] = o;
    }
  }
  if (!block_barrier(P, rank, k, 1, epoch, timeout_ns, status)) return;
  for (int r = 0; r < k; ++r) {
    const int64_t lo = slice_lo(r), hi = slice_lo(r + 1);
    const uint4* src = reinterpret_cast<const uint4*>(P.base[r] + red_off);
    uint4* dst = reinterpret_cast<uint4*>(out);
    for (int64_t v = lo + blockIdx.x * int64_t(blockDim.x) + threadIdx.x; v < hi;
         v += int64_t(gridDim.x) * blockDim.x)
      dst[v] = __ldcg(src + v);
  }
  __syncthreads();
  if (threadIdx.x == 0) epochs[blockIdx.x] = epoch;
}

// out [n] bf16 (local); bases: int64 [k] byte addresses of the symmetric
// allocations; in_off / red_off: byte offsets of this call's buffers.
void tp_allreduce(torch::Tensor out, std::vector<int64_t> bases, int64_t rank, int64_t in_off,
                  int64_t red_off, torch::Tensor epochs, double timeout_s) {
  CHECK_BF16(out);
  CHECK_CONTIG(out);
  const int k = static_cast<int>(bases.size());
  TORCH_CHECK(k >= 1 && k <= kArMaxRanks);
  TORCH_CHECK(epochs.scalar_type() == at::kInt && epochs.numel() >= kArBlocks);
  const int64_t n = out.numel();
  TORCH_CHECK(n % 8 == 0, "all-reduce size must be a multiple of 8 elements");
  TORCH_CHECK(in_off % 16 == 0 && red_off % 16 == 0);
  ArPeers P;
  for (int r = 0; r < kArMaxRanks; ++r) P.base[r] = r < k ? static_cast<uint64_t>(bases[r]) : 0;
  tp_allreduce_kernel<<<kArBlocks, kArThreads, 0, cur_stream()>>>(
      P, static_cast<int>(rank), k, in_off, red_off,
      reinterpret_cast<__nv_bfloat16*>(out.data_ptr<at::BFloat16>()), n,
      reinterpret_cast<uint32_t*>(epochs.data_ptr<int32_t>()),
      static_cast<int64_t>(timeout_s * 1e9), status_word_ptr());
  SWIFT_CHECK_LAUNCH();
}

// Second half of the fused GEMM -> all-reduce. gemm_rs has stored every
// rank's partial rows of this rank's tokens [lo, hi) into this rank's
// receive buffer ([src][row - lo][H], local memory) and published its
// completion epoch to flag[src]. Block b:
//   1. waits until every rank's flag reached this call's epoch (bounded);
//   2. sums the k partials of its share of [lo, hi) x H in fixed rank order
//      (fp32) and stores the bf16 result into EVERY rank's output buffer
//      (all-gather by push over NVLink);
//   3. per-block barrier with its peers (phase 1 slots): after it, block b
//      of every rank has pushed its share, so when the kernel has finished
//      on this rank, the whole [T, H] output is present locally.
__global__ void __launch_bounds__(kArThreads)
    tp_rs_finish_kernel(ArPeers P, int rank, int k, int64_t in_off, int64_t out_off, int s_max,
                        int T, int H, int64_t flag_off, uint32_t* __restrict__ gemm_epochs,
                        uint32_t* __restrict__ epochs, int64_t timeout_ns, int* status) {
  const uint32_t want = gemm_epochs[blockIdx.x] + 1;
  __shared__ int ok;
  if (threadIdx.x == 0) ok = 1;
  __syncthreads();
  if (threadIdx.x < k) {
    const uint32_t* f = reinterpret_cast<const uint32_t*>(P.base[rank] + flag_off) + threadIdx.x;
    const uint64_t deadline = globaltimer_ns() + static_cast<uint64_t>(timeout_ns);
    while (static_cast<int32_t>(ld_acquire_sys(f) - want) < 0) {
      if (globaltimer_ns() > deadline) {
        set_status(status, kErrPeerTimeout, 210);
        atomicExch(&ok, 0);
        break;
      }
    }
  }
  __syncthreads();
  if (!ok) return;
  const int lo = static_cast<int>(int64_t(T) * rank / k), hi = static_cast<int>(int64_t(T) * (rank + 1) / k);
  const int hv = H / 8;  // 16-byte vectors per row
  const int64_t nv = int64_t(hi - lo) * hv;
  for (int64_t v = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; v < nv;
       v += int64_t(gridDim.x) * blockDim.x) {
    const int row = static_cast<int>(v / hv), col = static_cast<int>(v % hv);
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int r = 0; r < k; ++r) {
      const uint4* src = reinterpret_cast<const uint4*>(P.base[rank] + in_off) +
                         (int64_t(r) * s_max + row) * hv + col;
      uint4 x = __ldcg(src);
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&x);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float2 f = __bfloat1622float2(h[j]);
        acc[2 * j] += f.x;
        acc[2 * j + 1] += f.y;
      }
    }
    uint4 o;
    __nv_bfloat162* oh = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
    for (int j = 0; j < 4; ++j) oh[j] = __floats2bfloat162_rn(acc[2 * j], acc[2 * j + 1]);
    for (int p = 0; p < k; ++p) {
      const int q = (rank + p) % k;  // stagger destinations across ranks
      uint4* dst = reinterpret_cast<uint4*>(P.base[q] + out_off) + (int64_t(lo) + row) * hv + col;
      *dst = o;
    }
  }
  const uint32_t epoch = epochs[blockIdx.x] + 1;
  if (!block_barrier(P, rank, k, 1, epoch, timeout_ns, status)) return;
  __syncthreads();
  if (threadIdx.x == 0) {
    epochs[blockIdx.x] = epoch;
    gemm_epochs[blockIdx.x] = want;
  }
}

void tp_rs_finish(std::vector<int64_t> bases, int64_t rank, int64_t in_off, int64_t out_off,
                  int64_t s_max, int64_t T, int64_t H, int64_t flag_off, torch::Tensor gemm_epochs,
                  torch::Tensor epochs, double timeout_s) {
  const int k = static_cast<int>(bases.size());
  TORCH_CHECK(k >= 2 && k <= kArMaxRanks);
  TORCH_CHECK(H % 8 == 0 && in_off % 16 == 0 && out_off % 16 == 0 && flag_off % 4 == 0);
  TORCH_CHECK(epochs.scalar_type() == at::kInt && epochs.numel() >= kArBlocks);
  TORCH_CHECK(gemm_epochs.scalar_type() == at::kInt && gemm_epochs.numel() >= kArBlocks);
  ArPeers P;
  for (int r = 0; r < kArMaxRanks; ++r) P.base[r] = r < k ? static_cast<uint64_t>(bases[r]) : 0;
  // every finish kernel runs kArBlocks blocks: block b owns the per-block
  // epoch counters b of gemm_epochs / epochs, shared by all of them
  tp_rs_finish_kernel<<<kArBlocks, kArThreads, 0, cur_stream()>>>(
      P, static_cast<int>(rank), k, in_off, out_off, static_cast<int>(s_max), static_cast<int>(T),
      static_cast<int>(H), flag_off, reinterpret_cast<uint32_t*>(gemm_epochs.data_ptr<int32_t>()),
      reinterpret_cast<uint32_t*>(epochs.data_ptr<int32_t>()),
      static_cast<int64_t>(timeout_s * 1e9), status_word_ptr());
  SWIFT_CHECK_LAUNCH();
}

// tp_rs_finish with the following fused add + RMSNorm (the norm that opens
// the next sub-block). Block b owns whole token rows of this rank's shard
// (row lo + b, lo + b + gridDim, ...): it sums the k partials in rank order
// (fp32, rounded to bf16 like the unfused reduce), adds the residual row
// (rounded to bf16, the new residual), computes the RMS scale over the row,
// and pushes both the new residual row and the normalised row to every
// rank's `res_off` / `out_off` buffers. Same flags and barrier as
// tp_rs_finish. H <= 4 * 8 * blockDim.x.
__global__ void __launch_bounds__(kArThreads)
    tp_rs_finish_norm_kernel(ArPeers P, int rank, int k, int64_t in_off, int64_t out_off,
                             int64_t res_off, const __nv_bfloat16* __restrict__ residual,
                             const __nv_bfloat16* __restrict__ w, float eps, int s_max, int T,
                             int H, int64_t flag_off, uint32_t* __restrict__ gemm_epochs,
                             uint32_t* __restrict__ epochs, int64_t timeout_ns, int* status) {
  const uint32_t want = gemm_epochs[blockIdx.x] + 1;
  __shared__ int ok;
  __shared__ float red[33];
  if (threadIdx.x == 0) ok = 1;
  __syncthreads();
  if (threadIdx.x < k) {
    const uint32_t* f = reinterpret_cast<const uint32_t*>(P.base[rank] + flag_off) + threadIdx.x;
    const uint64_t deadline = globaltimer_ns() + static_cast<uint64_t>(timeout_ns);
    while (static_cast<int32_t>(ld_acquire_sys(f) - want) < 0) {
      if (globaltimer_ns() > deadline) {
        set_status(status, kErrPeerTimeout, 220);
        atomicExch(&ok, 0);
        break;
      }
    }
  }
  __syncthreads();
  if (!ok) return;
  const int lo = static_cast<int>(int64_t(T) * rank / k), hi = static_cast<int>(int64_t(T) * (rank + 1) / k);
  const int hv = H / 8;
  for (int row = blockIdx.x; row < hi - lo; row += gridDim.x) {
    float v[4][8];
    float s2 = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int col = threadIdx.x + j * blockDim.x;
      if (col >= hv) continue;
      float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      for (int r = 0; r < k; ++r) {
        uint4 x = __ldcg(reinterpret_cast<const uint4*>(P.base[rank] + in_off) +
                         (int64_t(r) * s_max + row) * hv + col);
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&x);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float2 f = __bfloat1622float2(h[e]);
          acc[2 * e] += f.x;
          acc[2 * e + 1] += f.y;
        }
      }
      float rr[8];
      load8(residual + (int64_t(lo) + row) * H + col * 8, rr);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float sum = __bfloat162float(__float2bfloat16(acc[e]));  // the reduced output, bf16
        v[j][e] = __bfloat162float(__float2bfloat16(sum + rr[e]));  // new residual, bf16
        s2 += v[j][e] * v[j][e];
      }
    }
    const float scale = rsqrtf(block_sum(s2, red) / H + eps);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int col = threadIdx.x + j * blockDim.x;
      if (col >= hv) continue;
      float wf[8], o[8];
      load8(w + col * 8, wf);
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = v[j][e] * scale * wf[e];
      uint4 ov, rv;
      __nv_bfloat162* oh = reinterpret_cast<__nv_bfloat162*>(&ov);
      __nv_bfloat162* rh = reinterpret_cast<__nv_bfloat162*>(&rv);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        oh[e] = __floats2bfloat162_rn(o[2 * e], o[2 * e + 1]);
        rh[e] = __floats2bfloat162_rn(v[j][2 * e], v[j][2 * e + 1]);
      }
      const int64_t idx = (int64_t(lo) + row) * hv + col;
      for (int p = 0; p < k; ++p) {
        const int q = (rank + p) % k;
        reinterpret_cast<uint4*>(P.base[q] + out_off)[idx] = ov;
        reinterpret_cast<uint4*>(P.base[q] + res_off)[idx] = rv;
      }
    }
  }
  const uint32_t epoch = epochs[blockIdx.x] + 1;
  if (!block_barrier(P, rank, k, 1, epoch, timeout_ns, status)) return;
  __syncthreads();
  if (threadIdx.x == 0) {
    epochs[blockIdx.x] = epoch;
    gemm_epochs[blockIdx.x] = want;
  }
}

void tp_rs_finish_norm(std::vector<int64_t> bases, int64_t rank, int64_t in_off, int64_t out_off,
                       int64_t res_off, torch::Tensor residual, torch::Tensor w, double eps,
                       int64_t s_max, int64_t T, int64_t H, int64_t flag_off,
                       torch::Tensor gemm_epochs, torch::Tensor epochs, double timeout_s) {
  const int k = static_cast<int>(bases.size());
  TORCH_CHECK(k >= 2 && k <= kArMaxRanks);
  CHECK_BF16(residual);
  CHECK_BF16(w);
  TORCH_CHECK(residual.is_contiguous() && residual.numel() >= T * H && w.numel() == H);
  TORCH_CHECK(H % 8 == 0 && H <= 4 * 8 * kArThreads, "tp_rs_finish_norm: H too large");
  TORCH_CHECK(in_off % 16 == 0 && out_off % 16 == 0 && res_off % 16 == 0 && flag_off % 4 == 0);
  TORCH_CHECK(epochs.numel() >= kArBlocks && gemm_epochs.numel() >= kArBlocks);
  ArPeers P;
  for (int r = 0; r < kArMaxRanks; ++r) P.base[r] = r < k ? static_cast<uint64_t>(bases[r]) : 0;
  tp_rs_finish_norm_kernel<<<kArBlocks, kArThreads, 0, cur_stream()>>>(
      P, static_cast<int>(rank), k, in_off, out_off, res_off,
      reinterpret_cast<const __nv_bfloat16*>(residual.data_ptr<at::BFloat16>()),
      reinterpret_cast<const __nv_bfloat16*>(w.data_ptr<at::BFloat16>()), static_cast<float>(eps),
      static_cast<int>(s_max), static_cast<int>(T), static_cast<int>(H), flag_off,
      reinterpret_cast<uint32_t*>(gemm_epochs.data_ptr<int32_t>()),
      reinterpret_cast<uint32_t*>(epochs.data_ptr<int32_t>()),
      static_cast<int64_t>(timeout_s * 1e9), status_word_ptr());
  SWIFT_CHECK_LAUNCH();
}

// Test hook: one bounded wait on a flag nobody sets (single GPU, no peer):
// must return with kErrPeerTimeout recorded, the context still usable.
__global__ void flag_wait_probe_kernel(const uint32_t* flag, uint32_t want, int64_t timeout_ns,
                                       int* status) {
  const uint64_t deadline = globaltimer_ns() + static_cast<uint64_t>(timeout_ns);
  while (static_cast<int32_t>(ld_acquire_sys(flag) - want) < 0) {
    if (globaltimer_ns() > deadline) {
      set_status(status, kErrPeerTimeout, 299);
      return;
    }
  }
}

void flag_wait_probe(torch::Tensor flag, int64_t want, double timeout_s) {
  TORCH_CHECK(flag.scalar_type() == at::kInt && flag.is_cuda());
  flag_wait_probe_kernel<<<1, 1, 0, cur_stream()>>>(
      reinterpret_cast<const uint32_t*>(flag.data_ptr<int32_t>()), static_cast<uint32_t>(want),
      static_cast<int64_t>(timeout_s * 1e9), status_word_ptr());
  SWIFT_CHECK_LAUNCH();
}

}  // namespace swift
