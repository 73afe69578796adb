// Shared device helpers for the sm_100a kernels.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdlib>
#include <utility>

#include <c10/cuda/CUDAStream.h>
#include <torch/extension.h>

#define SWIFT_CHECK_CUDA(x)                                                              \
  do {                                                                                   \
    cudaError_t e_ = (x);                                                                \
    TORCH_CHECK(e_ == cudaSuccess, "CUDA error: ", cudaGetErrorString(e_), " at ", __FILE__, \
                ":", __LINE__);                                                          \
  } while (0)

#define SWIFT_CHECK_LAUNCH() SWIFT_CHECK_CUDA(cudaGetLastError())

#define CHECK_CUDA_TENSOR(t) TORCH_CHECK((t).is_cuda(), #t " must be a CUDA tensor")
#define CHECK_CONTIG(t) TORCH_CHECK((t).is_contiguous(), #t " must be contiguous")
#define CHECK_BF16(t) TORCH_CHECK((t).scalar_type() == at::kBFloat16, #t " must be bfloat16")

namespace swift {

// Device status word: kernels that give up a bounded wait, or whose
// always-on index guards find an out-of-range index, record a code here and
// return (or skip the access) instead of trapping. The host reads and clears
// it.
enum StatusCode : int {
  kOk = 0,
  kErrWaitTimeout = 1,
  kErrPeerTimeout = 2,
  kErrBadIndex = 3,
};

// Defined in elementwise.cu.
int* status_word_ptr();

__device__ __forceinline__ void set_status(int* st, int code, int where) {
  if (st) {
    atomicCAS(st, 0, code);
    atomicCAS(st + 1, 0, where);
  }
}

inline cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream().stream(); }

// ---- programmatic dependent launch (PDL)
// Kernels launched with launch_pdl() may start while the previous kernel on
// the stream is still finishing; they must call pdl_wait() before touching
// memory the previous kernel writes (or before any write a previous kernel
// might still read). pdl_trigger() lets the next PDL kernel start early.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// SWIFT_PDL=0 turns the overlap off (plain stream order); read once.
inline bool pdl_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("SWIFT_PDL");
    return !(v && v[0] == '0');
  }();
  return on;
}

template <typename... KArgs, typename... Args>
inline void launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                       Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  SWIFT_CHECK_CUDA(cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Block-wide sum over up to 32 warps; `buf` has >= 33 floats of shared memory.
__device__ __forceinline__ float block_sum(float v, float* buf) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) buf[wid] = v;
  __syncthreads();
  float r = lane < nw ? buf[lane] : 0.f;
  r = warp_sum(r);
  if (threadIdx.x == 0) buf[32] = r;
  __syncthreads();
  return buf[32];
}

// 8 x bf16 <-> float helpers over a 16-byte vector.
struct alignas(16) bf16x8 {
  __nv_bfloat162 v[4];
};

__device__ __forceinline__ void load8(const __nv_bfloat16* p, float f[8]) {
  bf16x8 x = *reinterpret_cast<const bf16x8*>(p);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 t = __bfloat1622float2(x.v[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}
__device__ __forceinline__ void store8(__nv_bfloat16* p, const float f[8]) {
  bf16x8 x;
#pragma unroll
  for (int i = 0; i < 4; ++i) x.v[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
  *reinterpret_cast<bf16x8*>(p) = x;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- mbarrier + bulk-copy (TMA engine) helpers, PTX ISA 8.x semantics ----
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Warp-uniform bounded wait: every lane returns the same verdict, so the
// callers' __syncwarp() / shuffles never see a split warp.
__device__ __forceinline__ bool mbar_wait_warp(uint64_t* bar, uint32_t parity, int* status,
                                               int where, uint32_t limit = (1u << 26)) {
  for (uint32_t i = 0; i < limit; ++i) {
    bool ok = mbar_try_wait(bar, parity);
    if (__all_sync(0xffffffffu, ok)) return true;
  }
  if ((threadIdx.x & 31) == 0) set_status(status, kErrWaitTimeout, where);
  return false;
}

// 1-D bulk copy global -> shared, completion counted on `bar` (bytes).
// Both addresses 16-byte aligned, size a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* smem_dst, const void* gsrc, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Philox4x32-10 (Salmon, Moraes, Dror, Shaw, SC'11): round multipliers and
// Weyl key increments from the paper. Same stream as csrc/core/sampler.cpp.
__device__ __forceinline__ void philox4x32(uint64_t key, uint32_t c0, uint32_t c1, uint32_t c2,
                                           uint32_t c3, uint32_t out[4]) {
  uint32_t k0 = static_cast<uint32_t>(key), k1 = static_cast<uint32_t>(key >> 32);
  uint32_t x0 = c0, x1 = c1, x2 = c2, x3 = c3;
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    uint32_t hi0 = __umulhi(0xD2511F53u, x0), lo0 = 0xD2511F53u * x0;
    uint32_t hi1 = __umulhi(0xCD9E8D57u, x2), lo1 = 0xCD9E8D57u * x2;
    uint32_t y0 = hi1 ^ x1 ^ k0, y1 = lo1, y2 = hi0 ^ x3 ^ k1, y3 = lo0;
    x0 = y0; x1 = y1; x2 = y2; x3 = y3;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  out[0] = x0; out[1] = x1; out[2] = x2; out[3] = x3;
}

}  // namespace swift
