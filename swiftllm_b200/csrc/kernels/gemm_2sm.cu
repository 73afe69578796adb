// Y[T, M] = X[T, K] . W[M, K]^T (+ bias) on CTA pairs: tcgen05.mma.cta_group::2.
//
// The reference has no GEMM (Linear::forward returns zeros,
// crates/swiftllm-models/src/layers/mod.rs:65-78); this kernel serves the
// dense projections (QKV, o_proj, gate_up, down, lm_head) of prefill, mixed
// and decode steps.
//
// Orientation: weights are the MMA "A" operand (output features fill the
// TMEM lanes), tokens are "B" (the MMA N dimension, any multiple of 16 up to
// 256, picked per call so the token tiles pad T the least).
//
// One cluster of two CTAs (two SMs) computes a 256-feature x BN-token tile:
// each CTA loads its own 128 weight rows and BN/2 token rows per K step with
// plain (non-multicast) TMA loads whose completion is counted on the even
// CTA's mbarrier; the even CTA's single issuing thread runs
// tcgen05.mma.cta_group::2 (M = 256), which reads the B halves of both CTAs,
// so each SM streams half the token tile of a one-SM kernel per MMA and the
// tensor pipe is not starved by shared-memory bandwidth. The accumulator of
// each CTA's 128 features lives in its own TMEM, double-buffered (2 x BN
// columns) so the epilogue of tile i overlaps the MMAs of tile i+1.
//
// Warp roles (6 warps per CTA, one CTA per SM, persistent over tiles):
//   warp 0      TMA producer (both CTAs)
//   warp 1      TMEM allocation (both CTAs); MMA issue (even CTA only)
//   warps 2-5   epilogue: tcgen05.ld 32 lanes x 32 columns, bias, bf16,
//               transposed through shared memory into 16-byte row stores
// Split-K (few tiles): fp32 partials into a workspace, summed by
// splitk2_reduce_kernel.
// Every wait is bounded: on expiry the waiter records kErrWaitTimeout, raises
// the CTA's abort flag and the roles drain; both CTAs always reach the final
// cluster barrier, then free TMEM and return.
#include <cudaTypedefs.h>

#include <algorithm>

#include "common.cuh"

namespace swift {

namespace g2 {

constexpr int kBM = 128;          // weight rows per CTA (256 per pair)
constexpr int kBK = 64;           // K elements per stage (one 128-byte swizzle row)
constexpr int kMaxBN = 256;       // tokens per pair tile
constexpr int kThreads = 192;
constexpr uint32_t kWaitLimit = 1u << 25;
constexpr int kABytes = kBM * kBK * 2;            // 16 KB
constexpr int kBBytesMax = (kMaxBN / 2) * kBK * 2;  // 16 KB
constexpr int kStageBytes = kABytes + kBBytesMax;
constexpr int kStages = 6;
constexpr int kEpiPitch = 40;  // bf16 per staged row (32 + 8 padding)
constexpr size_t kSmemBytes = 1024 + size_t(kStages) * kStageBytes + 4 * 32 * kEpiPitch * 2 + 256;

__device__ __forceinline__ uint32_t cta_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t mapa(uint32_t smem_addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr), "r"(rank));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}
// 2-D tiled TMA load into this CTA's shared memory; completion (bytes) is
// counted on the mbarrier at cluster address `mbar` (the even CTA's).
__device__ __forceinline__ void tma_load_2sm(void* smem_dst, const CUtensorMap* tm, int x, int y,
                                             uint32_t mbar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(tm)), "r"(x), "r"(y), "r"(mbar)
      : "memory");
}
__device__ __forceinline__ bool try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ void arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
               : "memory");
}
__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                              int* status, int where, bool cluster_scope = false) {
  for (uint32_t i = 0; i < kWaitLimit; ++i) {
    if (cluster_scope ? try_wait_cluster(bar, parity) : mbar_try_wait(bar, parity)) return true;
    if ((i & 255) == 255 && *abort_flag) return false;
  }
  set_status(status, kErrWaitTimeout, where);
  *abort_flag = 1;
  return false;
}
// K-major, 128-byte swizzle, 8-row atoms 1024 B apart (SBO), descriptor v1.
__device__ __forceinline__ uint64_t desc_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr & 0x3FFFF) >> 4);
  d |= static_cast<uint64_t>(1) << 16;
  d |= static_cast<uint64_t>(1024 >> 4) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}
// kind::f16: f32 accumulate, A and B bf16, both K-major, N >> 3, M >> 4 (M = 256).
__device__ __forceinline__ uint32_t idesc_bf16_m256(int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
         (static_cast<uint32_t>(256 >> 4) << 24);
}
__device__ __forceinline__ void umma2(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc));
}
// Arrive (once the MMAs issued so far complete) on the barrier at this
// shared offset in both CTAs of the pair.
__device__ __forceinline__ void commit_both(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 "
      "[%0], %1;" ::"r"(smem_u32(bar)),
      "h"(static_cast<uint16_t>(3))
      : "memory");
}
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]),
        "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]),
        "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

}  // namespace g2

// One launch: tiles are (256 features, BN tokens) x split; pair p handles
// tiles p, p + pairs, ... (feature tile outer, token tile inner, split
// outermost), so pairs running together share each weight tile through L2.
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(g2::kThreads, 1)
    gemm2_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x,
                 __nv_bfloat16* __restrict__ y, int64_t ldy, const __nv_bfloat16* __restrict__ bias,
                 float* __restrict__ ws, int M, int N, int K, int BN, int splits, int vec_out,
                 int* status) {
  using namespace g2;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* tiles =
      reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __nv_bfloat16* epi = reinterpret_cast<__nv_bfloat16*>(tiles + size_t(kStages) * kStageBytes);
  uint64_t* full = reinterpret_cast<uint64_t*>(epi + 4 * 32 * kEpiPitch);
  uint64_t* empty = full + kStages;
  uint64_t* tfull = empty + kStages;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t crank = cta_rank();
  const bool leader = crank == 0;
  const int pair = blockIdx.x >> 1, pairs = gridDim.x >> 1;
  const int m_tiles = (M + 2 * kBM - 1) / (2 * kBM);
  const int n_tiles = (N + BN - 1) / BN;
  const int k_iters = (K + kBK - 1) / kBK;
  const int k_per = (k_iters + splits - 1) / splits;
  const int total = m_tiles * n_tiles * splits;
  const int half_bn = BN / 2;
  const uint32_t b_bytes = static_cast<uint32_t>(half_bn) * kBK * 2;
  // accumulator buffers start 32-column aligned; the epilogue reads whole
  // 32-column chunks, so a partial last chunk stays inside the allocation
  const uint32_t buf_cols = static_cast<uint32_t>((BN + 31) / 32 * 32);
  const uint32_t tmem_cols = 2 * buf_cols <= 32 ? 32 : 2 * buf_cols <= 64 ? 64 : 2 * buf_cols <= 128 ? 128 : 2 * buf_cols <= 256 ? 256 : 512;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 8);  // 4 epilogue warps in each CTA of the pair
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(tmem_cols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
  }
  fence_before();
  cluster_sync();  // barriers of both CTAs initialised, TMEM allocated
  fence_after();
  const uint32_t tmem_base = *tmem_slot;

  auto decode = [&](int t, int& m0, int& x0, int& s) {
    s = t / (m_tiles * n_tiles);
    const int r = t % (m_tiles * n_tiles);
    m0 = (r / n_tiles) * 2 * kBM;
    x0 = (r % n_tiles) * BN;
  };

  if (warp == 0) {
    if (lane == 0) {
      const uint32_t full_leader = mapa(smem_u32(full), 0);
      uint32_t it = 0;
      bool ok = true;
      for (int t = pair; t < total && ok; t += pairs) {
        int m0, x0, s;
        decode(t, m0, x0, s);
        const int k0 = s * k_per, k1 = min(k_iters, k0 + k_per);
        for (int kk = k0; kk < k1; ++kk, ++it) {
          const int st = it % kStages;
          if (!wait_or_abort(&empty[st], ((it / kStages) & 1) ^ 1, abort_flag, status, 40)) {
            ok = false;
            break;
          }
          uint8_t* a = tiles + size_t(st) * kStageBytes;
          if (leader) mbar_arrive_expect_tx(&full[st], 2 * (kABytes + b_bytes));
          const uint32_t fb = full_leader + st * 8;
          tma_load_2sm(a, &tm_w, kk * kBK, m0 + int(crank) * kBM, fb);
          tma_load_2sm(a + kABytes, &tm_x, kk * kBK, x0 + int(crank) * half_bn, fb);
        }
      }
      if (!ok) {  // let the loads already issued land before the CTA leaves
        for (uint32_t p = 0; p < (1u << 22); ++p) __nanosleep(0);
      }
    }
  } else if (warp == 1) {
    if (leader && lane == 0) {
      const uint32_t idesc = idesc_bf16_m256(BN);
      uint32_t it = 0, tc = 0;
      bool ok = true;
      for (int t = pair; t < total && ok; t += pairs, ++tc) {
        int m0, x0, s;
        decode(t, m0, x0, s);
        const int k0 = s * k_per, k1 = min(k_iters, k0 + k_per);
        const uint32_t buf = tc & 1;
        if (!wait_or_abort(&tempty[buf], ((tc >> 1) & 1) ^ 1, abort_flag, status, 41, true)) {
          ok = false;
          break;
        }
        fence_after();
        const uint32_t d_tmem = tmem_base + buf * buf_cols;
        for (int kk = k0; kk < k1; ++kk, ++it) {
          const int st = it % kStages;
          if (!wait_or_abort(&full[st], (it / kStages) & 1, abort_flag, status, 42)) {
            ok = false;
            break;
          }
          fence_after();
          const uint32_t a = smem_u32(tiles + size_t(st) * kStageBytes);
          const uint64_t ad = desc_sw128(a), bd = desc_sw128(a + kABytes);
#pragma unroll
          for (int j = 0; j < kBK / 16; ++j)  // +32 B along K inside the swizzle atom
            umma2(d_tmem, ad + 2 * j, bd + 2 * j, idesc, (kk > k0 || j > 0) ? 1u : 0u);
          commit_both(&empty[st]);
        }
        if (!ok) break;
        commit_both(&tfull[buf]);
      }
      if (!ok) {
        for (uint32_t p = 0; p < (1u << 22); ++p) __nanosleep(0);
      }
    }
  } else {
    const int q = warp & 3;  // TMEM lane quarter of this warp
    const uint32_t tempty_leader = mapa(smem_u32(tempty), 0);
    __nv_bfloat16* stage = epi + q * 32 * kEpiPitch;
    uint32_t tc = 0;
    for (int t = pair; t < total; t += pairs, ++tc) {
      int m0, x0, s;
      decode(t, m0, x0, s);
      const uint32_t buf = tc & 1;
      bool ok = true;
      for (uint32_t i = 0;; ++i) {
        const bool r = mbar_try_wait(&tfull[buf], (tc >> 1) & 1);
        if (__all_sync(0xffffffffu, r)) break;
        if (i > kWaitLimit || ((i & 255) == 255 && *abort_flag)) {
          if (lane == 0 && i > kWaitLimit) {
            set_status(status, kErrWaitTimeout, 43);
            *abort_flag = 1;
          }
          ok = false;
          break;
        }
      }
      if (!ok) break;
      fence_after();
      const int fbase = m0 + int(crank) * kBM + q * 32;
      const int f = fbase + lane;
      const float b = (bias != nullptr && f < M && splits == 1) ? __bfloat162float(bias[f]) : 0.f;
      const uint32_t tq = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + buf * buf_cols;
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        float v[32];
        g2::tmem_ld32(tq + c, v);  // columns past BN are not this tile's: masked below
        const int t0 = x0 + c;
        const int nvalid = min(min(32, BN - c), N - t0);
        if (splits > 1) {
          if (f < M)
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (j < nvalid) ws[(int64_t(s) * N + t0 + j) * M + f] = v[j];
        } else if (vec_out) {
#pragma unroll
          for (int j = 0; j < 32; ++j) stage[j * kEpiPitch + lane] = __float2bfloat16(v[j] + b);
          __syncwarp();
#pragma unroll
          for (int r0 = 0; r0 < 32; r0 += 8) {
            const int row = r0 + (lane >> 2), part = lane & 3;
            const int fo = fbase + part * 8;
            if (row < nvalid && fo < M)
              *reinterpret_cast<uint4*>(y + int64_t(t0 + row) * ldy + fo) =
                  *reinterpret_cast<const uint4*>(stage + row * kEpiPitch + part * 8);
          }
          __syncwarp();
        } else if (f < M) {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (j < nvalid) y[int64_t(t0 + j) * ldy + f] = __float2bfloat16(v[j] + b);
        }
      }
      fence_before();
      __syncwarp();
      if (lane == 0) g2::arrive_remote(tempty_leader + buf * 8);
    }
  }
  fence_before();
  __syncthreads();
  cluster_sync();  // no CTA leaves while its peer may still signal it
  if (warp == 1) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                 "r"(tmem_cols));
  }
}

__global__ void splitk2_reduce_kernel(__nv_bfloat16* __restrict__ y, int64_t ldy,
                                      const float* __restrict__ ws,
                                      const __nv_bfloat16* __restrict__ bias, int M, int N,
                                      int splits) {
  const int64_t total = int64_t(M) * N;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total;
       i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t t = i / M;
    const int f = static_cast<int>(i % M);
    float acc = bias ? __bfloat162float(bias[f]) : 0.f;
    for (int s = 0; s < splits; ++s) acc += ws[int64_t(s) * total + i];
    y[t * ldy + f] = __float2bfloat16(acc);
  }
}

// ---------------------------------------------------------------- host side
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    SWIFT_CHECK_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q));
    TORCH_CHECK(q == cudaDriverEntryPointSuccess && p, "cuTensorMapEncodeTiled unavailable");
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// bf16 [rows, cols] with row stride ld elements; box 64 columns x box_rows.
static CUtensorMap tmap_bf16(const void* ptr, int64_t rows, int64_t cols, int64_t ld, int box_rows) {
  CUtensorMap tm;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * 2)};
  cuuint32_t box[2] = {64, static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn()(&tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims,
                           strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                           CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed (", static_cast<int>(r), ")");
  return tm;
}

static int sm_count() {
  static int n[64] = {0};
  int dev;
  cudaGetDevice(&dev);
  if (!n[dev]) cudaDeviceGetAttribute(&n[dev], cudaDevAttrMultiProcessorCount, dev);
  return n[dev];
}

// Token tile and split count: the fewest token tiles of width <= 256, the
// width rounded up to 16 (padding under 16 per tile); split K while the
// tiles fill under 3/4 of the SM pairs and each split keeps >= 8 K steps.
void gemm2_plan(int64_t M, int64_t N, int64_t K, int* bn, int* splits) {
  const int pairs = sm_count() / 2;
  const int64_t nt = (N + 255) / 256;
  int b = static_cast<int>(((N + nt - 1) / nt + 15) / 16 * 16);
  b = std::max(16, std::min(256, b));
  const int64_t tiles = ((M + 255) / 256) * ((N + b - 1) / b);
  const int k_iters = static_cast<int>((K + 63) / 64);
  int s = 1;
  while (tiles * s * 4 < int64_t(pairs) * 3 && k_iters / (s * 2) >= 8 && s < 8) s *= 2;
  *bn = b;
  *splits = s;
}

// y [T, M] (row stride ldy), x [T, K], w [M, K], bias [M] or null.
// Returns the number of kernels launched.
int64_t gemm2_launch(__nv_bfloat16* y, int64_t ldy, const torch::Tensor& x, const torch::Tensor& w,
                     const __nv_bfloat16* bias) {
  const int64_t K = x.size(-1), T = x.numel() / K, M = w.size(0);
  if (T == 0) return 0;
  const int64_t ldx = x.dim() >= 2 ? x.stride(-2) : K;
  int bn, splits;
  gemm2_plan(M, T, K, &bn, &splits);
  static bool attr[64] = {false};
  int dev;
  cudaGetDevice(&dev);
  if (!attr[dev]) {
    SWIFT_CHECK_CUDA(cudaFuncSetAttribute(gemm2_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          static_cast<int>(g2::kSmemBytes)));
    attr[dev] = true;
  }
  CUtensorMap tw = tmap_bf16(w.data_ptr(), M, K, w.stride(0), g2::kBM);
  CUtensorMap tx = tmap_bf16(x.data_ptr(), T, K, ldx, bn / 2);
  const int64_t tiles = ((M + 255) / 256) * ((T + bn - 1) / bn) * splits;
  const int pairs = static_cast<int>(std::min<int64_t>(tiles, sm_count() / 2));
  torch::Tensor ws;
  float* wsp = nullptr;
  if (splits > 1) {
    ws = torch::empty({splits, T, M}, x.options().dtype(torch::kFloat));
    wsp = ws.data_ptr<float>();
  }
  const int vec_out = (M % 8 == 0 && ldy % 8 == 0 && reinterpret_cast<uintptr_t>(y) % 16 == 0) ? 1 : 0;
  gemm2_kernel<<<2 * pairs, g2::kThreads, g2::kSmemBytes, cur_stream()>>>(
      tw, tx, y, ldy, bias, wsp, static_cast<int>(M), static_cast<int>(T), static_cast<int>(K), bn,
      splits, vec_out, status_word_ptr());
  SWIFT_CHECK_LAUNCH();
  if (splits > 1) {
    const int64_t n = M * T;
    const int blocks = static_cast<int>(std::min<int64_t>((n + 255) / 256, 148 * 8));
    splitk2_reduce_kernel<<<blocks, 256, 0, cur_stream()>>>(y, ldy, wsp, bias, static_cast<int>(M),
                                                           static_cast<int>(T), splits);
    SWIFT_CHECK_LAUNCH();
    return 2;
  }
  return 1;
}

// Python binding: out [T, M] (row stride may exceed M), x [T, K], w [M, K].
int64_t gemm2(torch::Tensor out, torch::Tensor x, torch::Tensor w, c10::optional<torch::Tensor> bias) {
  CHECK_BF16(out);
  CHECK_BF16(x);
  CHECK_BF16(w);
  const int64_t K = x.size(-1);
  TORCH_CHECK(w.size(1) == K && K % 8 == 0, "gemm2: K must match and be a multiple of 8");
  TORCH_CHECK(x.stride(-1) == 1 && w.stride(1) == 1 && out.stride(-1) == 1);
  const int64_t ldx = x.dim() >= 2 ? x.stride(-2) : K;
  TORCH_CHECK(ldx % 8 == 0 && w.stride(0) % 8 == 0, "gemm2: row strides must be 16-byte multiples");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0 &&
                  reinterpret_cast<uintptr_t>(w.data_ptr()) % 16 == 0,
              "gemm2: operands must be 16-byte aligned");
  const int64_t ldy = out.dim() >= 2 ? out.stride(-2) : w.size(0);
  const __nv_bfloat16* bp =
      bias.has_value() ? reinterpret_cast<const __nv_bfloat16*>(bias.value().data_ptr<at::BFloat16>())
                       : nullptr;
  return gemm2_launch(reinterpret_cast<__nv_bfloat16*>(out.data_ptr<at::BFloat16>()), ldy, x, w, bp);
}

std::vector<int64_t> gemm2_plan_py(int64_t M, int64_t N, int64_t K) {
  int bn, s;
  gemm2_plan(M, N, K, &bn, &s);
  return {bn, s};
}

}  // namespace swift
