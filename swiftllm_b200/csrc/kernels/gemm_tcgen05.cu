// Y[T, N] = X[T, K] . W[N, K]^T (+ bias) on the 5th-generation tensor cores.
//
// The reference has no GEMM (Linear::forward returns zeros,
// crates/swiftllm-models/src/layers/mod.rs:65-78). This kernel serves every
// projection: QKV, o_proj, gate_up, down, lm_head and the MoE experts.
//
// Orientation: the weight is the MMA "A" operand (its rows, the output
// features, fill the 128 TMEM lanes) and the activations are "B" (tokens
// are the MMA N dimension, 16..256). Decode steps with few tokens therefore
// still issue full 128-row MMAs, and the weight - the bytes that matter in
// decode - is streamed once per token tile.
//
// Structure (one CTA of 6 warps per SM, persistent over output tiles):
//   warp 0      TMA producer: cp.async.bulk.tensor 2-D loads (128B swizzle,
//               plain per-CTA loads) of a 128x64 weight tile and a BNx64 token tile
//               per stage into an STAGES-deep shared-memory ring;
//   warp 1      allocates TMEM; one thread issues
//               tcgen05.mma.cta_group::1.kind::f16 (bf16 in, fp32 in TMEM);
//               tcgen05.commit frees ring stages and signals finished tiles;
//   warps 2-5   epilogue: tcgen05.ld 32 lanes x 32 columns per warp, bias
//               add, bf16 store (or fp32 split-K partials); two TMEM
//               accumulators let the epilogue of tile i overlap the MMAs of
//               tile i+1.
// Split-K (shapes with too few tiles to fill the SMs) writes fp32 partials
// into a caller workspace that splitk_reduce_kernel sums.
// All mbarrier waits are bounded: on expiry the waiting role records
// kErrWaitTimeout in the status word and raises a CTA-wide abort flag the
// other roles poll; in-flight copies / MMAs are drained (bounded), TMEM is
// freed and the CTA returns.
#include <cudaTypedefs.h>

#include "common.cuh"

namespace swift {

constexpr int kGemmBM = 128, kGemmBK = 64;
constexpr int kGemmThreads = 192;
constexpr uint32_t kWaitLimit = 1u << 25;

__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* tm, int x, int y,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, "
      "%3}], [%4];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(tm)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity,
                                              volatile int* abort_flag, int* status, int where) {
  for (uint32_t i = 0; i < kWaitLimit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255) == 255 && *abort_flag) return false;
  }
  set_status(status, kErrWaitTimeout, where);
  *abort_flag = 1;
  return false;
}

// K-major, 128-byte swizzle: rows of 128 B, 8-row atoms 1024 B apart
// (SBO = 1024 B), LBO unused (1), descriptor version 1, layout type 2.
__device__ __forceinline__ uint64_t smem_desc_sw128(const void* p) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_u32(p) & 0x3FFFF) >> 4);
  d |= static_cast<uint64_t>(1) << 16;
  d |= static_cast<uint64_t>(1024 >> 4) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}

// c_format f32 (bits 4-5 = 1), a/b format bf16 (bits 7-9, 10-12 = 1), both
// K-major, N >> 3 at bits 17-22, M >> 4 at bits 24-28.
template <int BN>
__host__ __device__ constexpr uint32_t instr_desc_bf16() {
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(BN >> 3) << 17) |
         (static_cast<uint32_t>(kGemmBM >> 4) << 24);
}

__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

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
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

template <int BN, int STAGES>
struct GemmSmem {
  static constexpr int A_BYTES = kGemmBM * kGemmBK * 2;
  static constexpr int B_BYTES = BN * kGemmBK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int TMEM_COLS = (2 * BN) <= 32    ? 32
                                   : (2 * BN) <= 64  ? 64
                                   : (2 * BN) <= 128 ? 128
                                   : (2 * BN) <= 256 ? 256
                                                     : 512;
  static constexpr size_t BYTES = 1024 + size_t(STAGES) * STAGE_BYTES + 256;
};

template <int BN, int STAGES>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_tcgen05_kernel(const __grid_constant__ CUtensorMap tm_w,
                        const __grid_constant__ CUtensorMap tm_x, __nv_bfloat16* __restrict__ y,
                        int64_t ldy, const __nv_bfloat16* __restrict__ bias,
                        float* __restrict__ ws, int M, int N, int K, int splits, int* status,
                        const int32_t* __restrict__ goff, int groups) {
  using S = GemmSmem<BN, STAGES>;
  // Grouped mode (goff != nullptr, MoE experts): group g multiplies the token
  // rows [goff[g], goff[g+1]) by weight rows [g*M, (g+1)*M); tiles never
  // straddle groups, rows past a group's end are loaded but not stored.
  __shared__ int g_off[65];
  __shared__ int g_tiles[65];
  extern __shared__ uint8_t smem_raw[];
  uint8_t* tiles =
      reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(tiles + size_t(STAGES) * S::STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m_tiles = (M + kGemmBM - 1) / kGemmBM;
  const int n_tiles = (N + BN - 1) / BN;
  const int k_iters = (K + kGemmBK - 1) / kGemmBK;
  const int k_per = (k_iters + splits - 1) / splits;
  int total = m_tiles * n_tiles * splits;
  if (goff) {
    if (threadIdx.x == 0) {
      int acc = 0;
      for (int g = 0; g < groups; ++g) {
        g_off[g] = goff[g];
        g_tiles[g] = acc;
        acc += m_tiles * ((goff[g + 1] - goff[g] + BN - 1) / BN);
      }
      g_off[groups] = goff[groups];
      g_tiles[groups] = acc;
    }
    __syncthreads();
    total = g_tiles[groups];
  }

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 4);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(S::TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  // tile -> (split outermost, then m, n fastest: CTAs running at the same
  // time share the weight tile through L2)
  // -> split s, feature tile m, first token row x0, token row limit xend,
  // first weight row w0
  auto decode_tile = [&](int t, int& m, int& x0, int& xend, int& w0, int& s) {
    if (goff) {
      int g = 0;
      while (g + 1 < groups && g_tiles[g + 1] <= t) ++g;
      const int r = t - g_tiles[g];
      const int nt = (g_off[g + 1] - g_off[g] + BN - 1) / BN;
      m = r / nt;
      x0 = g_off[g] + (r % nt) * BN;
      xend = g_off[g + 1];
      w0 = g * M + m * kGemmBM;
      s = 0;
      return;
    }
    s = t / (m_tiles * n_tiles);
    int r = t % (m_tiles * n_tiles);
    m = r / n_tiles;
    x0 = (r % n_tiles) * BN;
    xend = N;
    w0 = m * kGemmBM;
  };

  if (warp == 0) {
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
        int m, x0, xend, w0, s;
        decode_tile(t, m, x0, xend, w0, s);
        const int k0 = s * k_per, k1 = min(k_iters, k0 + k_per);
        for (int kk = k0; kk < k1; ++kk, ++it) {
          const int st = it % STAGES;
          if (!wait_or_abort(&empty[st], ((it / STAGES) & 1) ^ 1, abort_flag, status, 10)) {
            ok = false;
            break;
          }
          uint8_t* a = tiles + size_t(st) * S::STAGE_BYTES;
          mbar_arrive_expect_tx(&full[st], S::STAGE_BYTES);
          tma_load_2d(a, &tm_w, kk * kGemmBK, w0, &full[st]);
          tma_load_2d(a + S::A_BYTES, &tm_x, kk * kGemmBK, x0, &full[st]);
        }
      }
      if (!ok) {  // let the loads already issued land before the CTA exits
        for (uint32_t j = it > STAGES ? it - STAGES : 0; j < it; ++j)
          for (uint32_t p = 0; p < (1u << 20); ++p)
            if (mbar_try_wait(&full[j % STAGES], (j / STAGES) & 1)) break;
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = instr_desc_bf16<BN>();
      uint32_t it = 0, tc = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x, ++tc) {
        int m, x0, xend, w0, s;
        decode_tile(t, m, x0, xend, w0, s);
        const int k0 = s * k_per, k1 = min(k_iters, k0 + k_per);
        const uint32_t buf = tc & 1;
        if (!wait_or_abort(&tempty[buf], ((tc >> 1) & 1) ^ 1, abort_flag, status, 11)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * BN;
        for (int kk = k0; kk < k1; ++kk, ++it) {
          const int st = it % STAGES;
          if (!wait_or_abort(&full[st], (it / STAGES) & 1, abort_flag, status, 12)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint8_t* a = tiles + size_t(st) * S::STAGE_BYTES;
          const uint64_t ad = smem_desc_sw128(a);
          const uint64_t bd = smem_desc_sw128(a + S::A_BYTES);
#pragma unroll
          for (int j = 0; j < kGemmBK / 16; ++j)  // +32 B along K inside the swizzle atom
            umma_bf16(d_tmem, ad + 2 * j, bd + 2 * j, idesc, (kk > k0 || j > 0) ? 1u : 0u);
          umma_commit(&empty[st]);
        }
        if (!ok) break;
        umma_commit(&tfull[buf]);
      }
      if (!ok) {  // MMAs already issued finish (their commits arrive on empty[])
        for (uint32_t j = it > STAGES ? it - STAGES : 0; j < it; ++j)
          for (uint32_t p = 0; p < (1u << 20); ++p)
            if (mbar_try_wait(&empty[j % STAGES], (j / STAGES) & 1)) break;
      }
    }
  } else {
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    uint32_t tc = 0;
    for (int t = blockIdx.x; t < total; t += gridDim.x, ++tc) {
      int m, x0, xend, w0, s;
      decode_tile(t, m, x0, xend, w0, s);
      const uint32_t buf = tc & 1;
      bool ok = true;
      for (uint32_t i = 0;; ++i) {
        bool r = mbar_try_wait(&tfull[buf], (tc >> 1) & 1);
        if (__all_sync(0xffffffffu, r)) break;
        if (i > kWaitLimit || ((i & 255) == 255 && *abort_flag)) {
          if (lane == 0 && i > kWaitLimit) {
            set_status(status, kErrWaitTimeout, 13);
            *abort_flag = 1;
          }
          ok = false;
          break;
        }
      }
      if (!ok) break;
      tc_fence_after();
      const int f = m * kGemmBM + q * 32 + lane;
      const float b = (bias != nullptr && f < M && splits == 1) ? __bfloat162float(bias[f]) : 0.f;
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + buf * BN;
      if constexpr (BN >= 32) {
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          float v[32];
          tmem_ld32(tbase + c * 32, v);
          const int t0 = x0 + c * 32;
          if (f < M) {
            if (splits == 1) {
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (t0 + j < xend) y[int64_t(t0 + j) * ldy + f] = __float2bfloat16(v[j] + b);
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (t0 + j < N) ws[(int64_t(s) * N + t0 + j) * M + f] = v[j];
            }
          }
        }
      } else {
        float v[16];
        tmem_ld16(tbase, v);
        const int t0 = x0;
        if (f < M) {
          if (splits == 1) {
#pragma unroll
            for (int j = 0; j < 16; ++j)
              if (t0 + j < xend) y[int64_t(t0 + j) * ldy + f] = __float2bfloat16(v[j] + b);
          } else {
#pragma unroll
            for (int j = 0; j < 16; ++j)
              if (t0 + j < N) ws[(int64_t(s) * N + t0 + j) * M + f] = v[j];
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[buf]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                 "r"(S::TMEM_COLS));
  }
}

__global__ void splitk_reduce_kernel(__nv_bfloat16* __restrict__ y, int64_t ldy,
                                     const float* __restrict__ ws,
                                     const __nv_bfloat16* __restrict__ bias, int M, int N,
                                     int splits) {
  const int64_t total = int64_t(M) * N;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total;
       i += int64_t(gridDim.x) * blockDim.x) {
    int64_t t = i / M;
    int f = static_cast<int>(i % M);
    float acc = bias ? __bfloat162float(bias[f]) : 0.f;
    for (int s = 0; s < splits; ++s) acc += ws[int64_t(s) * total + i];
    y[t * ldy + f] = __float2bfloat16(acc);
  }
}

// ---------------------------------------------------------------- host side
static PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
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

// 2-D bf16 tensor [rows, cols] with row stride `ld` elements; box 64 x box_rows.
static CUtensorMap make_tmap(const void* ptr, int64_t rows, int64_t cols, int64_t ld, int box_rows) {
  CUtensorMap tm;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * 2)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(kGemmBK), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = get_encode()(&tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims,
                            strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed (", static_cast<int>(r), ")");
  return tm;
}

static int num_sms() {
  static int n[64] = {0};
  int dev;
  cudaGetDevice(&dev);
  if (!n[dev]) cudaDeviceGetAttribute(&n[dev], cudaDevAttrMultiProcessorCount, dev);
  return n[dev];
}

template <int BN, int STAGES>
static void launch_gemm(const CUtensorMap& tw, const CUtensorMap& tx, __nv_bfloat16* y, int64_t ldy,
                        const __nv_bfloat16* bias, float* ws, int M, int N, int K, int splits,
                        const int32_t* goff = nullptr, int groups = 0) {
  using S = GemmSmem<BN, STAGES>;
  auto kern = gemm_tcgen05_kernel<BN, STAGES>;
  static bool attr[64] = {false};
  int dev;
  cudaGetDevice(&dev);
  if (!attr[dev]) {
    SWIFT_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          static_cast<int>(S::BYTES)));
    attr[dev] = true;
  }
  // grouped: tile count is only known on the device; N bounds it
  const int tiles = ((M + kGemmBM - 1) / kGemmBM) * ((N + BN - 1) / BN + (goff ? groups : 0)) * splits;
  const int grid = std::min(tiles, num_sms());
  kern<<<grid, kGemmThreads, S::BYTES, cur_stream()>>>(tw, tx, y, ldy, bias, ws, M, N, K, splits,
                                                       status_word_ptr(), goff, groups);
  SWIFT_CHECK_LAUNCH();
}

// Token-tile width and split count for a (features M, tokens N, K) problem.
static void plan(int M, int N, int K, int* bn, int* splits) {
  const int sms = num_sms();
  const int m_tiles = (M + kGemmBM - 1) / kGemmBM;
  int b;
  if (N > 512) {
    b = 256;
  } else {
    b = 16;
    while (b < N && b < 256) b *= 2;
    // narrower token tiles until the grid covers the SMs (weights re-read from L2)
    while (b > 32 && int64_t(m_tiles) * ((N + b - 1) / b) < sms * 3 / 4) b /= 2;
  }
  int tiles = m_tiles * ((N + b - 1) / b);
  int k_iters = (K + kGemmBK - 1) / kGemmBK;
  int s = 1;
  if (tiles < sms * 3 / 4) s = std::max(1, std::min({(sms + tiles - 1) / tiles, k_iters / 4, 8}));
  *bn = b;
  *splits = s;
}

// out [T, N] (row stride may exceed N), x [T, K], w [N, K], bias [N] or None.
// Split-K partials go to `ws` when given (fp32, >= splits*T*N), else to a
// fresh tensor. Returns the number of kernels launched.
int64_t gemm(torch::Tensor out, torch::Tensor x, torch::Tensor w, c10::optional<torch::Tensor> bias) {
  CHECK_BF16(x);
  CHECK_BF16(w);
  CHECK_BF16(out);
  const int64_t K = x.size(-1);
  const int64_t T = x.numel() / K;
  const int64_t M = w.size(0);
  TORCH_CHECK(w.size(1) == K, "gemm: K mismatch");
  TORCH_CHECK(x.stride(-1) == 1 && w.stride(1) == 1 && out.stride(-1) == 1,
              "gemm: inner dim must be contiguous");
  TORCH_CHECK(K % 8 == 0, "gemm: K must be a multiple of 8 (16-byte TMA rows)");
  const int64_t ldx = x.dim() >= 2 ? x.stride(-2) : K;
  const int64_t ldy = out.dim() >= 2 ? out.stride(-2) : M;
  TORCH_CHECK(ldx % 8 == 0 && w.stride(0) % 8 == 0, "gemm: row strides must be 16-byte multiples");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0 &&
                  reinterpret_cast<uintptr_t>(w.data_ptr()) % 16 == 0,
              "gemm: operands must be 16-byte aligned");
  if (T == 0) return 0;
  int bn, splits;
  plan(static_cast<int>(M), static_cast<int>(T), static_cast<int>(K), &bn, &splits);
  CUtensorMap tw = make_tmap(w.data_ptr(), M, K, w.stride(0), kGemmBM);
  CUtensorMap tx = make_tmap(x.data_ptr(), T, K, ldx, bn);
  auto y = reinterpret_cast<__nv_bfloat16*>(out.data_ptr<at::BFloat16>());
  const __nv_bfloat16* bp =
      bias.has_value() ? reinterpret_cast<const __nv_bfloat16*>(bias.value().data_ptr<at::BFloat16>())
                       : nullptr;
  torch::Tensor ws;
  float* wsp = nullptr;
  if (splits > 1) {
    ws = torch::empty({splits, T, M}, x.options().dtype(torch::kFloat));
    wsp = ws.data_ptr<float>();
  }
  const int Mi = static_cast<int>(M), Ni = static_cast<int>(T), Ki = static_cast<int>(K);
  switch (bn) {
    case 16: launch_gemm<16, 8>(tw, tx, y, ldy, bp, wsp, Mi, Ni, Ki, splits); break;
    case 32: launch_gemm<32, 8>(tw, tx, y, ldy, bp, wsp, Mi, Ni, Ki, splits); break;
    case 64: launch_gemm<64, 8>(tw, tx, y, ldy, bp, wsp, Mi, Ni, Ki, splits); break;
    case 128: launch_gemm<128, 6>(tw, tx, y, ldy, bp, wsp, Mi, Ni, Ki, splits); break;
    default: launch_gemm<256, 4>(tw, tx, y, ldy, bp, wsp, Mi, Ni, Ki, splits); break;
  }
  if (splits > 1) {
    int64_t n = M * T;
    int blocks = static_cast<int>(std::min<int64_t>((n + 255) / 256, 148 * 8));
    splitk_reduce_kernel<<<blocks, 256, 0, cur_stream()>>>(y, ldy, wsp, bp, Mi, Ni, splits);
    SWIFT_CHECK_LAUNCH();
    return 2;
  }
  return 1;
}

std::vector<int64_t> gemm_plan(int64_t M, int64_t N, int64_t K) {
  int bn, s;
  plan(static_cast<int>(M), static_cast<int>(N), static_cast<int>(K), &bn, &s);
  return {bn, s};
}

}  // namespace swift

namespace swift {

// Grouped GEMM for MoE experts: out [n_max, M] rows of group g (token rows
// [offsets[g], offsets[g+1]) of x [n_max, K]) = x_rows . w[g]^T with
// w [groups, M, K]. offsets (int32, groups + 1) live on the device, so the
// call needs no host synchronisation and can be captured in a CUDA graph.
int64_t gemm_grouped(torch::Tensor out, torch::Tensor x, torch::Tensor w, torch::Tensor offsets,
                     int64_t avg_rows) {
  CHECK_BF16(x);
  CHECK_BF16(w);
  CHECK_BF16(out);
  TORCH_CHECK(w.dim() == 3 && w.is_contiguous() && x.is_contiguous() && out.is_contiguous());
  TORCH_CHECK(offsets.scalar_type() == at::kInt && offsets.numel() == w.size(0) + 1);
  const int groups = static_cast<int>(w.size(0));
  TORCH_CHECK(groups <= 64, "at most 64 groups");
  const int64_t M = w.size(1), K = w.size(2), T = x.size(0);
  TORCH_CHECK(x.size(1) == K && K % 8 == 0);
  if (T == 0) return 0;
  int bn = 16;
  while (bn < avg_rows && bn < 256) bn *= 2;
  CUtensorMap tw = make_tmap(w.data_ptr(), groups * M, K, K, kGemmBM);
  CUtensorMap tx = make_tmap(x.data_ptr(), T, K, K, bn);
  auto y = reinterpret_cast<__nv_bfloat16*>(out.data_ptr<at::BFloat16>());
  const int Mi = static_cast<int>(M), Ni = static_cast<int>(T), Ki = static_cast<int>(K);
  const int32_t* go = offsets.data_ptr<int32_t>();
  switch (bn) {
    case 16: launch_gemm<16, 8>(tw, tx, y, M, nullptr, nullptr, Mi, Ni, Ki, 1, go, groups); break;
    case 32: launch_gemm<32, 8>(tw, tx, y, M, nullptr, nullptr, Mi, Ni, Ki, 1, go, groups); break;
    case 64: launch_gemm<64, 8>(tw, tx, y, M, nullptr, nullptr, Mi, Ni, Ki, 1, go, groups); break;
    case 128: launch_gemm<128, 6>(tw, tx, y, M, nullptr, nullptr, Mi, Ni, Ki, 1, go, groups); break;
    default: launch_gemm<256, 4>(tw, tx, y, M, nullptr, nullptr, Mi, Ni, Ki, 1, go, groups); break;
  }
  return 1;
}

}  // namespace swift
