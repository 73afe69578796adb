// Paged decode attention (one query token per sequence), split-KV.
//
// Replaces the reference's paged_attention_v1/v2 kernels
// (crates/swiftllm-cuda/kernels/paged_attention.cu:35-163, which cannot run:
// zero dynamic smem, a register atomicMax, and an empty v2 body).
//
// Design (decode is bound by reading the KV pool from HBM):
//  * grid (seq, kv_head, split); a CTA serves all G query heads that share
//    its KV head (GQA packing), so every KV page is read once per step;
//  * 4 warps per CTA, each warp streams whole pages (block_size x D bf16,
//    contiguous in the pool) with the TMA bulk-copy engine
//    (cp.async.bulk + mbarrier complete_tx) through a private ring;
//  * scores on CUDA cores (at most 2 flops per KV byte, far under the FMA
//    rate), online softmax per warp, warps merged in shared memory;
//  * with split > 1 each CTA writes a normalised partial plus (max, sum) to
//    a caller-provided fp32 workspace and decode_combine_kernel merges the
//    splits (FlashDecoding).
// Every mbarrier wait is bounded; on expiry the kernel records
// kErrWaitTimeout in the status word, lets its issued copies land (bounded)
// and returns.
#include "common.cuh"

namespace swift {

// attention_decode_tc.cu: tensor-core kernel for block size 16, head_dim 64/128
bool paged_decode_tc(torch::Tensor out, torch::Tensor q, torch::Tensor kv, int64_t layer,
                     torch::Tensor bt, torch::Tensor seq_lens, int rows, int splits, double scale,
                     int window, torch::Tensor ws);

constexpr int kDecWarps = 4;
constexpr int kDecStages = 2;
constexpr int kMaxGroup = 8;

template <int D, int BS>
struct DecodeCfg {
  static constexpr int LPT = 32 / BS;            // lanes per token in QK
  static constexpr int DL = D / LPT;             // channels per lane in QK
  static constexpr int CH = DL * 2 / 16;         // 16-byte chunks per lane in QK
  static constexpr int DP = (D + 31) / 32;       // channels per lane in PV
  // PV channel ownership: contiguous (lane*DP + d, bf16x2 loads) when DP is
  // even, else strided (lane + 32*d)
  static constexpr bool CONTIG = (D % 64) == 0;
  static constexpr int PAGE = BS * D * 2;        // bytes of one (layer, k|v, head) page
  static constexpr int STAGE = 2 * PAGE;
  static constexpr int NST = STAGE >= 16384 ? 1 : kDecStages;  // ring depth per warp
  static constexpr size_t RING = size_t(kDecWarps) * NST * STAGE;
  // shared bytes for GQA group g: ring + q + per-warp merge buffers + barriers
  static constexpr size_t smem_for(int g) {
    return RING + size_t(g) * D * 4 + size_t(kDecWarps) * g * (D + 2) * 4 + kDecWarps * NST * 8 + 16;
  }
  static constexpr size_t SMEM = smem_for(kMaxGroup);
  static_assert((DL * 2) % 16 == 0, "QK lane slice must be whole 16-byte chunks");
};

template <int D, int BS>
__global__ void __launch_bounds__(kDecWarps * 32, 3)
    paged_decode_kernel(__nv_bfloat16* __restrict__ out, const __nv_bfloat16* __restrict__ q,
                        const __nv_bfloat16* __restrict__ kv, int64_t blk_stride,
                        int64_t layer_off, int64_t kv_stride, const int32_t* __restrict__ bt,
                        int64_t bt_stride, const int32_t* __restrict__ seq_lens, int Hq, int Hkv,
                        int splits, float scale, int window, float* __restrict__ ws,
                        int* status, const float* __restrict__ alibi) {
  using C = DecodeCfg<D, BS>;
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* ring = smem;
  const int G = Hq / Hkv;
  float* q_s = reinterpret_cast<float*>(smem + C::RING);
  float* merge = q_s + G * D;  // [warps][G][D] acc, then [warps][G][2] (m, l)
  uint64_t* bars = reinterpret_cast<uint64_t*>(merge + kDecWarps * G * (D + 2));

  const int row = blockIdx.x, kvh = blockIdx.y, split = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int len = seq_lens[row];

  for (int i = threadIdx.x; i < G * D; i += blockDim.x)
    q_s[i] = __bfloat162float(q[(int64_t(row) * Hq + kvh * G) * D + i]);
  if (threadIdx.x < kDecWarps * C::NST) mbar_init(&bars[threadIdx.x], 1);
  fence_mbar_init();
  __syncthreads();

  const int first = window > 0 ? max(0, len - window) : 0;
  const int p_lo_all = first / BS;
  const int n_pages = (len + BS - 1) / BS;
  const int span = max(0, n_pages - p_lo_all);
  const int pps = (span + splits - 1) / splits;
  const int p_lo = p_lo_all + split * pps;
  const int p_hi = min(n_pages, p_lo + pps);

  float m[kMaxGroup], l[kMaxGroup], acc[kMaxGroup][C::DP];
#pragma unroll
  for (int g = 0; g < kMaxGroup; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
#pragma unroll
    for (int i = 0; i < C::DP; ++i) acc[g][i] = 0.f;
  }

  uint8_t* my_ring = ring + size_t(warp) * C::NST * C::STAGE;
  uint64_t* my_bars = bars + warp * C::NST;
  const int n_mine = p_hi > p_lo + warp ? (p_hi - p_lo - warp + kDecWarps - 1) / kDecWarps : 0;
  const int32_t* my_bt = bt + int64_t(row) * bt_stride;
  const int64_t head_off = layer_off + int64_t(kvh) * BS * D;

  auto issue = [&](int i) {
    int page = p_lo + warp + i * kDecWarps;
    int64_t blk = my_bt[page];
    const __nv_bfloat16* kp = kv + blk * blk_stride + head_off;
    uint8_t* dst = my_ring + (i % C::NST) * C::STAGE;
    uint64_t* bar = &my_bars[i % C::NST];
    mbar_arrive_expect_tx(bar, C::STAGE);
    bulk_g2s(dst, kp, C::PAGE, bar);
    bulk_g2s(dst + C::PAGE, kp + kv_stride, C::PAGE, bar);
  };
  if (lane == 0)
    for (int i = 0; i < min(n_mine, C::NST); ++i) issue(i);
  __syncwarp();

  const int tok = lane / C::LPT, part = lane % C::LPT;
  bool failed = false;
  int fail_at = 0;
  for (int i = 0; i < n_mine; ++i) {
    const int stage = i % C::NST;
    if (!mbar_wait_warp(&my_bars[stage], (i / C::NST) & 1, status, 1)) {
      failed = true;
      fail_at = i;
      break;
    }
    const __nv_bfloat16* ks = reinterpret_cast<const __nv_bfloat16*>(my_ring + stage * C::STAGE);
    const __nv_bfloat16* vs = ks + BS * D;
    const int page = p_lo + warp + i * kDecWarps;
    const int t_abs = page * BS + tok;
    const bool valid = t_abs < len && t_abs >= first;
    float s[kMaxGroup];
#pragma unroll
    for (int g = 0; g < kMaxGroup; ++g) s[g] = 0.f;
    const __nv_bfloat16* krow = ks + tok * D + part * C::DL;
#pragma unroll
    for (int c0 = 0; c0 < C::CH; ++c0) {
      const int c = (c0 + lane) % C::CH;  // rotate chunks: conflict-free shared reads
      float kf[8];
      load8(krow + c * 8, kf);
#pragma unroll
      for (int g = 0; g < kMaxGroup; ++g) {
        if (g < G) {
          const float* qg = q_s + g * D + part * C::DL + c * 8;
#pragma unroll
          for (int e = 0; e < 8; ++e) s[g] += qg[e] * kf[e];
        }
      }
    }
#pragma unroll
    for (int g = 0; g < kMaxGroup; ++g) {
      if (g < G) {
#pragma unroll
        for (int o = C::LPT / 2; o > 0; o >>= 1) s[g] += __shfl_xor_sync(0xffffffffu, s[g], o);
        // ALiBi: + slope(head) * (key position - query position)
        const float bias = alibi != nullptr ? alibi[kvh * G + g] * float(t_abs - (len - 1)) : 0.f;
        s[g] = valid ? s[g] * scale + bias : -INFINITY;
        float pm = warp_max(s[g]);
        float mn = fmaxf(m[g], pm);
        float corr = mn == -INFINITY ? 1.f : __expf(m[g] - mn);
        float p = mn == -INFINITY ? 0.f : __expf(s[g] - mn);
        float ps = warp_sum(part == 0 ? p : 0.f);
        l[g] = l[g] * corr + ps;
        m[g] = mn;
#pragma unroll
        for (int d = 0; d < C::DP; ++d) acc[g][d] *= corr;
        s[g] = p;
      }
    }
#pragma unroll 4
    for (int t = 0; t < BS; ++t) {
      float vf[C::DP];
      if constexpr (C::CONTIG) {
#pragma unroll
        for (int d = 0; d < C::DP; d += 2) {
          float2 f2 = __bfloat1622float2(
              *reinterpret_cast<const __nv_bfloat162*>(vs + t * D + lane * C::DP + d));
          vf[d] = f2.x;
          vf[d + 1] = f2.y;
        }
      } else {
#pragma unroll
        for (int d = 0; d < C::DP; ++d) {
          int ch = lane + 32 * d;
          vf[d] = ch < D ? __bfloat162float(vs[t * D + ch]) : 0.f;
        }
      }
#pragma unroll
      for (int g = 0; g < kMaxGroup; ++g) {
        if (g < G) {
          float p = __shfl_sync(0xffffffffu, s[g], t * C::LPT);
#pragma unroll
          for (int d = 0; d < C::DP; ++d) acc[g][d] += p * vf[d];
        }
      }
    }
    __syncwarp();
    if (lane == 0 && i + C::NST < n_mine) issue(i + C::NST);
    __syncwarp();
  }
  if (failed) {
    // give up, but first let copies already issued into this warp's ring land
    // (bounded) so no bulk copy writes shared memory after the CTA exits
    for (int j = fail_at + 1; j < min(n_mine, fail_at + C::NST); ++j)
      mbar_wait_warp(&my_bars[j % C::NST], (j / C::NST) & 1, status, 2, 1u << 22);
  }

  float* macc = merge;                             // [W][G][D]
  float* mml = merge + kDecWarps * G * D;  // [W][G][2]
#pragma unroll
  for (int g = 0; g < kMaxGroup; ++g) {
    if (g < G) {
#pragma unroll
      for (int d = 0; d < C::DP; ++d) {
        int ch = C::CONTIG ? lane * C::DP + d : lane + 32 * d;
        if (ch < D) macc[(warp * G + g) * D + ch] = acc[g][d];
      }
      if (lane == 0) {
        mml[(warp * G + g) * 2] = m[g];
        mml[(warp * G + g) * 2 + 1] = l[g];
      }
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < G * D; i += blockDim.x) {
    int g = i / D, ch = i % D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kDecWarps; ++w) M = fmaxf(M, mml[(w * G + g) * 2]);
    float L = 0.f, O = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < kDecWarps; ++w) {
        float mw = mml[(w * G + g) * 2];
        if (mw == -INFINITY) continue;
        float f = __expf(mw - M);
        L += mml[(w * G + g) * 2 + 1] * f;
        O += macc[(w * G + g) * D + ch] * f;
      }
    }
    const int h = kvh * G + g;
    float o = L > 0.f ? O / L : 0.f;
    if (splits == 1) {
      out[(int64_t(row) * Hq + h) * D + ch] = __float2bfloat16(o);
    } else {
      const int64_t base = (int64_t(row) * Hq + h) * splits + split;
      ws[base * D + ch] = o;
      if (ch == 0) {
        float* ml = ws + int64_t(gridDim.x) * Hq * splits * D;
        ml[base * 2] = M;
        ml[base * 2 + 1] = L;
      }
    }
  }
}

template <int D>
__global__ void decode_combine_kernel(__nv_bfloat16* __restrict__ out, const float* __restrict__ ws,
                                      int rows, int Hq, int splits) {
  pdl_wait();  // previous kernel done (programmatic dependent launch)
  pdl_trigger();
  const int row = blockIdx.x, h = blockIdx.y;
  const int64_t base = (int64_t(row) * Hq + h) * splits;
  const float* ml = ws + int64_t(rows) * Hq * splits * D;
  float M = -INFINITY;
  for (int s = 0; s < splits; ++s) M = fmaxf(M, ml[(base + s) * 2]);
  for (int ch = threadIdx.x; ch < D; ch += blockDim.x) {
    float L = 0.f, O = 0.f;
    if (M != -INFINITY) {
      for (int s = 0; s < splits; ++s) {
        float ms = ml[(base + s) * 2];
        if (ms == -INFINITY) continue;
        float f = __expf(ms - M) * ml[(base + s) * 2 + 1];
        L += f;
        O += ws[(base + s) * D + ch] * f;
      }
    }
    out[(int64_t(row) * Hq + h) * D + ch] = __float2bfloat16(L > 0.f ? O / L : 0.f);
  }
}

template <int D, int BS>
static void launch_decode(torch::Tensor out, torch::Tensor q, torch::Tensor kv, int64_t layer,
                          torch::Tensor bt, torch::Tensor seq_lens, int rows, int splits,
                          double scale, int window, torch::Tensor ws, const float* alibi) {
  using C = DecodeCfg<D, BS>;
  const int Hq = static_cast<int>(q.size(1)), Hkv = static_cast<int>(kv.size(3));
  TORCH_CHECK(Hq % Hkv == 0 && Hq / Hkv <= kMaxGroup, "GQA group must be <= 8");
  auto kern = paged_decode_kernel<D, BS>;
  static bool attr_set[64] = {false};
  int dev;
  cudaGetDevice(&dev);
  if (!attr_set[dev]) {
    SWIFT_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          static_cast<int>(C::SMEM)));
    attr_set[dev] = true;
  }
  if (splits > 1)
    TORCH_CHECK(ws.numel() >= int64_t(rows) * Hq * splits * (D + 2), "decode workspace too small");
  dim3 grid(rows, Hkv, splits);
  auto st = cur_stream();
  kern<<<grid, kDecWarps * 32, C::smem_for(Hq / Hkv), st>>>(
      reinterpret_cast<__nv_bfloat16*>(out.data_ptr<at::BFloat16>()),
      reinterpret_cast<const __nv_bfloat16*>(q.data_ptr<at::BFloat16>()),
      reinterpret_cast<const __nv_bfloat16*>(kv.data_ptr<at::BFloat16>()), kv.stride(0),
      layer * kv.stride(1), kv.stride(2), bt.data_ptr<int32_t>(), bt.stride(0),
      seq_lens.data_ptr<int32_t>(), Hq, Hkv, splits, static_cast<float>(scale), window,
      splits > 1 ? ws.data_ptr<float>() : nullptr, status_word_ptr(), alibi);
  SWIFT_CHECK_LAUNCH();
  if (splits > 1) {
    decode_combine_kernel<D><<<dim3(rows, Hq), 128, 0, st>>>(
        reinterpret_cast<__nv_bfloat16*>(out.data_ptr<at::BFloat16>()), ws.data_ptr<float>(), rows,
        Hq, splits);
    SWIFT_CHECK_LAUNCH();
  }
}

// out, q: [T, Hq, D] (the first `rows` rows are decode rows); kv pool
// [blocks, layers, 2, Hkv, BS, D]; bt [S, max_blocks]; seq_lens [S].
// Returns the number of kernels launched.
// alibi: optional fp32 [Hq] ALiBi slopes (then the CUDA-core kernel runs;
// the tensor-core kernel has no bias term).
int64_t paged_decode(torch::Tensor out, torch::Tensor q, torch::Tensor kv, int64_t layer,
                     torch::Tensor bt, torch::Tensor seq_lens, int64_t rows, int64_t splits,
                     double scale, int64_t window, torch::Tensor ws,
                     c10::optional<torch::Tensor> alibi) {
  CHECK_BF16(q);
  CHECK_BF16(kv);
  CHECK_CONTIG(kv);
  TORCH_CHECK(q.is_contiguous() && out.is_contiguous());
  TORCH_CHECK(bt.scalar_type() == at::kInt && seq_lens.scalar_type() == at::kInt);
  TORCH_CHECK(bt.stride(1) == 1);
  if (rows <= 0) return 0;
  const int D = static_cast<int>(q.size(2)), BS = static_cast<int>(kv.size(4));
  splits = std::max<int64_t>(1, splits);
  if (splits > 1)
    TORCH_CHECK(ws.numel() >= rows * q.size(1) * splits * (D + 2), "decode workspace too small");
  const float* ap = nullptr;
  if (alibi.has_value()) {
    TORCH_CHECK(alibi->scalar_type() == at::kFloat && alibi->is_contiguous() &&
                    alibi->numel() == q.size(1) && alibi->is_cuda(),
                "paged_decode: alibi slopes must be fp32 [num_heads] on the device");
    ap = alibi->data_ptr<float>();
  }
  // tensor-core path (block size 16, head_dim 64 / 128)
  if (ap == nullptr && paged_decode_tc(out, q, kv, layer, bt, seq_lens, static_cast<int>(rows),
                      static_cast<int>(splits), scale, static_cast<int>(window), ws)) {
    if (splits == 1) return 1;
    const int Hq = static_cast<int>(q.size(1));
    auto* op = reinterpret_cast<__nv_bfloat16*>(out.data_ptr<at::BFloat16>());
    if (D == 128)
      launch_pdl(decode_combine_kernel<128>, dim3(rows, Hq), dim3(128), 0, cur_stream(), op,
                 static_cast<const float*>(ws.data_ptr<float>()), static_cast<int>(rows), Hq,
                 static_cast<int>(splits));
    else
      launch_pdl(decode_combine_kernel<64>, dim3(rows, Hq), dim3(128), 0, cur_stream(), op,
                 static_cast<const float*>(ws.data_ptr<float>()), static_cast<int>(rows), Hq,
                 static_cast<int>(splits));
    SWIFT_CHECK_LAUNCH();
    return 2;
  }
#define DEC_CASE(d, bs)                                                                  \
  if (D == d && BS == bs) {                                                              \
    launch_decode<d, bs>(out, q, kv, layer, bt, seq_lens, static_cast<int>(rows),         \
                         static_cast<int>(splits), scale, static_cast<int>(window), ws, ap); \
    return splits > 1 ? 2 : 1;                                                           \
  }
  DEC_CASE(128, 16)
  DEC_CASE(128, 32)
  DEC_CASE(128, 8)
  DEC_CASE(64, 16)
  DEC_CASE(64, 32)
  DEC_CASE(80, 16)
  DEC_CASE(96, 16)
#undef DEC_CASE
  TORCH_CHECK(false, "paged_decode: unsupported head_dim/block_size ", D, "/", BS);
  return 0;
}

}  // namespace swift

// ---------------------------------------------------------------------------
// Allocation-free C entry point (declared in swift_noalloc.h; no counterpart
// in the reference). The split-KV scratch that paged_decode takes from the
// caller lives here in a fixed device array instead.
#include "swift_noalloc.h"

static __device__ __align__(256) float g_noalloc_scratch[SWIFT_NOALLOC_SCRATCH_BYTES / sizeof(float)];
// Status word of the allocation-free calls ([code, site], the same codes as
// the library's own status word): a kernel that gives up a bounded wait
// records it here; swift_noalloc_status() reads it back.
static __device__ int g_noalloc_status[2];

namespace swift {
namespace {

constexpr int kNoallocMaxDevices = 64;
float* g_noalloc_ptr[kNoallocMaxDevices] = {nullptr};
int* g_noalloc_status_ptr[kNoallocMaxDevices] = {nullptr};

// Once per device, with that device current: the device addresses of the
// scratch array and the status word (host code must not use the arrays'
// names as pointers).
int noalloc_setup(float** scratch, int** status) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return SWIFT_NOALLOC_ERR_CUDA;
  if (dev < 0 || dev >= kNoallocMaxDevices) return SWIFT_NOALLOC_ERR_CUDA;
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    void* ps = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr)
      return SWIFT_NOALLOC_ERR_CUDA;
    if (cudaGetSymbolAddress(&ps, g_noalloc_status) != cudaSuccess || ps == nullptr)
      return SWIFT_NOALLOC_ERR_CUDA;
    g_noalloc_status_ptr[dev] = static_cast<int*>(ps);
    g_noalloc_ptr[dev] = static_cast<float*>(p);
  }
  *scratch = g_noalloc_ptr[dev];
  *status = g_noalloc_status_ptr[dev];
  return SWIFT_NOALLOC_OK;
}

template <int D, int BS>
int noalloc_decode(void* out, const void* q, const void* kv, int64_t blk_stride, int64_t layer_off,
                   int64_t kv_stride, const int32_t* bt, int64_t bt_stride,
                   const int32_t* seq_lens, int rows, int Hq, int Hkv, int splits, float scale,
                   int window, float* scratch, int* status, cudaStream_t stream) {
  using C = DecodeCfg<D, BS>;
  auto kern = paged_decode_kernel<D, BS>;
  static bool attr_set[kNoallocMaxDevices] = {false};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return SWIFT_NOALLOC_ERR_CUDA;
  if (!attr_set[dev]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(C::SMEM)) != cudaSuccess)
      return SWIFT_NOALLOC_ERR_CUDA;
    attr_set[dev] = true;
  }
  dim3 grid(rows, Hkv, splits);
  kern<<<grid, kDecWarps * 32, C::smem_for(Hq / Hkv), stream>>>(
      static_cast<__nv_bfloat16*>(out), static_cast<const __nv_bfloat16*>(q),
      static_cast<const __nv_bfloat16*>(kv), blk_stride, layer_off, kv_stride, bt, bt_stride,
      seq_lens, Hq, Hkv, splits, scale, window, splits > 1 ? scratch : nullptr, status, nullptr);
  if (cudaGetLastError() != cudaSuccess) return SWIFT_NOALLOC_ERR_CUDA;
  if (splits > 1) {
    decode_combine_kernel<D><<<dim3(rows, Hq), 128, 0, stream>>>(
        static_cast<__nv_bfloat16*>(out), scratch, rows, Hq, splits);
    if (cudaGetLastError() != cudaSuccess) return SWIFT_NOALLOC_ERR_CUDA;
  }
  return SWIFT_NOALLOC_OK;
}

}  // namespace
}  // namespace swift

extern "C" __attribute__((visibility("default"))) int swift_paged_decode_noalloc(
    void* out, const void* q, const void* kv, int64_t blk_stride, int64_t layer_off,
    int64_t kv_stride, int block_size, int head_dim, const int32_t* bt, int64_t bt_stride,
    const int32_t* seq_lens, int rows, int Hq, int Hkv, int splits, float scale, int window,
    cudaStream_t stream) {
  using namespace swift;
  if (!out || !q || !kv || !bt || !seq_lens || rows <= 0 || Hq <= 0 || Hkv <= 0 || splits <= 0)
    return SWIFT_NOALLOC_ERR_ARGS;
  if (Hq % Hkv != 0 || Hq / Hkv > kMaxGroup) return SWIFT_NOALLOC_ERR_UNSUPPORTED;
  const bool shape_ok = (head_dim == 128 && (block_size == 8 || block_size == 16 || block_size == 32)) ||
                        (head_dim == 64 && (block_size == 16 || block_size == 32)) ||
                        ((head_dim == 80 || head_dim == 96) && block_size == 16);
  if (!shape_ok) return SWIFT_NOALLOC_ERR_UNSUPPORTED;
  // the kernel moves 16-byte pieces of q, out and every KV page (bulk
  // copies): the pointers must be 16-byte aligned and the element offsets
  // multiples of 8 bf16
  auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  if (!al16(out) || !al16(q) || !al16(kv) || blk_stride % 8 || layer_off % 8 || kv_stride % 8 ||
      blk_stride <= 0 || kv_stride <= 0 || layer_off < 0 || bt_stride <= 0)
    return SWIFT_NOALLOC_ERR_ARGS;
  const uint64_t need = splits > 1
      ? static_cast<uint64_t>(rows) * Hq * splits * (static_cast<uint64_t>(head_dim) + 2) * sizeof(float)
      : 0;
  if (need > SWIFT_NOALLOC_SCRATCH_BYTES) return SWIFT_NOALLOC_ERR_TOO_LARGE;
  float* scratch = nullptr;
  int* status = nullptr;
  int st = noalloc_setup(&scratch, &status);
  if (st != SWIFT_NOALLOC_OK) return st;
#define NOALLOC_CASE(d, bs)                                                                     \
  if (head_dim == d && block_size == bs)                                                        \
    return noalloc_decode<d, bs>(out, q, kv, blk_stride, layer_off, kv_stride, bt, bt_stride,   \
                                 seq_lens, rows, Hq, Hkv, splits, scale, window, scratch, status, \
                                 stream);
  NOALLOC_CASE(128, 16)
  NOALLOC_CASE(128, 32)
  NOALLOC_CASE(128, 8)
  NOALLOC_CASE(64, 16)
  NOALLOC_CASE(64, 32)
  NOALLOC_CASE(80, 16)
  NOALLOC_CASE(96, 16)
#undef NOALLOC_CASE
  return SWIFT_NOALLOC_ERR_UNSUPPORTED;
}

// Reads (and with clear != 0 resets) the status word of the allocation-free
// calls on the current device. Synchronous: it waits for the device.
extern "C" __attribute__((visibility("default"))) int swift_noalloc_status(int* code, int* site,
                                                                           int clear) {
  using namespace swift;
  if (!code || !site) return SWIFT_NOALLOC_ERR_ARGS;
  float* scratch = nullptr;
  int* status = nullptr;
  int st = noalloc_setup(&scratch, &status);
  if (st != SWIFT_NOALLOC_OK) return st;
  int h[2] = {0, 0};
  if (cudaMemcpyFromSymbol(h, g_noalloc_status, sizeof(h)) != cudaSuccess) return SWIFT_NOALLOC_ERR_CUDA;
  *code = h[0];
  *site = h[1];
  if (clear) {
    const int z[2] = {0, 0};
    if (cudaMemcpyToSymbol(g_noalloc_status, z, sizeof(z)) != cudaSuccess) return SWIFT_NOALLOC_ERR_CUDA;
  }
  return SWIFT_NOALLOC_OK;
}
