// Paged decode attention on the tensor cores (block size 16, head_dim 64/128).
//
// Same contract and split-KV workspace layout as paged_decode_kernel in
// attention_decode.cu (which remains the path for other page/head sizes);
// paged_decode dispatches here when it can.
//
// Per warp and per 16-token page:
//   * the page's K and V tiles arrive by 2-D TMA (cp.async.bulk.tensor,
//     per-CTA loads) with the 128-byte swizzle, so ldmatrix reads them without
//     bank conflicts; each warp owns a 2-stage ring and mbarriers;
//   * S = Q K^T with mma.m16n8k16 (bf16 in, fp32 out): the MMA rows are the
//     G query heads that share this KV head (GQA packing, rows >= G are 0),
//     so grouped-query models cost the same as single-head ones;
//   * online softmax on the accumulator fragments (quad shuffles only);
//   * O += P V with P re-packed from the score fragments as the A operand.
// Roughly 120 warp instructions per page instead of ~900 for the CUDA-core
// loop, which was issue-bound at 41% of HBM bandwidth.
// Every mbarrier wait is bounded (status word + early return after letting
// issued copies land).
#include "tma_util.cuh"

namespace swift {

namespace {

constexpr int kTcWarps = 4;
constexpr int kTcBS = 16;
constexpr int kTcMaxG = 8;

__device__ __forceinline__ void tc_ldsm_x4(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3,
                                           uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void tc_ldsm_x4_t(uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                             uint32_t& r3, uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void tc_mma(float d[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t tc_pack(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Shared address of element (row r, column c) of a page tile stored as
// D/64 TMA boxes of [16 rows x 128 B] with the 128-byte swizzle.
__device__ __forceinline__ uint32_t swz(uint32_t base, int r, int c) {
  const int box = c >> 6, j = (c & 63) >> 3;
  return base + box * (kTcBS * 128) + r * 128 + ((j ^ (r & 7)) << 4) + (c & 7) * 2;
}

template <int D>
struct TcCfg {
  static constexpr int NKT = D / 16, NDT = D / 8, BOXES = D / 64;
  static constexpr int PAGE = kTcBS * D * 2;
  static constexpr int STAGE = 2 * PAGE;
  static constexpr int NST = D >= 128 ? 2 : 4;
  static constexpr size_t RING = size_t(kTcWarps) * NST * STAGE;
  static constexpr size_t smem_for(int g) {
    return 1024 + RING + size_t(kTcWarps) * g * (D + 2) * 4 + kTcWarps * NST * 8 + 16;
  }
};

template <int D>
__global__ void __launch_bounds__(kTcWarps * 32, 3)
    paged_decode_tc_kernel(const __grid_constant__ CUtensorMap tm_kv,
                           __nv_bfloat16* __restrict__ out, const __nv_bfloat16* __restrict__ q,
                           int rows_per_blk, int layer_row_off, const int32_t* __restrict__ bt,
                           int64_t bt_stride, const int32_t* __restrict__ seq_lens, int Hq, int Hkv,
                           int splits, float scale_log2, int window, float* __restrict__ ws,
                           int* status) {
  pdl_wait();  // previous kernel done (programmatic dependent launch)
  pdl_trigger();
  using C = TcCfg<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* ring =
      reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int G = Hq / Hkv;
  float* merge = reinterpret_cast<float*>(ring + C::RING);  // [W][G][D] then [W][G][2]
  uint64_t* bars = reinterpret_cast<uint64_t*>(merge + kTcWarps * G * (D + 2));

  const int row = blockIdx.x, kvh = blockIdx.y, split = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int len = seq_lens[row];
  if (threadIdx.x < kTcWarps * C::NST) mbar_init(&bars[threadIdx.x], 1);
  fence_mbar_init();
  __syncthreads();

  // Q as the A operand: rows = query heads of this KV head (g < G), 8..15 zero.
  const int g0 = lane >> 2;
  uint32_t qf[C::NKT][4];
  {
    const __nv_bfloat16* qrow = q + (int64_t(row) * Hq + kvh * G + g0) * D + (lane & 3) * 2;
#pragma unroll
    for (int kk = 0; kk < C::NKT; ++kk) {
      qf[kk][0] = g0 < G ? *reinterpret_cast<const uint32_t*>(qrow + kk * 16) : 0u;
      qf[kk][1] = 0u;
      qf[kk][2] = g0 < G ? *reinterpret_cast<const uint32_t*>(qrow + kk * 16 + 8) : 0u;
      qf[kk][3] = 0u;
    }
  }

  const int first = window > 0 ? max(0, len - window) : 0;
  const int p_lo_all = first / kTcBS;
  const int n_pages = (len + kTcBS - 1) / kTcBS;
  const int span = max(0, n_pages - p_lo_all);
  const int pps = (span + splits - 1) / splits;
  const int p_lo = p_lo_all + split * pps;
  const int p_hi = min(n_pages, p_lo + pps);
  const int n_mine = p_hi > p_lo + warp ? (p_hi - p_lo - warp + kTcWarps - 1) / kTcWarps : 0;
  const int32_t* my_bt = bt + int64_t(row) * bt_stride;
  uint8_t* my_ring = ring + size_t(warp) * C::NST * C::STAGE;
  uint64_t* my_bars = bars + warp * C::NST;
  const int head_row = layer_row_off + kvh * kTcBS;
  const int v_rows = Hkv * kTcBS;

  auto issue = [&](int i) {
    const int page = p_lo + warp + i * kTcWarps;
    const int y = my_bt[page] * rows_per_blk + head_row;
    uint8_t* dst = my_ring + (i % C::NST) * C::STAGE;
    uint64_t* bar = &my_bars[i % C::NST];
    mbar_arrive_expect_tx(bar, C::STAGE);
#pragma unroll
    for (int b = 0; b < C::BOXES; ++b) {
      tma_load_2d_nomc(dst + b * (kTcBS * 128), &tm_kv, b * 64, y, bar);
      tma_load_2d_nomc(dst + C::PAGE + b * (kTcBS * 128), &tm_kv, b * 64, y + v_rows, bar);
    }
  };
  if (lane == 0)
    for (int i = 0; i < min(n_mine, C::NST); ++i) issue(i);
  __syncwarp();

  float o[C::NDT][4];
#pragma unroll
  for (int n = 0; n < C::NDT; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float m = -INFINITY, l = 0.f;
  bool failed = false;
  int fail_at = 0;
  for (int i = 0; i < n_mine; ++i) {
    const int stage = i % C::NST;
    if (!mbar_wait_warp(&my_bars[stage], (i / C::NST) & 1, status, 20)) {
      failed = true;
      fail_at = i;
      break;
    }
    const uint32_t ks = smem_u32(my_ring + stage * C::STAGE);
    const uint32_t vs = ks + C::PAGE;
    float s[2][4];
#pragma unroll
    for (int n = 0; n < 2; ++n) {
      s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll
      for (int kk = 0; kk < C::NKT; kk += 2) {
        uint32_t b0, b1, b2, b3;
        tc_ldsm_x4(b0, b1, b2, b3, swz(ks, n * 8 + (lane & 7), kk * 16 + (lane >> 3) * 8));
        tc_mma(s[n], qf[kk], b0, b1);
        tc_mma(s[n], qf[kk + 1], b2, b3);
      }
    }
    const int t0 = (p_lo + warp + i * kTcWarps) * kTcBS + (lane & 3) * 2;
    float mx = -INFINITY;
#pragma unroll
    for (int n = 0; n < 2; ++n)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int t = t0 + n * 8 + e;
        float v = s[n][e] * scale_log2;
        v = (t >= len || t < first) ? -INFINITY : v;
        s[n][e] = v;
        mx = fmaxf(mx, v);
      }
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    const float mn = fmaxf(m, mx);
    const float corr = mn == -INFINITY ? 1.f : exp2f(m - mn);
    float ps = 0.f;
#pragma unroll
    for (int n = 0; n < 2; ++n)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        float p = mn == -INFINITY ? 0.f : exp2f(s[n][e] - mn);
        s[n][e] = p;
        ps += p;
      }
    l = l * corr + ps;
    m = mn;
#pragma unroll
    for (int n = 0; n < C::NDT; ++n) {
      o[n][0] *= corr;
      o[n][1] *= corr;
    }
    uint32_t a[4];
    a[0] = tc_pack(s[0][0], s[0][1]);
    a[1] = 0u;
    a[2] = tc_pack(s[1][0], s[1][1]);
    a[3] = 0u;
#pragma unroll
    for (int n = 0; n < C::NDT; n += 2) {
      uint32_t b0, b1, b2, b3;
      tc_ldsm_x4_t(b0, b1, b2, b3,
                   swz(vs, (lane & 7) + ((lane >> 3) & 1) * 8, n * 8 + (lane >> 4) * 8));
      tc_mma(o[n], a, b0, b1);
      tc_mma(o[n + 1], a, b2, b3);
    }
    __syncwarp();
    if (lane == 0 && i + C::NST < n_mine) issue(i + C::NST);
    __syncwarp();
  }
  if (failed) {
    for (int j = fail_at + 1; j < min(n_mine, fail_at + C::NST); ++j)
      mbar_wait_warp(&my_bars[j % C::NST], (j / C::NST) & 1, status, 21, 1u << 22);
  }
  l += __shfl_xor_sync(0xffffffffu, l, 1);
  l += __shfl_xor_sync(0xffffffffu, l, 2);

  float* macc = merge;
  float* mml = merge + kTcWarps * G * D;
  if (g0 < G) {
#pragma unroll
    for (int n = 0; n < C::NDT; ++n) {
      const int ch = n * 8 + (lane & 3) * 2;
      macc[(warp * G + g0) * D + ch] = o[n][0];
      macc[(warp * G + g0) * D + ch + 1] = o[n][1];
    }
    if ((lane & 3) == 0) {
      mml[(warp * G + g0) * 2] = m;
      mml[(warp * G + g0) * 2 + 1] = l;
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < G * D; i += blockDim.x) {
    const int g = i / D, ch = i % D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kTcWarps; ++w) M = fmaxf(M, mml[(w * G + g) * 2]);
    float L = 0.f, O = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < kTcWarps; ++w) {
        const float mw = mml[(w * G + g) * 2];
        if (mw == -INFINITY) continue;
        const float f = exp2f(mw - M);
        L += mml[(w * G + g) * 2 + 1] * f;
        O += macc[(w * G + g) * D + ch] * f;
      }
    }
    const int h = kvh * G + g;
    const float res = L > 0.f ? O / L : 0.f;
    if (splits == 1) {
      out[(int64_t(row) * Hq + h) * D + ch] = __float2bfloat16(res);
    } else {
      // (max, sum) in natural-log units, matching decode_combine_kernel
      const int64_t base = (int64_t(row) * Hq + h) * splits + split;
      ws[base * D + ch] = res;
      if (ch == 0) {
        float* ml = ws + int64_t(gridDim.x) * Hq * splits * D;
        ml[base * 2] = M == -INFINITY ? -INFINITY : M * 0.6931471805599453f;
        ml[base * 2 + 1] = L;
      }
    }
  }
}

template <int D>
void launch_tc(torch::Tensor out, torch::Tensor q, torch::Tensor kv, int64_t layer,
               torch::Tensor bt, torch::Tensor seq_lens, int rows, int splits, double scale,
               int window, torch::Tensor ws) {
  using C = TcCfg<D>;
  const int Hq = static_cast<int>(q.size(1)), Hkv = static_cast<int>(kv.size(3));
  const int L = static_cast<int>(kv.size(1));
  const int64_t total_rows = kv.numel() / D;
  TORCH_CHECK(total_rows < (int64_t(1) << 31), "KV pool too large for 32-bit TMA rows");
  CUtensorMap tm = make_tmap_2d(kv.data_ptr(), total_rows, D, D, 64, kTcBS);
  auto kern = paged_decode_tc_kernel<D>;
  static bool attr[64] = {false};
  int dev;
  cudaGetDevice(&dev);
  if (!attr[dev]) {
    SWIFT_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          static_cast<int>(C::smem_for(kTcMaxG))));
    attr[dev] = true;
  }
  const int rows_per_blk = L * 2 * Hkv * kTcBS;
  const int layer_row_off = static_cast<int>(layer) * 2 * Hkv * kTcBS;
  dim3 grid(rows, Hkv, splits);
  launch_pdl(kern, dim3(grid), dim3(kTcWarps * 32), C::smem_for(Hq / Hkv), cur_stream(), 
      tm, reinterpret_cast<__nv_bfloat16*>(out.data_ptr<at::BFloat16>()),
      reinterpret_cast<const __nv_bfloat16*>(q.data_ptr<at::BFloat16>()), rows_per_blk,
      layer_row_off, bt.data_ptr<int32_t>(), bt.stride(0), seq_lens.data_ptr<int32_t>(), Hq, Hkv,
      splits, static_cast<float>(scale * 1.4426950408889634), window,
      splits > 1 ? ws.data_ptr<float>() : nullptr, status_word_ptr());
  SWIFT_CHECK_LAUNCH();
}

}  // namespace

// Launches the tensor-core decode kernel when the shape is supported; the
// caller launches the split combine. Returns false if unsupported.
bool paged_decode_tc(torch::Tensor out, torch::Tensor q, torch::Tensor kv, int64_t layer,
                     torch::Tensor bt, torch::Tensor seq_lens, int rows, int splits, double scale,
                     int window, torch::Tensor ws) {
  const int D = static_cast<int>(q.size(2)), BS = static_cast<int>(kv.size(4));
  const int Hq = static_cast<int>(q.size(1)), Hkv = static_cast<int>(kv.size(3));
  if (BS != kTcBS || Hq % Hkv || Hq / Hkv > kTcMaxG) return false;
  if (reinterpret_cast<uintptr_t>(kv.data_ptr()) % 16) return false;
  if (D == 128) {
    launch_tc<128>(out, q, kv, layer, bt, seq_lens, rows, splits, scale, window, ws);
    return true;
  }
  if (D == 64) {
    launch_tc<64>(out, q, kv, layer, bt, seq_lens, rows, splits, scale, window, ws);
    return true;
  }
  return false;
}

}  // namespace swift
