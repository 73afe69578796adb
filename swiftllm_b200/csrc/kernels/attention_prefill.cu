// Paged prefill attention: varlen causal attention of new query tokens against
// the paged KV pool (which already holds them), covering chunked prefill
// (queries start at seq_len - q_len), GQA and sliding windows.
//
// Replaces the reference's paged_attention_prefill stub
// (crates/swiftllm-cuda/src/bindings.rs:33-54).
//
// Tiling: CTA = (64-query tile, sequence, query head), 4 warps x 16 query
// rows; keys in 64-token tiles gathered page by page from the pool with
// cp.async (zero-fill past the end), double-buffered; S = Q K^T and O += P V
// on the tensor cores (mma.sync bf16, fp32 accumulate), online softmax in
// registers. Shared rows are padded by 16 bytes so ldmatrix is conflict-free
// for every supported head size.
#include "common.cuh"

namespace swift {

constexpr int kPfBM = 64, kPfBN = 64, kPfWarps = 4;

__device__ __forceinline__ void cp_async16(void* smem, const void* g, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem)), "l"(g),
               "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void ldsm_x4(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3,
                                        const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3,
                                          const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void mma_bf16(float d[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

template <int D>
__global__ void __launch_bounds__(kPfWarps * 32)
    paged_prefill_kernel(__nv_bfloat16* __restrict__ out, const __nv_bfloat16* __restrict__ q,
                         const __nv_bfloat16* __restrict__ kv, int64_t blk_stride,
                         int64_t layer_off, int64_t kv_stride, int block_size,
                         const int32_t* __restrict__ bt, int64_t bt_stride,
                         const int32_t* __restrict__ q_start, const int32_t* __restrict__ seq_lens,
                         int seq0, int Hq, int Hkv, float scale, int window,
                         const float* __restrict__ alibi) {
  constexpr int LD = D + 8;   // padded row (elements)
  constexpr int NKT = D / 16; // k-steps over head_dim
  constexpr int NDT = D / 8;  // n-tiles over head_dim
  constexpr int CH = D / 8;   // 16-byte chunks per row
  extern __shared__ __align__(128) uint8_t smem[];
  __nv_bfloat16* Qs = reinterpret_cast<__nv_bfloat16*>(smem);
  __nv_bfloat16* Ks = Qs + kPfBM * LD;      // [2][BN][LD]
  __nv_bfloat16* Vs = Ks + 2 * kPfBN * LD;  // [2][BN][LD]

  const int seq = seq0 + blockIdx.y, head = blockIdx.z, kvh = head / (Hq / Hkv);
  const int qs = q_start[seq], q_len = q_start[seq + 1] - qs;
  const int tile0 = blockIdx.x * kPfBM;
  if (tile0 >= q_len) return;
  const int L = seq_lens[seq];
  const int pos0 = L - q_len;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int32_t* mybt = bt + int64_t(seq) * bt_stride;
  const int64_t head_off = layer_off + int64_t(kvh) * block_size * D;

  for (int i = threadIdx.x; i < kPfBM * CH; i += blockDim.x) {
    int r = i / CH, c = i % CH;
    int t = tile0 + r;
    bool ok = t < q_len;
    const __nv_bfloat16* src = q + (int64_t(qs + (ok ? t : 0)) * Hq + head) * D + c * 8;
    cp_async16(Qs + r * LD + c * 8, src, ok);
  }
  auto load_kv = [&](int kb, int buf) {
    __nv_bfloat16* kd = Ks + buf * kPfBN * LD;
    __nv_bfloat16* vd = Vs + buf * kPfBN * LD;
    for (int i = threadIdx.x; i < kPfBN * CH; i += blockDim.x) {
      int r = i / CH, c = i % CH;
      int j = kb * kPfBN + r;
      bool ok = j < L;
      int jj = ok ? j : 0;
      int64_t blk = mybt[jj / block_size];
      const __nv_bfloat16* src = kv + blk * blk_stride + head_off + int64_t(jj % block_size) * D + c * 8;
      cp_async16(kd + r * LD + c * 8, src, ok);
      cp_async16(vd + r * LD + c * 8, src + kv_stride, ok);
    }
  };

  const int last_pos = pos0 + min(q_len, tile0 + kPfBM) - 1;
  const int kb_end = last_pos / kPfBN + 1;
  int kb_begin = 0;
  if (window > 0) kb_begin = max(0, pos0 + tile0 - window + 1) / kPfBN;
  load_kv(kb_begin, 0);
  cp_async_commit();

  const int rA = warp * 16 + (lane >> 2);
  const int qposA = pos0 + tile0 + rA, qposB = qposA + 8;
  const int warp_pos0 = pos0 + tile0 + warp * 16;
  float o[NDT][4];
#pragma unroll
  for (int i = 0; i < NDT; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float mA = -INFINITY, mB = -INFINITY, lA = 0.f, lB = 0.f;
  uint32_t qf[NKT][4];
  const float sl2 = scale * 1.4426950408889634f;  // exp(x) = exp2(x * log2 e)
  // ALiBi slope of this head in the exp2 domain (0: no bias)
  const float ab2 = alibi != nullptr ? alibi[head] * 1.4426950408889634f : 0.f;

  for (int kb = kb_begin; kb < kb_end; ++kb) {
    const int buf = (kb - kb_begin) & 1;
    if (kb + 1 < kb_end) {
      load_kv(kb + 1, buf ^ 1);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    if (kb == kb_begin) {
#pragma unroll
      for (int kk = 0; kk < NKT; ++kk) {
        const __nv_bfloat16* p = Qs + (warp * 16 + (lane & 15)) * LD + kk * 16 + (lane >> 4) * 8;
        ldsm_x4(qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3], p);
      }
    }
    const __nv_bfloat16* Kb = Ks + buf * kPfBN * LD;
    const __nv_bfloat16* Vb = Vs + buf * kPfBN * LD;
    float s[kPfBN / 8][4];
#pragma unroll
    for (int n = 0; n < kPfBN / 8; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll
    for (int n = 0; n < kPfBN / 8; ++n) {
#pragma unroll
      for (int kk = 0; kk < NKT; kk += 2) {
        uint32_t b0, b1, b2, b3;
        if (kk + 1 < NKT) {
          const __nv_bfloat16* p = Kb + (n * 8 + (lane & 7)) * LD + kk * 16 + (lane >> 3) * 8;
          ldsm_x4(b0, b1, b2, b3, p);
          mma_bf16(s[n], qf[kk], b0, b1);
          mma_bf16(s[n], qf[kk + 1], b2, b3);
        } else {
          const __nv_bfloat16* p = Kb + (n * 8 + (lane & 7)) * LD + kk * 16 + ((lane >> 3) & 1) * 8;
          ldsm_x4(b0, b1, b2, b3, p);
          mma_bf16(s[n], qf[kk], b0, b1);
        }
      }
    }
    float mxA = mA, mxB = mB;
    const bool need_mask = (kb + 1) * kPfBN - 1 > warp_pos0 || window > 0 || (kb + 1) * kPfBN > L;
#pragma unroll
    for (int n = 0; n < kPfBN / 8; ++n) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        int key = kb * kPfBN + n * 8 + (lane & 3) * 2 + (e & 1);
        int qp = e < 2 ? qposA : qposB;
        float v = s[n][e] * sl2 + ab2 * float(key - qp);
        if (need_mask) {
          bool bad = key > qp || key >= L || (window > 0 && key <= qp - window);
          v = bad ? -INFINITY : v;
        }
        s[n][e] = v;
      }
      mxA = fmaxf(mxA, fmaxf(s[n][0], s[n][1]));
      mxB = fmaxf(mxB, fmaxf(s[n][2], s[n][3]));
    }
    mxA = fmaxf(mxA, __shfl_xor_sync(0xffffffffu, mxA, 1));
    mxA = fmaxf(mxA, __shfl_xor_sync(0xffffffffu, mxA, 2));
    mxB = fmaxf(mxB, __shfl_xor_sync(0xffffffffu, mxB, 1));
    mxB = fmaxf(mxB, __shfl_xor_sync(0xffffffffu, mxB, 2));
    const float cA = mxA == -INFINITY ? 1.f : exp2f(mA - mxA);
    const float cB = mxB == -INFINITY ? 1.f : exp2f(mB - mxB);
    mA = mxA;
    mB = mxB;
    float sumA = 0.f, sumB = 0.f;
#pragma unroll
    for (int n = 0; n < kPfBN / 8; ++n) {
      s[n][0] = mxA == -INFINITY ? 0.f : exp2f(s[n][0] - mxA);
      s[n][1] = mxA == -INFINITY ? 0.f : exp2f(s[n][1] - mxA);
      s[n][2] = mxB == -INFINITY ? 0.f : exp2f(s[n][2] - mxB);
      s[n][3] = mxB == -INFINITY ? 0.f : exp2f(s[n][3] - mxB);
      sumA += s[n][0] + s[n][1];
      sumB += s[n][2] + s[n][3];
    }
    lA = lA * cA + sumA;
    lB = lB * cB + sumB;
#pragma unroll
    for (int i = 0; i < NDT; ++i) {
      o[i][0] *= cA;
      o[i][1] *= cA;
      o[i][2] *= cB;
      o[i][3] *= cB;
    }
#pragma unroll
    for (int kk = 0; kk < kPfBN / 16; ++kk) {
      uint32_t a[4];
      a[0] = pack_bf16(s[2 * kk][0], s[2 * kk][1]);
      a[1] = pack_bf16(s[2 * kk][2], s[2 * kk][3]);
      a[2] = pack_bf16(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      a[3] = pack_bf16(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int n = 0; n < NDT; n += 2) {
        uint32_t b0, b1, b2, b3;
        const __nv_bfloat16* p = Vb + (kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8) * LD + n * 8 +
                                 (lane >> 4) * 8;
        ldsm_x4_t(b0, b1, b2, b3, p);
        mma_bf16(o[n], a, b0, b1);
        mma_bf16(o[n + 1], a, b2, b3);
      }
    }
    __syncthreads();
  }
  lA += __shfl_xor_sync(0xffffffffu, lA, 1);
  lA += __shfl_xor_sync(0xffffffffu, lA, 2);
  lB += __shfl_xor_sync(0xffffffffu, lB, 1);
  lB += __shfl_xor_sync(0xffffffffu, lB, 2);
  const float iA = lA > 0.f ? 1.f / lA : 0.f, iB = lB > 0.f ? 1.f / lB : 0.f;
  const int tA = tile0 + rA, tB = tA + 8;
#pragma unroll
  for (int n = 0; n < NDT; ++n) {
    int col = n * 8 + (lane & 3) * 2;
    if (tA < q_len)
      *reinterpret_cast<__nv_bfloat162*>(out + (int64_t(qs + tA) * Hq + head) * D + col) =
          __floats2bfloat162_rn(o[n][0] * iA, o[n][1] * iA);
    if (tB < q_len)
      *reinterpret_cast<__nv_bfloat162*>(out + (int64_t(qs + tB) * Hq + head) * D + col) =
          __floats2bfloat162_rn(o[n][2] * iB, o[n][3] * iB);
  }
}

template <int D>
static void launch_prefill(torch::Tensor out, torch::Tensor q, torch::Tensor kv, int64_t layer,
                           torch::Tensor bt, torch::Tensor q_start, torch::Tensor seq_lens,
                           int seq0, int seq1, int max_q_len, double scale, int window,
                           const float* alibi) {
  static_assert((D / 8) % 2 == 0, "head_dim/8 must be even");
  constexpr int LD = D + 8;
  const size_t smem = size_t(kPfBM + 4 * kPfBN) * LD * 2;
  auto kern = paged_prefill_kernel<D>;
  static bool attr[64] = {false};
  int dev;
  cudaGetDevice(&dev);
  if (!attr[dev]) {
    SWIFT_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          static_cast<int>(smem)));
    attr[dev] = true;
  }
  const int Hq = static_cast<int>(q.size(1)), Hkv = static_cast<int>(kv.size(3));
  dim3 grid((max_q_len + kPfBM - 1) / kPfBM, seq1 - seq0, Hq);
  kern<<<grid, kPfWarps * 32, smem, cur_stream()>>>(
      reinterpret_cast<__nv_bfloat16*>(out.data_ptr<at::BFloat16>()),
      reinterpret_cast<const __nv_bfloat16*>(q.data_ptr<at::BFloat16>()),
      reinterpret_cast<const __nv_bfloat16*>(kv.data_ptr<at::BFloat16>()), kv.stride(0),
      layer * kv.stride(1), kv.stride(2), static_cast<int>(kv.size(4)), bt.data_ptr<int32_t>(),
      bt.stride(0), q_start.data_ptr<int32_t>(), seq_lens.data_ptr<int32_t>(), seq0, Hq, Hkv,
      static_cast<float>(scale), window, alibi);
  SWIFT_CHECK_LAUNCH();
}

bool paged_prefill_tc_supported(int D, int block_size, int Hq, int Hkv);
void paged_prefill_tc(torch::Tensor out, torch::Tensor q, torch::Tensor kv, int64_t layer,
                      torch::Tensor bt, torch::Tensor q_start, torch::Tensor seq_lens, int seq0,
                      int seq1, int max_q_len, double scale, int window);

// impl: -1 the tcgen05 kernel (attention_prefill_tc.cu) where it applies
// (head_dim 128, 16-token pages), else this one; 0 this one; 1 tcgen05.
// alibi: optional fp32 [Hq] ALiBi slopes (this kernel only).
void paged_prefill(torch::Tensor out, torch::Tensor q, torch::Tensor kv, int64_t layer,
                   torch::Tensor bt, torch::Tensor q_start, torch::Tensor seq_lens, int64_t seq0,
                   int64_t seq1, int64_t max_q_len, double scale, int64_t window, int64_t impl,
                   c10::optional<torch::Tensor> alibi) {
  CHECK_BF16(q);
  CHECK_BF16(kv);
  CHECK_CONTIG(kv);
  TORCH_CHECK(q.is_contiguous() && out.is_contiguous());
  if (seq1 <= seq0 || max_q_len <= 0) return;
  const int D = static_cast<int>(q.size(2));
  const int w = static_cast<int>(window);
  const int a = static_cast<int>(seq0), b = static_cast<int>(seq1), mq = static_cast<int>(max_q_len);
  const bool tc_ok = paged_prefill_tc_supported(D, static_cast<int>(kv.size(4)),
                                                static_cast<int>(q.size(1)), static_cast<int>(kv.size(3)));
  const float* ap = nullptr;
  if (alibi.has_value()) {
    TORCH_CHECK(alibi->scalar_type() == at::kFloat && alibi->is_contiguous() &&
                    alibi->numel() == q.size(1) && alibi->is_cuda(),
                "paged_prefill: alibi slopes must be fp32 [num_heads] on the device");
    TORCH_CHECK(impl != 1, "paged_prefill: the tcgen05 kernel has no ALiBi bias");
    ap = alibi->data_ptr<float>();
  }
  TORCH_CHECK(impl != 1 || tc_ok, "paged_prefill: the tcgen05 kernel needs head_dim 128 and 16-token pages");
  if (impl != 0 && tc_ok && ap == nullptr) {
    paged_prefill_tc(out, q, kv, layer, bt, q_start, seq_lens, a, b, mq, scale, w);
    return;
  }
  switch (D) {
    case 64: launch_prefill<64>(out, q, kv, layer, bt, q_start, seq_lens, a, b, mq, scale, w, ap); break;
    case 80: launch_prefill<80>(out, q, kv, layer, bt, q_start, seq_lens, a, b, mq, scale, w, ap); break;
    case 96: launch_prefill<96>(out, q, kv, layer, bt, q_start, seq_lens, a, b, mq, scale, w, ap); break;
    case 128: launch_prefill<128>(out, q, kv, layer, bt, q_start, seq_lens, a, b, mq, scale, w, ap); break;
    default: TORCH_CHECK(false, "paged_prefill: unsupported head_dim ", D);
  }
}

}  // namespace swift
