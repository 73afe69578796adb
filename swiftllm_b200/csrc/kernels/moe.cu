// MoE routing: softmax over experts, top-k, renormalised weights, and the
// token permutation that groups rows by (local) expert.
//
// The reference's MoeMlp returns zeros (crates/swiftllm-models/src/layers/
// mlp.rs:207-258) and create_model rejects Mixtral (architectures/mod.rs:68-76).
//
// moe_route_kernel: one warp per token, E <= 64 experts, k <= 8.
// moe_permute: one CTA counts rows per local expert, scans, and orders the
//   (token, slot) pairs expert-contiguously (warp match + per-warp scan) so
//   every expert's rows form one dense block for the grouped tcgen05 GEMM.
//   Deterministic: rows keep token order inside an expert.
// moe_gather: the expert-ordered activation rows the grouped GEMM reads.
// moe_combine: weighted sum of a token's expert outputs in slot order.
#include <algorithm>

#include "common.cuh"

namespace swift {

__global__ void moe_route_kernel(const float* __restrict__ logits, int T, int E, int k,
                                 bool renorm, float* __restrict__ w_out, int32_t* __restrict__ id_out) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= T) return;
  const float* row = logits + int64_t(warp) * E;
  float v0 = lane < E ? row[lane] : -INFINITY;
  float v1 = lane + 32 < E ? row[lane + 32] : -INFINITY;
  float mx = warp_max(fmaxf(v0, v1));
  float e0 = lane < E ? __expf(v0 - mx) : 0.f, e1 = lane + 32 < E ? __expf(v1 - mx) : 0.f;
  const float z = warp_sum(e0 + e1);
  float p0 = e0 / z, p1 = e1 / z;
  float wsum = 0.f;
  float sel_w[8];
  int sel_i[8];
  for (int j = 0; j < k; ++j) {
    // arg-max over the remaining probabilities (ties: lower index)
    float bv = p0;
    int bi = lane < E ? lane : 1 << 20;
    if (p1 > bv || (p1 == bv && lane + 32 < E && lane + 32 < bi)) {
      bv = p1;
      bi = lane + 32 < E ? lane + 32 : bi;
    }
    for (int o = 16; o > 0; o >>= 1) {
      float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
    sel_w[j] = bv;
    sel_i[j] = bi;
    wsum += bv;
    if (bi == lane) p0 = -1.f;
    if (bi == lane + 32) p1 = -1.f;
  }
  if (lane == 0) {
    for (int j = 0; j < k; ++j) {
      w_out[int64_t(warp) * k + j] = renorm ? sel_w[j] / wsum : sel_w[j];
      id_out[int64_t(warp) * k + j] = sel_i[j];
    }
  }
}

// ids [T, k] global expert ids; local experts are [e0, e0 + E_local).
// Outputs: offsets [E_local + 1] (rows per local expert, exclusive scan),
// perm_token [T*k] (token of each expert-ordered row, rows past the total
// stay 0) and inv_slot [T*k] (row of each (token, slot), -1 if the expert is
// not local).
// One CTA of 1024 threads. Pass 1 counts rows per expert (shared atomics).
// Pass 2 walks the (token, slot) list in chunks of 1024: inside a warp,
// __match_any_sync groups lanes of the same expert and ranks them; a scan
// over the 32 warps' per-expert counts (one thread per expert) turns them
// into positions. Rows keep (token, slot) order inside an expert, so the
// result is deterministic.
constexpr int kPermThreads = 1024;
__global__ void __launch_bounds__(kPermThreads)
    moe_permute_kernel(const int32_t* __restrict__ ids, int T, int k, int e0, int E_local,
                       int32_t* __restrict__ offsets, int32_t* __restrict__ perm_token,
                       int32_t* __restrict__ inv_slot) {
  __shared__ int cnt[64];
  __shared__ int base[64];
  __shared__ int wcnt[32][64];  // per warp, per expert: count, then first position
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n = T * k;
  for (int e = tid; e < 64; e += blockDim.x) cnt[e] = 0;
  for (int j = tid; j < 32 * 64; j += blockDim.x) (&wcnt[0][0])[j] = 0;
  for (int i = tid; i < n; i += blockDim.x) perm_token[i] = 0;
  __syncthreads();
  for (int i = tid; i < n; i += blockDim.x) {
    const int e = ids[i] - e0;
    if (e >= 0 && e < E_local) atomicAdd(&cnt[e], 1);
  }
  __syncthreads();
  if (tid == 0) {
    int acc = 0;
    for (int e = 0; e < E_local; ++e) {
      offsets[e] = acc;
      base[e] = acc;
      acc += cnt[e];
    }
    offsets[E_local] = acc;
  }
  __syncthreads();
  const unsigned lt = (1u << lane) - 1u;
  for (int c0 = 0; c0 < n; c0 += blockDim.x) {
    const int i = c0 + tid;
    int e = i < n ? ids[i] - e0 : -1;
    const bool local = e >= 0 && e < E_local;
    if (!local) e = -1;
    const unsigned same = __match_any_sync(0xffffffffu, e);
    const int rk = __popc(same & lt);
    if (local && rk == 0) wcnt[warp][e] = __popc(same);
    __syncthreads();
    if (tid < E_local) {
      int run = base[tid];
      for (int w = 0; w < 32; ++w) {
        const int c = wcnt[w][tid];
        wcnt[w][tid] = run;
        run += c;
      }
      base[tid] = run;
    }
    __syncthreads();
    if (i < n) {
      if (local) {
        const int pos = wcnt[warp][e] + rk;
        perm_token[pos] = i / k;
        inv_slot[i] = pos;
      } else {
        inv_slot[i] = -1;
      }
    }
    __syncthreads();
    for (int j = tid; j < 32 * 64; j += blockDim.x) (&wcnt[0][0])[j] = 0;
    __syncthreads();
  }
}

// xg[r] = x[perm_token[r]] for every expert-ordered row r < rows (16-byte
// vectors; replaces a framework index_select before the grouped GEMM).
__global__ void moe_gather_kernel(__nv_bfloat16* __restrict__ xg, const __nv_bfloat16* __restrict__ x,
                                  const int32_t* __restrict__ perm, int rows, int H, int64_t ldx) {
  const int vec = H / 8;
  const int64_t total = int64_t(rows) * vec;
  for (int64_t j = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; j < total;
       j += int64_t(gridDim.x) * blockDim.x) {
    const int r = static_cast<int>(j / vec), c = static_cast<int>(j % vec);
    const uint4 v = reinterpret_cast<const uint4*>(x + int64_t(perm[r]) * ldx)[c];
    reinterpret_cast<uint4*>(xg + int64_t(r) * H)[c] = v;
  }
}

// out[t] = sum_j w[t, j] * y[inv_slot[t*k + j]] over local slots, fixed order
// (deterministic), fp32 accumulate, bf16 store. One CTA per token.
__global__ void moe_combine_kernel(__nv_bfloat16* __restrict__ out, const __nv_bfloat16* __restrict__ y,
                                   const float* __restrict__ w, const int32_t* __restrict__ inv,
                                   int k, int H) {
  const int t = blockIdx.x;
  for (int c = threadIdx.x * 8; c < H; c += blockDim.x * 8) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int j = 0; j < k; ++j) {
      const int r = inv[t * k + j];
      if (r < 0) continue;
      const float wj = w[t * k + j];
      float v[8];
      load8(y + int64_t(r) * H + c, v);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] += wj * v[e];
    }
    store8(out + int64_t(t) * H + c, acc);
  }
}

void moe_route(torch::Tensor logits, int64_t k, bool renorm, torch::Tensor w_out,
               torch::Tensor id_out) {
  TORCH_CHECK(logits.scalar_type() == at::kFloat && logits.is_contiguous());
  const int T = static_cast<int>(logits.size(0)), E = static_cast<int>(logits.size(1));
  TORCH_CHECK(E <= 64 && k >= 1 && k <= 8 && k <= E, "moe_route: E <= 64, 1 <= k <= 8");
  if (!T) return;
  const int threads = 256, warps = threads / 32;
  moe_route_kernel<<<(T + warps - 1) / warps, threads, 0, cur_stream()>>>(
      logits.data_ptr<float>(), T, E, static_cast<int>(k), renorm, w_out.data_ptr<float>(),
      id_out.data_ptr<int32_t>());
  SWIFT_CHECK_LAUNCH();
}

void moe_permute(torch::Tensor ids, int64_t e0, int64_t E_local, torch::Tensor offsets,
                 torch::Tensor perm_token, torch::Tensor inv_slot) {
  TORCH_CHECK(ids.scalar_type() == at::kInt && ids.is_contiguous());
  TORCH_CHECK(E_local >= 1 && E_local <= 64, "moe_permute: 1 <= local experts <= 64");
  const int T = static_cast<int>(ids.size(0)), k = static_cast<int>(ids.size(1));
  if (T * k == 0) return;
  moe_permute_kernel<<<1, kPermThreads, 0, cur_stream()>>>(
      ids.data_ptr<int32_t>(), T, k, static_cast<int>(e0), static_cast<int>(E_local),
      offsets.data_ptr<int32_t>(), perm_token.data_ptr<int32_t>(), inv_slot.data_ptr<int32_t>());
  SWIFT_CHECK_LAUNCH();
}

void moe_gather(torch::Tensor xg, torch::Tensor x, torch::Tensor perm_token) {
  CHECK_BF16(xg);
  CHECK_BF16(x);
  TORCH_CHECK(perm_token.scalar_type() == at::kInt && perm_token.is_contiguous());
  const int rows = static_cast<int>(perm_token.numel()), H = static_cast<int>(x.size(1));
  TORCH_CHECK(xg.is_contiguous() && xg.size(0) >= rows && xg.size(1) == H && H % 8 == 0);
  TORCH_CHECK(x.stride(1) == 1 && x.stride(0) % 8 == 0 &&
              reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0, "moe_gather: 16-byte rows");
  if (!rows) return;
  const int64_t vecs = int64_t(rows) * (H / 8);
  const int blocks = static_cast<int>(std::min<int64_t>((vecs + 255) / 256, 148 * 16));
  moe_gather_kernel<<<blocks, 256, 0, cur_stream()>>>(
      reinterpret_cast<__nv_bfloat16*>(xg.data_ptr<at::BFloat16>()),
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr<at::BFloat16>()),
      perm_token.data_ptr<int32_t>(), rows, H, x.stride(0));
  SWIFT_CHECK_LAUNCH();
}

void moe_combine(torch::Tensor out, torch::Tensor y, torch::Tensor weights, torch::Tensor inv_slot) {
  CHECK_BF16(out);
  CHECK_BF16(y);
  const int T = static_cast<int>(out.size(0)), H = static_cast<int>(out.size(1));
  const int k = static_cast<int>(weights.size(1));
  TORCH_CHECK(H % 8 == 0 && out.is_contiguous() && y.is_contiguous());
  if (!T) return;
  moe_combine_kernel<<<T, 128, 0, cur_stream()>>>(
      reinterpret_cast<__nv_bfloat16*>(out.data_ptr<at::BFloat16>()),
      reinterpret_cast<const __nv_bfloat16*>(y.data_ptr<at::BFloat16>()), weights.data_ptr<float>(),
      inv_slot.data_ptr<int32_t>(), k, H);
  SWIFT_CHECK_LAUNCH();
}

}  // namespace swift
