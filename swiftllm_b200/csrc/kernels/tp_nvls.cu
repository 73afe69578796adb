// Sequence-parallel tensor-parallel reduction with the residual add, the
// following norm and the all-gather fused in one kernel, over NVSwitch
// multicast (NVLS `multimem`) or, where the driver offers no multicast
// object, plain NVLink peer loads / stores.
//
// The reference declares all_reduce / reduce_scatter / all_gather and
// returns NotImplemented (crates/swiftllm-core/src/execution/
// tensor_parallel.rs:115-141); its RowParallelLinear would all-reduce
// (crates/swiftllm-models/src/layers/mod.rs:145-149).
//
// Row-parallel GEMMs (o_proj, down_proj) store their partial [T, H] output
// in this rank's `in` buffer of the symmetric allocation (local stores).
// Token rows are owned by ranks in contiguous shards: rank j owns
// [T*j/k, T*(j+1)/k). This kernel, per owned row:
//   1. sums the k partials: one `multimem.ld_reduce ... .acc::f32` per
//      16-byte vector through the switch (or k peer loads, fp32, rank order);
//   2. adds the row of the residual stream, which each rank keeps only for
//      its own token shard (rounded to bf16 like an unfused add);
//   3. RMS-normalises it with the next sub-block's weight (optional);
//   4. stores the normalised row into EVERY rank's `out` buffer with one
//      `multimem.st` (or k peer stores): the all-gather of the next GEMM's
//      input, so the next QKV / gate_up GEMM reads it locally.
// Ordering: block b of every rank handles the same rows, so each block only
// synchronises with block b of its peers, on a per-block u32 counter in the
// symmetric allocation that every arrival increments on every rank
// (`multimem.red.add`, or one `red.add` per peer): arrival 1 after the
// previous kernel (the GEMM) finished on this rank, arrival 2 after this
// block's stores; a block waits until the counter reaches k * arrivals so
// far. The counters only grow (the target is kept per block in local device
// memory), so CUDA-graph replays need no reset. Every wait is bounded by a
// %globaltimer deadline; on expiry the block records kErrPeerTimeout and
// returns (the host raises CommTimeoutError).
//
// Buffer reuse needs no double buffering: a rank's next GEMM writes `in`
// only after this kernel completed on that rank, i.e. after every block
// passed arrival 2, which every rank makes only after reading `in`; `out` is
// written only after arrival 1, which a rank makes only after its consumer
// of the previous `out` (the GEMM before this kernel) has finished.
#include <algorithm>

#include "common.cuh"

namespace swift {

constexpr int kRnMaxRanks = 8;
constexpr int kRnBlocks = 128;
constexpr int kRnThreads = 512;
constexpr int kRnMaxVecs = 4;  // 16-byte vectors per thread per row: H <= 4*8*512

struct RnPeers {
  uint64_t base[kRnMaxRanks];  // byte address of each rank's symmetric allocation
  uint64_t mc;                 // multicast address of the allocation (0: none)
};

__device__ __forceinline__ uint64_t rn_now() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ uint32_t rn_ld_acquire(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void rn_red_release(uint32_t* p, uint32_t v) {
  asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void mc_red_release(uint64_t mc_addr, uint32_t v) {
  asm volatile("multimem.red.release.sys.global.add.u32 [%0], %1;" ::"l"(mc_addr), "r"(v)
               : "memory");
}
// Sum over all ranks of the 8 bf16 at this multicast address, fp32 accumulate.
__device__ __forceinline__ uint4 mc_ld_reduce_bf16x8(uint64_t mc_addr) {
  uint4 r;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(mc_addr)
               : "memory");
  return r;
}
__device__ __forceinline__ void mc_st_bf16x8(uint64_t mc_addr, uint4 v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.bf16x2 [%0], {%1,%2,%3,%4};" ::"l"(mc_addr),
               "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

__device__ __forceinline__ void mc_st_f32x4(uint64_t mc_addr, float4 v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(mc_addr),
               "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w)
               : "memory");
}

__device__ __forceinline__ void unpack8(uint4 x, float f[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&x);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float2 t = __bfloat1622float2(h[j]);
    f[2 * j] = t.x;
    f[2 * j + 1] = t.y;
  }
}
__device__ __forceinline__ uint4 pack8(const float f[8]) {
  uint4 x;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&x);
#pragma unroll
  for (int j = 0; j < 4; ++j) h[j] = __floats2bfloat162_rn(f[2 * j], f[2 * j + 1]);
  return x;
}

// Cross-rank barrier of block b (thread 0 arrives and waits; the block then
// syncs). Returns false on timeout.
template <bool MC>
__device__ __forceinline__ bool rn_barrier(const RnPeers& P, int rank, int k, int64_t ctr_off,
                                           uint32_t target, int64_t timeout_ns, int* status,
                                           int where) {
  __shared__ int ok;
  __syncthreads();
  if (threadIdx.x == 0) {
    ok = 1;
    // no separate fence: the block's stores are ordered before thread 0 by
    // the barrier above, and the release of the arrival is cumulative over
    // them (release at system scope covers the peers' view of them)
    const int64_t off = ctr_off + int64_t(blockIdx.x) * 4;
    if constexpr (MC) {
      mc_red_release(P.mc + off, 1u);
    } else {
      for (int p = 0; p < k; ++p) rn_red_release(reinterpret_cast<uint32_t*>(P.base[p] + off), 1u);
    }
    const uint32_t* mine = reinterpret_cast<const uint32_t*>(P.base[rank] + off);
    const uint64_t deadline = rn_now() + static_cast<uint64_t>(timeout_ns);
    while (static_cast<int32_t>(rn_ld_acquire(mine) - target) < 0) {
      if (rn_now() > deadline) {
        set_status(status, kErrPeerTimeout, where);
        ok = 0;
        break;
      }
    }
  }
  __syncthreads();
  return ok != 0;
}

// residual == nullptr: out = plain sum (an all-reduce). w == nullptr: no
// norm (out = the new residual row). layer_norm: w/b LayerNorm instead of RMS.
template <bool MC>
__global__ void __launch_bounds__(kRnThreads)
    tp_reduce_norm_kernel(RnPeers P, int rank, int k, int64_t in_off, int64_t out_off,
                          int64_t ctr_off, __nv_bfloat16* __restrict__ residual,
                          const __nv_bfloat16* __restrict__ w, float eps, int T, int H,
                          uint32_t* __restrict__ epochs, int64_t timeout_ns, int* status) {
  pdl_wait();  // previous kernel done (programmatic dependent launch)
  pdl_trigger();
  __shared__ float red[33];
  const uint32_t e = epochs[blockIdx.x];
  if (!rn_barrier<MC>(P, rank, k, ctr_off, (2 * e + 1) * uint32_t(k), timeout_ns, status, 230))
    return;
  const int lo = static_cast<int>(int64_t(T) * rank / k);
  const int hi = static_cast<int>(int64_t(T) * (rank + 1) / k);
  const int hv = H / 8;
  for (int row = lo + blockIdx.x; row < hi; row += gridDim.x) {
    float v[kRnMaxVecs][8];
    float s2 = 0.f;
    const int64_t rbase = int64_t(row) * hv;
#pragma unroll
    for (int j = 0; j < kRnMaxVecs; ++j) {
      const int col = threadIdx.x + j * kRnThreads;
      if (col >= hv) continue;
      const int64_t byte = (rbase + col) * 16;
      float acc[8];
      if constexpr (MC) {
        unpack8(mc_ld_reduce_bf16x8(P.mc + in_off + byte), acc);
      } else {
#pragma unroll
        for (int e2 = 0; e2 < 8; ++e2) acc[e2] = 0.f;
        for (int r = 0; r < k; ++r) {
          float f[8];
          unpack8(__ldcg(reinterpret_cast<const uint4*>(P.base[r] + in_off + byte)), f);
#pragma unroll
          for (int e2 = 0; e2 < 8; ++e2) acc[e2] += f[e2];
        }
      }
      if (residual != nullptr) {
        float rr[8];
        uint4* rp = reinterpret_cast<uint4*>(residual) + rbase + col;
        unpack8(*rp, rr);
#pragma unroll
        for (int e2 = 0; e2 < 8; ++e2) {
          const float sum = __bfloat162float(__float2bfloat16(acc[e2]));
          v[j][e2] = __bfloat162float(__float2bfloat16(sum + rr[e2]));
          s2 += v[j][e2] * v[j][e2];
        }
        *rp = pack8(v[j]);
      } else {
#pragma unroll
        for (int e2 = 0; e2 < 8; ++e2) v[j][e2] = acc[e2];
      }
    }
    float scale = 1.f;
    if (w != nullptr) scale = rsqrtf(block_sum(s2, red) / H + eps);
#pragma unroll
    for (int j = 0; j < kRnMaxVecs; ++j) {
      const int col = threadIdx.x + j * kRnThreads;
      if (col >= hv) continue;
      float o[8];
      if (w != nullptr) {
        float wf[8];
        load8(w + col * 8, wf);
#pragma unroll
        for (int e2 = 0; e2 < 8; ++e2) o[e2] = v[j][e2] * scale * wf[e2];
      } else {
#pragma unroll
        for (int e2 = 0; e2 < 8; ++e2) o[e2] = v[j][e2];
      }
      const uint4 ov = pack8(o);
      const int64_t byte = (rbase + col) * 16;
      if constexpr (MC) {
        mc_st_bf16x8(P.mc + out_off + byte, ov);
      } else {
        for (int p = 0; p < k; ++p) {
          const int q = (rank + p) % k;  // stagger destinations across ranks
          *reinterpret_cast<uint4*>(P.base[q] + out_off + byte) = ov;
        }
      }
    }
  }
  if (!rn_barrier<MC>(P, rank, k, ctr_off, (2 * e + 2) * uint32_t(k), timeout_ns, status, 231))
    return;
  if (threadIdx.x == 0) epochs[blockIdx.x] = e + 1;
}

static RnPeers rn_peers(const std::vector<int64_t>& bases, int64_t mc) {
  const int k = static_cast<int>(bases.size());
  TORCH_CHECK(k >= 2 && k <= kRnMaxRanks, "tp_reduce_norm: 2..8 ranks");
  RnPeers P;
  for (int r = 0; r < kRnMaxRanks; ++r) P.base[r] = r < k ? static_cast<uint64_t>(bases[r]) : 0;
  P.mc = static_cast<uint64_t>(mc);
  return P;
}

// bases: byte addresses of every rank's symmetric allocation; mc: its
// multicast address or 0; in_off / out_off: byte offsets of the [T, H] bf16
// partial and output buffers; ctr_off: byte offset of kRnBlocks u32
// counters; residual: local [>= T, H] bf16 (own shard rows read and
// updated) or None; w: norm weight [H] or None; epochs: int32 [kRnBlocks]
// local. Returns the number of kernels launched.
int64_t tp_reduce_norm(std::vector<int64_t> bases, int64_t mc, int64_t rank, int64_t in_off,
                       int64_t out_off, int64_t ctr_off, c10::optional<torch::Tensor> residual,
                       c10::optional<torch::Tensor> w, double eps, int64_t T, int64_t H,
                       torch::Tensor epochs, double timeout_s) {
  const RnPeers P = rn_peers(bases, mc);
  const int k = static_cast<int>(bases.size());
  TORCH_CHECK(H % 8 == 0 && H <= kRnMaxVecs * 8 * kRnThreads, "tp_reduce_norm: H");
  TORCH_CHECK(in_off % 16 == 0 && out_off % 16 == 0 && ctr_off % 4 == 0);
  TORCH_CHECK(epochs.scalar_type() == at::kInt && epochs.numel() >= kRnBlocks && epochs.is_cuda());
  __nv_bfloat16* rp = nullptr;
  if (residual.has_value()) {
    CHECK_BF16(residual.value());
    TORCH_CHECK(residual->is_contiguous() && residual->numel() >= T * H);
    TORCH_CHECK(reinterpret_cast<uintptr_t>(residual->data_ptr()) % 16 == 0);
    rp = reinterpret_cast<__nv_bfloat16*>(residual->data_ptr<at::BFloat16>());
  }
  const __nv_bfloat16* wp = nullptr;
  if (w.has_value()) {
    CHECK_BF16(w.value());
    TORCH_CHECK(w->numel() == H && w->is_contiguous());
    wp = reinterpret_cast<const __nv_bfloat16*>(w->data_ptr<at::BFloat16>());
  }
  const int64_t tns = static_cast<int64_t>(timeout_s * 1e9);
  auto ep = reinterpret_cast<uint32_t*>(epochs.data_ptr<int32_t>());
  // one block per owned row up to kRnBlocks: a block takes part in both
  // cross-rank barriers whether or not it owns rows, so idle blocks only add
  // arrivals. Every rank computes the same grid from (T, k), and block b's
  // counter and epoch advance only when block b runs, on every rank alike.
  const int blocks = static_cast<int>(std::min<int64_t>(kRnBlocks, std::max<int64_t>(1, (T + k - 1) / k)));
  if (P.mc)
    launch_pdl(tp_reduce_norm_kernel<true>, dim3(blocks), dim3(kRnThreads), 0, cur_stream(), 
        P, static_cast<int>(rank), k, in_off, out_off, ctr_off, rp, wp, static_cast<float>(eps),
        static_cast<int>(T), static_cast<int>(H), ep, tns, status_word_ptr());
  else
    launch_pdl(tp_reduce_norm_kernel<false>, dim3(blocks), dim3(kRnThreads), 0, cur_stream(), 
        P, static_cast<int>(rank), k, in_off, out_off, ctr_off, rp, wp, static_cast<float>(eps),
        static_cast<int>(T), static_cast<int>(H), ep, tns, status_word_ptr());
  SWIFT_CHECK_LAUNCH();
  return 1;
}

// ---- vocab-parallel greedy sampling
// Each rank holds the logits of its vocabulary slice [v0, v0 + V). Block r
// reduces row r to (max, first index of the max, sum exp(l - max)), stores
// that candidate into slot [rank][r] of every rank's candidate buffer
// (multimem.st or peer stores), meets block r of its peers on the same
// counter scheme as above, and merges the k candidates in rank order: the
// token is the first index of the global max (what a full-vocabulary argmax
// returns) and its log-probability is -log(sum_r z_r exp(m_r - M)).
constexpr int kVaThreads = 256;

template <bool MC>
__global__ void __launch_bounds__(kVaThreads)
    tp_vocab_argmax_kernel(RnPeers P, int rank, int k, const float* __restrict__ logits,
                           int64_t ld, int V, int v0, int rows, int64_t cand_off, int64_t ctr_off,
                           int32_t* __restrict__ tokens, float* __restrict__ lps,
                           uint32_t* __restrict__ epochs, int64_t timeout_ns, int* status) {
  pdl_wait();  // previous kernel done (programmatic dependent launch)
  pdl_trigger();
  __shared__ float sm[32];
  __shared__ int si[32];
  __shared__ float red[33];
  const int r = blockIdx.x;
  const uint32_t e = epochs[r];
  const float* row = logits + int64_t(r) * ld;
  float m = -INFINITY;
  int mi = 0x7fffffff;
  for (int i = threadIdx.x; i < V; i += kVaThreads) {
    const float x = row[i];
    if (x > m) {  // ascending i per thread: the first max wins ties
      m = x;
      mi = i;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float om = __shfl_xor_sync(0xffffffffu, m, o);
    const int oi = __shfl_xor_sync(0xffffffffu, mi, o);
    if (om > m || (om == m && oi < mi)) {
      m = om;
      mi = oi;
    }
  }
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  if (lane == 0) {
    sm[wid] = m;
    si[wid] = mi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int q = 1; q < kVaThreads / 32; ++q)
      if (sm[q] > sm[0] || (sm[q] == sm[0] && si[q] < si[0])) {
        sm[0] = sm[q];
        si[0] = si[q];
      }
  }
  __syncthreads();
  const float mx = sm[0];
  const int arg = si[0];
  float z = 0.f;
  for (int i = threadIdx.x; i < V; i += kVaThreads) z += __expf(row[i] - mx);
  z = block_sum(z, red);
  if (threadIdx.x == 0) {
    // the vocabulary index travels as an exactly representable float
    const float4 c = make_float4(mx, static_cast<float>(arg + v0), z, 0.f);
    const int64_t byte = cand_off + (int64_t(rank) * rows + r) * 16;
    if constexpr (MC) {
      mc_st_f32x4(P.mc + byte, c);
    } else {
      for (int p = 0; p < k; ++p) *reinterpret_cast<float4*>(P.base[p] + byte) = c;
    }
  }
  if (!rn_barrier<MC>(P, rank, k, ctr_off, (e + 1) * uint32_t(k), timeout_ns, status, 240)) return;
  if (threadIdx.x == 0) {
    float M = -INFINITY;
    int tok = 0;
    float4 c[kRnMaxRanks];
    for (int p = 0; p < k; ++p) {
      c[p] = __ldcg(reinterpret_cast<const float4*>(P.base[rank] + cand_off) + int64_t(p) * rows + r);
      if (c[p].x > M) {  // ranks hold ascending vocabulary slices: first max wins
        M = c[p].x;
        tok = static_cast<int>(c[p].y);
      }
    }
    float Z = 0.f;
    for (int p = 0; p < k; ++p) Z += c[p].z * __expf(c[p].x - M);
    tokens[r] = tok;
    lps[r] = -logf(Z);
    epochs[r] = e + 1;
  }
}

// logits: local fp32 [rows, V] (this rank's vocabulary slice starting at
// v0); cand_off: byte offset of [k][rows] float4 candidate slots; ctr_off:
// byte offset of >= rows u32 counters; epochs: int32 [>= rows] local.
int64_t tp_vocab_argmax(std::vector<int64_t> bases, int64_t mc, int64_t rank, torch::Tensor logits,
                        int64_t v0, int64_t cand_off, int64_t ctr_off, torch::Tensor tokens,
                        torch::Tensor lps, torch::Tensor epochs, double timeout_s) {
  const RnPeers P = rn_peers(bases, mc);
  const int k = static_cast<int>(bases.size());
  TORCH_CHECK(logits.scalar_type() == at::kFloat && logits.dim() == 2 && logits.stride(1) == 1);
  const int rows = static_cast<int>(logits.size(0));
  TORCH_CHECK(tokens.scalar_type() == at::kInt && tokens.numel() >= rows);
  TORCH_CHECK(lps.scalar_type() == at::kFloat && lps.numel() >= rows);
  TORCH_CHECK(epochs.scalar_type() == at::kInt && epochs.numel() >= rows);
  TORCH_CHECK(cand_off % 16 == 0 && ctr_off % 4 == 0);
  if (rows == 0) return 0;
  const int64_t tns = static_cast<int64_t>(timeout_s * 1e9);
  auto ep = reinterpret_cast<uint32_t*>(epochs.data_ptr<int32_t>());
  if (P.mc)
    launch_pdl(tp_vocab_argmax_kernel<true>, dim3(rows), dim3(kVaThreads), 0, cur_stream(), 
        P, static_cast<int>(rank), k, logits.data_ptr<float>(), logits.stride(0),
        static_cast<int>(logits.size(1)), static_cast<int>(v0), rows, cand_off, ctr_off,
        tokens.data_ptr<int32_t>(), lps.data_ptr<float>(), ep, tns, status_word_ptr());
  else
    launch_pdl(tp_vocab_argmax_kernel<false>, dim3(rows), dim3(kVaThreads), 0, cur_stream(), 
        P, static_cast<int>(rank), k, logits.data_ptr<float>(), logits.stride(0),
        static_cast<int>(logits.size(1)), static_cast<int>(v0), rows, cand_off, ctr_off,
        tokens.data_ptr<int32_t>(), lps.data_ptr<float>(), ep, tns, status_word_ptr());
  SWIFT_CHECK_LAUNCH();
  return 1;
}

// ---- vocab-parallel logits all-gather (sampled / logprob steps)
// Rank j holds the fp32 logits of vocabulary slice [j*Vs, (j+1)*Vs) for
// every sampled row. Block b pushes rows b, b + grid, ... of this rank's
// slice into column block j of every rank's [rows, k*Vs] gather buffer (one
// multimem.st of 16 bytes per 4 logits, or k peer stores), then meets block
// b of the peers on its counter (arrival after its stores); when every block
// has passed, each rank holds the full rows locally. The gather buffer is
// only rewritten after a later step's TP reductions, which order every rank
// past its readers of this one.
constexpr int kGaThreads = 256;
constexpr int kGaBlocks = 64;

template <bool MC>
__global__ void __launch_bounds__(kGaThreads)
    tp_gather_vocab_kernel(RnPeers P, int rank, int k, const float* __restrict__ logits,
                           int64_t ld, int Vs, int rows, int64_t dst_off, int64_t ctr_off,
                           uint32_t* __restrict__ epochs, int64_t timeout_ns, int* status) {
  pdl_wait();
  pdl_trigger();
  const uint32_t e = epochs[blockIdx.x];
  const int V = Vs * k, nv = Vs / 4;
  for (int r = blockIdx.x; r < rows; r += gridDim.x) {
    const float4* src = reinterpret_cast<const float4*>(logits + int64_t(r) * ld);
    const int64_t byte0 = dst_off + (int64_t(r) * V + int64_t(rank) * Vs) * 4;
    for (int i = threadIdx.x; i < nv; i += kGaThreads) {
      const float4 v = src[i];
      if constexpr (MC) {
        mc_st_f32x4(P.mc + byte0 + int64_t(i) * 16, v);
      } else {
        for (int p = 0; p < k; ++p) {
          const int q = (rank + p) % k;
          *reinterpret_cast<float4*>(P.base[q] + byte0 + int64_t(i) * 16) = v;
        }
      }
    }
  }
  if (!rn_barrier<MC>(P, rank, k, ctr_off, (e + 1) * uint32_t(k), timeout_ns, status, 240)) return;
  if (threadIdx.x == 0) epochs[blockIdx.x] = e + 1;
}

// logits: this rank's fp32 [rows, Vs] slice (row stride may exceed Vs);
// dst_off: byte offset of the [rows, k*Vs] fp32 gather buffer in the
// symmetric allocation; ctr_off: kGaBlocks u32 counters; epochs: int32
// [kGaBlocks] local. Returns the number of kernels launched.
int64_t tp_gather_vocab(std::vector<int64_t> bases, int64_t mc, int64_t rank, torch::Tensor logits,
                        int64_t dst_off, int64_t ctr_off, torch::Tensor epochs, double timeout_s) {
  const RnPeers P = rn_peers(bases, mc);
  const int k = static_cast<int>(bases.size());
  TORCH_CHECK(logits.scalar_type() == at::kFloat && logits.dim() == 2 && logits.stride(1) == 1);
  const int rows = static_cast<int>(logits.size(0)), Vs = static_cast<int>(logits.size(1));
  TORCH_CHECK(Vs % 4 == 0 && logits.stride(0) % 4 == 0 &&
                  reinterpret_cast<uintptr_t>(logits.data_ptr()) % 16 == 0,
              "tp_gather_vocab: 16-byte rows");
  TORCH_CHECK(dst_off % 16 == 0 && ctr_off % 4 == 0);
  TORCH_CHECK(epochs.scalar_type() == at::kInt && epochs.numel() >= kGaBlocks && epochs.is_cuda());
  if (rows == 0) return 0;
  const int64_t tns = static_cast<int64_t>(timeout_s * 1e9);
  auto ep = reinterpret_cast<uint32_t*>(epochs.data_ptr<int32_t>());
  // every rank computes the same grid from rows, so block b's counter and
  // epoch advance alike on all ranks
  const int blocks = std::min(kGaBlocks, rows);
  if (P.mc)
    launch_pdl(tp_gather_vocab_kernel<true>, dim3(blocks), dim3(kGaThreads), 0, cur_stream(),
               P, static_cast<int>(rank), k, logits.data_ptr<float>(), logits.stride(0), Vs, rows,
               dst_off, ctr_off, ep, tns, status_word_ptr());
  else
    launch_pdl(tp_gather_vocab_kernel<false>, dim3(blocks), dim3(kGaThreads), 0, cur_stream(),
               P, static_cast<int>(rank), k, logits.data_ptr<float>(), logits.stride(0), Vs, rows,
               dst_off, ctr_off, ep, tns, status_word_ptr());
  SWIFT_CHECK_LAUNCH();
  return 1;
}

// Test hook: one bounded wait on a flag nobody sets (single GPU, no peer):
// must return with kErrPeerTimeout recorded, the context still usable.
__global__ void flag_wait_probe_kernel(const uint32_t* flag, uint32_t want, int64_t timeout_ns,
                                       int* status) {
  const uint64_t deadline = rn_now() + static_cast<uint64_t>(timeout_ns);
  while (static_cast<int32_t>(rn_ld_acquire(flag) - want) < 0) {
    if (rn_now() > deadline) {
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
