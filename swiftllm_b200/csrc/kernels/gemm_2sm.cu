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
#include <cstring>

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
// epilogue staging: per epilogue warp two [32 tokens][32 features] bf16
// boxes (dense 64-byte rows, the TMA store box)
constexpr int kEpiBox = 32 * 32;
constexpr size_t kSmemBytes = 1024 + size_t(kStages) * kStageBytes + 4 * 2 * kEpiBox * 2 + 256;

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
// Warp-uniform bounded wait: every lane polls, all agree before leaving.
__device__ __forceinline__ bool wait_warp_or_abort(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                                   int* status, int where) {
  for (uint32_t i = 0; i < kWaitLimit; ++i) {
    const bool ok = mbar_try_wait(bar, parity);
    if (__all_sync(0xffffffffu, ok)) return true;
    if ((i & 255) == 255 && __any_sync(0xffffffffu, *abort_flag != 0)) return false;
  }
  if ((threadIdx.x & 31) == 0) {
    set_status(status, kErrWaitTimeout, where);
    *abort_flag = 1;
  }
  return false;
}
__device__ __forceinline__ bool elect_one() {
  uint32_t pred;
  asm volatile(
      "{\n .reg .pred p;\n elect.sync _|p, 0xffffffff;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(pred));
  return pred != 0;
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
// tcgen05.ld without the wait: the registers are valid after tmem_wait().
__device__ __forceinline__ void tmem_ld32_async(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]),
        "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]),
        "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// TMA store of one [32 tokens][32 features] bf16 box from shared memory
// (bulk async-group; out-of-range rows / columns are clipped).
__device__ __forceinline__ void tma_store_box(const CUtensorMap* tm, const void* smem, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(tm)),
      "r"(smem_u32(smem)), "r"(x), "r"(y)
      : "memory");
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
__device__ __forceinline__ void tma_store_wait_read1() {
  asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
}
__device__ __forceinline__ void tma_store_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// silu(g) * u = g * u / (1 + e^-g)
__device__ __forceinline__ float silu_mul(float g, float u) { return g * u / (1.f + __expf(-g)); }

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

// Work decomposition of one launch (identical for both CTAs of a pair):
//  data-parallel / split-K (sk_per == 0): tiles are (256 features, BN tokens)
//    x split; pair p takes tiles p, p + pairs, ... (feature tile outer, token
//    tile inner, split outermost), so pairs running together share each
//    weight tile through L2;
//  stream-K (sk_per > 0, one token tile): the (feature tile, k-step) space is
//    cut into one contiguous range of sk_per k-steps per pair, so every SM
//    streams the same share of the weights. A tile whose k-steps span
//    several pairs is finished by whichever pair arrives last: the others
//    store fp32 partials into their workspace slot and bump the tile's
//    counter; the last one adds them in pair order (bitwise the same result
//    whichever pair finishes) and stores bf16. No pair waits for another.
struct Seg {
  int m0, x0, k0, k1, tile, split;
};
struct SegIter {
  int pair, pairs, m_tiles, n_tiles, k_iters, k_per, splits, BN, sk_per, total;
  int it_begin, it_end, first_tile, nseg;
  __device__ void init(int pair_, int pairs_, int M, int N, int K, int BN_, int splits_, int sk_per_) {
    pair = pair_;
    pairs = pairs_;
    BN = BN_;
    m_tiles = (M + 255) / 256;
    n_tiles = (N + BN - 1) / BN;
    k_iters = (K + g2::kBK - 1) / g2::kBK;
    splits = splits_;
    k_per = (k_iters + splits - 1) / splits;
    sk_per = sk_per_;
    if (sk_per > 0) {
      const int all = m_tiles * k_iters;
      it_begin = min(all, pair * sk_per);
      it_end = min(all, it_begin + sk_per);
      first_tile = it_begin / k_iters;
      nseg = it_end > it_begin ? (it_end - 1) / k_iters - first_tile + 1 : 0;
    } else {
      total = m_tiles * n_tiles * splits;
      nseg = pair < total ? (total - pair + pairs - 1) / pairs : 0;
    }
  }
  __device__ Seg get(int i) const {
    Seg g;
    if (sk_per > 0) {
      // a partial LAST segment goes first: it is the head of a tile whose
      // tail the next pair computes first, so both halves of a split tile
      // are computed early and the finishing pair finds the partial ready
      const bool tail_first = nseg >= 2 && ((it_end - 1) % k_iters + 1) < k_iters;
      if (tail_first) i = i == 0 ? nseg - 1 : i - 1;
      g.tile = first_tile + i;
      g.m0 = g.tile * 256;
      g.x0 = 0;
      g.k0 = i == 0 ? it_begin % k_iters : 0;
      g.k1 = i == nseg - 1 ? (it_end - 1) % k_iters + 1 : k_iters;
      g.split = 0;
    } else {
      const int t = pair + i * pairs;
      g.split = t / (m_tiles * n_tiles);
      const int r = t % (m_tiles * n_tiles);
      g.tile = r;
      g.m0 = (r / n_tiles) * 256;
      g.x0 = (r % n_tiles) * BN;
      g.k0 = g.split * k_per;
      g.k1 = min(k_iters, g.k0 + k_per);
    }
    return g;
  }
  // stream-K: first and last pair contributing to tile t
  __device__ int first_pair(int t) const { return (t * k_iters) / sk_per; }
  __device__ int last_pair(int t) const { return ((t + 1) * k_iters - 1) / sk_per; }
  // workspace slot of pair o's partial of tile t (each pair has one slot
  // for its first tile and one for its last)
  __device__ int slot(int o, int t) const { return (o * sk_per) / k_iters == t ? 2 * o : 2 * o + 1; }
};

__device__ __forceinline__ void epi_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// SWAP = false: A = weights (M = output features), B = tokens (N).
// SWAP = true (decode, at most 256 tokens): A = tokens (one 256-row tile:
// 128 per CTA), B = weights in BN-feature tiles, so the feature tile width
// (any multiple of 16) spreads the weights over every SM pair in one wave;
// the accumulator lanes are tokens and each thread stores contiguous
// features of its token row. M / N are the row counts of A / B.
template <bool SWAP>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(g2::kThreads, 1)
    gemm2_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x,
                 const __grid_constant__ CUtensorMap tm_y, __nv_bfloat16* __restrict__ y, int64_t ldy, const __nv_bfloat16* __restrict__ bias,
                 float* __restrict__ ws, int M, int N, int K, int BN, int splits, int sk_per,
                 float* __restrict__ skws, int* __restrict__ skctr, int vec_out, int act,
                 int* status) {
  using namespace g2;
  extern __shared__ uint8_t smem_raw[];
  __shared__ int sh_ok[2][4];
  __shared__ int sh_last;
  uint8_t* tiles =
      reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __nv_bfloat16* epi = reinterpret_cast<__nv_bfloat16*>(tiles + size_t(kStages) * kStageBytes);
  uint64_t* full = reinterpret_cast<uint64_t*>(epi + 4 * 2 * kEpiBox);
  uint64_t* empty = full + kStages;
  uint64_t* tfull = empty + kStages;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t crank = cta_rank();
  const bool leader = crank == 0;
  SegIter S;
  S.init(blockIdx.x >> 1, gridDim.x >> 1, M, N, K, BN, splits, sk_per);
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

  if (warp == 0) {
    if (lane == 0) {
      const uint32_t full_leader = mapa(smem_u32(full), 0);
      uint32_t it = 0;
      bool ok = true;
      // Under programmatic dependent launch the weights (not written by the
      // previous kernel) of the first ring's worth of k-steps are requested
      // before waiting for the previous kernel; the token tiles after.
      // operand loads of k-step kk into stage smem `a`: A rows from m0, B rows from x0
      auto load_w = [&](uint8_t* a, int kk, const Seg& g, uint32_t fb) {
        if constexpr (SWAP)
          tma_load_2sm(a + kABytes, &tm_w, kk * kBK, g.x0 + int(crank) * half_bn, fb);
        else
          tma_load_2sm(a, &tm_w, kk * kBK, g.m0 + int(crank) * kBM, fb);
      };
      auto load_x = [&](uint8_t* a, int kk, const Seg& g, uint32_t fb) {
        if constexpr (SWAP)
          tma_load_2sm(a, &tm_x, kk * kBK, g.m0 + int(crank) * kBM, fb);
        else
          tma_load_2sm(a + kABytes, &tm_x, kk * kBK, g.x0 + int(crank) * half_bn, fb);
      };
      int pre = 0;
      if (S.nseg > 0) {
        const Seg g = S.get(0);
        pre = min(kStages, g.k1 - g.k0);
        for (int j = 0; j < pre; ++j) {
          if (leader) mbar_arrive_expect_tx(&full[j], 2 * (kABytes + b_bytes));
          load_w(tiles + size_t(j) * kStageBytes, g.k0 + j, g, full_leader + j * 8);
        }
      }
      pdl_wait();
      for (int i = 0; i < S.nseg && ok; ++i) {
        const Seg g = S.get(i);
        for (int kk = g.k0; kk < g.k1; ++kk, ++it) {
          const int st = it % kStages;
          uint8_t* a = tiles + size_t(st) * kStageBytes;
          const uint32_t fb = full_leader + st * 8;
          if (i == 0 && kk - g.k0 < pre) {  // weights already requested
            load_x(a, kk, g, fb);
            continue;
          }
          if (!wait_or_abort(&empty[st], ((it / kStages) & 1) ^ 1, abort_flag, status, 40)) {
            ok = false;
            break;
          }
          if (leader) mbar_arrive_expect_tx(&full[st], 2 * (kABytes + b_bytes));
          load_w(a, kk, g, fb);
          load_x(a, kk, g, fb);
        }
      }
      pdl_trigger();  // every load issued: the next kernel may start its prologue
      if (!ok) {  // let the loads already issued land before the CTA leaves
        for (uint32_t p = 0; p < (1u << 22); ++p) __nanosleep(0);
      }
    }
  } else if (warp == 1) {
    // MMA issue: the whole warp runs the loop with warp-uniform waits and
    // one elected lane issues the MMAs and commits. (A single-lane loop
    // beside 31 parked lanes issued measurably slower: about 400 ns per
    // 64-wide k-step at 64-feature tiles, against 290 ns converged.)
    if (leader) {
      const uint32_t idesc = idesc_bf16_m256(BN);
      uint32_t it = 0;
      bool ok = true;
      for (int i = 0; i < S.nseg && ok; ++i) {
        const Seg g = S.get(i);
        const uint32_t buf = i & 1;
        if (!wait_warp_or_abort(&tempty[buf], ((i >> 1) & 1) ^ 1, abort_flag, status, 41)) {
          ok = false;
          break;
        }
        fence_after();
        const uint32_t d_tmem = tmem_base + buf * buf_cols;
        for (int kk = g.k0; kk < g.k1; ++kk, ++it) {
          const int st = it % kStages;
          if (!wait_warp_or_abort(&full[st], (it / kStages) & 1, abort_flag, status, 42)) {
            ok = false;
            break;
          }
          fence_after();
          if (elect_one()) {
            const uint32_t a = smem_u32(tiles + size_t(st) * kStageBytes);
            const uint64_t ad = desc_sw128(a), bd = desc_sw128(a + kABytes);
#pragma unroll
            for (int j = 0; j < kBK / 16; ++j)  // +32 B along K inside the swizzle atom
              umma2(d_tmem, ad + 2 * j, bd + 2 * j, idesc, (kk > g.k0 || j > 0) ? 1u : 0u);
            commit_both(&empty[st]);
          }
          __syncwarp();
        }
        if (!ok) break;
        if (elect_one()) commit_both(&tfull[buf]);
        __syncwarp();
      }
      if (!ok && lane == 0) {
        for (uint32_t p = 0; p < (1u << 22); ++p) __nanosleep(0);
      }
    }
  } else {
    const int q = warp & 3;  // TMEM lane quarter of this warp
    const int fl = q * 32 + lane;  // feature within this CTA's 128
    const uint32_t tempty_leader = mapa(smem_u32(tempty), 0);
    __nv_bfloat16* stage = epi + q * 2 * kEpiBox;  // two boxes per warp
    uint32_t nbox = 0;                              // boxes stored by this warp
    constexpr int kSlotFloats = kBM * kMaxBN;
    for (int i = 0; i < S.nseg; ++i) {
      const Seg g = S.get(i);
      const uint32_t buf = i & 1;
      bool ok = true;
      for (uint32_t w = 0;; ++w) {
        const bool r = mbar_try_wait(&tfull[buf], (i >> 1) & 1);
        if (__all_sync(0xffffffffu, r)) break;
        if (w > kWaitLimit || ((w & 255) == 255 && *abort_flag)) {
          if (lane == 0 && w > kWaitLimit) {
            set_status(status, kErrWaitTimeout, 43);
            *abort_flag = 1;
          }
          ok = false;
          break;
        }
      }
      // the four epilogue warps agree before any named barrier, so a warp
      // that gave up never leaves the others waiting at bar.sync
      if (lane == 0) sh_ok[i & 1][q] = ok;
      epi_sync();
      ok = sh_ok[i & 1][0] && sh_ok[i & 1][1] && sh_ok[i & 1][2] && sh_ok[i & 1][3];
      if (!ok) break;
      fence_after();
      const int fbase = g.m0 + int(crank) * kBM + q * 32;
      const int f = fbase + lane;
      const uint32_t tq = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + buf * buf_cols;
      const bool whole = g.k0 == 0 && g.k1 == S.k_iters;
      // ---- stream-K partial tile: store the partial or finish the tile
      bool finish = true;
      int cf = S.pair, cl = S.pair;
      if (S.sk_per > 0 && !whole) {
        cf = S.first_pair(g.tile);
        cl = S.last_pair(g.tile);
        const int others = cl - cf;
        int* ctr = skctr + g.tile * 2 + int(crank);
        if (threadIdx.x == 64) {
          const int done = *reinterpret_cast<volatile int*>(ctr);
          const int lst = done == others;
          if (lst) {
            __threadfence();  // acquire the other partials
            *ctr = 0;         // ready for the next launch
          }
          sh_last = lst;
        }
        epi_sync();
        finish = sh_last != 0;
        epi_sync();
        if (!finish) {
          float* wp = skws + (size_t(S.slot(S.pair, g.tile)) * 2 + crank) * kSlotFloats;
#pragma unroll 1
          for (int c = 0; c < BN; c += 32) {
            float v[32];
            g2::tmem_ld32(tq + c, v);
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (c + j < BN) __stcg(wp + size_t(c + j) * kBM + fl, v[j]);
          }
          epi_sync();  // every partial store happens-before the counter bump
          if (threadIdx.x == 64) {
            __threadfence();
            const int old = atomicAdd(ctr, 1);
            const int lst = old == others;
            if (lst) {
              __threadfence();
              *ctr = 0;
            }
            sh_last = lst;
          }
          epi_sync();
          finish = sh_last != 0;
        }
      }
      if (finish) {
        const float b = (!SWAP && bias != nullptr && f < M && splits == 1) ? __bfloat162float(bias[f]) : 0.f;
        // TMEM loads run one chunk ahead of the conversion and the stores
        uint32_t nxt[32];
        g2::tmem_ld32_async(tq, nxt);
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
          g2::tmem_wait();
          float v[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(nxt[j]);
          // columns past BN are not this tile's: masked below
          if (c + 32 < BN) g2::tmem_ld32_async(tq + c + 32, nxt);
          if (cl > cf) {  // fixed order over the tile's pairs
            float acc[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) acc[j] = 0.f;
            // two other pairs' partials per round: 64 independent loads in
            // flight per thread instead of one latency per partial
            for (int o = cf; o <= cl; o += 2) {
              const bool use0 = o != S.pair, use1 = o + 1 <= cl && o + 1 != S.pair;
              const float* r0 = skws + (size_t(S.slot(o, g.tile)) * 2 + crank) * kSlotFloats +
                                size_t(c) * kBM + fl;
              const float* r1 = skws + (size_t(S.slot(min(o + 1, cl), g.tile)) * 2 + crank) * kSlotFloats +
                                size_t(c) * kBM + fl;
              float p0[32], p1[32];
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                const bool in = c + j < BN;
                p0[j] = (use0 && in) ? __ldcg(r0 + size_t(j) * kBM) : 0.f;
                p1[j] = (use1 && in) ? __ldcg(r1 + size_t(j) * kBM) : 0.f;
              }
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                acc[j] += o == S.pair ? v[j] : p0[j];
                if (o + 1 <= cl) acc[j] += o + 1 == S.pair ? v[j] : p1[j];
              }
            }
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = acc[j];
          }
          const int t0 = g.x0 + c;
          const int nvalid = min(min(32, BN - c), N - t0);
          if constexpr (SWAP) {
            // this thread's row is token f (= m0 + lane row); columns are
            // features t0 .. t0 + nvalid - 1
            if (act && f < M && nvalid > 0) {
              // interleaved (gate, up) column pairs -> silu(gate) * up, 16 outputs
              __nv_bfloat16* yr = y + int64_t(f) * ldy + t0 / 2;
              float o[16];
#pragma unroll
              for (int i = 0; i < 16; ++i) o[i] = silu_mul(v[2 * i], v[2 * i + 1]);
              if (vec_out && nvalid == 32) {
                store8(yr, o);
                store8(yr + 8, o + 8);
              } else {
#pragma unroll
                for (int i = 0; i < 16; ++i)
                  if (2 * i + 1 < nvalid) yr[i] = __float2bfloat16(o[i]);
              }
            } else if (f < M && nvalid > 0) {
              __nv_bfloat16* yr = y + int64_t(f) * ldy + t0;
              if (bias != nullptr) {
#pragma unroll
                for (int j = 0; j < 32; ++j)
                  if (j < nvalid) v[j] += __bfloat162float(bias[t0 + j]);
              }
              if (vec_out && nvalid == 32) {
#pragma unroll
                for (int q8 = 0; q8 < 4; ++q8) {
                  uint4 pk;
                  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&pk);
#pragma unroll
                  for (int e = 0; e < 4; ++e)
                    h[e] = __floats2bfloat162_rn(v[q8 * 8 + 2 * e], v[q8 * 8 + 2 * e + 1]);
                  *reinterpret_cast<uint4*>(yr + q8 * 8) = pk;
                }
              } else {
#pragma unroll
                for (int j = 0; j < 32; ++j)
                  if (j < nvalid) yr[j] = __float2bfloat16(v[j]);
              }
            }
            continue;
          }
          if (act) {
            // lanes hold interleaved (gate, up) feature rows: the even lane
            // of each pair takes the odd lane's value, outputs feature f / 2
            float o[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const float other = __shfl_xor_sync(0xffffffffu, v[j], 1);
              o[j] = silu_mul(v[j], other);
            }
            __nv_bfloat16* box = stage + (nbox & 1) * kEpiBox;  // [32 tokens][16 outputs]
            if (lane == 0 && nbox >= 2) g2::tma_store_wait_read1();
            __syncwarp();
            if ((lane & 1) == 0) {
#pragma unroll
              for (int j = 0; j < 32; ++j) box[j * 16 + (lane >> 1)] = __float2bfloat16(o[j]);
            }
            __syncwarp();
            // 32 rows x 32 bytes: lane stores both 16-byte halves of row `lane`
            const int fo = fbase / 2;
            if (lane < nvalid && fo < M / 2) {
              __nv_bfloat16* yr = y + int64_t(t0 + lane) * ldy + fo;
              if (vec_out) {
                *reinterpret_cast<uint4*>(yr) = *reinterpret_cast<const uint4*>(box + lane * 16);
                *reinterpret_cast<uint4*>(yr + 8) = *reinterpret_cast<const uint4*>(box + lane * 16 + 8);
              } else {
                for (int i = 0; i < 16 && fo + i < M / 2; ++i) yr[i] = box[lane * 16 + i];
              }
            }
            __syncwarp();
            continue;
          }
          if (splits > 1) {
            if (f < M)
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (j < nvalid) ws[(int64_t(g.split) * N + t0 + j) * M + f] = v[j];
          } else if (vec_out) {
            // [token][feature] box in shared memory, then one TMA store; the
            // box written two chunks ago must have been read out first
            __nv_bfloat16* box = stage + (nbox & 1) * kEpiBox;
            if (lane == 0 && nbox >= 2) g2::tma_store_wait_read1();
            __syncwarp();
#pragma unroll
            for (int j = 0; j < 32; ++j) box[j * 32 + lane] = __float2bfloat16(v[j] + b);
            if (BN - c >= 32) {
              g2::fence_proxy_async_smem();
              __syncwarp();
              if (lane == 0) g2::tma_store_box(&tm_y, box, fbase, t0);
              ++nbox;
            } else {
              // last chunk of a tile narrower than a multiple of 32: the box
              // would reach into the next token tile, so store only its rows
              __syncwarp();
#pragma unroll
              for (int r0 = 0; r0 < 32; r0 += 8) {
                const int row = r0 + (lane >> 2), part = lane & 3;
                const int fo = fbase + part * 8;
                if (row < nvalid && fo < M)
                  *reinterpret_cast<uint4*>(y + int64_t(t0 + row) * ldy + fo) =
                      *reinterpret_cast<const uint4*>(box + row * 32 + part * 8);
              }
              __syncwarp();
            }
          } else if (f < M) {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (j < nvalid) y[int64_t(t0 + j) * ldy + f] = __float2bfloat16(v[j] + b);
          }
        }
        g2::tmem_wait();
      }
      fence_before();
      __syncwarp();
      if (lane == 0) g2::arrive_remote(tempty_leader + buf * 8);
    }
  }
  if (warp >= 2 && lane == 0) g2::tma_store_wait_all();  // stores read out of smem and done
  fence_before();
  __syncthreads();
  cluster_sync();  // no CTA leaves while its peer may still signal it
  if (warp == 1) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                 "r"(tmem_cols));
  }
}

// y[t, f] = bias[f] + sum_s ws[s, t, f]; 8 features per thread (M % 8 == 0).
__global__ void splitk2_reduce_kernel(__nv_bfloat16* __restrict__ y, int64_t ldy,
                                      const float* __restrict__ ws,
                                      const __nv_bfloat16* __restrict__ bias, int M, int N,
                                      int splits) {
  pdl_wait();
  const int mv = M / 8;
  const int64_t total = int64_t(M) * N, nvec = int64_t(mv) * N;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < nvec;
       i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t t = i / mv;
    const int f = static_cast<int>(i - t * mv) * 8;
    float acc[8];
    if (bias) {
      load8(bias + f, acc);
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] = 0.f;
    }
    const float* p = ws + t * M + f;
    for (int sp = 0; sp < splits; ++sp) {
      const float4 a = __ldcg(reinterpret_cast<const float4*>(p + sp * total));
      const float4 c = __ldcg(reinterpret_cast<const float4*>(p + sp * total + 4));
      acc[0] += a.x; acc[1] += a.y; acc[2] += a.z; acc[3] += a.w;
      acc[4] += c.x; acc[5] += c.y; acc[6] += c.z; acc[7] += c.w;
    }
    store8(y + t * ldy + f, acc);
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

// Stream-K state per device: two partial slots of 128 x 256 fp32 per CTA
// and zeroed per-(tile, CTA half) counters that the finishing pair resets;
// allocated once and kept for the process (CUDA graphs capture the
// pointers).
constexpr int kSk2MaxTiles = 4096;
struct Sk2Buffers {
  float* ws = nullptr;
  int* ctr = nullptr;
};
static Sk2Buffers& sk2_buffers() {
  static Sk2Buffers b[64];
  int dev;
  cudaGetDevice(&dev);
  if (!b[dev].ws) {
    const size_t slots = size_t(sm_count()) * 2;
    SWIFT_CHECK_CUDA(cudaMalloc(&b[dev].ws, slots * g2::kBM * g2::kMaxBN * sizeof(float)));
    SWIFT_CHECK_CUDA(cudaMalloc(&b[dev].ctr, 2 * kSk2MaxTiles * sizeof(int)));
    SWIFT_CHECK_CUDA(cudaMemset(b[dev].ctr, 0, 2 * kSk2MaxTiles * sizeof(int)));
    SWIFT_CHECK_CUDA(cudaDeviceSynchronize());
  }
  return b[dev];
}

// Plan: token tile BN (the fewest tiles of width <= 256, rounded up to 16),
// split count, and k-steps per pair for stream-K (0: data-parallel).
// One token tile (N <= 256, decode and small mixed steps): stream-K over all
// pairs, at least 16 k-steps per pair. Otherwise data-parallel tiles, split K
// while they fill under 3/4 of the pairs and each split keeps >= 8 k-steps.
// plan force: -1 automatic, 0 data-parallel (optionally with the given
// token tile / split), 1 stream-K, 2 swapped operands (tokens as A).
void gemm2_plan(int64_t M, int64_t N, int64_t K, int* bn, int* splits, int* sk_per, int* pairs_out,
                int* swap, int force = -1, int force_bn = 0, int force_splits = 0) {
  const int pairs = sm_count() / 2;
  *swap = 0;
  if ((force < 0 && N <= 256) || (force == 2 && N <= 256)) {
    // swapped operands: one 256-token A tile; feature tiles as wide as
    // needed to give every SM pair one tile (whole waves when there are
    // more features than 256 x pairs); width a multiple of 16
    int64_t nf = (M + 255) / 256;
    if (nf < pairs) nf = std::min<int64_t>(pairs, (M + 15) / 16);
    else nf = (nf + pairs - 1) / pairs * pairs;
    int w = static_cast<int>(((M + nf - 1) / nf + 15) / 16 * 16);
    w = std::max(16, std::min(256, w));
    if (force_bn > 0) w = force_bn;
    *bn = w;
    *splits = 1;
    *sk_per = 0;
    *swap = 1;
    *pairs_out = static_cast<int>(std::min<int64_t>((M + w - 1) / w, pairs));
    return;
  }
  const int64_t nt = (N + 255) / 256;
  int b = static_cast<int>(((N + nt - 1) / nt + 15) / 16 * 16);
  b = std::max(16, std::min(256, b));
  const int64_t m_tiles = (M + 255) / 256;
  const int64_t tiles = m_tiles * ((N + b - 1) / b);
  const int k_iters = static_cast<int>((K + 63) / 64);
  *bn = b;
  if (force == 0) {  // data-parallel with the given token tile / split (defaults: BN above, 1)
    if (force_bn > 0) b = force_bn;
    *bn = b;
    *splits = force_splits > 0 ? force_splits : 1;
    *sk_per = 0;
    *pairs_out = static_cast<int>(
        std::min<int64_t>(m_tiles * ((N + b - 1) / b) * *splits, pairs));
    return;
  }
  if ((force == 1 || (force < 0 && nt == 1)) && nt == 1 && m_tiles <= kSk2MaxTiles) {
    const int64_t all = m_tiles * k_iters;
    int64_t g = std::min<int64_t>(pairs, (all + 15) / 16);
    g = std::max<int64_t>(g, 1);
    const int64_t per = (all + g - 1) / g;
    *splits = 1;
    *sk_per = static_cast<int>(per);
    *pairs_out = static_cast<int>((all + per - 1) / per);
    return;
  }
  int s = 1;
  while (tiles * s * 4 < int64_t(pairs) * 3 && k_iters / (s * 2) >= 8 && s < 8) s *= 2;
  *splits = s;
  *sk_per = 0;
  *pairs_out = static_cast<int>(std::min<int64_t>(tiles * s, pairs));
}

// y [T, M] (row stride ldy), x [T, K], w [M, K], bias [M] or null.
// Returns the number of kernels launched.
int64_t gemm2_launch(__nv_bfloat16* y, int64_t ldy, const torch::Tensor& x, const torch::Tensor& w,
                     const __nv_bfloat16* bias, int force = -1, int force_bn = 0,
                     int force_splits = 0, int act = 0) {
  const int64_t K = x.size(-1), T = x.numel() / K, M = w.size(0);
  if (T == 0) return 0;
  const int64_t ldx = x.dim() >= 2 ? x.stride(-2) : K;
  int bn, splits, sk_per, pairs, swap;
  gemm2_plan(M, T, K, &bn, &splits, &sk_per, &pairs, &swap, force, force_bn, force_splits);
  static bool attr[64] = {false};
  int dev;
  cudaGetDevice(&dev);
  if (!attr[dev]) {
    SWIFT_CHECK_CUDA(cudaFuncSetAttribute(gemm2_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          static_cast<int>(g2::kSmemBytes)));
    SWIFT_CHECK_CUDA(cudaFuncSetAttribute(gemm2_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          static_cast<int>(g2::kSmemBytes)));
    attr[dev] = true;
  }
  // A operand boxes are 128 rows per CTA, B operand boxes bn / 2
  CUtensorMap tw = tmap_bf16(w.data_ptr(), M, K, w.stride(0), swap ? bn / 2 : g2::kBM);
  CUtensorMap tx = tmap_bf16(x.data_ptr(), T, K, ldx, swap ? g2::kBM : bn / 2);
  const int64_t out_w = act ? M / 2 : M;  // silu-mul halves the output width
  const int vec_out = (out_w % 8 == 0 && ldy % 8 == 0 && reinterpret_cast<uintptr_t>(y) % 16 == 0) ? 1 : 0;
  TORCH_CHECK(!act || (splits == 1 && M % 2 == 0), "gemm2: silu-mul needs whole (gate, up) pairs, no split-K");
  // output boxes of 32 features x 32 tokens, no swizzle (dense 64-byte rows)
  CUtensorMap ty;
  if (vec_out && !swap && !act) {
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(M), static_cast<cuuint64_t>(T)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(ldy * 2)};
    cuuint32_t box[2] = {32, 32};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = encode_fn()(&ty, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, static_cast<void*>(y), dims,
                             strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                             CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (output) failed (", static_cast<int>(r), ")");
  } else {
    std::memset(&ty, 0, sizeof(ty));
  }
  float* skws = nullptr;
  int* skctr = nullptr;
  if (sk_per > 0) {
    Sk2Buffers& b = sk2_buffers();
    skws = b.ws;
    skctr = b.ctr;
  }
  torch::Tensor ws;
  float* wsp = nullptr;
  if (splits > 1) {
    ws = torch::empty({splits, T, M}, x.options().dtype(torch::kFloat));
    wsp = ws.data_ptr<float>();
  }
  if (swap)
    launch_pdl(gemm2_kernel<true>, dim3(2 * pairs), dim3(g2::kThreads), g2::kSmemBytes, cur_stream(),
               tw, tx, ty, y, ldy, bias, wsp, static_cast<int>(T), static_cast<int>(M),
               static_cast<int>(K), bn, 1, 0, skws, skctr, vec_out, act, status_word_ptr());
  else
    launch_pdl(gemm2_kernel<false>, dim3(2 * pairs), dim3(g2::kThreads), g2::kSmemBytes, cur_stream(),
               tw, tx, ty, y, ldy, bias, wsp, static_cast<int>(M), static_cast<int>(T),
               static_cast<int>(K), bn, splits, sk_per, skws, skctr, vec_out, act, status_word_ptr());
  if (splits > 1) {
    TORCH_CHECK(M % 8 == 0 && ldy % 8 == 0 && reinterpret_cast<uintptr_t>(y) % 16 == 0,
                "gemm2: split-K needs 8-aligned output rows");
    const int64_t n = M / 8 * T;
    const int blocks = static_cast<int>(std::min<int64_t>((n + 255) / 256, 148 * 8));
    launch_pdl(splitk2_reduce_kernel, dim3(blocks), dim3(256), 0, cur_stream(), y, ldy,
               static_cast<const float*>(wsp), bias, static_cast<int>(M), static_cast<int>(T), splits);
    return 2;
  }
  return 1;
}

// Gate/up projection with the SwiGLU activation in the epilogue: w13 rows
// interleaved (gate_0, up_0, gate_1, up_1, ...), out [T, M / 2] =
// silu(x . gate^T) * (x . up^T). Swapped operands for at most 256 tokens,
// data-parallel tiles without split-K above. Returns the launches.
int64_t gemm_swiglu(torch::Tensor out, torch::Tensor x, torch::Tensor w13) {
  CHECK_BF16(out);
  CHECK_BF16(x);
  CHECK_BF16(w13);
  const int64_t K = x.size(-1), T = x.numel() / K, M = w13.size(0);
  TORCH_CHECK(w13.size(1) == K && K % 8 == 0 && M % 2 == 0, "gemm_swiglu: shapes");
  TORCH_CHECK(x.stride(-1) == 1 && w13.stride(1) == 1 && out.stride(-1) == 1);
  TORCH_CHECK(out.numel() == T * (M / 2), "gemm_swiglu: out must be [T, M / 2]");
  const int64_t ldx = x.dim() >= 2 ? x.stride(-2) : K;
  TORCH_CHECK(ldx % 8 == 0 && w13.stride(0) % 8 == 0);
  const int64_t ldy = out.dim() >= 2 ? out.stride(-2) : M / 2;
  return gemm2_launch(reinterpret_cast<__nv_bfloat16*>(out.data_ptr<at::BFloat16>()), ldy, x, w13,
                      nullptr, T <= 256 ? 2 : 0, 0, 1, 1);
}

// Python binding: out [T, M] (row stride may exceed M), x [T, K], w [M, K].
// plan: -1 automatic, 0 data-parallel without split, 1 stream-K (one token
// tile only); the explicit plans exist for measurements and tests.
int64_t gemm2(torch::Tensor out, torch::Tensor x, torch::Tensor w, c10::optional<torch::Tensor> bias,
              int64_t plan, int64_t bn, int64_t splits) {
  TORCH_CHECK(bn == 0 || (bn % 16 == 0 && bn >= 16 && bn <= 256), "gemm2: bn");
  TORCH_CHECK(splits >= 0 && splits <= 16, "gemm2: splits");
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
  return gemm2_launch(reinterpret_cast<__nv_bfloat16*>(out.data_ptr<at::BFloat16>()), ldy, x, w, bp,
                      static_cast<int>(plan), static_cast<int>(bn), static_cast<int>(splits));
}

// [B tile width, splits, stream-K k-steps per pair (0: none), pairs, swapped]
std::vector<int64_t> gemm2_plan_py(int64_t M, int64_t N, int64_t K) {
  int bn, s, per, pairs, swap;
  gemm2_plan(M, N, K, &bn, &s, &per, &pairs, &swap);
  return {bn, s, per, pairs, swap};
}

}  // namespace swift
