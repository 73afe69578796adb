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

#include <algorithm>
#include <cstdlib>

#include <cuda_fp8.h>

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

// Warp-uniform variant for the MMA-issue warp (all lanes poll, all agree).
__device__ __forceinline__ bool wait_warp_or_abort(uint64_t* bar, uint32_t parity,
                                                   volatile int* abort_flag, int* status, int where);
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
__device__ __forceinline__ bool wait_warp_or_abort(uint64_t* bar, uint32_t parity,
                                                   volatile int* abort_flag, int* status, int where) {
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
// kind::f8f6f4 with A and B both E4M3 (format code 0), fp32 accumulate.
template <int BN>
__host__ __device__ constexpr uint32_t instr_desc_e4m3() {
  return (1u << 4) | (static_cast<uint32_t>(BN >> 3) << 17) |
         (static_cast<uint32_t>(kGemmBM >> 4) << 24);
}
__device__ __forceinline__ void umma_e4m3(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
}
// kind::i8 with A and B signed int8 (format code 1), s32 accumulate (c
// format 2), 32 elements of K per instruction like kind::f8f6f4.
template <int BN>
__host__ __device__ constexpr uint32_t instr_desc_s8() {
  return (2u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(BN >> 3) << 17) |
         (static_cast<uint32_t>(kGemmBM >> 4) << 24);
}
__device__ __forceinline__ void umma_s8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                        uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
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

// ---- fused GEMM -> reduce-scatter over NVLink (tensor parallelism)
// When k > 0 the epilogue does not store into `y`: output row t (a token) is
// stored straight into the symmetric receive buffer of the rank that owns
// that token, at [src = this rank][t - lo(owner)][:], with plain stores
// through the peer mapping (NVLink). Token ownership is contiguous:
// lo(j) = T*j/k. After the last CTA has finished, the kernel publishes its
// completion epoch to every peer's flag slot (st.release.sys), and
// tp_rs_finish (tp_allreduce.cu) reduces each rank's own tokens.
struct ScatterDesc {
  uint64_t base[8];   // symmetric allocation of every rank (byte address)
  int64_t in_off;     // byte offset of this call's receive buffer
  int64_t flag_off;   // byte offset of the [src rank] u32 completion flags
  uint32_t* ctr;      // this rank's device counters: [0] epoch, [2] CTA done count
  int k, rank, s_max, T, H;
  int fence_all;      // 1: every thread fences its own stores before the CTA publishes
};

__device__ __forceinline__ int sc_owner(const ScatterDesc& sc, int t) {
  return static_cast<int>((int64_t(t + 1) * sc.k - 1) / sc.T);
}
// row base pointer of output row t
__device__ __forceinline__ __nv_bfloat16* sc_row(const ScatterDesc& sc, __nv_bfloat16* y,
                                                 int64_t ldy, int t) {
  if (sc.k == 0) return y + int64_t(t) * ldy;
  const int j = sc_owner(sc, t);
  const int lo = static_cast<int>(int64_t(sc.T) * j / sc.k);
  return reinterpret_cast<__nv_bfloat16*>(sc.base[j] + sc.in_off) +
         (int64_t(sc.rank) * sc.s_max + (t - lo)) * sc.H;
}
// Rows t0 .. t0+n-1 as base + j*stride when they share an owner (else null).
__device__ __forceinline__ __nv_bfloat16* sc_run(const ScatterDesc& sc, __nv_bfloat16* y,
                                                 int64_t ldy, int t0, int n, int64_t* stride) {
  if (sc.k == 0) {
    *stride = ldy;
    return y + int64_t(t0) * ldy;
  }
  *stride = sc.H;
  const int last = min(t0 + n - 1, sc.T - 1);
  if (t0 >= sc.T || sc_owner(sc, t0) != sc_owner(sc, last)) return nullptr;
  return sc_row(sc, y, ldy, t0);
}

__device__ __forceinline__ void st_release_sys_u32(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// End of a fused GEMM (all threads, after the CTA's final __syncthreads):
// the last CTA to finish bumps the epoch and publishes it to every rank.
__device__ __forceinline__ void sc_publish(const ScatterDesc& sc) {
  if (sc.k == 0) return;
  if (sc.fence_all) __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    const uint32_t old = atomicAdd(&sc.ctr[2], 1u);
    if (old == gridDim.x - 1) {
      __threadfence_system();
      sc.ctr[2] = 0;
      const uint32_t ep = sc.ctr[0] + 1;
      sc.ctr[0] = ep;
      for (int r = 0; r < sc.k; ++r)
        st_release_sys_u32(reinterpret_cast<uint32_t*>(sc.base[r] + sc.flag_off) + sc.rank, ep);
    }
  }
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

// Q: 0 bf16 operands; 1 E4M3 (kind::f8f6f4); 2 signed int8 (kind::i8, s32
// accumulators converted to float in the epilogue). For Q != 0 both
// operands carry per-row fp32 scales applied in the epilogue.
template <int BN, int STAGES, int Q = 0>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_tcgen05_kernel(const __grid_constant__ CUtensorMap tm_w,
                        const __grid_constant__ CUtensorMap tm_x, __nv_bfloat16* __restrict__ y,
                        int64_t ldy, const __nv_bfloat16* __restrict__ bias,
                        float* __restrict__ ws, int M, int N, int K, int splits, int* status,
                        const int32_t* __restrict__ goff, int groups, const ScatterDesc sc,
                        const float* __restrict__ wscale = nullptr,
                        const float* __restrict__ xscale = nullptr) {
  // FP8 (E4M3 weights and activations, per-row scales): a 128-byte smem row
  // holds 128 elements, so one stage covers 128 of K; scales are applied in
  // the epilogue.
  constexpr int kBK = Q ? 128 : kGemmBK;
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
  const int k_iters = (K + kBK - 1) / kBK;
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
          tma_load_2d(a, &tm_w, kk * kBK, w0, &full[st]);
          tma_load_2d(a + S::A_BYTES, &tm_x, kk * kBK, x0, &full[st]);
        }
      }
      if (!ok) {  // let the loads already issued land before the CTA exits
        for (uint32_t j = it > STAGES ? it - STAGES : 0; j < it; ++j)
          for (uint32_t p = 0; p < (1u << 20); ++p)
            if (mbar_try_wait(&full[j % STAGES], (j / STAGES) & 1)) break;
      }
    }
  } else if (warp == 1) {
    // whole warp: warp-uniform waits, one elected lane issues
    {
      constexpr uint32_t idesc =
          Q == 1 ? instr_desc_e4m3<BN>() : Q == 2 ? instr_desc_s8<BN>() : instr_desc_bf16<BN>();
      uint32_t it = 0, tc = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x, ++tc) {
        int m, x0, xend, w0, s;
        decode_tile(t, m, x0, xend, w0, s);
        const int k0 = s * k_per, k1 = min(k_iters, k0 + k_per);
        const uint32_t buf = tc & 1;
        if (!wait_warp_or_abort(&tempty[buf], ((tc >> 1) & 1) ^ 1, abort_flag, status, 11)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * BN;
        for (int kk = k0; kk < k1; ++kk, ++it) {
          const int st = it % STAGES;
          if (!wait_warp_or_abort(&full[st], (it / STAGES) & 1, abort_flag, status, 12)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (elect_one()) {
            const uint8_t* a = tiles + size_t(st) * S::STAGE_BYTES;
            const uint64_t ad = smem_desc_sw128(a);
            const uint64_t bd = smem_desc_sw128(a + S::A_BYTES);
#pragma unroll
            for (int j = 0; j < kGemmBK / 16; ++j)  // +32 B along K inside the swizzle atom
              if constexpr (Q == 1)
                umma_e4m3(d_tmem, ad + 2 * j, bd + 2 * j, idesc, (kk > k0 || j > 0) ? 1u : 0u);
              else if constexpr (Q == 2)
                umma_s8(d_tmem, ad + 2 * j, bd + 2 * j, idesc, (kk > k0 || j > 0) ? 1u : 0u);
              else
                umma_bf16(d_tmem, ad + 2 * j, bd + 2 * j, idesc, (kk > k0 || j > 0) ? 1u : 0u);
            umma_commit(&empty[st]);
          }
          __syncwarp();
        }
        if (!ok) break;
        if (elect_one()) umma_commit(&tfull[buf]);
        __syncwarp();
      }
      if (!ok && lane == 0) {  // MMAs already issued finish (their commits arrive on empty[])
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
      const float wsf = (Q && f < M) ? wscale[f] : 1.f;
      // 8-bit: scales applied once per chunk, before the stores (independent loads)
      auto dq = [&](float a, int) { return a; };
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + buf * BN;
      if constexpr (BN >= 32) {
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          float v[32];
          tmem_ld32(tbase + c * 32, v);
          const int t0 = x0 + c * 32;
          if constexpr (Q == 2) {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = static_cast<float>(__float_as_int(v[j]));
          }
          if constexpr (Q != 0) {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] *= wsf * xscale[min(t0 + j, N - 1)];
          }
          if (f < M) {
            if (splits == 1) {
              int64_t rs;
              __nv_bfloat16* run = sc_run(sc, y, ldy, t0, 32, &rs);
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (t0 + j < xend)
                  (run ? run + j * rs : sc_row(sc, y, ldy, t0 + j))[f] = __float2bfloat16(dq(v[j], t0 + j) + b);
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (t0 + j < N) ws[(int64_t(s) * N + t0 + j) * M + f] = dq(v[j], t0 + j);
            }
          }
        }
      } else {
        float v[16];
        tmem_ld16(tbase, v);
        const int t0 = x0;
        if constexpr (Q == 2) {
#pragma unroll
          for (int j = 0; j < 16; ++j) v[j] = static_cast<float>(__float_as_int(v[j]));
        }
        if constexpr (Q != 0) {
#pragma unroll
          for (int j = 0; j < 16; ++j) v[j] *= wsf * xscale[min(t0 + j, N - 1)];
        }
        if (f < M) {
          if (splits == 1) {
            int64_t rs;
            __nv_bfloat16* run = sc_run(sc, y, ldy, t0, 16, &rs);
#pragma unroll
            for (int j = 0; j < 16; ++j)
              if (t0 + j < xend)
                (run ? run + j * rs : sc_row(sc, y, ldy, t0 + j))[f] = __float2bfloat16(dq(v[j], t0 + j) + b);
          } else {
#pragma unroll
            for (int j = 0; j < 16; ++j)
              if (t0 + j < N) ws[(int64_t(s) * N + t0 + j) * M + f] = dq(v[j], t0 + j);
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
  sc_publish(sc);
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                 "r"(S::TMEM_COLS));
  }
}

// ------------------------------------------------------------ stream-K
// Decode-shaped GEMMs (at most 256 tokens): one token tile covers every
// token, so the weight is read exactly once; a CTA owns MT x 128 features at
// a time, so the token tile is re-read from L2 only M / (128 MT) times. The
// (tile, k-iteration) space is cut into one contiguous range per CTA (all
// SMs busy, no wave tail). A tile whose K range spans several CTAs is
// finished by whichever CTA arrives last: every CTA writes its fp32 partial
// to its own workspace slot, fences, bumps the tile's counter; the one that
// sees the count complete adds the other partials and stores bf16 (and resets
// the counter for the next launch). No CTA ever waits for another.
constexpr int pow2_cols(int c) { return c <= 32 ? 32 : c <= 64 ? 64 : c <= 128 ? 128 : c <= 256 ? 256 : 512; }

template <int BN, int MT, int STAGES>
struct SkSmem {
  static constexpr int UM = kGemmBM * MT;
  static constexpr int A_BYTES = UM * kGemmBK * 2;
  static constexpr int B_BYTES = BN * kGemmBK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int ACC_COLS = MT * BN;
  static constexpr int NBUF = 2 * ACC_COLS <= 512 ? 2 : 1;
  static constexpr int TMEM_COLS = pow2_cols(NBUF * ACC_COLS);
  static constexpr size_t BYTES = 1024 + size_t(STAGES) * STAGE_BYTES + 256;
};

__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

template <int BN, int MT, int STAGES>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_streamk_kernel(const __grid_constant__ CUtensorMap tm_w,
                        const __grid_constant__ CUtensorMap tm_x, __nv_bfloat16* __restrict__ y,
                        int64_t ldy, const __nv_bfloat16* __restrict__ bias,
                        float* __restrict__ ws, int* __restrict__ counters, int M, int N, int K,
                        int per, int* status, int vec_out, int packed_kt,
                        const ScatterDesc sc) {
  using S = SkSmem<BN, MT, STAGES>;
  constexpr int UM = S::UM, NBUF = S::NBUF;
  extern __shared__ uint8_t smem_raw[];
  __shared__ int sh_last;
  __shared__ int sh_ok[2][4];
  __shared__ __align__(8) uint64_t fixbar;  // partner partials fetched into the idle ring
  __shared__ __align__(16) __nv_bfloat16 epi_stage[4 * 32 * 40];
  uint8_t* tiles =
      reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(tiles + size_t(STAGES) * S::STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_tiles = (N + BN - 1) / BN;
  const int m_units = (M + UM - 1) / UM;
  const int k_iters = (K + kGemmBK - 1) / kGemmBK;
  const int total = m_units * n_tiles * k_iters;
  const int cta = blockIdx.x;
  const int it_begin = min(total, cta * per), it_end = min(total, it_begin + per);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 4);
    }
    mbar_init(&fixbar, 1);
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

  // Segments of this CTA's range, natural order j = 0..nseg-1 (tile
  // first_tile + j). Processing order: a partial LAST segment goes first
  // (it is the beginning of a tile whose end the next CTA computes as its
  // first processed segment), then the rest in order. So both halves of a
  // split tile are computed early, and the CTA that finishes the tile finds
  // the other partials ready and never stores its own.
  const int first_tile = it_begin / k_iters;
  const int nseg = it_end > it_begin ? (it_end - 1) / k_iters - first_tile + 1 : 0;
  const bool tail_first = nseg >= 2 && ((it_end - 1) % k_iters + 1) < k_iters;
  auto seg_of = [&](int p, int& j, int& t, int& k0, int& k1) {
    j = tail_first ? (p == 0 ? nseg - 1 : p - 1) : p;
    t = first_tile + j;
    k0 = j == 0 ? it_begin % k_iters : 0;
    k1 = j == nseg - 1 ? (it_end - 1) % k_iters + 1 : k_iters;
  };

  if (warp == 0) {
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      for (int p = 0; p < nseg && ok; ++p) {
        int j, t, k0, k1;
        seg_of(p, j, t, k0, k1);
        const int w0 = (t / n_tiles) * UM, x0 = (t % n_tiles) * BN;
        for (int kk = k0; kk < k1; ++kk, ++it) {
          const int st = it % STAGES;
          if (!wait_or_abort(&empty[st], ((it / STAGES) & 1) ^ 1, abort_flag, status, 20)) {
            ok = false;
            break;
          }
          uint8_t* a = tiles + size_t(st) * S::STAGE_BYTES;
          mbar_arrive_expect_tx(&full[st], S::STAGE_BYTES);
          if (packed_kt) {  // tile-packed weights: one contiguous 16 KB box per 128 rows
#pragma unroll
            for (int mi = 0; mi < MT; ++mi)
              tma_load_2d(a + mi * kGemmBM * kGemmBK * 2, &tm_w, 0,
                          ((w0 / kGemmBM + mi) * packed_kt + kk) * kGemmBM, &full[st]);
          } else {
            tma_load_2d(a, &tm_w, kk * kGemmBK, w0, &full[st]);
          }
          tma_load_2d(a + S::A_BYTES, &tm_x, kk * kGemmBK, x0, &full[st]);
        }
      }
      if (!ok) {
        for (uint32_t j = it > STAGES ? it - STAGES : 0; j < it; ++j)
          for (uint32_t p = 0; p < (1u << 20); ++p)
            if (mbar_try_wait(&full[j % STAGES], (j / STAGES) & 1)) break;
      }
    }
  } else if (warp == 1) {
    // whole warp: warp-uniform waits, one elected lane issues
    {
      constexpr uint32_t idesc = instr_desc_bf16<BN>();
      uint32_t it = 0, tc = 0;
      bool ok = true;
      for (int p = 0; p < nseg && ok; ++p, ++tc) {
        int j, t, k0, k1;
        seg_of(p, j, t, k0, k1);
        const uint32_t buf = tc % NBUF;
        if (!wait_warp_or_abort(&tempty[buf], ((tc / NBUF) & 1) ^ 1, abort_flag, status, 21)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * S::ACC_COLS;
        for (int kk = k0; kk < k1; ++kk, ++it) {
          const int st = it % STAGES;
          if (!wait_warp_or_abort(&full[st], (it / STAGES) & 1, abort_flag, status, 22)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (elect_one()) {
            const uint8_t* a = tiles + size_t(st) * S::STAGE_BYTES;
            const uint64_t bd = smem_desc_sw128(a + S::A_BYTES);
#pragma unroll
            for (int q = 0; q < kGemmBK / 16; ++q) {
#pragma unroll
              for (int i = 0; i < MT; ++i) {
                const uint64_t ad = smem_desc_sw128(a + i * kGemmBM * kGemmBK * 2);
                umma_bf16(d_tmem + i * BN, ad + 2 * q, bd + 2 * q, idesc,
                          (kk > k0 || q > 0) ? 1u : 0u);
              }
            }
            umma_commit(&empty[st]);
          }
          __syncwarp();
        }
        if (!ok) break;
        if (elect_one()) umma_commit(&tfull[buf]);
        __syncwarp();
      }
      if (!ok && lane == 0) {
        for (uint32_t j = it > STAGES ? it - STAGES : 0; j < it; ++j)
          for (uint32_t p = 0; p < (1u << 20); ++p)
            if (mbar_try_wait(&empty[j % STAGES], (j / STAGES) & 1)) break;
      }
    }
  } else {
    const int q = warp & 3;
    const int slot_floats = UM * BN;
    uint32_t tc = 0, fix_uses = 0;
    for (int p = 0; p < nseg; ++p, ++tc) {
      int j, t, k0, k1;
      seg_of(p, j, t, k0, k1);
      const int m0 = (t / n_tiles) * UM, x0 = (t % n_tiles) * BN;
      const uint32_t buf = tc % NBUF;
      bool ok = true;
      for (uint32_t i = 0;; ++i) {
        bool r = mbar_try_wait(&tfull[buf], (tc / NBUF) & 1);
        if (__all_sync(0xffffffffu, r)) break;
        if (i > kWaitLimit || ((i & 255) == 255 && *abort_flag)) {
          if (lane == 0 && i > kWaitLimit) {
            set_status(status, kErrWaitTimeout, 23);
            *abort_flag = 1;
          }
          ok = false;
          break;
        }
      }
      // the four epilogue warps agree before any named barrier, so a warp
      // that gave up never leaves the others waiting at bar.sync
      if (lane == 0) sh_ok[tc & 1][q] = ok;
      epi_bar();
      ok = sh_ok[tc & 1][0] && sh_ok[tc & 1][1] && sh_ok[tc & 1][2] && sh_ok[tc & 1][3];
      if (!ok) break;
      tc_fence_after();
      const bool whole = k0 == 0 && k1 == k_iters;
      const uint32_t tq = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + buf * S::ACC_COLS;
      const int fl = q * 32 + lane;  // feature within a 128-row sub-tile
      bool last = whole;
      int cf = 0, cl = -1;
      if (!whole) {
        cf = (t * k_iters) / per;
        cl = ((t + 1) * k_iters - 1) / per;
        // every other CTA of this tile already done? then this one finishes
        // it without storing its own partial
        if (threadIdx.x == 64) {
          int done = *reinterpret_cast<volatile int*>(&counters[t]);
          int lst = done == cl - cf;
          if (lst) {
            __threadfence();  // acquire the other partials
            counters[t] = 0;
          }
          sh_last = lst;
        }
        epi_bar();
        last = sh_last != 0;
        epi_bar();
        if (!last) {
          // partial slot layout: [token column (BN)][feature (UM)] fp32: a
          // warp moves 32 consecutive features of one column per instruction
          float* wp = ws + size_t(j == 0 ? 2 * cta : 2 * cta + 1) * slot_floats;
#pragma unroll 1
          for (int i = 0; i < MT; ++i)
#pragma unroll 1
            for (int c = 0; c < BN / 32; ++c) {
              float v[32];
              tmem_ld32(tq + i * BN + c * 32, v);
#pragma unroll
              for (int jj = 0; jj < 32; ++jj)
                __stcg(wp + size_t(c * 32 + jj) * UM + i * kGemmBM + fl, v[jj]);
            }
          // release: the partial stores happen-before the counter bump
          epi_bar();
          if (threadIdx.x == 64) {
            __threadfence();
            const int old = atomicAdd(&counters[t], 1);
            const int lst = old == cl - cf;
            if (lst) {
              __threadfence();
              counters[t] = 0;
            }
            sh_last = lst;
          }
          epi_bar();
          last = sh_last != 0;
        }
      }
      // The CTA's last processed segment: producer and MMAs are done, so the
      // other CTAs' partials are fetched with bulk copies into the idle
      // shared-memory ring (one latency instead of one per chunk).
      const int others = whole ? 0 : cl - cf;
      const bool staged = last && others > 0 && p == nseg - 1 &&
                          size_t(others) * slot_floats * 4 <= size_t(STAGES) * S::STAGE_BYTES;
      if (staged) {
        if (threadIdx.x == 64) {
          asm volatile("fence.proxy.async;" ::: "memory");
          constexpr uint32_t kPiece = 32768;
          const uint32_t slot_bytes = uint32_t(slot_floats) * 4;
          mbar_arrive_expect_tx(&fixbar, uint32_t(others) * slot_bytes);
          int idx = 0;
          for (int o = cf; o <= cl; ++o) {
            if (o == cta) continue;
            const int slot = ((o * per) / k_iters == t) ? 2 * o : 2 * o + 1;
            const uint8_t* src = reinterpret_cast<const uint8_t*>(ws + size_t(slot) * slot_floats);
            for (uint32_t off = 0; off < slot_bytes; off += kPiece)
              bulk_g2s(tiles + size_t(idx) * slot_bytes + off, src + off,
                       min(kPiece, slot_bytes - off), &fixbar);
            ++idx;
          }
        }
        if (!mbar_wait_warp(&fixbar, fix_uses & 1, status, 24)) *abort_flag = 1;
        ++fix_uses;
      }
      if (last) {
        __nv_bfloat16* stage = epi_stage + q * 32 * 40;  // [32 tokens][40] bf16, padded rows
#pragma unroll 1
        for (int i = 0; i < MT; ++i) {
          const int f = m0 + i * kGemmBM + fl;
          const float b = (bias != nullptr && f < M) ? __bfloat162float(bias[f]) : 0.f;
#pragma unroll 1
          for (int c = 0; c < BN / 32; ++c) {
            float own[32], v[32];
            tmem_ld32(tq + i * BN + c * 32, own);
            // fixed summation order over the tile's CTAs (bitwise identical
            // results whichever CTA finishes the tile)
#pragma unroll
            for (int jj = 0; jj < 32; ++jj) v[jj] = (cf == cta || whole) ? own[jj] : 0.f;
            int idx = 0;
            for (int o = cf; o <= cl; ++o) {
              if (o == cta) {
                if (o != cf) {
#pragma unroll
                  for (int jj = 0; jj < 32; ++jj) v[jj] += own[jj];
                }
                continue;
              }
              const size_t off = size_t(c * 32) * UM + i * kGemmBM + fl;
              float r[32];
              if (staged) {
                const float* sp = reinterpret_cast<const float*>(tiles) + size_t(idx) * slot_floats + off;
#pragma unroll
                for (int jj = 0; jj < 32; ++jj) r[jj] = sp[size_t(jj) * UM];
              } else {
                const int slot = ((o * per) / k_iters == t) ? 2 * o : 2 * o + 1;
                const float* rp = ws + size_t(slot) * slot_floats + off;
#pragma unroll
                for (int jj = 0; jj < 32; ++jj) r[jj] = __ldcg(rp + size_t(jj) * UM);
              }
#pragma unroll
              for (int jj = 0; jj < 32; ++jj) v[jj] += r[jj];
              ++idx;
            }
            const int t0 = x0 + c * 32;
            if (vec_out) {
              // transpose through shared memory: 4 lanes write one token's
              // 32 features as 16-byte vectors
#pragma unroll
              for (int jj = 0; jj < 32; ++jj) stage[jj * 40 + lane] = __float2bfloat16(v[jj] + b);
              __syncwarp();
              const int fbase = m0 + i * kGemmBM + q * 32;
              int64_t rs;
              __nv_bfloat16* run = sc_run(sc, y, ldy, t0, 32, &rs);
#pragma unroll
              for (int r0 = 0; r0 < 32; r0 += 8) {
                const int row = r0 + (lane >> 2), part = lane & 3;
                const int fo = fbase + part * 8;
                if (t0 + row < N && fo < M)
                  *reinterpret_cast<uint4*>((run ? run + row * rs : sc_row(sc, y, ldy, t0 + row)) + fo) =
                      *reinterpret_cast<const uint4*>(stage + row * 40 + part * 8);
              }
              __syncwarp();
            } else if (f < M) {
#pragma unroll
              for (int jj = 0; jj < 32; ++jj)
                if (t0 + jj < N) sc_row(sc, y, ldy, t0 + jj)[f] = __float2bfloat16(v[jj] + b);
            }
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
  sc_publish(sc);
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
int64_t gemm2_launch(__nv_bfloat16* y, int64_t ldy, const torch::Tensor& x, const torch::Tensor& w,
                     const __nv_bfloat16* bias, int force, int force_bn, int force_splits,
                     int act);

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
// fp8 = true: 1-byte elements, 128 per 128-byte box row.
static CUtensorMap make_tmap(const void* ptr, int64_t rows, int64_t cols, int64_t ld, int box_rows,
                             bool fp8 = false) {
  CUtensorMap tm;
  const int es = fp8 ? 1 : 2;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * es)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(128 / es), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = get_encode()(&tm, fp8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                            2, const_cast<void*>(ptr), dims,
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

template <int BN, int STAGES, int Q = 0>
static void launch_gemm(const CUtensorMap& tw, const CUtensorMap& tx, __nv_bfloat16* y, int64_t ldy,
                        const __nv_bfloat16* bias, float* ws, int M, int N, int K, int splits,
                        const int32_t* goff = nullptr, int groups = 0,
                        const ScatterDesc& sc = ScatterDesc{}, const float* wscale = nullptr,
                        const float* xscale = nullptr) {
  using S = GemmSmem<BN, STAGES>;
  auto kern = gemm_tcgen05_kernel<BN, STAGES, Q>;
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
                                                       status_word_ptr(), goff, groups, sc, wscale,
                                                       xscale);
  SWIFT_CHECK_LAUNCH();
}

// ---- stream-K host side
struct SkBuffers {
  float* ws = nullptr;
  int* counters = nullptr;
};
constexpr int kSkMaxTiles = 8192;
constexpr size_t kSkSlotFloats = 256 * 256;  // UM * BN at most

// Per-device workspace (two partial slots per CTA) and zeroed tile counters,
// allocated once and kept for the process (CUDA graphs capture the pointers).
static SkBuffers& sk_buffers() {
  static SkBuffers b[64];
  int dev;
  cudaGetDevice(&dev);
  if (!b[dev].ws) {
    SWIFT_CHECK_CUDA(cudaMalloc(&b[dev].ws, size_t(2) * num_sms() * kSkSlotFloats * sizeof(float)));
    SWIFT_CHECK_CUDA(cudaMalloc(&b[dev].counters, kSkMaxTiles * sizeof(int)));
    SWIFT_CHECK_CUDA(cudaMemset(b[dev].counters, 0, kSkMaxTiles * sizeof(int)));
    SWIFT_CHECK_CUDA(cudaDeviceSynchronize());
  }
  return b[dev];
}

// Stream-K planning parameters, process wide. mode: 1 (default) stream-K
// where the plan below picks it, 0 never, 2 for every shape it supports
// (initial value from SWIFT_GEMM_STREAMK, read once); mt: 128-row feature
// sub-tiles per unit (1 or 2); min_per: fewest k-iterations per CTA. Only
// gemm_streamk_config() changes them (tests force split tiles with it).
struct SkConfig {
  int mode = -1, mt = 1, min_per = 32;
};
static SkConfig& sk_config() {
  static SkConfig c;
  if (c.mode < 0) {
    const char* v = std::getenv("SWIFT_GEMM_STREAMK");
    c.mode = v && *v ? std::atoi(v) : 1;
  }
  return c;
}

void gemm_streamk_config(int64_t mode, int64_t mt, int64_t min_per) {
  TORCH_CHECK(mode >= 0 && mode <= 2 && (mt == 1 || mt == 2) && min_per >= 1);
  SkConfig& c = sk_config();
  c.mode = static_cast<int>(mode);
  c.mt = static_cast<int>(mt);
  c.min_per = static_cast<int>(min_per);
}

template <int BN, int MT>
static void launch_sk(const void* w, int64_t ldw, const void* x, int64_t ldx, __nv_bfloat16* y,
                      int64_t ldy, const __nv_bfloat16* bias, int M, int N, int K, int grid,
                      int per, int packed_kt = 0, const ScatterDesc& sc = ScatterDesc{}) {
  // 16-byte output vectors need 8-feature groups that stay inside rows
  const int vec_out = (M % 8 == 0 && ldy % 8 == 0 && reinterpret_cast<uintptr_t>(y) % 16 == 0) ? 1 : 0;
  constexpr int SB = SkSmem<BN, MT, 1>::STAGE_BYTES;
  constexpr int STAGES = std::min(8, (200 * 1024) / SB);
  using S = SkSmem<BN, MT, STAGES>;
  auto kern = gemm_streamk_kernel<BN, MT, STAGES>;
  static bool attr[64] = {false};
  int dev;
  cudaGetDevice(&dev);
  if (!attr[dev]) {
    SWIFT_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          static_cast<int>(S::BYTES)));
    attr[dev] = true;
  }
  SkBuffers& b = sk_buffers();
  // packed: [ceil(M/128) * KT * 128 rows, 64 cols], one 128-row box per tile
  CUtensorMap tw = packed_kt
                       ? make_tmap(w, int64_t((M + kGemmBM - 1) / kGemmBM) * packed_kt * kGemmBM,
                                   kGemmBK, kGemmBK, kGemmBM)
                       : make_tmap(w, M, K, ldw, S::UM);
  CUtensorMap tx = make_tmap(x, N, K, ldx, BN);
  kern<<<grid, kGemmThreads, S::BYTES, cur_stream()>>>(tw, tx, y, ldy, bias, b.ws, b.counters, M,
                                                       N, K, per, status_word_ptr(), vec_out,
                                                       packed_kt, sc);
  SWIFT_CHECK_LAUNCH();
}


// Stream-K plan for tokens N <= 256: token tile BN (one tile), MT x 128
// features per unit, grid and iterations per CTA. false: not applicable.
static void plan(int M, int N, int K, int* bn, int* splits);

// Stream-K for decode-shaped GEMMs (N <= 256 tokens, and mixed steps of up
// to 2048 tokens where the rule below says so; SWIFT_GEMM_STREAMK=0 turns it
// off, 2 forces it). Token tile: the smallest power of two >= N (>= 32), halved
// from 256 to 128 while the feature tiles x 2 still fit two waves (measured
// on B200 for the Llama-2-7B projections: the narrower tile halves the
// partial-sum traffic, which outweighs the second read of each weight tile,
// served from L2). At least 32 k-iterations per CTA.
static bool sk_plan(int M, int N, int K, int* bn, int* mt, int* grid, int* per,
                    bool force = false) {
  const SkConfig& cfg = sk_config();
  const int mode = force ? 2 : cfg.mode;
  if (N > 2048 || mode == 0) return false;
  const int sms = num_sms();
  if (mode == 1 && N > 256) {
    // more tokens: stream-K only where the data-parallel plan would split K
    // or, up to 512 tokens, has few feature tiles (measured on B200)
    int dbn, dsplits;
    plan(M, N, K, &dbn, &dsplits);
    const int m_tiles = (M + kGemmBM - 1) / kGemmBM;
    if (!(dsplits > 1 || (N <= 512 && m_tiles <= 96))) return false;
  }
  int b = 32;
  while (b < N && b < 256) b *= 2;
  if (N > 256) {
    // several token tiles: the width (128 or 256) that pads N the least
    const int pad128 = (N + 127) / 128 * 128 - N, pad256 = (N + 255) / 256 * 256 - N;
    b = pad128 < pad256 ? 128 : 256;
  } else if (b == 256 && int64_t((M + kGemmBM - 1) / kGemmBM) * 2 <= int64_t(2) * sms) {
    b = 128;
  }
  const int k_iters = (K + kGemmBK - 1) / kGemmBK;
  const int m = cfg.mt;
  const int units = (M + 128 * m - 1) / (128 * m) * ((N + b - 1) / b);
  if (units > kSkMaxTiles) return false;
  const int64_t total = int64_t(units) * k_iters;
  // at least 32 k-iterations per CTA, but never more than one tile's worth
  // (short K: one CTA per tile keeps every tile's CTA busy)
  const int min_per = std::max(1, std::min(cfg.min_per, k_iters));
  int g = static_cast<int>(std::min<int64_t>(sms, (total + min_per - 1) / min_per));
  g = std::max(g, 1);
  int p = static_cast<int>((total + g - 1) / g);
  g = static_cast<int>((total + p - 1) / p);
  *bn = b;
  *mt = m;
  *grid = g;
  *per = p;
  return true;
}

static bool gemm_streamk(__nv_bfloat16* y, torch::Tensor x, torch::Tensor w,
                         const __nv_bfloat16* bias, int64_t T, int64_t ldx, int64_t ldy,
                         int Mp = 0, int packed_kt = 0, const ScatterDesc& sc = ScatterDesc{}) {
  const int M = packed_kt ? Mp : static_cast<int>(w.size(0));
  const int K = static_cast<int>(x.size(-1));
  const int N = static_cast<int>(T);
  int bn, mt, grid, per;
  if (!sk_plan(M, N, K, &bn, &mt, &grid, &per, sc.k > 0)) return false;
  const void* wp = w.data_ptr();
  const void* xp = x.data_ptr();
  const int64_t ldw = w.stride(0);
#define SK_CASE(B, MTV) \
  if (bn == B && mt == MTV) { launch_sk<B, MTV>(wp, ldw, xp, ldx, y, ldy, bias, M, N, K, grid, per, packed_kt, sc); return true; }
  SK_CASE(32, 1) SK_CASE(32, 2) SK_CASE(64, 1) SK_CASE(64, 2)
  SK_CASE(128, 1) SK_CASE(128, 2) SK_CASE(256, 1) SK_CASE(256, 2)
#undef SK_CASE
  return false;
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
  // only as many splits as non-empty K ranges of ceil(k_iters / s) steps
  if (s > 1) s = (k_iters + (k_iters + s - 1) / s - 1) / ((k_iters + s - 1) / s);
  *bn = b;
  *splits = s;
}

// out [T, N] (row stride may exceed N), x [T, K], w [N, K], bias [N] or None.
// Split-K partials go to `ws` when given (fp32, >= splits*T*N), else to a
// fresh tensor. Returns the number of kernels launched.
static int64_t gemm_impl(__nv_bfloat16* y, int64_t ldy, torch::Tensor x, torch::Tensor w,
                         c10::optional<torch::Tensor> bias, const ScatterDesc& sc) {
  CHECK_BF16(x);
  CHECK_BF16(w);
  const int64_t K = x.size(-1);
  const int64_t T = x.numel() / K;
  const int64_t M = w.size(0);
  TORCH_CHECK(w.size(1) == K, "gemm: K mismatch");
  TORCH_CHECK(x.stride(-1) == 1 && w.stride(1) == 1, "gemm: inner dim must be contiguous");
  TORCH_CHECK(K % 8 == 0, "gemm: K must be a multiple of 8 (16-byte TMA rows)");
  const int64_t ldx = x.dim() >= 2 ? x.stride(-2) : K;
  TORCH_CHECK(ldx % 8 == 0 && w.stride(0) % 8 == 0, "gemm: row strides must be 16-byte multiples");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0 &&
                  reinterpret_cast<uintptr_t>(w.data_ptr()) % 16 == 0,
              "gemm: operands must be 16-byte aligned");
  if (T == 0) return 0;
  const __nv_bfloat16* bp =
      bias.has_value() ? reinterpret_cast<const __nv_bfloat16*>(bias.value().data_ptr<at::BFloat16>())
                       : nullptr;
  // The 2-SM kernel (gemm_2sm.cu) where it measured faster on B200 (graph
  // replays of back-to-back calls, weights streamed from HBM): every shape
  // with more than 256 tokens; with at most 256 tokens, weights of >= 12288
  // rows (data-parallel 256 x 256 pair tiles up to 16384 rows, swapped
  // operands above). Narrower decode weights stay on the one-SM stream-K
  // kernel below.
  if (sc.k == 0 && (T > 256 || M >= 12288))
    return gemm2_launch(y, ldy, x, w, bp, T > 256 ? -1 : (M > 16384 ? 2 : 0), 0, 1, 0);
  if (gemm_streamk(y, x, w, bp, T, ldx, ldy, 0, 0, sc)) return 1;
  int bn, splits;
  plan(static_cast<int>(M), static_cast<int>(T), static_cast<int>(K), &bn, &splits);
  if (sc.k > 0) splits = 1;  // the fused scatter stores final values only
  CUtensorMap tw = make_tmap(w.data_ptr(), M, K, w.stride(0), kGemmBM);
  CUtensorMap tx = make_tmap(x.data_ptr(), T, K, ldx, bn);
  torch::Tensor ws;
  float* wsp = nullptr;
  if (splits > 1) {
    ws = torch::empty({splits, T, M}, x.options().dtype(torch::kFloat));
    wsp = ws.data_ptr<float>();
  }
  const int Mi = static_cast<int>(M), Ni = static_cast<int>(T), Ki = static_cast<int>(K);
  switch (bn) {
    case 16: launch_gemm<16, 8>(tw, tx, y, ldy, bp, wsp, Mi, Ni, Ki, splits, nullptr, 0, sc); break;
    case 32: launch_gemm<32, 8>(tw, tx, y, ldy, bp, wsp, Mi, Ni, Ki, splits, nullptr, 0, sc); break;
    case 64: launch_gemm<64, 8>(tw, tx, y, ldy, bp, wsp, Mi, Ni, Ki, splits, nullptr, 0, sc); break;
    case 128: launch_gemm<128, 6>(tw, tx, y, ldy, bp, wsp, Mi, Ni, Ki, splits, nullptr, 0, sc); break;
    default: launch_gemm<256, 4>(tw, tx, y, ldy, bp, wsp, Mi, Ni, Ki, splits, nullptr, 0, sc); break;
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

int64_t gemm(torch::Tensor out, torch::Tensor x, torch::Tensor w, c10::optional<torch::Tensor> bias) {
  CHECK_BF16(out);
  TORCH_CHECK(out.stride(-1) == 1, "gemm: inner dim must be contiguous");
  const int64_t ldy = out.dim() >= 2 ? out.stride(-2) : w.size(0);
  return gemm_impl(reinterpret_cast<__nv_bfloat16*>(out.data_ptr<at::BFloat16>()), ldy, x, w,
                   bias, ScatterDesc{});
}

// Weights in tile-packed order: w_packed [ceil(M/128), ceil(K/64), 128, 64]
// (zero padded), so every 128 x 64 weight tile is one contiguous 16 KB block.
// Decode-shaped only (tokens <= 256). out [T, M], x [T, K].
int64_t gemm_packed(torch::Tensor out, torch::Tensor x, torch::Tensor wp, int64_t M,
                    c10::optional<torch::Tensor> bias) {
  CHECK_BF16(x);
  CHECK_BF16(wp);
  CHECK_BF16(out);
  TORCH_CHECK(wp.dim() == 4 && wp.size(2) == kGemmBM && wp.size(3) == kGemmBK && wp.is_contiguous());
  const int64_t K = x.size(-1), T = x.numel() / K;
  TORCH_CHECK(wp.size(0) == (M + kGemmBM - 1) / kGemmBM && wp.size(1) == (K + kGemmBK - 1) / kGemmBK);
  TORCH_CHECK(T <= 256, "gemm_packed: at most 256 tokens");
  if (T == 0) return 0;
  const int64_t ldx = x.dim() >= 2 ? x.stride(-2) : K;
  const int64_t ldy = out.dim() >= 2 ? out.stride(-2) : M;
  const __nv_bfloat16* bp =
      bias.has_value() ? reinterpret_cast<const __nv_bfloat16*>(bias.value().data_ptr<at::BFloat16>())
                       : nullptr;
  TORCH_CHECK(gemm_streamk(reinterpret_cast<__nv_bfloat16*>(out.data_ptr<at::BFloat16>()), x, wp,
                           bp, T, ldx, ldy, static_cast<int>(M), static_cast<int>(wp.size(1))),
              "gemm_packed: no stream-K plan");
  return 1;
}

// ---- FP8 (E4M3) weights and activations
// Per-row symmetric quantisation: scale = max|row| / 448 (the largest finite
// E4M3 value), q = round-to-nearest E4M3 of x / scale, saturating. Used for
// weights at load time (one scale per output feature) and for activations
// before every FP8 GEMM (one scale per token).
__global__ void quantize_e4m3_kernel(uint8_t* __restrict__ q, float* __restrict__ scale,
                                     const __nv_bfloat16* __restrict__ x, int K, int64_t ldx) {
  const int64_t r = blockIdx.x;
  const __nv_bfloat16* row = x + r * ldx;
  float m = 0.f;
  for (int k = threadIdx.x; k < K; k += blockDim.x) m = fmaxf(m, fabsf(__bfloat162float(row[k])));
  __shared__ float red[32];
  m = warp_max(m);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x + 31) / 32 ? red[threadIdx.x] : 0.f;
    v = warp_max(v);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  const float s = fmaxf(red[0] / 448.f, 1e-12f);
  const float inv = 1.f / s;
  if (threadIdx.x == 0) scale[r] = s;
  for (int k = threadIdx.x; k < K; k += blockDim.x)
    q[r * K + k] = __nv_cvt_float_to_fp8(__bfloat162float(row[k]) * inv, __NV_SATFINITE, __NV_E4M3);
}

void quantize_e4m3(torch::Tensor q, torch::Tensor scale, torch::Tensor x) {
  CHECK_BF16(x);
  TORCH_CHECK(q.scalar_type() == at::kByte && q.is_contiguous() && scale.scalar_type() == at::kFloat);
  const int64_t K = x.size(-1), R = x.numel() / K;
  TORCH_CHECK(x.stride(-1) == 1 && q.numel() == R * K && scale.numel() == R);
  if (R == 0) return;
  const int64_t ldx = x.dim() >= 2 ? x.stride(-2) : K;
  quantize_e4m3_kernel<<<static_cast<unsigned>(R), 256, 0, cur_stream()>>>(
      q.data_ptr<uint8_t>(), scale.data_ptr<float>(),
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr<at::BFloat16>()), static_cast<int>(K), ldx);
  SWIFT_CHECK_LAUNCH();
}

// out [T, M] bf16 = (xq * xscale) . (wq * wscale)^T (+ bias), on
// tcgen05.mma kind::f8f6f4. xq [T, K], wq [M, K] uint8 holding E4M3 bits,
// K a multiple of 16. Returns launches.
template <int Q>
static int64_t gemm_q8(torch::Tensor out, torch::Tensor xq, torch::Tensor xscale, torch::Tensor wq,
                       torch::Tensor wscale, c10::optional<torch::Tensor> bias) {
  CHECK_BF16(out);
  TORCH_CHECK((xq.scalar_type() == at::kByte || xq.scalar_type() == at::kChar) &&
              (wq.scalar_type() == at::kByte || wq.scalar_type() == at::kChar));
  TORCH_CHECK(xq.is_contiguous() && wq.is_contiguous() && out.stride(-1) == 1);
  TORCH_CHECK(xscale.scalar_type() == at::kFloat && wscale.scalar_type() == at::kFloat);
  const int64_t K = xq.size(-1), T = xq.numel() / K, M = wq.size(0);
  TORCH_CHECK(wq.size(1) == K && K % 16 == 0, "8-bit GEMM: K must match and be a multiple of 16");
  TORCH_CHECK(xscale.numel() == T && wscale.numel() == M);
  if (T == 0) return 0;
  const int64_t ldy = out.dim() >= 2 ? out.stride(-2) : M;
  int bn, splits;
  plan(static_cast<int>(M), static_cast<int>(T), static_cast<int>(K / 2), &bn, &splits);
  CUtensorMap tw = make_tmap(wq.data_ptr(), M, K, K, kGemmBM, true);
  CUtensorMap tx = make_tmap(xq.data_ptr(), T, K, K, bn, true);
  auto y = reinterpret_cast<__nv_bfloat16*>(out.data_ptr<at::BFloat16>());
  const __nv_bfloat16* bp =
      bias.has_value() ? reinterpret_cast<const __nv_bfloat16*>(bias.value().data_ptr<at::BFloat16>())
                       : nullptr;
  torch::Tensor ws;
  float* wsp = nullptr;
  if (splits > 1) {
    ws = torch::empty({splits, T, M}, out.options().dtype(torch::kFloat));
    wsp = ws.data_ptr<float>();
  }
  const int Mi = static_cast<int>(M), Ni = static_cast<int>(T), Ki = static_cast<int>(K);
  const float* wsc = wscale.data_ptr<float>();
  const float* xsc = xscale.data_ptr<float>();
  const ScatterDesc none{};
  switch (bn) {
    case 16: launch_gemm<16, 8, Q>(tw, tx, y, ldy, bp, wsp, Mi, Ni, Ki, splits, nullptr, 0, none, wsc, xsc); break;
    case 32: launch_gemm<32, 8, Q>(tw, tx, y, ldy, bp, wsp, Mi, Ni, Ki, splits, nullptr, 0, none, wsc, xsc); break;
    case 64: launch_gemm<64, 8, Q>(tw, tx, y, ldy, bp, wsp, Mi, Ni, Ki, splits, nullptr, 0, none, wsc, xsc); break;
    case 128: launch_gemm<128, 6, Q>(tw, tx, y, ldy, bp, wsp, Mi, Ni, Ki, splits, nullptr, 0, none, wsc, xsc); break;
    default: launch_gemm<256, 4, Q>(tw, tx, y, ldy, bp, wsp, Mi, Ni, Ki, splits, nullptr, 0, none, wsc, xsc); break;
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

int64_t gemm_e4m3(torch::Tensor out, torch::Tensor xq, torch::Tensor xscale, torch::Tensor wq,
                  torch::Tensor wscale, c10::optional<torch::Tensor> bias) {
  return gemm_q8<1>(out, xq, xscale, wq, wscale, bias);
}

// out [T, M] bf16 = (xq * xscale) . (wq * wscale)^T (+ bias) on
// tcgen05.mma kind::i8 (exact int32 accumulation). xq [T, K], wq [M, K]
// int8 (per-row symmetric), K a multiple of 16. Returns launches.
int64_t gemm_s8(torch::Tensor out, torch::Tensor xq, torch::Tensor xscale, torch::Tensor wq,
                torch::Tensor wscale, c10::optional<torch::Tensor> bias) {
  return gemm_q8<2>(out, xq, xscale, wq, wscale, bias);
}

// Per-row symmetric int8: scale = max|row| / 127, q = round-to-nearest of
// x / scale (ties to even), so |q| <= 127.
__global__ void quantize_s8_kernel(int8_t* __restrict__ q, float* __restrict__ scale,
                                   const __nv_bfloat16* __restrict__ x, int K, int64_t ldx) {
  const int64_t r = blockIdx.x;
  const __nv_bfloat16* row = x + r * ldx;
  float m = 0.f;
  for (int k = threadIdx.x; k < K; k += blockDim.x) m = fmaxf(m, fabsf(__bfloat162float(row[k])));
  __shared__ float red[32];
  m = warp_max(m);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x + 31) / 32 ? red[threadIdx.x] : 0.f;
    v = warp_max(v);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  const float sc = fmaxf(red[0] / 127.f, 1e-12f);
  const float inv = 1.f / sc;
  if (threadIdx.x == 0) scale[r] = sc;
  for (int k = threadIdx.x; k < K; k += blockDim.x) {
    const int v = __float2int_rn(__bfloat162float(row[k]) * inv);
    q[r * K + k] = static_cast<int8_t>(max(-127, min(127, v)));
  }
}

void quantize_s8(torch::Tensor q, torch::Tensor scale, torch::Tensor x) {
  CHECK_BF16(x);
  TORCH_CHECK(q.scalar_type() == at::kChar && q.is_contiguous() && scale.scalar_type() == at::kFloat);
  const int64_t K = x.size(-1), R = x.numel() / K;
  TORCH_CHECK(x.stride(-1) == 1 && q.numel() == R * K && scale.numel() == R);
  if (R == 0) return;
  const int64_t ldx = x.dim() >= 2 ? x.stride(-2) : K;
  quantize_s8_kernel<<<static_cast<unsigned>(R), 256, 0, cur_stream()>>>(
      q.data_ptr<int8_t>(), scale.data_ptr<float>(),
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr<at::BFloat16>()), static_cast<int>(K), ldx);
  SWIFT_CHECK_LAUNCH();
}

// [token tile, splits, stream-K features-per-unit / 128 (0: not stream-K),
//  grid, k-iterations per CTA]
std::vector<int64_t> gemm_plan(int64_t M, int64_t N, int64_t K) {
  int bn, s, mt, grid, per;
  if (sk_plan(static_cast<int>(M), static_cast<int>(N), static_cast<int>(K), &bn, &mt, &grid, &per))
    return {bn, 1, mt, grid, per};
  plan(static_cast<int>(M), static_cast<int>(N), static_cast<int>(K), &bn, &s);
  return {bn, s, 0, 0, 0};
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
