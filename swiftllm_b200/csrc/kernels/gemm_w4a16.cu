// Weight-only int4 GEMM (W4A16: GPTQ / AWQ style group quantisation) on the
// 5th-generation tensor cores.
//
//   Y[T, M] = X[T, K] . W[M, K]^T (+ bias),  W[m, k] = (q[m, k] - z[g, m]) * s[g, m]
//   with q in [0, 15], g = k / group, bf16 activations and outputs.
//
// The reference declares gemm_int4 (crates/swiftllm-cuda/src/bindings.rs:245-288)
// and the GPTQ / AWQ methods (crates/swiftllm-core/src/config.rs:184-215)
// without a kernel. Decode is bound by weight bytes, so a 4-bit weight moves a
// quarter of the bf16 bytes; the dequantisation happens in shared memory,
// next to the tensor cores, and the MMA itself is the plain bf16
// tcgen05.mma.kind::f16 with fp32 accumulators in TMEM.
//
// Weight layout (built once at load by ops.int4): qp [ceil(M/128), 2*ceil(K/128),
// 128, 32] bytes: the 128 x 64 code tile of one (feature tile, 64-wide K
// slice) is one contiguous 4 KB block, and a k step (128 of K) fetches two
// consecutive tiles with one 256-row tensor-TMA box. Inside a row,
// the 4 bytes of 16-byte output chunk c (K elements 8c .. 8c+7) form one
// little-endian word whose nibble at bit 4j holds element 2j and the nibble at
// bit 16 + 4j holds element 2j + 1 (j = 0..3); then
//   ((word >> 4j) & 0x000F000F) | 0x43004300
// is the bf16 pair (128 + q[2j], 128 + q[2j+1]) with one LOP3 and a shift.
// Per-(group, feature) parameters sz [G, Mpad] are bf16 pairs (128 + z, s):
// (pair - (128 + z)) is exact in bf16 and the multiply by s rounds once, so
// each dequantised weight equals bf16((q - z) * s) exactly.
//
// CTA (14 warps, one per SM, persistent over output tiles), two rings:
//   codes ring (RSTAGES slots of 9 KB: the two 4 KB code tiles of one k step
//   and the 512-byte scale row of each tile's group) and operand ring
//   (STAGES slots: two 128 x 64 bf16 A sub-tiles the dequantisation writes
//   and the two BN x 64 activation sub-tiles). The codes ring runs several
//   k steps ahead of the dequantisation.
//   warp 0      codes producer: three tensor-TMA loads per k step;
//   warp 1      TMEM allocation; one elected lane issues the eight MMAs of a
//               k step; tcgen05.commit frees operand stages / publishes
//               finished tiles;
//   warps 2-5   epilogue: tcgen05.ld, bias, bf16 stores or fp32 split-K
//               partials; two TMEM accumulators overlap tile i's epilogue
//               with tile i+1's MMAs;
//   warps 6-13  dequantisation, 2 groups of 4 warps taking k steps in turn:
//               wait for the operand stage to be free (the group's first
//               warp then requests its activation sub-tiles by 2-D TMA,
//               128-byte swizzle, no multicast), read the codes (freeing the
//               codes slot), one thread per weight row expands 2 x 64
//               nibbles into the K-major 128-byte-swizzled bf16 A sub-tiles
//               (chunk c of row r stored at chunk c ^ (r & 7)), then
//               fence.proxy.async so the tensor core sees the writes.
// Every mbarrier wait is bounded (status word + CTA abort flag; in-flight
// copies and MMAs are drained and TMEM freed before the CTA returns).
#include <cudaTypedefs.h>

#include <algorithm>

#include <cuda_fp8.h>

#include "common.cuh"
#include "tma_util.cuh"

namespace swift {
namespace w4 {

constexpr int BM = 128, BK = 64;               // one packed code tile: 128 rows x 64 K
constexpr int KSUB = 2, KSTEP = BK * KSUB;      // a k step covers two code tiles (128 K)
constexpr int kDqGroups = 2;                     // dequantisation groups of 4 warps
constexpr int kThreads = (6 + 4 * kDqGroups) * 32;  // 448
constexpr int kRawBytes = KSUB * BM * BK / 2;   // 8 KB of codes per k step
constexpr int kScBytes = KSUB * BM * 4;         // a scale word per row and code tile
constexpr int kRawRegion = kRawBytes + kScBytes;  // one codes-ring slot
constexpr uint32_t kWaitLimit = 1u << 25;

template <int BN, int STAGES, int RSTAGES>
struct Smem {
  static constexpr int A_SUB = BM * BK * 2;   // one 128 x 64 bf16 swizzled sub-tile
  static constexpr int B_SUB = BN * BK * 2;
  static constexpr int A_BYTES = KSUB * A_SUB;
  static constexpr int B_BYTES = KSUB * B_SUB;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;  // bf16 operands of one k step
  static constexpr int TMEM_COLS = (2 * BN) <= 32    ? 32
                                   : (2 * BN) <= 64  ? 64
                                   : (2 * BN) <= 128 ? 128
                                   : (2 * BN) <= 256 ? 256
                                                     : 512;
  static constexpr size_t BYTES =
      1024 + size_t(STAGES) * STAGE_BYTES + size_t(RSTAGES) * kRawRegion + 512;
};

__device__ __forceinline__ bool wait_one(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                         int* status, int where) {
  for (uint32_t i = 0; i < kWaitLimit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255) == 255 && *abort_flag) return false;
  }
  set_status(status, kErrWaitTimeout, where);
  *abort_flag = 1;
  return false;
}
// all lanes poll; the warp proceeds together
__device__ __forceinline__ bool wait_warp(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
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
__device__ __forceinline__ bool elect() {
  uint32_t pred;
  asm volatile("{\n .reg .pred p;\n elect.sync _|p, 0xffffffff;\n selp.u32 %0, 1, 0, p;\n}\n"
               : "=r"(pred));
  return pred != 0;
}
// K-major, 128-byte swizzle descriptor (8-row atoms 1024 B apart, version 1)
__device__ __forceinline__ uint64_t desc_sw128(const void* p) {
  uint64_t d = static_cast<uint64_t>((smem_u32(p) & 0x3FFFF) >> 4);
  d |= static_cast<uint64_t>(1) << 16;
  d |= static_cast<uint64_t>(1024 >> 4) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}
// bf16 x bf16 -> f32, both K-major, N = BN, M = 128
template <int BN>
__host__ __device__ constexpr uint32_t idesc() {
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(BN >> 3) << 17) |
         (static_cast<uint32_t>(BM >> 4) << 24);
}
__device__ __forceinline__ void mma(uint32_t d, uint64_t a, uint64_t b, uint32_t id, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d),
      "l"(a), "l"(b), "r"(id), "r"(acc));
}
__device__ __forceinline__ void commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void ld32(uint32_t taddr, float (&v)[32]) {
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
__device__ __forceinline__ void ld16(uint32_t taddr, float (&v)[16]) {
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
__device__ __forceinline__ uint32_t bf2_as_u32(__nv_bfloat162 v) {
  return *reinterpret_cast<uint32_t*>(&v);
}
__device__ __forceinline__ __nv_bfloat162 u32_as_bf2(uint32_t v) {
  return *reinterpret_cast<__nv_bfloat162*>(&v);
}
// 8 int4 (one packed word, order above) -> 4 bf16 pairs (q - z) * s
__device__ __forceinline__ uint4 dequant8(uint32_t w, __nv_bfloat162 zb, __nv_bfloat162 s) {
  uint32_t o[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t p = ((w >> (4 * j)) & 0x000F000Fu) | 0x43004300u;
    o[j] = bf2_as_u32(__hmul2(__hsub2(u32_as_bf2(p), zb), s));
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}
// NVFP4 codes: each nibble is E2M1 (bit 3 sign, bits 0-2 magnitude code
// 0..7 = 0, 0.5, 1, 1.5, 2, 3, 4, 6), same nibble order as above. The bf16
// bits of the magnitudes are looked up with byte permutes: high bytes
// {00,3F,3F,3F,40,40,40,40}, low bytes {00,00,80,C0,00,40,80,C0}; the sign
// bit moves to bit 15 / 31; one multiply by the block scale (a bf16 pair)
// rounds once.
__device__ __forceinline__ uint4 dequant8_fp4(uint32_t w, __nv_bfloat162 s) {
  constexpr uint32_t kHi0 = 0x3F3F3F00u, kHi1 = 0x40404040u;
  constexpr uint32_t kLo0 = 0xC0800000u, kLo1 = 0xC0804000u;
  const uint32_t mag = w & 0x77777777u;
  const uint32_t se = mag & 0xFFFFu, so = mag >> 16;  // elements 0,2,4,6 / 1,3,5,7
  const uint32_t hiE = __byte_perm(kHi0, kHi1, se), loE = __byte_perm(kLo0, kLo1, se);
  const uint32_t hiO = __byte_perm(kHi0, kHi1, so), loO = __byte_perm(kLo0, kLo1, so);
  const uint32_t a0 = __byte_perm(loE, loO, 0x5140), b0 = __byte_perm(hiE, hiO, 0x5140);
  const uint32_t a1 = __byte_perm(loE, loO, 0x7362), b1 = __byte_perm(hiE, hiO, 0x7362);
  uint32_t o[4] = {__byte_perm(a0, b0, 0x5140), __byte_perm(a0, b0, 0x7362),
                   __byte_perm(a1, b1, 0x5140), __byte_perm(a1, b1, 0x7362)};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    o[j] |= ((w >> (4 * j)) & 0x00080008u) << 12;
    o[j] = bf2_as_u32(__hmul2(u32_as_bf2(o[j]), s));
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// qp: packed int4 tiles; sz: [G, Mpad] (128 + z, s) bf16 pairs; group is a
// multiple of 64. ws: fp32 split-K partials [splits, N, M] when splits > 1.
// FMT 0: int4 codes with (128 + z, s) bf16 pairs per group; FMT 1: NVFP4
// (E2M1 codes, four E4M3 block scales per row and k step in the scale word,
// times the per-tensor gscale).
template <int BN, int STAGES, int RSTAGES, int FMT>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_w4a16_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_q,
                      const __grid_constant__ CUtensorMap tm_s, __nv_bfloat16* __restrict__ y, int64_t ldy,
                      const __nv_bfloat16* __restrict__ bias, float* __restrict__ ws, int M, int N,
                      int K, int Mpad, int group, int splits, int* status, float gscale) {
  using S = Smem<BN, STAGES, RSTAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* tiles =
      reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* rring = tiles + size_t(STAGES) * S::STAGE_BYTES;  // int4 codes + (z, s) rows
  uint64_t* bfull = reinterpret_cast<uint64_t*>(rring + size_t(RSTAGES) * kRawRegion);
  uint64_t* afull = bfull + STAGES;    // dequantised A tile written (4 warp arrivals)
  uint64_t* abempty = afull + STAGES;  // MMAs of the operand stage done
  uint64_t* rfull = abempty + STAGES;  // codes + scales landed
  uint64_t* rempty = rfull + RSTAGES;  // codes read by the dequantisation warps (4 arrivals)
  uint64_t* tfull = rempty + RSTAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m_tiles = (M + BM - 1) / BM;
  const int n_tiles = (N + BN - 1) / BN;
  const int k_iters = (K + KSTEP - 1) / KSTEP;  // code tiles per feature tile: KSUB * k_iters
  const int k_per = (k_iters + splits - 1) / splits;
  const int total = m_tiles * n_tiles * splits;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&bfull[s], 1);
      mbar_init(&afull[s], 4);
      mbar_init(&abempty[s], 1);
    }
    for (int s = 0; s < RSTAGES; ++s) {
      mbar_init(&rfull[s], 1);
      mbar_init(&rempty[s], 4);
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
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem_base = *tmem_slot;

  // tile t -> split s (outermost), feature tile m, token tile (n fastest, so
  // CTAs running together share the weight tile through L2)
  auto decode = [&](int t, int& m, int& x0, int& s) {
    s = t / (m_tiles * n_tiles);
    const int r = t % (m_tiles * n_tiles);
    m = r / n_tiles;
    x0 = (r % n_tiles) * BN;
  };
  auto stage = [&](int st) { return tiles + size_t(st) * S::STAGE_BYTES; };
  auto rstage = [&](int r) { return rring + size_t(r) * kRawRegion; };

  if (warp == 0) {
    // codes producer: runs up to RSTAGES k steps ahead of the dequantisation
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
        int m, x0, s;
        decode(t, m, x0, s);
        const int k0 = s * k_per, k1 = min(k_iters, k0 + k_per);
        for (int kk = k0; kk < k1; ++kk, ++it) {
          const int r = it % RSTAGES;
          if (!wait_one(&rempty[r], ((it / RSTAGES) & 1) ^ 1, abort_flag, status, 40)) {
            ok = false;
            break;
          }
          uint8_t* dst = rstage(r);
          mbar_arrive_expect_tx(&rfull[r], kRawBytes + kScBytes);
          // two consecutive code tiles (one 256-row box) and the scale row of
          // each tile's group
          tma_load_2d_nomc(dst, &tm_q, 0, (m * k_iters + kk) * KSUB * BM, &rfull[r]);
#pragma unroll
          for (int sub = 0; sub < KSUB; ++sub)
            tma_load_2d_nomc(dst + kRawBytes + sub * BM * 4, &tm_s, m * BM,
                             (kk * KSTEP + sub * BK) / group, &rfull[r]);
        }
      }
      if (!ok) {  // let issued copies land before the CTA exits
        for (uint32_t j = it > RSTAGES ? it - RSTAGES : 0; j < it; ++j)
          for (uint32_t p = 0; p < (1u << 20); ++p)
            if (mbar_try_wait(&rfull[j % RSTAGES], (j / RSTAGES) & 1)) break;
      }
    }
  } else if (warp == 1) {
    constexpr uint32_t id = idesc<BN>();
    uint32_t it = 0, tc = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < total && ok; t += gridDim.x, ++tc) {
      int m, x0, s;
      decode(t, m, x0, s);
      const int k0 = s * k_per, k1 = min(k_iters, k0 + k_per);
      const uint32_t buf = tc & 1;
      if (!wait_warp(&tempty[buf], ((tc >> 1) & 1) ^ 1, abort_flag, status, 41)) {
        ok = false;
        break;
      }
      fence_after();
      const uint32_t d_tmem = tmem_base + buf * BN;
      for (int kk = k0; kk < k1; ++kk, ++it) {
        const int st = it % STAGES;
        const uint32_t ph = (it / STAGES) & 1;
        if (!wait_warp(&bfull[st], ph, abort_flag, status, 42) ||
            !wait_warp(&afull[st], ph, abort_flag, status, 43)) {
          ok = false;
          break;
        }
        fence_after();
        if (elect()) {
          const uint8_t* a = stage(st);
#pragma unroll
          for (int j = 0; j < KSTEP / 16; ++j) {  // sub-tile j / 4, +32 B along K inside its atom
            const int sub = j / (BK / 16), jj = j % (BK / 16);
            const uint64_t ad = desc_sw128(a + sub * S::A_SUB);
            const uint64_t bd = desc_sw128(a + S::A_BYTES + sub * S::B_SUB);
            mma(d_tmem, ad + 2 * jj, bd + 2 * jj, id, (kk > k0 || j > 0) ? 1u : 0u);
          }
          commit(&abempty[st]);
        }
        __syncwarp();
      }
      if (!ok) break;
      if (elect()) commit(&tfull[buf]);
      __syncwarp();
    }
    if (!ok && lane == 0) {  // issued MMAs finish (their commits arrive on abempty[])
      for (uint32_t j = it > STAGES ? it - STAGES : 0; j < it; ++j)
        for (uint32_t p = 0; p < (1u << 20); ++p)
          if (mbar_try_wait(&abempty[j % STAGES], (j / STAGES) & 1)) break;
    }
  } else if (warp < 6) {
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    uint32_t tc = 0;
    for (int t = blockIdx.x; t < total; t += gridDim.x, ++tc) {
      int m, x0, s;
      decode(t, m, x0, s);
      const uint32_t buf = tc & 1;
      if (!wait_warp(&tfull[buf], (tc >> 1) & 1, abort_flag, status, 44)) break;
      fence_after();
      const int f = m * BM + q * 32 + lane;
      const float b = (bias != nullptr && f < M && splits == 1) ? __bfloat162float(bias[f]) : 0.f;
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + buf * BN;
      if constexpr (BN >= 32) {
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          float v[32];
          ld32(tbase + c * 32, v);
          const int t0 = x0 + c * 32;
          if (f < M) {
            if (splits == 1) {
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (t0 + j < N) y[int64_t(t0 + j) * ldy + f] = __float2bfloat16(v[j] + b);
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (t0 + j < N) ws[(int64_t(s) * N + t0 + j) * M + f] = v[j];
            }
          }
        }
      } else {
        float v[16];
        ld16(tbase, v);
        if (f < M) {
          if (splits == 1) {
#pragma unroll
            for (int j = 0; j < 16; ++j)
              if (x0 + j < N) y[int64_t(x0 + j) * ldy + f] = __float2bfloat16(v[j] + b);
          } else {
#pragma unroll
            for (int j = 0; j < 16; ++j)
              if (x0 + j < N) ws[(int64_t(s) * N + x0 + j) * M + f] = v[j];
          }
        }
      }
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[buf]);
    }
  } else {
    // dequantisation (warps 6..): kDqGroups groups of 4 warps take k steps
    // round robin, so that many stages are expanded at once (one group's
    // wait / convert / fence chain is ~0.5 us per k step); thread r of a
    // group expands weight row r. Before writing operand stage st the group
    // waits for its previous MMAs; the group's first warp then requests that
    // stage's activation tile.
    const int dw = warp - 6, grp = dw >> 2;
    const bool leader = (dw & 3) == 0;
    const int r = (dw & 3) * 32 + lane;
    uint32_t it = 0;
    for (int t = blockIdx.x; t < total; t += gridDim.x) {
      int m, x0, s;
      decode(t, m, x0, s);
      const int k0 = s * k_per, k1 = min(k_iters, k0 + k_per);
      bool ok = true;
      for (int kk = k0; kk < k1; ++kk, ++it) {
        if (static_cast<int>(it % kDqGroups) != grp) continue;
        const int st = it % STAGES, rs = it % RSTAGES;
        if (!wait_warp(&abempty[st], ((it / STAGES) & 1) ^ 1, abort_flag, status, 45)) {
          ok = false;
          break;
        }
        uint8_t* a = stage(st);
        if (leader && lane == 0) {
          mbar_arrive_expect_tx(&bfull[st], S::B_BYTES);
#pragma unroll
          for (int sub = 0; sub < KSUB; ++sub)
            tma_load_2d_nomc(a + S::A_BYTES + sub * S::B_SUB, &tm_x, kk * KSTEP + sub * BK, x0,
                             &bfull[st]);
        }
        if (!wait_warp(&rfull[rs], (it / RSTAGES) & 1, abort_flag, status, 46)) {
          ok = false;
          break;
        }
        const uint8_t* raw = rstage(rs);
        uint32_t p[KSUB];
        uint32_t wv[KSUB][8];
#pragma unroll
        for (int sub = 0; sub < KSUB; ++sub) {
          p[sub] = reinterpret_cast<const uint32_t*>(raw + kRawBytes + sub * BM * 4)[r];
          const uint4 w0 = reinterpret_cast<const uint4*>(raw + (sub * BM + r) * 32)[0];
          const uint4 w1 = reinterpret_cast<const uint4*>(raw + (sub * BM + r) * 32)[1];
          wv[sub][0] = w0.x; wv[sub][1] = w0.y; wv[sub][2] = w0.z; wv[sub][3] = w0.w;
          wv[sub][4] = w1.x; wv[sub][5] = w1.y; wv[sub][6] = w1.z; wv[sub][7] = w1.w;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&rempty[rs]);  // codes consumed: the slot may refill
#pragma unroll
        for (int sub = 0; sub < KSUB; ++sub) {
          uint8_t* row = a + sub * S::A_SUB + r * 128;
          if constexpr (FMT == 0) {
            const __nv_bfloat162 zb = __bfloat162bfloat162(u32_as_bf2(p[sub]).x);
            const __nv_bfloat162 sc = __bfloat162bfloat162(u32_as_bf2(p[sub]).y);
#pragma unroll
            for (int c = 0; c < 8; ++c)
              *reinterpret_cast<uint4*>(row + ((c ^ (r & 7)) << 4)) = dequant8(wv[sub][c], zb, sc);
          } else {
            __nv_bfloat162 sb[4];  // block b covers K elements 16b .. 16b + 15 (chunks 2b, 2b + 1)
#pragma unroll
            for (int b = 0; b < 4; ++b) {
              const __half_raw h = __nv_cvt_fp8_to_halfraw(
                  static_cast<__nv_fp8_storage_t>((p[sub] >> (8 * b)) & 0xFFu), __NV_E4M3);
              sb[b] = __float2bfloat162_rn(__half2float(__half(h)) * gscale);
            }
#pragma unroll
            for (int c = 0; c < 8; ++c)
              *reinterpret_cast<uint4*>(row + ((c ^ (r & 7)) << 4)) =
                  dequant8_fp4(wv[sub][c], sb[c >> 1]);
          }
        }
        // generic-proxy smem writes -> visible to the tensor core (async proxy)
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) mbar_arrive(&afull[st]);
      }
      if (!ok) break;
    }
    if (warp == 6 && lane == 0) {  // activation tiles already requested land before exit
      for (uint32_t j = it > STAGES ? it - STAGES : 0; j < it; ++j)
        for (uint32_t p = 0; p < (1u << 20); ++p)
          if (mbar_try_wait(&bfull[j % STAGES], (j / STAGES) & 1)) break;
    }
  }
  fence_before();
  __syncthreads();
  if (warp == 1) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                 "r"(S::TMEM_COLS));
  }
}

__global__ void w4_splitk_reduce(__nv_bfloat16* __restrict__ y, int64_t ldy,
                                 const float* __restrict__ ws, const __nv_bfloat16* __restrict__ bias,
                                 int M, int N, int splits) {
  const int64_t n = int64_t(M) * N;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n;
       i += int64_t(gridDim.x) * blockDim.x) {
    const int t = static_cast<int>(i / M), f = static_cast<int>(i % M);
    float acc = bias ? __bfloat162float(bias[f]) : 0.f;
    for (int s = 0; s < splits; ++s) acc += ws[int64_t(s) * n + i];
    y[int64_t(t) * ldy + f] = __float2bfloat16(acc);
  }
}

// 2-D map without swizzle: [rows, cols] elements, row pitch in bytes, box
// box_cols x box_rows.
inline CUtensorMap make_tmap_plain(const void* ptr, CUtensorMapDataType dt, int64_t rows,
                                   int64_t cols, int64_t pitch, int box_cols, int box_rows) {
  CUtensorMap tm;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(pitch)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = tma_encode_fn()(&tm, dt, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed (", static_cast<int>(r), ")");
  return tm;
}

template <int BN, int STAGES, int RSTAGES, int FMT>
void launch(const CUtensorMap& tx, const CUtensorMap& tq, const CUtensorMap& ts, __nv_bfloat16* y,
            int64_t ldy, const __nv_bfloat16* bias, float* ws, int M, int N, int K, int Mpad,
            int group, int splits, int sms, float gscale) {
  using S = Smem<BN, STAGES, RSTAGES>;
  static_assert(S::BYTES <= 232448, "shared memory");
  auto kern = gemm_w4a16_kernel<BN, STAGES, RSTAGES, FMT>;
  static bool attr[64] = {false};
  int dev;
  cudaGetDevice(&dev);
  if (!attr[dev]) {
    SWIFT_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          static_cast<int>(S::BYTES)));
    attr[dev] = true;
  }
  const int tiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN) * splits;
  kern<<<std::min(tiles, sms), kThreads, S::BYTES, cur_stream()>>>(
      tx, tq, ts, y, ldy, bias, ws, M, N, K, Mpad, group, splits, status_word_ptr(), gscale);
  SWIFT_CHECK_LAUNCH();
}

}  // namespace w4

// Shared host path of the two weight formats (checks, plan, launch).
template <int FMT>
static int64_t gemm_w4_impl(torch::Tensor out, torch::Tensor x, torch::Tensor qp, torch::Tensor sz,
                            int64_t M, int64_t group, c10::optional<torch::Tensor> bias,
                            float gscale) {
  CHECK_BF16(x);
  CHECK_BF16(out);
  TORCH_CHECK(qp.scalar_type() == at::kByte && qp.is_contiguous() && qp.dim() == 4 &&
                  qp.size(2) == w4::BM && qp.size(3) == w4::BK / 2,
              "gemm_w4a16: qp must be uint8 [Mt, Kt, 128, 32]");
  TORCH_CHECK(sz.scalar_type() == at::kInt && sz.is_contiguous() && sz.dim() == 2,
              "gemm_w4a16: sz must be int32 [G, Mpad]");
  TORCH_CHECK(group > 0 && group % w4::BK == 0, "gemm_w4a16: group must be a multiple of 64");
  const int64_t K = x.size(-1), T = x.numel() / K;
  const int64_t Mt = (M + w4::BM - 1) / w4::BM;
  const int64_t Kt = w4::KSUB * ((K + w4::KSTEP - 1) / w4::KSTEP);  // code tiles, even
  TORCH_CHECK(qp.size(0) == Mt && qp.size(1) == Kt,
              "gemm_w4a16: qp must hold [ceil(M/128), 2*ceil(K/128)] code tiles");
  TORCH_CHECK(sz.size(1) == Mt * w4::BM && sz.size(0) >= (Kt * w4::BK + group - 1) / group,
              "gemm_w4a16: sz shape");
  TORCH_CHECK(x.stride(-1) == 1 && out.stride(-1) == 1, "gemm_w4a16: inner dims contiguous");
  TORCH_CHECK(K % 8 == 0, "gemm_w4a16: K must be a multiple of 8 (16-byte TMA rows)");
  const int64_t ldx = x.dim() >= 2 ? x.stride(-2) : K;
  TORCH_CHECK(ldx % 8 == 0 && reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0 &&
                  reinterpret_cast<uintptr_t>(qp.data_ptr()) % 16 == 0 &&
                  reinterpret_cast<uintptr_t>(sz.data_ptr()) % 16 == 0,
              "gemm_w4a16: 16-byte alignment");
  TORCH_CHECK(out.numel() / out.size(-1) == T && out.size(-1) >= M);
  if (T == 0) return 0;
  const int64_t ldy = out.dim() >= 2 ? out.stride(-2) : M;
  int dev;
  cudaGetDevice(&dev);
  static int sms_cache[64] = {0};
  if (!sms_cache[dev]) cudaDeviceGetAttribute(&sms_cache[dev], cudaDevAttrMultiProcessorCount, dev);
  const int sms = sms_cache[dev];
  // Token tile: one tile covers up to 256 tokens (each weight tile read once
  // from HBM); narrower tiles while the grid leaves SMs idle (weight re-reads
  // come from L2); split K only when that still leaves a quarter idle.
  int bn;
  if (T > 128) {
    bn = 256;
  } else {
    bn = 16;
    while (bn < T) bn *= 2;
  }
  while (bn > 32 && Mt * ((T + bn - 1) / bn) < sms * 3 / 4) bn /= 2;
  const int64_t tiles = Mt * ((T + bn - 1) / bn);
  int splits = 1;
  if (tiles < sms * 3 / 4)
    splits = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>({(sms + tiles - 1) / tiles, Kt / 8, 8})));
  {  // only as many splits as non-empty K ranges (the kernel gives each
     // split ceil(k_iters / splits) steps; a split past the end would publish
     // an accumulator it never wrote)
    const int k_iters = static_cast<int>(Kt / w4::KSUB);
    const int k_per = (k_iters + splits - 1) / splits;
    splits = (k_iters + k_per - 1) / k_per;
  }
  CUtensorMap tx = make_tmap_2d(x.data_ptr(), T, K, ldx, w4::BK, bn);
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
  // codes as a [Mt * Kt * 128, 32] byte matrix (one 128-row box = one 4 KB
  // tile of a k step) and scales as [G, Mpad] u32 (one 128-word box = the
  // (z, s) row of a group): both fetched by tensor TMA, no swizzle
  const CUtensorMap q = w4::make_tmap_plain(qp.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_UINT8, Mt * Kt * w4::BM,
                                        32, 32, 32, w4::KSUB * w4::BM);
  const CUtensorMap s = w4::make_tmap_plain(sz.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_UINT32, sz.size(0),
                                        sz.size(1), sz.size(1) * 4, w4::BM, 1);
  const int Mi = static_cast<int>(M), Ni = static_cast<int>(T), Ki = static_cast<int>(K),
            Mp = static_cast<int>(sz.size(1)), g = static_cast<int>(group);
  switch (bn) {
    case 16: w4::launch<16, 4, 8, FMT>(tx, q, s, y, ldy, bp, wsp, Mi, Ni, Ki, Mp, g, splits, sms, gscale); break;
    case 32: w4::launch<32, 3, 10, FMT>(tx, q, s, y, ldy, bp, wsp, Mi, Ni, Ki, Mp, g, splits, sms, gscale); break;
    case 64: w4::launch<64, 3, 8, FMT>(tx, q, s, y, ldy, bp, wsp, Mi, Ni, Ki, Mp, g, splits, sms, gscale); break;
    case 128: w4::launch<128, 2, 10, FMT>(tx, q, s, y, ldy, bp, wsp, Mi, Ni, Ki, Mp, g, splits, sms, gscale); break;
    default: w4::launch<256, 2, 3, FMT>(tx, q, s, y, ldy, bp, wsp, Mi, Ni, Ki, Mp, g, splits, sms, gscale); break;
  }
  if (splits > 1) {
    const int64_t n = M * T;
    const int blocks = static_cast<int>(std::min<int64_t>((n + 255) / 256, sms * 8));
    w4::w4_splitk_reduce<<<blocks, 256, 0, cur_stream()>>>(y, ldy, wsp, bp, Mi, Ni, splits);
    SWIFT_CHECK_LAUNCH();
    return 2;
  }
  return 1;
}

// out [T, M] bf16 = x [T, K] . dequant(qp, sz)^T (+ bias). qp uint8
// [ceil(M/128), 2*ceil(K/128), 128, 32] (tile-packed int4), sz int32 [G, Mpad]
// ((128 + z, s) bf16 pairs), group a multiple of 64. Returns launches.
int64_t gemm_w4a16(torch::Tensor out, torch::Tensor x, torch::Tensor qp, torch::Tensor sz,
                   int64_t M, int64_t group, c10::optional<torch::Tensor> bias) {
  return gemm_w4_impl<0>(out, x, qp, sz, M, group, bias, 1.f);
}

// NVFP4 weights: qp as above holding E2M1 codes, sc int32 [2*ceil(K/128), Mpad]
// (four E4M3 block scales per row and k step, block b in byte b), gscale the
// per-tensor fp32 scale. w = bf16(e2m1 * bf16(e4m3 * gscale)).
int64_t gemm_nvfp4w(torch::Tensor out, torch::Tensor x, torch::Tensor qp, torch::Tensor sc,
                    int64_t M, double gscale, c10::optional<torch::Tensor> bias) {
  return gemm_w4_impl<1>(out, x, qp, sc, M, 64, bias, static_cast<float>(gscale));
}

}  // namespace swift
