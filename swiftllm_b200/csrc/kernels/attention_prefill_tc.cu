// Paged prefill attention on the 5th-generation tensor cores (head_dim 128,
// KV block size 16): varlen causal attention of new query tokens against
// the paged KV pool (which already holds them), chunked prefill (queries
// start at seq_len - q_len), GQA and sliding windows.
//
// Replaces the reference's paged_attention_prefill stub
// (crates/swiftllm-cuda/src/bindings.rs:33-54).
//
// One CTA = (128 query rows, sequence, KV head). The 128 rows are the G query
// heads of the KV head's group for 128 / G consecutive positions (row r =
// position r / G, head r % G), so each KV tile is loaded once for the whole
// group. Per 128-key tile j:
//   warp 0      TMA: the Q tile once (3-D map over [tokens, heads, dim]),
//               then the K and V pages of each tile (2-D map over pool rows,
//               two 64-column halves per 16-token page) into a 2-stage ring;
//   warp 1      one thread issues tcgen05.mma.cta_group::1.kind::f16:
//               S_j = Q K_j^T into a double-buffered TMEM accumulator
//               (issued one tile ahead, so the next scores are computed
//               while this tile's softmax runs), then O += P_j V_j with V
//               read as an MN-major operand (no transpose);
//   warps 2-5   one thread per row: tcgen05.ld of the score row, mask,
//               online softmax in base 2, P (bf16) into shared memory in the
//               128-byte-swizzled K-major layout the MMA reads. The running
//               maximum used for P is only raised (and O, l rescaled through
//               tcgen05.ld / tcgen05.st) when the true maximum exceeds it by
//               more than 2^8, so most tiles skip the O round trip; the
//               final division by l makes the result exact either way.
// Epilogue: O / l, bf16, one 256-byte row store per thread.
// Every mbarrier wait is bounded: on expiry the waiter records
// kErrWaitTimeout in the status word and raises the CTA's abort flag; the
// roles drain, TMEM is freed and the CTA returns.
#include <cudaTypedefs.h>

#include <algorithm>

#include "common.cuh"

namespace swift {

namespace pft {

constexpr int kD = 128;            // head_dim
constexpr int kBM = 128;           // query rows per CTA
constexpr int kBN = 128;           // keys per tile
constexpr int kPage = 16;          // KV block size (tokens per page)
constexpr int kThreads = 192;
constexpr int kHalf = 128 * 64 * 2;        // one 128-row x 64-column bf16 half: 16 KB
constexpr int kQBytes = 2 * kHalf;         // 32 KB
constexpr int kKVStage = 4 * kHalf;        // K (2 halves) + V (2 halves): 64 KB
constexpr int kStages = 2;
constexpr int kPBytes = 2 * kHalf;         // 32 KB per P buffer (two buffers)
constexpr size_t kSmem = 1024 + kQBytes + size_t(kStages) * kKVStage + 2 * kPBytes + 256;
constexpr float kRescaleLog2 = 8.f;        // raise the P reference max past 2^8 growth only

__device__ __forceinline__ void tma2d(void* dst, const CUtensorMap* tm, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, "
      "%3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(tm)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void tma3d(void* dst, const CUtensorMap* tm, int x, int y, int z,
                                      uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, "
      "%3, %4}], [%5];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(tm)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}
// K-major SW128 (rows of 128 B, 8-row atoms 1024 B apart).
__device__ __forceinline__ uint64_t desc_k(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr & 0x3FFFF) >> 4);
  d |= static_cast<uint64_t>(1) << 16;
  d |= static_cast<uint64_t>(1024 >> 4) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}
// MN-major SW128 for V [keys][dim] (dim contiguous): 64-element dim blocks
// `lbo` bytes apart, 8-key groups 1024 B apart.
__device__ __forceinline__ uint64_t desc_mn(uint32_t saddr, uint32_t lbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr & 0x3FFFF) >> 4);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFF) << 16;
  d |= static_cast<uint64_t>(1024 >> 4) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}
// kind::f16, f32 accumulate, bf16 A and B, M = 128, N = 128; b_mn: B is MN-major.
__device__ __forceinline__ constexpr uint32_t idesc(bool b_mn) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((b_mn ? 1u : 0u) << 16) | ((128u >> 3) << 17) |
         ((128u >> 4) << 24);
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
__device__ __forceinline__ void ld32(uint32_t taddr, uint32_t (&r)[32]) {
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
__device__ __forceinline__ void st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ uint64_t now_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Bounded waits: give up after kWaitNs (or once another role of the CTA gave
// up), record the site and raise the CTA's abort flag.
constexpr uint64_t kWaitNs = 2000000000ull;
__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                         int* status, int where) {
  const uint64_t t0 = now_ns();
  for (uint32_t i = 0;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255) == 255) {
      if (*abort_flag) return false;
      if (now_ns() - t0 > kWaitNs) break;
    }
  }
  set_status(status, kErrWaitTimeout, where);
  *abort_flag = 1;
  return false;
}
// warp-uniform variant for the softmax warps
__device__ __forceinline__ bool wait_bar_warp(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                              int* status, int where) {
  const uint64_t t0 = now_ns();
  for (uint32_t i = 0;; ++i) {
    const bool r = mbar_try_wait(bar, parity);
    if (__all_sync(0xffffffffu, r)) return true;
    if ((i & 255) == 255) {
      const bool give_up = *abort_flag || now_ns() - t0 > kWaitNs;
      if (__any_sync(0xffffffffu, give_up)) {
        if ((threadIdx.x & 31) == 0 && !*abort_flag) {
          set_status(status, kErrWaitTimeout, where);
          *abort_flag = 1;
        }
        return false;
      }
    }
  }
}

}  // namespace pft

__global__ void __launch_bounds__(pft::kThreads, 1)
    paged_prefill_tc_kernel(const __grid_constant__ CUtensorMap tm_q,
                            const __grid_constant__ CUtensorMap tm_kv,
                            __nv_bfloat16* __restrict__ out, int rows_per_blk, int layer_row_off,
                            const int32_t* __restrict__ bt, int64_t bt_stride,
                            const int32_t* __restrict__ q_start,
                            const int32_t* __restrict__ seq_lens, int seq0, int Hq, int Hkv,
                            int n_qtiles, float sl2, int window, int* status) {
  using namespace pft;
  pdl_wait();
  pdl_trigger();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base =
      reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = base;
  uint8_t* sKV = base + kQBytes;
  uint8_t* sP = sKV + kStages * kKVStage;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + 2 * kPBytes);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;      // [2] per KV stage
  uint64_t* v_full = bars + 3;      // [2]
  uint64_t* kv_empty = bars + 5;    // [2]
  uint64_t* s_full = bars + 7;      // [2] per S accumulator
  uint64_t* s_empty = bars + 9;     // [2]
  uint64_t* p_full = bars + 11;     // [2] per P buffer
  uint64_t* o_done = bars + 13;     // [2] per P buffer: the P.V that read it finished
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 15);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = Hq / Hkv, P = kBM / G;  // heads per group, positions per tile
  const int qt = n_qtiles - 1 - static_cast<int>(blockIdx.x);  // longest causal rows first
  const int seq = seq0 + blockIdx.y, h = blockIdx.z;
  const int qs = q_start[seq], q_len = q_start[seq + 1] - qs;
  const int p0 = qt * P;  // first query position (within the new tokens) of this tile
  if (p0 >= q_len) return;
  const int L = seq_lens[seq];
  const int pos0 = L - q_len;  // absolute position of new token 0
  const int last_pos = pos0 + min(q_len, p0 + P) - 1;
  const int first_pos = pos0 + p0;
  const int n_end = min(L, last_pos + 1);
  const int j0 = window > 0 ? max(0, first_pos - window + 1) / kBN : 0;
  const int j1 = (n_end + kBN - 1) / kBN;  // key tiles [j0, j1)
  const int nt = j1 - j0;
  const int32_t* mybt = bt + int64_t(seq) * bt_stride;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&kv_empty[s], 1);
      mbar_init(&s_full[s], 1);
      mbar_init(&s_empty[s], 4);
      mbar_init(&p_full[s], 4);
      mbar_init(&o_done[s], 1);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(
        smem_u32(tmem_slot)));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tmem_slot;  // columns: S0 [0,128), S1 [128,256), O [256,384)
  const uint32_t tO = tmem + 256;

  if (warp == 0) {
    if (lane == 0) {
      bool ok = true;
      // Q: 128 rows = P positions x G heads, two 64-column halves
      mbar_arrive_expect_tx(q_full, kQBytes);
      for (int hf = 0; hf < 2; ++hf) tma3d(sQ + hf * kHalf, &tm_q, hf * 64, h * G, qs + p0, q_full);
      // block ids of the next tile's pages are read while this tile's
      // stage is awaited
      int blk[kBN / kPage];
      auto fetch_ids = [&](int t) {
#pragma unroll
        for (int pg = 0; pg < kBN / kPage; ++pg) {
          const int key = (j0 + t) * kBN + pg * kPage;
          // pages past the sequence end: any valid block (masked later)
          blk[pg] = mybt[min(key, L - 1) / kPage];
        }
      };
      if (nt > 0) fetch_ids(0);
      for (int t = 0; t < nt && ok; ++t) {
        const int st = t & 1;
        if (!pft::wait_bar(&kv_empty[st], ((t >> 1) & 1) ^ 1, abort_flag, status, 60)) {
          ok = false;
          break;
        }
        uint8_t* kvs = sKV + st * kKVStage;  // K half 0 | K half 1 | V half 0 | V half 1
        mbar_arrive_expect_tx(&k_full[st], 2 * kHalf);
#pragma unroll
        for (int pg = 0; pg < kBN / kPage; ++pg) {
          const int row = blk[pg] * rows_per_blk + layer_row_off + h * kPage;  // K rows
          for (int hf = 0; hf < 2; ++hf)
            tma2d(kvs + hf * kHalf + pg * kPage * 128, &tm_kv, hf * 64, row, &k_full[st]);
        }
        mbar_arrive_expect_tx(&v_full[st], 2 * kHalf);
#pragma unroll
        for (int pg = 0; pg < kBN / kPage; ++pg) {
          const int vrow = blk[pg] * rows_per_blk + layer_row_off + (Hkv + h) * kPage;  // V rows
          for (int hf = 0; hf < 2; ++hf)
            tma2d(kvs + (2 + hf) * kHalf + pg * kPage * 128, &tm_kv, hf * 64, vrow, &v_full[st]);
        }
        if (t + 1 < nt) fetch_ids(t + 1);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      bool ok = pft::wait_bar(q_full, 0, abort_flag, status, 61);
      const uint32_t qa = smem_u32(sQ);
      auto issue_s = [&](int t) {  // S_t = Q K_t^T into S[t & 1]
        const int st = t & 1;
        if (!pft::wait_bar(&k_full[st], (t >> 1) & 1, abort_flag, status, 62)) return false;
        if (!pft::wait_bar(&s_empty[st], ((t >> 1) & 1) ^ 1, abort_flag, status, 63)) return false;
        fence_after();
        const uint32_t ka = smem_u32(sKV + st * kKVStage);
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk) {
          const uint32_t off = (kk >> 2) * kHalf + (kk & 3) * 32;
          mma(tmem + st * 128, pft::desc_k(qa + off), pft::desc_k(ka + off), idesc(false),
              kk > 0 ? 1u : 0u);
        }
        commit(&s_full[st]);
        return true;
      };
      auto issue_pv = [&](int t) {  // O += P_t V_t
        const int st = t & 1;  // KV stage and P buffer
        if (!pft::wait_bar(&p_full[st], (t >> 1) & 1, abort_flag, status, 64)) return false;
        if (!pft::wait_bar(&v_full[st], (t >> 1) & 1, abort_flag, status, 68)) return false;
        fence_after();
        const uint32_t va = smem_u32(sKV + st * kKVStage + 2 * kHalf);
        const uint32_t pa = smem_u32(sP + st * kPBytes);
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk) {
          const uint32_t poff = (kk >> 2) * kHalf + (kk & 3) * 32;   // P: K-major, keys
          const uint32_t voff = kk * 16 * 128;                        // V: 16 keys = 2 KB
          mma(tO, pft::desc_k(pa + poff), pft::desc_mn(va + voff, kHalf), idesc(true),
              (t > 0 || kk > 0) ? 1u : 0u);
        }
        commit(&o_done[st]);
        commit(&kv_empty[st]);
        return true;
      };
      if (ok && nt > 0) ok = issue_s(0);
      for (int t = 0; t < nt && ok; ++t) {
        if (t + 1 < nt) ok = issue_s(t + 1);
        if (ok) ok = issue_pv(t);
      }
    }
  } else {
    // softmax / epilogue: thread = query row r
    const int q4 = warp & 3;
    const int r = q4 * 32 + lane;
    const int p = r / G, g = r % G;
    const int qpos = pos0 + p0 + p;  // absolute position of this row's query
    const bool row_valid = p0 + p < q_len;
    const uint32_t lane_off = static_cast<uint32_t>(q4 * 32) << 16;
    float m_used = -INFINITY, m_run = -INFINITY, l = 0.f;
    bool ok = true;
    for (int t = 0; t < nt; ++t) {
      const int st = t & 1;
      if (!pft::wait_bar_warp(&s_full[st], (t >> 1) & 1, abort_flag, status, 65)) {
        ok = false;
        break;
      }
      fence_after();
      const int key0 = (j0 + t) * kBN;
      const uint32_t tS = tmem + lane_off + st * 128;
      // pass 1: masked, scaled row maximum of this tile
      float mt = -INFINITY;
#pragma unroll 1
      for (int c = 0; c < kBN; c += 64) {
        uint32_t u[32], u2[32];
        pft::ld32(tS + c, u);
        pft::ld32(tS + c + 32, u2);
        pft::ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int key = key0 + c + 32 + i;
          const bool keep =
              row_valid && key <= qpos && key < L && (window <= 0 || key > qpos - window);
          if (keep) mt = fmaxf(mt, __uint_as_float(u2[i]) * sl2);
        }
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int key = key0 + c + i;
          const bool keep =
              row_valid && key <= qpos && key < L && (window <= 0 || key > qpos - window);
          if (keep) mt = fmaxf(mt, __uint_as_float(u[i]) * sl2);
        }
      }
      m_run = fmaxf(m_run, mt);
      // P buffer t & 1 free: the P.V of tile t - 2 finished
      if (t > 1 && !pft::wait_bar_warp(&o_done[st], ((t - 2) >> 1) & 1, abort_flag, status, 66)) {
        ok = false;
        break;
      }
      // raise the reference max of rows whose true max outgrew it; the O
      // round trip (tcgen05.ld / .st are warp-collective) runs for the whole
      // warp when any of its rows needs it, with factor 1 for the others
      const bool need = m_used != -INFINITY && m_run > m_used + kRescaleLog2;
      float f = 1.f;
      if (m_used == -INFINITY) {
        m_used = m_run;
      } else if (need) {
        f = exp2f(m_used - m_run);
        l *= f;
        m_used = m_run;
      }
      if (__any_sync(0xffffffffu, need)) {
        // O stable: the P.V of tile t - 1 finished
        if (!pft::wait_bar_warp(&o_done[(t - 1) & 1], ((t - 1) >> 1) & 1, abort_flag, status, 69)) {
          ok = false;
          break;
        }
        fence_after();
#pragma unroll 1
        for (int c = 0; c < kD; c += 32) {
          uint32_t u[32];
          pft::ld32(tO + lane_off + c, u);
          pft::ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) u[i] = __float_as_uint(__uint_as_float(u[i]) * f);
          pft::st32(tO + lane_off + c, u);
        }
        pft::st_wait();
      }
      // pass 2: P = 2^(s - m_used) in bf16, into the swizzled K-major layout
      const float mu = m_used == -INFINITY ? 0.f : m_used;
      float rs = 0.f;
#pragma unroll 1
      for (int c = 0; c < kBN; c += 32) {
        uint32_t u[32];
        pft::ld32(tS + c, u);
        pft::ld_wait();
#pragma unroll
        for (int ch = 0; ch < 4; ++ch) {  // 16-byte chunks of 8 keys
          float e[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int key = key0 + c + ch * 8 + i;
            const bool keep =
                row_valid && key <= qpos && key < L && (window <= 0 || key > qpos - window);
            e[i] = keep ? exp2f(__uint_as_float(u[ch * 8 + i]) * sl2 - mu) : 0.f;
            rs += e[i];
          }
          const int chunk = (c >> 3) + ch;  // 0..15
          const int hf = chunk >> 3, c16 = (chunk & 7) ^ (r & 7);
          store8(reinterpret_cast<__nv_bfloat16*>(sP + st * kPBytes + hf * kHalf + r * 128 + c16 * 16),
                 e);
        }
      }
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_empty[st]);  // S[st] may be overwritten
      l += rs;
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[st]);
    }
    // epilogue: wait for the last P.V, O / l, one 256-byte row per thread
    if (ok && nt > 0 &&
        pft::wait_bar_warp(&o_done[(nt - 1) & 1], ((nt - 1) >> 1) & 1, abort_flag, status, 67)) {
      fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      __nv_bfloat16* orow = out + (int64_t(qs + p0 + p) * Hq + h * G + g) * kD;
#pragma unroll 1
      for (int c = 0; c < kD; c += 32) {
        uint32_t u[32];
        pft::ld32(tO + lane_off + c, u);
        pft::ld_wait();
        if (row_valid) {
#pragma unroll
          for (int q8 = 0; q8 < 4; ++q8) {
            float f[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) f[i] = __uint_as_float(u[q8 * 8 + i]) * inv;
            store8(orow + c + q8 * 8, f);
          }
        }
      }
    }
  }
  fence_before();
  __syncthreads();
  if (warp == 1) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem));
  }
}

// ---------------------------------------------------------------- host side
static PFN_cuTensorMapEncodeTiled_v12000 pft_encode() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult qr;
    void* p = nullptr;
    SWIFT_CHECK_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &qr));
    TORCH_CHECK(qr == cudaDriverEntryPointSuccess && p, "cuTensorMapEncodeTiled unavailable");
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// Whether the tcgen05 kernel serves this call (head_dim 128, 16-token pages,
// a group size that divides 128).
bool paged_prefill_tc_supported(int D, int block_size, int Hq, int Hkv) {
  if (D != pft::kD || block_size != pft::kPage || Hkv <= 0 || Hq % Hkv) return false;
  const int G = Hq / Hkv;
  return G >= 1 && G <= 16 && pft::kBM % G == 0;
}

void paged_prefill_tc(torch::Tensor out, torch::Tensor q, torch::Tensor kv, int64_t layer,
                      torch::Tensor bt, torch::Tensor q_start, torch::Tensor seq_lens, int seq0,
                      int seq1, int max_q_len, double scale, int window) {
  using namespace pft;
  const int T = static_cast<int>(q.size(0)), Hq = static_cast<int>(q.size(1));
  const int L = static_cast<int>(kv.size(1)), Hkv = static_cast<int>(kv.size(3));
  const int G = Hq / Hkv, P = kBM / G;
  static bool attr[64] = {false};
  int dev;
  cudaGetDevice(&dev);
  if (!attr[dev]) {
    SWIFT_CHECK_CUDA(cudaFuncSetAttribute(paged_prefill_tc_kernel,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          static_cast<int>(kSmem)));
    attr[dev] = true;
  }
  // Q as [tokens][heads][dim]: box = 64 dims x G heads x P tokens
  CUtensorMap tq;
  {
    cuuint64_t dims[3] = {static_cast<cuuint64_t>(kD), static_cast<cuuint64_t>(Hq),
                          static_cast<cuuint64_t>(T)};
    cuuint64_t strides[2] = {static_cast<cuuint64_t>(kD) * 2, static_cast<cuuint64_t>(Hq) * kD * 2};
    cuuint32_t box[3] = {64, static_cast<cuuint32_t>(G), static_cast<cuuint32_t>(P)};
    cuuint32_t es[3] = {1, 1, 1};
    CUresult r = pft_encode()(&tq, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, q.data_ptr(), dims, strides,
                              box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    TORCH_CHECK(r == CUDA_SUCCESS, "paged_prefill_tc: Q tensor map (", static_cast<int>(r), ")");
  }
  // the pool as rows of head_dim: [blocks * layers * 2 * Hkv * 16, 128]
  CUtensorMap tkv;
  const int64_t pool_rows = kv.numel() / kD;
  TORCH_CHECK(pool_rows < (int64_t(1) << 31), "paged_prefill_tc: KV pool too large for int32 rows");
  {
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(kD), static_cast<cuuint64_t>(pool_rows)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(kD) * 2};
    cuuint32_t box[2] = {64, static_cast<cuuint32_t>(kPage)};
    cuuint32_t es[2] = {1, 1};
    CUresult r = pft_encode()(&tkv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, kv.data_ptr(), dims, strides,
                              box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    TORCH_CHECK(r == CUDA_SUCCESS, "paged_prefill_tc: KV tensor map (", static_cast<int>(r), ")");
  }
  const int rows_per_blk = L * 2 * Hkv * kPage;
  const int layer_row_off = static_cast<int>(layer) * 2 * Hkv * kPage;
  const int n_qtiles = (max_q_len + P - 1) / P;
  dim3 grid(n_qtiles, seq1 - seq0, Hkv);
  launch_pdl(paged_prefill_tc_kernel, grid, dim3(kThreads), kSmem, cur_stream(), tq, tkv,
             reinterpret_cast<__nv_bfloat16*>(out.data_ptr<at::BFloat16>()), rows_per_blk,
             layer_row_off, static_cast<const int32_t*>(bt.data_ptr<int32_t>()), bt.stride(0),
             static_cast<const int32_t*>(q_start.data_ptr<int32_t>()),
             static_cast<const int32_t*>(seq_lens.data_ptr<int32_t>()), seq0, Hq, Hkv, n_qtiles,
             static_cast<float>(scale * 1.4426950408889634), window, status_word_ptr());
}

}  // namespace swift
