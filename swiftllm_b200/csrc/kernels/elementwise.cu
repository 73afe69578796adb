// Memory-bound fused ops: (add +) RMSNorm / LayerNorm, SwiGLU, GELU(tanh),
// embedding gather, fused QKV split + bias + RoPE + paged KV write, KV block
// copy (copy-on-write), counter-based random init, and the status word.
//
// Parity (the reference declares these and stubs them):
//   rms_norm / fused_add_rms_norm  crates/swiftllm-cuda/src/bindings.rs:116-156
//   rotary_embedding               bindings.rs:159-180
//   silu_and_mul                   bindings.rs:183-199
//   reshape_and_cache              crates/swiftllm-cuda/kernels/paged_attention.cu:167-199
//   copy_blocks                    paged_attention.cu:202-227 (its launch uses
//                                  2048 threads per block and cannot run)
// All row kernels move 16-byte vectors (8 x bf16) and keep a row in registers
// between the reduction and the write, so each byte is read once.
#include "common.cuh"

namespace swift {

static __device__ int g_status[2];

int* status_word_ptr() {
  static int* cache[64] = {nullptr};
  int dev = 0;
  SWIFT_CHECK_CUDA(cudaGetDevice(&dev));
  if (dev < 64 && cache[dev]) return cache[dev];
  int* p = nullptr;
  SWIFT_CHECK_CUDA(cudaGetSymbolAddress(reinterpret_cast<void**>(&p), g_status));
  if (dev < 64) cache[dev] = p;
  return p;
}

// ---------------------------------------------------------------- norms
// One CTA per row; VEC vectors of 8 elements per thread held in registers.
template <int VEC, bool ADD, bool LAYERNORM>
__global__ void __launch_bounds__(1024) norm_kernel(__nv_bfloat16* __restrict__ out,
                                                    const __nv_bfloat16* __restrict__ x,
                                                    __nv_bfloat16* __restrict__ residual,
                                                    const __nv_bfloat16* __restrict__ w,
                                                    const __nv_bfloat16* __restrict__ b, int H,
                                                    float eps) {
  pdl_wait();  // previous kernel done (programmatic dependent launch)
  pdl_trigger();
  __shared__ float red[33];
  const int64_t row = blockIdx.x;
  const __nv_bfloat16* xr = x + row * H;
  __nv_bfloat16* rr = ADD ? residual + row * H : nullptr;
  float v[VEC][8];
  float s = 0.f, s2 = 0.f;
#pragma unroll
  for (int j = 0; j < VEC; ++j) {
    int c = (threadIdx.x + j * blockDim.x) * 8;
    if (c < H) {
      load8(xr + c, v[j]);
      if (ADD) {
        float r[8];
        load8(rr + c, r);
#pragma unroll
        for (int i = 0; i < 8; ++i) v[j][i] = __bfloat162float(__float2bfloat16(v[j][i] + r[i]));
        store8(rr + c, v[j]);
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        s += v[j][i];
        s2 += v[j][i] * v[j][i];
      }
    }
  }
  float mean = 0.f, scale;
  if (LAYERNORM) {
    mean = block_sum(s, red) / H;
    float var = block_sum(s2, red) / H - mean * mean;
    scale = rsqrtf(fmaxf(var, 0.f) + eps);
  } else {
    scale = rsqrtf(block_sum(s2, red) / H + eps);
  }
#pragma unroll
  for (int j = 0; j < VEC; ++j) {
    int c = (threadIdx.x + j * blockDim.x) * 8;
    if (c < H) {
      float wf[8], o[8];
      load8(w + c, wf);
      if (LAYERNORM && b) {
        float bf[8];
        load8(b + c, bf);
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = (v[j][i] - mean) * scale * wf[i] + bf[i];
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = (v[j][i] - mean) * scale * wf[i];
      }
      store8(out + row * H + c, o);
    }
  }
}

template <bool ADD, bool LN>
static void launch_norm(torch::Tensor out, torch::Tensor x, c10::optional<torch::Tensor> res,
                        torch::Tensor w, c10::optional<torch::Tensor> b, double eps) {
  CHECK_CUDA_TENSOR(x);
  CHECK_BF16(x);
  CHECK_CONTIG(x);
  CHECK_CONTIG(out);
  const int H = static_cast<int>(x.size(-1));
  TORCH_CHECK(H % 8 == 0, "hidden size must be a multiple of 8");
  const int64_t rows = x.numel() / H;
  if (rows == 0) return;
  int vecs = H / 8;
  int threads = std::min(1024, ((vecs + 31) / 32) * 32);
  int per = (vecs + threads - 1) / threads;
  auto* op = reinterpret_cast<__nv_bfloat16*>(out.data_ptr<at::BFloat16>());
  auto* xp = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr<at::BFloat16>());
  auto* rp = ADD ? reinterpret_cast<__nv_bfloat16*>(res.value().data_ptr<at::BFloat16>()) : nullptr;
  auto* wp = reinterpret_cast<const __nv_bfloat16*>(w.data_ptr<at::BFloat16>());
  const __nv_bfloat16* bp =
      (LN && b.has_value()) ? reinterpret_cast<const __nv_bfloat16*>(b.value().data_ptr<at::BFloat16>())
                            : nullptr;
  auto st = cur_stream();
  const float e = static_cast<float>(eps);
  switch (per) {
    case 1: launch_pdl(norm_kernel<1, ADD, LN>, dim3(rows), dim3(threads), 0, st, op, xp, rp, wp, bp, H, e); break;
    case 2: launch_pdl(norm_kernel<2, ADD, LN>, dim3(rows), dim3(threads), 0, st, op, xp, rp, wp, bp, H, e); break;
    case 3: launch_pdl(norm_kernel<3, ADD, LN>, dim3(rows), dim3(threads), 0, st, op, xp, rp, wp, bp, H, e); break;
    case 4: launch_pdl(norm_kernel<4, ADD, LN>, dim3(rows), dim3(threads), 0, st, op, xp, rp, wp, bp, H, e); break;
    default: TORCH_CHECK(false, "hidden size too large for the norm kernel");
  }
  SWIFT_CHECK_LAUNCH();
}

void rms_norm(torch::Tensor out, torch::Tensor x, torch::Tensor w, double eps) {
  launch_norm<false, false>(out, x, c10::nullopt, w, c10::nullopt, eps);
}
void fused_add_rms_norm(torch::Tensor out, torch::Tensor x, torch::Tensor residual,
                        torch::Tensor w, double eps) {
  CHECK_CONTIG(residual);
  launch_norm<true, false>(out, x, residual, w, c10::nullopt, eps);
}
void layer_norm(torch::Tensor out, torch::Tensor x, torch::Tensor w,
                c10::optional<torch::Tensor> b, double eps) {
  launch_norm<false, true>(out, x, c10::nullopt, w, b, eps);
}
void fused_add_layer_norm(torch::Tensor out, torch::Tensor x, torch::Tensor residual,
                          torch::Tensor w, c10::optional<torch::Tensor> b, double eps) {
  CHECK_CONTIG(residual);
  launch_norm<true, true>(out, x, residual, w, b, eps);
}

// ---------------------------------------------------------------- activations
__global__ void silu_mul_kernel(__nv_bfloat16* __restrict__ out, const __nv_bfloat16* __restrict__ x,
                                int64_t rows, int I) {
  pdl_wait();  // previous kernel done (programmatic dependent launch)
  pdl_trigger();
  const int vec = I / 8;
  const int64_t total = rows * vec;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    int64_t r = i / vec;
    int c = static_cast<int>(i % vec) * 8;
    float g[8], u[8], o[8];
    load8(x + r * 2 * I + c, g);
    load8(x + r * 2 * I + I + c, u);
#pragma unroll
    for (int k = 0; k < 8; ++k) o[k] = g[k] / (1.f + __expf(-g[k])) * u[k];
    store8(out + r * I + c, o);
  }
}

void silu_and_mul(torch::Tensor out, torch::Tensor x) {
  CHECK_BF16(x);
  CHECK_CONTIG(x);
  const int I = static_cast<int>(out.size(-1));
  TORCH_CHECK(I % 8 == 0 && x.size(-1) == 2 * I, "bad silu_and_mul shapes");
  int64_t rows = x.numel() / (2 * I);
  if (rows == 0) return;
  int64_t total = rows * (I / 8);
  int blocks = static_cast<int>(std::min<int64_t>((total + 255) / 256, 148 * 16));
  launch_pdl(silu_mul_kernel, dim3(blocks), dim3(256), 0, cur_stream(), 
      reinterpret_cast<__nv_bfloat16*>(out.data_ptr<at::BFloat16>()),
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr<at::BFloat16>()), rows, I);
  SWIFT_CHECK_LAUNCH();
}

__global__ void gelu_tanh_kernel(__nv_bfloat16* __restrict__ out, const __nv_bfloat16* __restrict__ x,
                                 int64_t n8) {
  pdl_wait();  // previous kernel done (programmatic dependent launch)
  pdl_trigger();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n8;
       i += (int64_t)gridDim.x * blockDim.x) {
    float v[8], o[8];
    load8(x + i * 8, v);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      float t = 0.7978845608028654f * (v[k] + 0.044715f * v[k] * v[k] * v[k]);
      o[k] = 0.5f * v[k] * (1.f + tanhf(t));
    }
    store8(out + i * 8, o);
  }
}

void gelu_tanh(torch::Tensor out, torch::Tensor x) {
  CHECK_BF16(x);
  CHECK_CONTIG(x);
  TORCH_CHECK(x.numel() % 8 == 0);
  int64_t n8 = x.numel() / 8;
  if (!n8) return;
  int blocks = static_cast<int>(std::min<int64_t>((n8 + 255) / 256, 148 * 16));
  launch_pdl(gelu_tanh_kernel, dim3(blocks), dim3(256), 0, cur_stream(), 
      reinterpret_cast<__nv_bfloat16*>(out.data_ptr<at::BFloat16>()),
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr<at::BFloat16>()), n8);
  SWIFT_CHECK_LAUNCH();
}

// ---------------------------------------------------------------- embedding
__global__ void embedding_kernel(__nv_bfloat16* __restrict__ out, const int32_t* __restrict__ ids,
                                 const __nv_bfloat16* __restrict__ w, int H, int64_t rows_w,
                                 int64_t vocab_start) {
  pdl_wait();  // previous kernel done (programmatic dependent launch)
  pdl_trigger();
  const int64_t t = blockIdx.x;
  int64_t id = static_cast<int64_t>(ids[t]) - vocab_start;
  bool ok = id >= 0 && id < rows_w;
  const uint4* src = reinterpret_cast<const uint4*>(w + (ok ? id : 0) * H);
  uint4* dst = reinterpret_cast<uint4*>(out + t * H);
  for (int c = threadIdx.x; c < H / 8; c += blockDim.x) dst[c] = ok ? src[c] : make_uint4(0, 0, 0, 0);
}

void embedding(torch::Tensor out, torch::Tensor ids, torch::Tensor w, int64_t vocab_start) {
  CHECK_BF16(w);
  TORCH_CHECK(ids.scalar_type() == at::kInt, "ids must be int32");
  const int H = static_cast<int>(w.size(1));
  TORCH_CHECK(H % 8 == 0);
  int64_t T = ids.numel();
  if (!T) return;
  launch_pdl(embedding_kernel, dim3(T), dim3(128), 0, cur_stream(), 
      reinterpret_cast<__nv_bfloat16*>(out.data_ptr<at::BFloat16>()), ids.data_ptr<int32_t>(),
      reinterpret_cast<const __nv_bfloat16*>(w.data_ptr<at::BFloat16>()), H, w.size(0), vocab_start);
  SWIFT_CHECK_LAUNCH();
}

// ------------------------------------------------- QKV split + RoPE + KV write
// One CTA per token. q heads and k heads get the neox (rotate-half) rotation
// over the first `rot` channels; k and v land in the paged pool
// [blocks, layers, 2, kv_heads, block_size, D] at slot_mapping[t] (-1 skips).
__global__ void qkv_rope_cache_kernel(__nv_bfloat16* __restrict__ q_out,
                                      const __nv_bfloat16* __restrict__ qkv,
                                      const __nv_bfloat16* __restrict__ bias,
                                      const int32_t* __restrict__ positions,
                                      const float* __restrict__ cos_sin,
                                      __nv_bfloat16* __restrict__ kv, int64_t blk_stride,
                                      int64_t layer_off, int64_t kv_stride, int block_size,
                                      const int32_t* __restrict__ slots, int Hq, int Hkv, int D,
                                      int rot, int max_pos, int64_t num_slots, int* status) {
  pdl_wait();  // previous kernel done (programmatic dependent launch)
  pdl_trigger();
  const int64_t t = blockIdx.x;
  const int row = (Hq + 2 * Hkv) * D;
  const __nv_bfloat16* src = qkv + t * row;
  int pos = positions[t];
  // index guards (always on, one compare each): a position outside the
  // RoPE table is clamped and a slot outside the pool is not written; both
  // are recorded as kErrBadIndex in the status word
  if ((pos < 0 || pos >= max_pos) && threadIdx.x == 0) set_status(status, kErrBadIndex, 100);
  pos = min(max(pos, 0), max_pos - 1);
  const int half = rot / 2;
  const float* cs = cos_sin + static_cast<int64_t>(pos) * rot;
  int slot = slots[t];
  if (slot >= num_slots) {
    if (threadIdx.x == 0) set_status(status, kErrBadIndex, 101);
    slot = -1;
  }
  const int64_t blk = slot >= 0 ? slot / block_size : 0;
  const int off = slot >= 0 ? slot % block_size : 0;
  __nv_bfloat16* kbase = kv + blk * blk_stride + layer_off;
  const int nrot = (Hq + Hkv) * half;
  for (int i = threadIdx.x; i < nrot; i += blockDim.x) {
    int h = i / half, j = i % half;
    int base = h * D;
    float x1 = __bfloat162float(src[base + j]);
    float x2 = __bfloat162float(src[base + j + half]);
    if (bias) {
      x1 += __bfloat162float(bias[base + j]);
      x2 += __bfloat162float(bias[base + j + half]);
    }
    float c = cs[j], s = cs[half + j];
    __nv_bfloat16 o1 = __float2bfloat16(x1 * c - x2 * s);
    __nv_bfloat16 o2 = __float2bfloat16(x2 * c + x1 * s);
    if (h < Hq) {
      q_out[t * Hq * D + base + j] = o1;
      q_out[t * Hq * D + base + j + half] = o2;
    } else if (slot >= 0) {
      int kh = h - Hq;
      __nv_bfloat16* dst = kbase + static_cast<int64_t>(kh) * block_size * D + off * D;
      dst[j] = o1;
      dst[j + half] = o2;
    }
  }
  const int pass = D - rot;
  const int npass = (Hq + Hkv) * pass;
  for (int i = threadIdx.x; i < npass; i += blockDim.x) {
    int h = i / pass, j = rot + i % pass;
    float x = __bfloat162float(src[h * D + j]) + (bias ? __bfloat162float(bias[h * D + j]) : 0.f);
    if (h < Hq) q_out[t * Hq * D + h * D + j] = __float2bfloat16(x);
    else if (slot >= 0)
      kbase[static_cast<int64_t>(h - Hq) * block_size * D + off * D + j] = __float2bfloat16(x);
  }
  if (slot >= 0) {
    const int nv = Hkv * D;
    const __nv_bfloat16* vs = src + (Hq + Hkv) * D;
    __nv_bfloat16* vbase = kbase + kv_stride;
    for (int i = threadIdx.x; i < nv; i += blockDim.x) {
      int h = i / D, j = i % D;
      float x = __bfloat162float(vs[i]) + (bias ? __bfloat162float(bias[(Hq + Hkv) * D + i]) : 0.f);
      vbase[static_cast<int64_t>(h) * block_size * D + off * D + j] = __float2bfloat16(x);
    }
  }
}

void qkv_rope_cache(torch::Tensor q, torch::Tensor qkv, torch::Tensor positions,
                    torch::Tensor cos_sin, torch::Tensor kv, int64_t layer, torch::Tensor slots,
                    int64_t Hq, int64_t Hkv, int64_t D, int64_t rot,
                    c10::optional<torch::Tensor> bias) {
  CHECK_BF16(qkv);
  CHECK_CONTIG(qkv);
  CHECK_BF16(kv);
  CHECK_CONTIG(kv);
  TORCH_CHECK(kv.dim() == 6, "kv pool must be [blocks, layers, 2, kv_heads, block, D]");
  TORCH_CHECK(cos_sin.scalar_type() == at::kFloat && cos_sin.size(1) == rot);
  TORCH_CHECK(rot % 2 == 0 && rot <= D);
  int64_t T = qkv.size(0);
  if (!T) return;
  const int bs = static_cast<int>(kv.size(4));
  launch_pdl(qkv_rope_cache_kernel, dim3(T), dim3(256), 0, cur_stream(), 
      reinterpret_cast<__nv_bfloat16*>(q.data_ptr<at::BFloat16>()),
      reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr<at::BFloat16>()),
      bias.has_value() ? reinterpret_cast<const __nv_bfloat16*>(bias.value().data_ptr<at::BFloat16>()) : nullptr,
      positions.data_ptr<int32_t>(), cos_sin.data_ptr<float>(),
      reinterpret_cast<__nv_bfloat16*>(kv.data_ptr<at::BFloat16>()), kv.stride(0),
      layer * kv.stride(1), kv.stride(2), bs, slots.data_ptr<int32_t>(), static_cast<int>(Hq),
      static_cast<int>(Hkv), static_cast<int>(D), static_cast<int>(rot),
      static_cast<int>(cos_sin.size(0)), static_cast<int64_t>(kv.size(0)) * bs, status_word_ptr());
  SWIFT_CHECK_LAUNCH();
}

// ---------------------------------------------------------------- copy_blocks
__global__ void copy_blocks_kernel(uint4* __restrict__ kv, const int32_t* __restrict__ pairs,
                                   int64_t blk_vec, int64_t num_blocks, int* status) {
  const int p = blockIdx.y;
  const int64_t src = pairs[2 * p], dst = pairs[2 * p + 1];
  if (src < 0 || src >= num_blocks || dst < 0 || dst >= num_blocks) {  // index guard
    if (blockIdx.x == 0 && threadIdx.x == 0) set_status(status, kErrBadIndex, 110);
    return;
  }
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < blk_vec;
       i += (int64_t)gridDim.x * blockDim.x)
    kv[dst * blk_vec + i] = kv[src * blk_vec + i];
}

void copy_blocks(torch::Tensor kv, torch::Tensor pairs) {
  CHECK_CONTIG(kv);
  TORCH_CHECK(pairs.scalar_type() == at::kInt && pairs.dim() == 2 && pairs.size(1) == 2);
  int64_t n = pairs.size(0);
  if (!n) return;
  int64_t bytes = kv.stride(0) * kv.element_size();
  TORCH_CHECK(bytes % 16 == 0);
  dim3 grid(64, static_cast<unsigned>(n));
  copy_blocks_kernel<<<grid, 256, 0, cur_stream()>>>(reinterpret_cast<uint4*>(kv.data_ptr()),
                                                     pairs.data_ptr<int32_t>(), bytes / 16,
                                                     static_cast<int64_t>(kv.size(0)),
                                                     status_word_ptr());
  SWIFT_CHECK_LAUNCH();
}

// ---------------------------------------------------------------- dummy init
// view [E, R, C] (any strides) of a logical [E, full_rows, full_cols] tensor
// at (row0, col0): element -> Philox(key, flat logical index) -> Box-Muller.
template <typename T>
__global__ void init_normal_kernel(T* __restrict__ out, int64_t E, int64_t R, int64_t C,
                                   int64_t se, int64_t sr, int64_t sc, uint64_t key, float std,
                                   int64_t full_rows, int64_t full_cols, int64_t row0, int64_t col0) {
  const int64_t n = E * R * C;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    int64_t e = i / (R * C), rc = i % (R * C), r = rc / C, c = rc % C;
    uint64_t idx = static_cast<uint64_t>(e * full_rows * full_cols + (row0 + r) * full_cols + (col0 + c));
    uint32_t o[4];
    philox4x32(key, static_cast<uint32_t>(idx), static_cast<uint32_t>(idx >> 32), 0, 0, o);
    float u1 = static_cast<float>((o[0] >> 8) + 1) * (1.0f / 16777216.0f);
    float u2 = static_cast<float>(o[1] >> 8) * (1.0f / 16777216.0f);
    float z = sqrtf(-2.0f * logf(u1)) * cosf(6.283185307179586f * u2);
    out[e * se + r * sr + c * sc] = static_cast<T>(z * std);
  }
}

void init_normal(torch::Tensor v, int64_t key, double std, int64_t full_rows, int64_t full_cols,
                 int64_t row0, int64_t col0) {
  TORCH_CHECK(v.dim() == 3);
  int64_t n = v.numel();
  if (!n) return;
  int blocks = static_cast<int>(std::min<int64_t>((n + 255) / 256, 148 * 32));
  auto st = cur_stream();
  const uint64_t k = static_cast<uint64_t>(key);
  const float sd = static_cast<float>(std);
  if (v.scalar_type() == at::kBFloat16) {
    init_normal_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(
        reinterpret_cast<__nv_bfloat16*>(v.data_ptr<at::BFloat16>()), v.size(0), v.size(1),
        v.size(2), v.stride(0), v.stride(1), v.stride(2), k, sd, full_rows, full_cols, row0, col0);
  } else if (v.scalar_type() == at::kFloat) {
    init_normal_kernel<float><<<blocks, 256, 0, st>>>(
        v.data_ptr<float>(), v.size(0), v.size(1), v.size(2), v.stride(0), v.stride(1),
        v.stride(2), k, sd, full_rows, full_cols, row0, col0);
  } else if (v.scalar_type() == at::kHalf) {
    init_normal_kernel<__half><<<blocks, 256, 0, st>>>(
        reinterpret_cast<__half*>(v.data_ptr<at::Half>()), v.size(0), v.size(1), v.size(2),
        v.stride(0), v.stride(1), v.stride(2), k, sd, full_rows, full_cols, row0, col0);
  } else {
    TORCH_CHECK(false, "init_normal: unsupported dtype");
  }
  SWIFT_CHECK_LAUNCH();
}

// ---------------------------------------------------------------- status
std::vector<int64_t> read_status(bool clear) {
  int h[2] = {0, 0};
  int* p = status_word_ptr();
  SWIFT_CHECK_CUDA(cudaMemcpy(h, p, sizeof(h), cudaMemcpyDeviceToHost));
  if (clear) SWIFT_CHECK_CUDA(cudaMemset(p, 0, sizeof(h)));
  return {h[0], h[1]};
}

}  // namespace swift
