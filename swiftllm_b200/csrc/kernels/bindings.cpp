// torch extension module swiftllm_b200._C: the sm_100a kernels.
#include <torch/extension.h>

#include <vector>

namespace swift {
void rms_norm(torch::Tensor out, torch::Tensor x, torch::Tensor w, double eps);
void fused_add_rms_norm(torch::Tensor out, torch::Tensor x, torch::Tensor residual, torch::Tensor w,
                        double eps);
void layer_norm(torch::Tensor out, torch::Tensor x, torch::Tensor w, c10::optional<torch::Tensor> b,
                double eps);
void fused_add_layer_norm(torch::Tensor out, torch::Tensor x, torch::Tensor residual,
                          torch::Tensor w, c10::optional<torch::Tensor> b, double eps);
void silu_and_mul(torch::Tensor out, torch::Tensor x);
void gelu_tanh(torch::Tensor out, torch::Tensor x);
void embedding(torch::Tensor out, torch::Tensor ids, torch::Tensor w, int64_t vocab_start);
void qkv_rope_cache(torch::Tensor q, torch::Tensor qkv, torch::Tensor positions,
                    torch::Tensor cos_sin, torch::Tensor kv, int64_t layer, torch::Tensor slots,
                    int64_t Hq, int64_t Hkv, int64_t D, int64_t rot,
                    c10::optional<torch::Tensor> bias);
void copy_blocks(torch::Tensor kv, torch::Tensor pairs);
void init_normal(torch::Tensor v, int64_t key, double std, int64_t full_rows, int64_t full_cols,
                 int64_t row0, int64_t col0);
std::vector<int64_t> read_status(bool clear);
int64_t paged_decode(torch::Tensor out, torch::Tensor q, torch::Tensor kv, int64_t layer,
                     torch::Tensor bt, torch::Tensor seq_lens, int64_t rows, int64_t splits,
                     double scale, int64_t window, torch::Tensor ws,
                     c10::optional<torch::Tensor> alibi);
void paged_prefill(torch::Tensor out, torch::Tensor q, torch::Tensor kv, int64_t layer,
                   torch::Tensor bt, torch::Tensor q_start, torch::Tensor seq_lens, int64_t seq0,
                   int64_t seq1, int64_t max_q_len, double scale, int64_t window, int64_t impl,
                   c10::optional<torch::Tensor> alibi);
void sample(torch::Tensor tokens, torch::Tensor lps, torch::Tensor logits, torch::Tensor fparams,
            torch::Tensor iparams, torch::Tensor keys, bool any_random);
int64_t gemm(torch::Tensor out, torch::Tensor x, torch::Tensor w, c10::optional<torch::Tensor> bias);
void apply_penalties(torch::Tensor logits, torch::Tensor offsets, torch::Tensor tokens,
                     torch::Tensor out_counts, torch::Tensor fparams);
std::vector<int64_t> gemm_plan(int64_t M, int64_t N, int64_t K);
void gemm_streamk_config(int64_t mode, int64_t mt, int64_t min_per);
void quantize_e4m3(torch::Tensor q, torch::Tensor scale, torch::Tensor x);
void quantize_s8(torch::Tensor q, torch::Tensor scale, torch::Tensor x);
int64_t gemm_s8(torch::Tensor out, torch::Tensor xq, torch::Tensor xscale, torch::Tensor wq,
                torch::Tensor wscale, c10::optional<torch::Tensor> bias);
int64_t gemm_e4m3(torch::Tensor out, torch::Tensor xq, torch::Tensor xscale, torch::Tensor wq,
                  torch::Tensor wscale, c10::optional<torch::Tensor> bias);
int64_t gemm_packed(torch::Tensor out, torch::Tensor x, torch::Tensor wp, int64_t M,
                    c10::optional<torch::Tensor> bias);
int64_t tp_reduce_norm(std::vector<int64_t> bases, int64_t mc, int64_t rank, int64_t in_off,
                       int64_t out_off, int64_t ctr_off, c10::optional<torch::Tensor> residual,
                       c10::optional<torch::Tensor> w, double eps, int64_t T, int64_t H,
                       torch::Tensor epochs, double timeout_s);
int64_t tp_vocab_argmax(std::vector<int64_t> bases, int64_t mc, int64_t rank, torch::Tensor logits,
                        int64_t v0, int64_t cand_off, int64_t ctr_off, torch::Tensor tokens,
                        torch::Tensor lps, torch::Tensor epochs, double timeout_s);
int64_t gemm2(torch::Tensor out, torch::Tensor x, torch::Tensor w, c10::optional<torch::Tensor> bias,
              int64_t plan, int64_t bn, int64_t splits);
std::vector<int64_t> gemm2_plan_py(int64_t M, int64_t N, int64_t K);
int64_t gemm_swiglu(torch::Tensor out, torch::Tensor x, torch::Tensor w13);
void flag_wait_probe(torch::Tensor flag, int64_t want, double timeout_s);
int64_t gemm_grouped(torch::Tensor out, torch::Tensor x, torch::Tensor w, torch::Tensor offsets,
                     int64_t avg_rows);
void moe_route(torch::Tensor logits, int64_t k, bool renorm, torch::Tensor w_out,
               torch::Tensor id_out);
void moe_permute(torch::Tensor ids, int64_t e0, int64_t E_local, torch::Tensor offsets,
                 torch::Tensor perm_token, torch::Tensor inv_slot);
void moe_combine(torch::Tensor out, torch::Tensor y, torch::Tensor weights, torch::Tensor inv_slot);
void moe_gather(torch::Tensor xg, torch::Tensor x, torch::Tensor perm_token);
int64_t tp_gather_vocab(std::vector<int64_t> bases, int64_t mc, int64_t rank, torch::Tensor logits,
                        int64_t dst_off, int64_t ctr_off, torch::Tensor epochs, double timeout_s);
void spec_verify_greedy(torch::Tensor logits, torch::Tensor pos, torch::Tensor draft,
                        torch::Tensor temp, torch::Tensor out);
int64_t gemm_w4a16(torch::Tensor out, torch::Tensor x, torch::Tensor qp, torch::Tensor sz,
                   int64_t M, int64_t group, c10::optional<torch::Tensor> bias);
int64_t gemm_nvfp4w(torch::Tensor out, torch::Tensor x, torch::Tensor qp, torch::Tensor sc,
                    int64_t M, double gscale, c10::optional<torch::Tensor> bias);
}  // namespace swift

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "swiftllm_b200 sm_100a kernels";
  m.def("rms_norm", &swift::rms_norm);
  m.def("fused_add_rms_norm", &swift::fused_add_rms_norm);
  m.def("layer_norm", &swift::layer_norm);
  m.def("fused_add_layer_norm", &swift::fused_add_layer_norm);
  m.def("silu_and_mul", &swift::silu_and_mul);
  m.def("gelu_tanh", &swift::gelu_tanh);
  m.def("embedding", &swift::embedding);
  m.def("qkv_rope_cache", &swift::qkv_rope_cache);
  m.def("copy_blocks", &swift::copy_blocks);
  m.def("init_normal", &swift::init_normal);
  m.def("read_status", &swift::read_status, pybind11::arg("clear") = true);
  m.def("paged_decode", &swift::paged_decode, pybind11::arg("out"), pybind11::arg("q"),
        pybind11::arg("kv"), pybind11::arg("layer"), pybind11::arg("bt"), pybind11::arg("seq_lens"),
        pybind11::arg("rows"), pybind11::arg("splits"), pybind11::arg("scale"),
        pybind11::arg("window"), pybind11::arg("ws"), pybind11::arg("alibi") = pybind11::none());
  m.def("paged_prefill", &swift::paged_prefill, pybind11::arg("out"), pybind11::arg("q"),
        pybind11::arg("kv"), pybind11::arg("layer"), pybind11::arg("bt"), pybind11::arg("q_start"),
        pybind11::arg("seq_lens"), pybind11::arg("seq0"), pybind11::arg("seq1"),
        pybind11::arg("max_q_len"), pybind11::arg("scale"), pybind11::arg("window"),
        pybind11::arg("impl") = -1, pybind11::arg("alibi") = pybind11::none());
  m.def("sample", &swift::sample);
  m.def("apply_penalties", &swift::apply_penalties);
  m.def("gemm", &swift::gemm);
  m.def("gemm_plan", &swift::gemm_plan);
  m.def("gemm_streamk_config", &swift::gemm_streamk_config);
  m.def("gemm_packed", &swift::gemm_packed);
  m.def("gemm_e4m3", &swift::gemm_e4m3);
  m.def("quantize_e4m3", &swift::quantize_e4m3);
  m.def("quantize_s8", &swift::quantize_s8);
  m.def("gemm_s8", &swift::gemm_s8);
  m.def("flag_wait_probe", &swift::flag_wait_probe);
  m.def("gemm2", &swift::gemm2, pybind11::arg("out"), pybind11::arg("x"), pybind11::arg("w"),
        pybind11::arg("bias"), pybind11::arg("plan") = -1, pybind11::arg("bn") = 0,
        pybind11::arg("splits") = 0);
  m.def("gemm2_plan", &swift::gemm2_plan_py);
  m.def("gemm_swiglu", &swift::gemm_swiglu);
  m.def("tp_reduce_norm", &swift::tp_reduce_norm);
  m.def("tp_vocab_argmax", &swift::tp_vocab_argmax);
  m.def("gemm_grouped", &swift::gemm_grouped);
  m.def("moe_route", &swift::moe_route);
  m.def("moe_permute", &swift::moe_permute);
  m.def("moe_combine", &swift::moe_combine);
  m.def("gemm_w4a16", &swift::gemm_w4a16);
  m.def("gemm_nvfp4w", &swift::gemm_nvfp4w);
  m.def("moe_gather", &swift::moe_gather);
  m.def("tp_gather_vocab", &swift::tp_gather_vocab);
  m.def("spec_verify_greedy", &swift::spec_verify_greedy);
}
