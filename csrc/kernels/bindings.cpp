// Python bindings for the sm_100a kernels (module lightbulb_b200._C).
#include <torch/extension.h>

namespace lb {
void gemm_bf16(const at::Tensor& A, const at::Tensor& W, at::Tensor& C,
               const c10::optional<at::Tensor>& residual, int64_t mode, at::Tensor& ws,
               at::Tensor& counters, at::Tensor& err, int64_t bt, int64_t splits,
               const c10::optional<at::Tensor>& trace);
std::vector<int64_t> gemm_plan(int64_t M, int64_t N, int64_t K, int64_t bt, int64_t splits);
void paged_attention(const at::Tensor& q, const at::Tensor& k_cache, const at::Tensor& v_cache,
                     at::Tensor& out, const at::Tensor& block_tables, const at::Tensor& seq_lens,
                     const at::Tensor& cu_q, const c10::optional<at::Tensor>& tile_seq,
                     const c10::optional<at::Tensor>& tile_row0, int64_t group, double scale,
                     bool decode, int64_t num_splits, const c10::optional<at::Tensor>& part_o,
                     const c10::optional<at::Tensor>& part_lse, bool causal);
void paged_decode_tma(const at::Tensor& q, const at::Tensor& k_cache, const at::Tensor& v_cache,
                      at::Tensor& out, const at::Tensor& block_tables, const at::Tensor& seq_lens,
                      int64_t group, double scale, int64_t num_splits,
                      const c10::optional<at::Tensor>& part_o,
                      const c10::optional<at::Tensor>& part_lse, at::Tensor& err);
void embedding(const at::Tensor& ids, const at::Tensor& table, at::Tensor& out, at::Tensor& err);
void rmsnorm(const at::Tensor& x, const c10::optional<at::Tensor>& residual, const at::Tensor& w,
             at::Tensor& y, double eps);
void rope_kv(at::Tensor& qkv, const at::Tensor& positions, const c10::optional<at::Tensor>& slots,
             const at::Tensor& cos_sin, at::Tensor& k_cache, at::Tensor& v_cache, int64_t hq,
             int64_t hkv, at::Tensor& err);
void sample_tokens(const at::Tensor& logits, const at::Tensor& temperature,
                   const at::Tensor& top_k, const at::Tensor& top_p, const at::Tensor& seeds,
                   at::Tensor& out_tokens, const c10::optional<at::Tensor>& out_logprob);
}  // namespace lb

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "lightbulb_b200 sm_100a kernels";
  m.def("gemm_bf16", &lb::gemm_bf16, "tcgen05 GEMM C = A W^T with fused epilogue",
        py::arg("A"), py::arg("W"), py::arg("C"), py::arg("residual"), py::arg("mode"),
        py::arg("ws"), py::arg("counters"), py::arg("err"), py::arg("bt"), py::arg("splits"),
        py::arg("trace") = py::none());
  m.def("gemm_plan", &lb::gemm_plan, "token tile, split-K and workspace size of a GEMM");
  m.def("paged_attention", &lb::paged_attention, "paged attention (decode / prefill)");
  m.def("paged_decode_tma", &lb::paged_decode_tma, "TMA-fed warp-specialised paged decode");
  m.def("embedding", &lb::embedding, "embedding gather");
  m.def("rmsnorm", &lb::rmsnorm, "RMSNorm with optional fused residual add");
  m.def("rope_kv", &lb::rope_kv, "RoPE + paged KV append");
  m.def("sample_tokens", &lb::sample_tokens, "greedy / top-k / top-p sampling");
}
