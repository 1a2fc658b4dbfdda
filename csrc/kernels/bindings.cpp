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
                     const c10::optional<at::Tensor>& part_lse, bool causal,
                     const c10::optional<at::Tensor>& err);
void paged_attention_tc(const at::Tensor& q, const at::Tensor& k_cache, const at::Tensor& v_cache,
                        at::Tensor& out, const at::Tensor& block_tables, const at::Tensor& seq_lens,
                        const at::Tensor& cu_q, const at::Tensor& tile_seq,
                        const at::Tensor& tile_row0, int64_t group, double scale, bool causal,
                        const c10::optional<at::Tensor>& err);
void paged_decode_tma(const at::Tensor& q, const at::Tensor& k_cache, const at::Tensor& v_cache,
                      at::Tensor& out, const at::Tensor& block_tables, const at::Tensor& seq_lens,
                      int64_t group, double scale, int64_t num_splits,
                      const c10::optional<at::Tensor>& part_o,
                      const c10::optional<at::Tensor>& part_lse, at::Tensor& err);
void gemm_bf16_tp(const at::Tensor& A, const at::Tensor& W, at::Tensor& C, int64_t mode,
                  at::Tensor& err, int64_t splits, std::vector<int64_t> scatter_ptrs,
                  std::vector<int64_t> signal_ptrs, int64_t rows_per_rank, int64_t src_rank,
                  int64_t slot_stride, int64_t wait_flag_ptr, int64_t wait_count,
                  int64_t done_counter_ptr, int64_t trace_ptr,
                  const c10::optional<at::Tensor>& ws);
int64_t allreduce_buffer_bytes(int64_t max_elems, int64_t world);
void gemm_bf16_pair(const at::Tensor& A, const at::Tensor& W, at::Tensor& C,
                    const c10::optional<at::Tensor>& residual, int64_t mode, at::Tensor& err,
                    int64_t bt);
void allreduce_prepare(int64_t base, int64_t max_elems, int64_t world);
void gemv_bf16(const at::Tensor& A, const at::Tensor& W, at::Tensor& C,
               const c10::optional<at::Tensor>& residual, int64_t mode);
bool allreduce_rmsnorm_p2p(at::Tensor& h, const at::Tensor& inp, at::Tensor& x,
                           const at::Tensor& w, std::vector<int64_t> bases, int64_t rank,
                           int64_t max_elems, int64_t ctas, double eps, at::Tensor& err);
void allreduce_p2p(at::Tensor& out, const at::Tensor& inp, std::vector<int64_t> bases,
                   int64_t rank, int64_t n_elems, int64_t max_elems, int64_t ctas,
                   at::Tensor& err);
int64_t rowpar_buffer_bytes(int64_t max_tokens, int64_t hidden, int64_t world);
std::vector<int64_t> rowpar_geometry(int64_t max_tokens, int64_t hidden, int64_t world);
void rowpar_prepare(int64_t base, int64_t max_tokens, int64_t hidden, int64_t world);
void rowpar_norm(at::Tensor& h, const c10::optional<at::Tensor>& partial, at::Tensor& x_own,
                 const at::Tensor& w, std::vector<int64_t> bases, int64_t rank, int64_t T,
                 int64_t max_tokens, double eps, int64_t ctas, at::Tensor& err,
                 int64_t trace_ptr);
void gemm_bf16_rowpar(const at::Tensor& A, const at::Tensor& W, at::Tensor& err,
                      std::vector<int64_t> recv1_ptrs, int64_t rank, int64_t rp_max,
                      int64_t epoch_ptr, const c10::optional<at::Tensor>& ws, int64_t splits,
                      int64_t trace_ptr);
void set_pdl_launch(bool on);
bool pdl_launch_enabled();
void set_comm_fence_mode(int64_t mode);
int64_t ipc_alloc(int64_t bytes);
void ipc_free(int64_t ptr);
at::Tensor ipc_export(int64_t ptr);
int64_t ipc_open(const at::Tensor& handle);
void ipc_close(int64_t ptr);
void rs_norm_ag(int64_t rs_ptr, const c10::optional<at::Tensor>& x_in, at::Tensor& residual,
                const at::Tensor& w, std::vector<int64_t> gather_ptrs,
                std::vector<int64_t> gather_flag_ptrs, int64_t rs_flag_ptr,
                int64_t done_counter_ptr, int64_t rank, int64_t R, int64_t rows, double eps,
                bool add_residual, at::Tensor& err, int64_t trace_ptr);
void h2o_accumulate(const at::Tensor& q, const at::Tensor& k_cache, const at::Tensor& block_tables,
                    const at::Tensor& seq_lens, at::Tensor& score, double decay, double scale,
                    at::Tensor& ws_logits, at::Tensor& ws_part);
void kv_compact(at::Tensor& storage, const at::Tensor& src, const at::Tensor& dst,
                const c10::optional<at::Tensor>& score);
void gemm_quant(const at::Tensor& X, const at::Tensor& qw, const at::Tensor& scales,
                const at::Tensor& offsets, int64_t bits, int64_t group, at::Tensor& C,
                int64_t mode, int64_t splits, at::Tensor& err, at::Tensor& ws);
void gemm_quant_iz(const at::Tensor& X, const at::Tensor& qw, const at::Tensor& scales,
                   const at::Tensor& offsets, int64_t group, at::Tensor& C, int64_t mode,
                   int64_t splits, at::Tensor& err, at::Tensor& ws);
void embedding(const at::Tensor& ids, const at::Tensor& table, at::Tensor& out, at::Tensor& err);
void forward_tokens(at::Tensor& ids, const at::Tensor& src, const at::Tensor& last,
                    at::Tensor& err);
void rmsnorm(const at::Tensor& x, const c10::optional<at::Tensor>& residual, const at::Tensor& w,
             at::Tensor& y, double eps);
void rope_kv(at::Tensor& qkv, const at::Tensor& positions, const c10::optional<at::Tensor>& slots,
             const at::Tensor& cos_sin, at::Tensor& k_cache, at::Tensor& v_cache, int64_t hq,
             int64_t hkv, at::Tensor& err, const c10::optional<at::Tensor>& q_norm,
             const c10::optional<at::Tensor>& k_norm, int64_t norm_dim, double eps);
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
  m.def("paged_attention", &lb::paged_attention, "paged attention (decode / prefill)",
        py::arg("q"), py::arg("k_cache"), py::arg("v_cache"), py::arg("out"),
        py::arg("block_tables"), py::arg("seq_lens"), py::arg("cu_q"), py::arg("tile_seq"),
        py::arg("tile_row0"), py::arg("group"), py::arg("scale"), py::arg("decode"),
        py::arg("num_splits"), py::arg("part_o"), py::arg("part_lse"), py::arg("causal"),
        py::arg("err") = py::none());
  m.def("paged_attention_tc", &lb::paged_attention_tc,
        "tcgen05 paged attention for chunked prefill / verify (S, O in TMEM, P from TMEM)");
  m.def("paged_decode_tma", &lb::paged_decode_tma, "TMA-fed warp-specialised paged decode");
  m.def("gemm_bf16_tp", &lb::gemm_bf16_tp, "tensor-parallel GEMM (wait / scatter / signal)",
        py::arg("A"), py::arg("W"), py::arg("C"), py::arg("mode"), py::arg("err"),
        py::arg("splits"), py::arg("scatter_ptrs"), py::arg("signal_ptrs"),
        py::arg("rows_per_rank"), py::arg("src_rank"), py::arg("slot_stride"),
        py::arg("wait_flag_ptr"), py::arg("wait_count"), py::arg("done_counter_ptr"),
        py::arg("trace_ptr") = 0, py::arg("ws") = py::none());
  m.def("allreduce_buffer_bytes", &lb::allreduce_buffer_bytes);
  m.def("allreduce_prepare", &lb::allreduce_prepare);
  m.def("gemv_bf16", &lb::gemv_bf16, "weight-streaming GEMV for 1-4 tokens");
  m.def("allreduce_rmsnorm_p2p", &lb::allreduce_rmsnorm_p2p,
        "x += allreduce(partial); h = rmsnorm(x) * w, over NVLink peer memory");
  m.def("gemm_bf16_pair", &lb::gemm_bf16_pair, "bf16 GEMM on SM pairs (tcgen05 cta_group::2)",
        py::arg("A"), py::arg("W"), py::arg("C"), py::arg("residual"), py::arg("mode"),
        py::arg("err"), py::arg("bt") = 0);
  m.def("allreduce_p2p", &lb::allreduce_p2p, "two-shot all-reduce over NVLink peer memory");
  m.def("rowpar_buffer_bytes", &lb::rowpar_buffer_bytes);
  m.def("rowpar_geometry", &lb::rowpar_geometry);
  m.def("rowpar_prepare", &lb::rowpar_prepare);
  m.def("rowpar_norm", &lb::rowpar_norm,
        "row-parallel exchange: reduce own rows + residual + RMSNorm, all-gather normed rows",
        py::arg("h"), py::arg("partial"), py::arg("x_own"), py::arg("w"), py::arg("bases"),
        py::arg("rank"), py::arg("T"), py::arg("max_tokens"), py::arg("eps"), py::arg("ctas"),
        py::arg("err"), py::arg("trace_ptr") = 0);
  m.def("gemm_bf16_rowpar", &lb::gemm_bf16_rowpar,
        "row-parallel GEMM pushing its output rows into the owners' exchange slots",
        py::arg("A"), py::arg("W"), py::arg("err"), py::arg("recv1_ptrs"), py::arg("rank"),
        py::arg("rp_max"), py::arg("epoch_ptr"), py::arg("ws") = py::none(),
        py::arg("splits") = 0, py::arg("trace_ptr") = 0);
  m.def("set_pdl", &lb::set_pdl_launch,
        "launch the decode-path kernels with programmatic dependent launch (default on)");
  m.def("pdl_enabled", &lb::pdl_launch_enabled);
  m.def("set_comm_fence_mode", &lb::set_comm_fence_mode,
        "peer-exchange launch-start fence: 1 every thread, 2 one per CTA, 0 none (measurement)");
  m.def("ipc_alloc", &lb::ipc_alloc);
  m.def("ipc_free", &lb::ipc_free);
  m.def("ipc_export", &lb::ipc_export);
  m.def("ipc_open", &lb::ipc_open);
  m.def("ipc_close", &lb::ipc_close);
  m.def("rs_norm_ag", &lb::rs_norm_ag, "reduce-scatter sum + residual + RMSNorm + all-gather",
        py::arg("rs_ptr"), py::arg("x_in"), py::arg("residual"), py::arg("w"),
        py::arg("gather_ptrs"), py::arg("gather_flag_ptrs"), py::arg("rs_flag_ptr"),
        py::arg("done_counter_ptr"), py::arg("rank"), py::arg("R"), py::arg("rows"),
        py::arg("eps"), py::arg("add_residual"), py::arg("err"), py::arg("trace_ptr") = 0);
  m.def("h2o_accumulate", &lb::h2o_accumulate, "H2O decayed attention-mass accumulation");
  m.def("kv_compact", &lb::kv_compact, "copy kept KV token slots (all layers)");
  m.def("gemm_quant", &lb::gemm_quant, "dequant-fused tcgen05 GEMM (int4 / int8 groups)");
  m.def("gemm_quant_iz", &lb::gemm_quant_iz,
        "small-batch 4-bit GEMM with integer zero points (weights in TMEM, per-group rescale)");
  m.def("embedding", &lb::embedding, "embedding gather");
  m.def("forward_tokens", &lb::forward_tokens, "patch input ids from the previous step's samples");
  m.def("rmsnorm", &lb::rmsnorm, "RMSNorm with optional fused residual add");
  m.def("rope_kv", &lb::rope_kv, "RoPE + paged KV append (optional per-head q/k RMSNorm)",
        py::arg("qkv"), py::arg("positions"), py::arg("slots"), py::arg("cos_sin"),
        py::arg("k_cache"), py::arg("v_cache"), py::arg("hq"), py::arg("hkv"), py::arg("err"),
        py::arg("q_norm") = py::none(), py::arg("k_norm") = py::none(), py::arg("norm_dim") = 0,
        py::arg("eps") = 1e-6);
  m.def("sample_tokens", &lb::sample_tokens, "greedy / top-k / top-p sampling");
}
