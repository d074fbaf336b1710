// Python bindings of the native sm_100a kernels (module braidinfer_b200._C).
#include <torch/extension.h>

namespace braid {
int64_t gemm(torch::Tensor out, torch::Tensor x, torch::Tensor w, c10::optional<torch::Tensor> bias,
             c10::optional<torch::Tensor> residual, int64_t epi, double rs_eps, c10::optional<torch::Tensor> rs_vec,
             c10::optional<torch::Tensor> sp);
void gemm_qkv(torch::Tensor q_out, torch::Tensor x, torch::Tensor w, c10::optional<torch::Tensor> bias,
              double rs_eps, torch::Tensor positions, torch::Tensor slots, torch::Tensor kv,
              c10::optional<torch::Tensor> q_norm, c10::optional<torch::Tensor> k_norm, double head_eps,
              torch::Tensor cos, torch::Tensor sin, int64_t Hq, int64_t Hkv, int64_t D, bool use_rope,
              c10::optional<torch::Tensor> rs_vec, c10::optional<torch::Tensor> sp);
void row_rstd(torch::Tensor x, double eps, torch::Tensor out);
unsigned long long bounds_status_gemm();
unsigned long long bounds_status_gemm_persistent();
unsigned long long bounds_status_attention();
unsigned long long bounds_status_attention_tc();
unsigned long long bounds_status_elementwise();
unsigned long long bounds_status_sampling();
unsigned long long bounds_status_comm();

// First bounds violation recorded since the last call (0: none), in the
// checked build: code << 48 | value; every file's word is read and cleared.
int64_t bounds_check_status() {
  unsigned long long first = 0;
  for (auto fn : {bounds_status_gemm, bounds_status_gemm_persistent, bounds_status_attention, bounds_status_attention_tc, bounds_status_elementwise, bounds_status_sampling, bounds_status_comm}) {
    const unsigned long long v = fn();
    if (first == 0) first = v;
  }
  return (int64_t)first;
}
bool bounds_check_enabled() {
#ifdef BRAID_BOUNDS_CHECK
  return true;
#else
  return false;
#endif
}
int64_t sp_reduce_allgather(torch::Tensor peers, int64_t recv_off, int64_t rs_flags_off, int64_t ag_flags_off,
                            int64_t g_off, int64_t rstd_off, int64_t rank, int64_t tp, int64_t rpr, int64_t T,
                            int64_t H, int64_t rs_expected, double eps, torch::Tensor status, double timeout_s);
void sp_wait(int64_t local_ptr, int64_t ag_flags_off, int64_t tp, int64_t rank, int64_t expected,
             torch::Tensor status, double timeout_s);
torch::Tensor comm_tensor(int64_t ptr, int64_t offset, std::vector<int64_t> shape, int64_t dtype, int64_t device);
int64_t gemm_check_error(int64_t device);
void gemm_set_trace(torch::Tensor buf);
void gemm_force_splits(int64_t n);
void gemm_force_bn(int64_t n);
int64_t span_trace(torch::Tensor buf);
int64_t gemm_prefetch_next(torch::Tensor w, int64_t T, int64_t skip);
std::vector<std::string> span_names();
void gemm_allreduce_add(torch::Tensor residual, torch::Tensor x, torch::Tensor w, torch::Tensor peers,
                        int64_t flags_off, int64_t tile_flags_off, int64_t max_tiles, int64_t rank, int64_t tp,
                        int64_t maxT, torch::Tensor epoch_state, torch::Tensor status, double timeout_s);
int64_t gemm_push(torch::Tensor x, torch::Tensor w, torch::Tensor peers, int64_t flags_off, int64_t rank, int64_t tp,
                  int64_t maxT, torch::Tensor epoch_state);
std::vector<torch::Tensor> comm_alloc(int64_t nbytes, int64_t device);
int64_t comm_open(torch::Tensor handle, int64_t device);
void comm_close(int64_t ptr, int64_t device);
void comm_free(int64_t ptr, int64_t device);
void tp_push(torch::Tensor x, torch::Tensor peers, int64_t flags_off, int64_t rank, int64_t tp, int64_t maxT,
             torch::Tensor epoch_state);
void tp_reduce_add(torch::Tensor out, torch::Tensor residual, bool add_residual, int64_t buf, int64_t flags_off,
                   int64_t tp, int64_t maxT, int64_t rank, int64_t arrivals_per_call, torch::Tensor epoch_state,
                   torch::Tensor status, double timeout_s);
void attention(torch::Tensor out, torch::Tensor q, torch::Tensor kv, torch::Tensor qo_indptr,
               torch::Tensor positions, torch::Tensor seg_indptr, torch::Tensor seg_page_indptr,
               torch::Tensor seg_offset, torch::Tensor seg_len, torch::Tensor seg_pos0, torch::Tensor seg_delta,
               torch::Tensor page_ids, torch::Tensor cos, torch::Tensor sin, double scale, bool use_rope,
               int64_t num_seqs, int64_t max_q_len, int64_t max_kv_len, bool decode, int64_t num_splits,
               c10::optional<torch::Tensor> part_o, c10::optional<torch::Tensor> part_lse,
               c10::optional<torch::Tensor> grp_qo_indptr, c10::optional<torch::Tensor> grp_seg_indptr,
               c10::optional<torch::Tensor> seq_nsh, int64_t shared_splits, int64_t grp_max_q);
void attn_set_trace(torch::Tensor buf);
void attn_tc_set_trace(torch::Tensor buf);
void attn_select_prefill_tc(int64_t mode);
int64_t attn_prefill_tile_rows(int64_t D);
void attn_set_exp2_poly(int64_t n);
void rms_norm(torch::Tensor out, torch::Tensor x, torch::Tensor w, double eps);
void add_rms_norm(torch::Tensor out, torch::Tensor residual, torch::Tensor x, torch::Tensor w, double eps);
void layer_norm(torch::Tensor out, torch::Tensor x, torch::Tensor w, torch::Tensor b, double eps);
void gelu_tanh(torch::Tensor out, torch::Tensor x);
void embedding(torch::Tensor out, torch::Tensor ids, torch::Tensor w, int64_t vocab_start);
void qkv_prepare(torch::Tensor q_out, torch::Tensor qkv, torch::Tensor positions, torch::Tensor slots,
                 torch::Tensor kv, c10::optional<torch::Tensor> q_norm, c10::optional<torch::Tensor> k_norm,
                 double eps, torch::Tensor cos, torch::Tensor sin, int64_t Hq, int64_t Hkv, int64_t D,
                 bool use_rope);
int64_t tp_sample_record_bytes();
void tp_sample(torch::Tensor out, torch::Tensor logits, int64_t vocab_start, int64_t vocab_size,
               torch::Tensor temperature, torch::Tensor top_k, torch::Tensor top_p, torch::Tensor min_p,
               torch::Tensor seed, torch::Tensor step, torch::Tensor peers, int64_t recv_off, int64_t flags_off,
               int64_t rank, int64_t tp, int64_t maxB, torch::Tensor epoch_state, torch::Tensor status,
               double timeout_s);
void sample(torch::Tensor out, torch::Tensor logits, torch::Tensor temperature, torch::Tensor top_k,
            torch::Tensor top_p, torch::Tensor min_p, torch::Tensor seed, torch::Tensor step, bool all_greedy);
}  // namespace braid

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "braidinfer_b200 native sm_100a kernels";
  m.def("gemm", &braid::gemm, "tcgen05 GEMM out = x @ w^T (+bias)(+residual); epi 1 = SwiGLU, 4 = reduce-scatter",
        py::arg("out"), py::arg("x"), py::arg("w"), py::arg("bias"), py::arg("residual"), py::arg("epi"),
        py::arg("rs_eps"), py::arg("rs_vec") = py::none(), py::arg("sp") = py::none());
  m.def("gemm_qkv", &braid::gemm_qkv, "tcgen05 QKV GEMM with fused q/k-norm, RoPE(k) and paged KV append",
        py::arg("q_out"), py::arg("x"), py::arg("w"), py::arg("bias"), py::arg("rs_eps"), py::arg("positions"),
        py::arg("slots"), py::arg("kv"), py::arg("q_norm"), py::arg("k_norm"), py::arg("head_eps"), py::arg("cos"),
        py::arg("sin"), py::arg("Hq"), py::arg("Hkv"), py::arg("D"), py::arg("use_rope"),
        py::arg("rs_vec") = py::none(), py::arg("sp") = py::none());
  m.def("row_rstd", &braid::row_rstd, "out[t] = 1/rms(x[t]) in fp32");
  m.def("bounds_check_status", &braid::bounds_check_status,
        "checked build: first recorded bounds violation (code << 48 | value), cleared; 0 = none");
  m.def("bounds_check_enabled", &braid::bounds_check_enabled, "true in the -DBRAID_BOUNDS_CHECK build");
  m.def("sp_reduce_allgather", &braid::sp_reduce_allgather,
        "sequence-parallel reduce of pushed partial rows + all-gather of the new rows and their 1/rms");
  m.def("sp_wait", &braid::sp_wait, "bounded wait for every owner's all-gather");
  m.def("comm_tensor", &braid::comm_tensor, "tensor view of comm-buffer memory");
  m.def("gemm_allreduce_add", &braid::gemm_allreduce_add,
        "row-parallel GEMM with the TP all-reduce (+ residual) done inside the kernel over peer memory");
  m.def("gemm_push", &braid::gemm_push, "row-parallel GEMM whose epilogue pushes bf16 tiles to TP peers");
  m.def("comm_alloc", &braid::comm_alloc, "cudaMalloc a comm buffer; returns (ptr, ipc handle)");
  m.def("comm_open", &braid::comm_open, "map a peer's comm buffer from its IPC handle");
  m.def("comm_close", &braid::comm_close);
  m.def("comm_free", &braid::comm_free);
  m.def("tp_push", &braid::tp_push, "push a bf16 partial to every TP peer");
  m.def("tp_reduce_add", &braid::tp_reduce_add, "bounded-wait sum of pushed partials (+ residual)");
  m.def("gemm_set_trace", &braid::gemm_set_trace, "profiling: per-CTA phase timestamps of later GEMMs");
  m.def("span_trace", &braid::span_trace,
        "profiling: record {first CTA start, first dependency-wait exit, last CTA end} of later GEMM/attention launches");
  m.def("gemm_prefetch_next", &braid::gemm_prefetch_next,
        "name the weight of a later decode GEMM; the next launch pulls its K-blocks [skip, skip + depth) of every "
        "K-slice into L2; returns depth", py::arg("w"), py::arg("T"), py::arg("skip") = 0);
  m.def("span_names", &braid::span_names, "profiling: names of the launches recorded by span_trace, in order");
  m.def("gemm_force_bn", &braid::gemm_force_bn, "tuning: force the decode token-tile width (0 = heuristic)");
  m.def("gemm_force_splits", &braid::gemm_force_splits, "tuning: force the split-K factor (0 = heuristic)");
  m.def("gemm_check_error", &braid::gemm_check_error, "read and clear the GEMM bounded-wait error flag");
  m.def("attention", &braid::attention, "paged cascade attention (decode/prefill; decode with a shared-prefix group)",
        py::arg("out"), py::arg("q"), py::arg("kv"), py::arg("qo_indptr"), py::arg("positions"),
        py::arg("seg_indptr"), py::arg("seg_page_indptr"), py::arg("seg_offset"), py::arg("seg_len"),
        py::arg("seg_pos0"), py::arg("seg_delta"), py::arg("page_ids"), py::arg("cos"), py::arg("sin"),
        py::arg("scale"), py::arg("use_rope"), py::arg("num_seqs"), py::arg("max_q_len"), py::arg("max_kv_len"),
        py::arg("decode"), py::arg("num_splits"), py::arg("part_o") = py::none(), py::arg("part_lse") = py::none(),
        py::arg("grp_qo_indptr") = py::none(), py::arg("grp_seg_indptr") = py::none(),
        py::arg("seq_nsh") = py::none(), py::arg("shared_splits") = 0, py::arg("grp_max_q") = 0);
  m.def("attn_prefill_tile_rows", &braid::attn_prefill_tile_rows,
        "query rows per CTA of the prefill attention kernel for head_dim D (256: tcgen05, one CTA per SM; 64: mma.sync, two)");
  m.def("attn_set_exp2_poly", &braid::attn_set_exp2_poly,
        "tcgen05 prefill softmax: every n-th exponential by polynomial on the FMA pipe (n = 0, 2, 4; -1: BRAID_ATTN_POLY)");
  m.def("attn_select_prefill_tc", &braid::attn_select_prefill_tc,
        "prefill attention for head_dim 128: 1 tcgen05 kernel, 0 mma.sync kernel, -1 BRAID_ATTN_TC");
  m.def("attn_tc_set_trace", &braid::attn_tc_set_trace,
        "profiling: per-tile softmax timestamps of later tcgen05 prefill attention (int64, 128 per CTA)");
  m.def("attn_set_trace", &braid::attn_set_trace, "profiling: per-CTA phase timestamps of later decode attention");
  m.def("rms_norm", &braid::rms_norm);
  m.def("add_rms_norm", &braid::add_rms_norm);
  m.def("layer_norm", &braid::layer_norm);
  m.def("gelu_tanh", &braid::gelu_tanh);
  m.def("embedding", &braid::embedding);
  m.def("qkv_prepare", &braid::qkv_prepare);
  m.def("sample", &braid::sample);
  m.def("tp_sample", &braid::tp_sample,
        "vocab-parallel sampling: per-shard records exchanged over peer memory, merged identically on every rank");
  m.def("tp_sample_record_bytes", &braid::tp_sample_record_bytes);
}
