// Python bindings of the sm_100a kernels (module sglang_neuron_b200._C).
#include <torch/extension.h>

// norm.cu
void rmsnorm_out(torch::Tensor out, torch::Tensor x, torch::Tensor weight, double eps, bool weight_plus_one);
void fused_add_rmsnorm(torch::Tensor x, torch::Tensor residual, torch::Tensor weight, double eps,
                       bool weight_plus_one);
void head_rmsnorm_(torch::Tensor x, torch::Tensor weight, int64_t heads, double eps);
// rope_kv.cu
void rope_qk_norm_kv_write(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor positions,
                           torch::Tensor cos_sin, int64_t num_q_heads, int64_t num_kv_heads, int64_t head_dim,
                           int64_t rot_dim, bool neox, c10::optional<torch::Tensor> q_norm_w,
                           c10::optional<torch::Tensor> k_norm_w, double norm_eps, torch::Tensor k_cache,
                           torch::Tensor v_cache, torch::Tensor slots, int64_t page_size, double k_scale,
                           double v_scale, c10::optional<torch::Tensor> status);
// attention.cu
void decode_attention(torch::Tensor out, torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache,
                      torch::Tensor block_table, torch::Tensor seq_lens, int64_t num_q_heads, int64_t num_kv_heads,
                      int64_t head_dim, int64_t page_size, int64_t window, double sm_scale, double k_scale,
                      double v_scale, c10::optional<torch::Tensor> sinks, int64_t num_splits, torch::Tensor o_part,
                      torch::Tensor lse_part, c10::optional<torch::Tensor> status,
                      c10::optional<torch::Tensor> merge_counters);
void extend_attention(torch::Tensor out, torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache,
                      torch::Tensor block_table, torch::Tensor qo_indptr, torch::Tensor kv_lens, int64_t max_extend,
                      int64_t num_q_heads, int64_t num_kv_heads, int64_t head_dim, int64_t page_size,
                      int64_t window, double sm_scale, double k_scale, double v_scale,
                      c10::optional<torch::Tensor> sinks);
// sampling.cu
void sample_tokens(torch::Tensor out_ids, torch::Tensor logits, c10::optional<torch::Tensor> temperature,
                   c10::optional<torch::Tensor> seeds, c10::optional<torch::Tensor> positions,
                   c10::optional<torch::Tensor> out_vals, int64_t vocab_offset, int64_t valid_vocab);
// moe_route.cu
void topk_route(torch::Tensor weights, torch::Tensor ids, torch::Tensor logits, int64_t k, int64_t mode, double scale);
void moe_align(torch::Tensor ids, int64_t e_lo, int64_t e_local, int64_t bn, torch::Tensor seg_offsets,
               torch::Tensor tile_offsets, torch::Tensor sorted_src, torch::Tensor inv_map);
void gather_quant_mxfp8(torch::Tensor q, torch::Tensor sf, torch::Tensor x, c10::optional<torch::Tensor> src,
                        int64_t bn, c10::optional<torch::Tensor> used, c10::optional<torch::Tensor> skip);
void moe_combine(torch::Tensor out, torch::Tensor y, torch::Tensor inv_map, torch::Tensor w, bool accumulate);
// mla_rope.cu
void mla_rope_latent(torch::Tensor kv_a, torch::Tensor q, int64_t H, int64_t nope, int64_t r, int64_t rope,
                     torch::Tensor norm_w, double eps, torch::Tensor positions, torch::Tensor cos_sin, bool neox,
                     torch::Tensor cache, torch::Tensor slots, int64_t page_size, torch::Tensor qf);
// sampling_topk.cu
void topk_pool(torch::Tensor logits, int64_t V, int64_t K, int64_t vocab_offset, torch::Tensor vals, torch::Tensor ids);
// moe_route_fused.cu
void moe_route_fused(torch::Tensor x, torch::Tensor w_tiled, int64_t E, c10::optional<torch::Tensor> bias,
                     int64_t k, int64_t mode, double scale, int64_t e_lo, int64_t e_local, int64_t bn,
                     torch::Tensor partial, torch::Tensor w_out, torch::Tensor id_out, torch::Tensor seg_offsets,
                     torch::Tensor tile_offsets, torch::Tensor sorted_src, torch::Tensor inv_map, torch::Tensor q,
                     torch::Tensor sf, torch::Tensor sync, torch::Tensor status, int64_t k_chunks);
// moe_gemm_sm100.cu
void moe_gemm(torch::Tensor out, torch::Tensor xq, torch::Tensor sfb, torch::Tensor w, torch::Tensor sfa,
              c10::optional<torch::Tensor> bias, torch::Tensor seg_offsets, torch::Tensor tile_offsets, int64_t bn,
              int64_t epi, double alpha, double limit, int64_t num_sms, torch::Tensor status, int64_t F, c10::optional<torch::Tensor> qout, c10::optional<torch::Tensor> sfout);
// activation.cu
void silu_and_mul(torch::Tensor out, torch::Tensor x);
// gemm_sm100.cu
void gemm_bf16(torch::Tensor out, torch::Tensor x, torch::Tensor w, c10::optional<torch::Tensor> bias,
               torch::Tensor status, int64_t bn, int64_t splits, c10::optional<torch::Tensor> workspace,
               bool reduce_partials, int64_t tiled_f);
void gemm_bf16_grouped(torch::Tensor out, torch::Tensor x, torch::Tensor w, int64_t tiled_f, torch::Tensor status,
                       int64_t group_k, int64_t x_rows, int64_t x_stride, int64_t o_rows, int64_t o_stride);
void set_pdl(bool on);
void set_decode_fp8_variant(int64_t v);
void mla_extend(torch::Tensor out, torch::Tensor q, torch::Tensor cache, torch::Tensor block_table,
                torch::Tensor seq_lens, torch::Tensor qo_indptr, int64_t max_extend, int64_t page_size,
                double sm_scale, int64_t dcp_size, int64_t dcp_rank, c10::optional<torch::Tensor> lse_out);
void mla_decode(torch::Tensor out, torch::Tensor q, torch::Tensor cache, torch::Tensor block_table,
                torch::Tensor seq_lens, int64_t page_size, double sm_scale, int64_t num_splits, torch::Tensor o_part,
                torch::Tensor lse_part);
void kv_page_copy(torch::Tensor src_bases, torch::Tensor dst_bases, torch::Tensor src_pages, torch::Tensor dst_pages,
                  int64_t page_bytes);
void kv_page_slice_copy(torch::Tensor src_bases, torch::Tensor dst_bases, torch::Tensor src_pages,
                        torch::Tensor dst_pages, int64_t src_page_bytes, int64_t dst_page_bytes, int64_t src_off,
                        int64_t dst_off, int64_t nbytes);
int64_t nvls_flag_bytes();
void nvls_allreduce(torch::Tensor out, torch::Tensor x, int64_t uc, int64_t mc, int64_t capacity, int64_t rank,
                    int64_t world, int64_t max_ctas, torch::Tensor status);
void nvls_combine_allreduce(torch::Tensor out, torch::Tensor y, torch::Tensor inv_map, torch::Tensor w, int64_t uc,
                            int64_t mc, int64_t capacity, int64_t rank, int64_t world, int64_t max_ctas,
                            torch::Tensor status);
void nvls_splitk_allreduce(torch::Tensor out, torch::Tensor partial, int64_t splits,
                           c10::optional<torch::Tensor> bias, int64_t uc, int64_t mc, int64_t capacity, int64_t rank,
                           int64_t world, int64_t max_ctas, torch::Tensor status);
bool get_pdl();
void splitk_allreduce(torch::Tensor out, torch::Tensor partial, int64_t splits, c10::optional<torch::Tensor> bias,
                      std::vector<int64_t> bufs, int64_t rank, int64_t capacity, int64_t num_ctas, torch::Tensor status,
                      c10::optional<torch::Tensor> residual, c10::optional<torch::Tensor> weight, double eps,
                      int64_t wait_ns);

void gemm_bf16_allreduce(torch::Tensor out, torch::Tensor x, torch::Tensor w, c10::optional<torch::Tensor> bias,
                         torch::Tensor status, std::vector<int64_t> bufs, int64_t rank, int64_t capacity,
                         int64_t num_sms, int64_t tiled_f);
// allreduce.cu
std::tuple<int64_t, py::bytes> symm_alloc(int64_t capacity, int64_t world);
int64_t symm_open(py::bytes handle);
void symm_close(int64_t ptr, bool owned);
void sp_allgather(torch::Tensor out, torch::Tensor in, std::vector<int64_t> bufs, int64_t rank, int64_t capacity,
                  int64_t num_ctas, torch::Tensor status, int64_t wait_ns);
void sp_reducescatter(torch::Tensor out, torch::Tensor in, std::vector<int64_t> bufs, int64_t rank, int64_t capacity,
                      int64_t num_ctas, torch::Tensor status, int64_t wait_ns);
void one_shot_allreduce(torch::Tensor out, torch::Tensor in, std::vector<int64_t> bufs, int64_t rank,
                        int64_t capacity, int64_t num_ctas, torch::Tensor status,
                        c10::optional<torch::Tensor> residual, c10::optional<torch::Tensor> weight, double eps,
                        int64_t wait_ns);
void moe_combine_allreduce(torch::Tensor out, torch::Tensor y, torch::Tensor inv_map, torch::Tensor w,
                           std::vector<int64_t> bufs, int64_t rank, int64_t capacity, int64_t num_ctas,
                           torch::Tensor status, c10::optional<torch::Tensor> residual,
                           c10::optional<torch::Tensor> weight, double eps, int64_t wait_ns);

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "sglang_neuron_b200 sm_100a kernels";
  m.def("rmsnorm_out", &rmsnorm_out);
  m.def("fused_add_rmsnorm", &fused_add_rmsnorm);
  m.def("head_rmsnorm_", &head_rmsnorm_);
  m.def("rope_qk_norm_kv_write", &rope_qk_norm_kv_write, py::arg("q"), py::arg("k"), py::arg("v"),
        py::arg("positions"), py::arg("cos_sin"), py::arg("num_q_heads"), py::arg("num_kv_heads"),
        py::arg("head_dim"), py::arg("rot_dim"), py::arg("neox"), py::arg("q_norm_w"), py::arg("k_norm_w"),
        py::arg("norm_eps"), py::arg("k_cache"), py::arg("v_cache"), py::arg("slots"), py::arg("page_size"),
        py::arg("k_scale"), py::arg("v_scale"), py::arg("status") = py::none());
  m.def("decode_attention", &decode_attention, py::arg("out"), py::arg("q"), py::arg("k_cache"), py::arg("v_cache"),
        py::arg("block_table"), py::arg("seq_lens"), py::arg("num_q_heads"), py::arg("num_kv_heads"),
        py::arg("head_dim"), py::arg("page_size"), py::arg("window"), py::arg("sm_scale"), py::arg("k_scale"),
        py::arg("v_scale"), py::arg("sinks"), py::arg("num_splits"), py::arg("o_part"), py::arg("lse_part"),
        py::arg("status") = py::none(), py::arg("merge_counters") = py::none());
  m.def("extend_attention", &extend_attention);
  m.def("sample_tokens", &sample_tokens);
  m.def("topk_route", &topk_route);
  m.def("moe_align", &moe_align);
  m.def("gather_quant_mxfp8", &gather_quant_mxfp8, py::arg("q"), py::arg("sf"), py::arg("x"), py::arg("src"),
        py::arg("bn"), py::arg("used") = py::none(), py::arg("skip") = py::none());
  m.def("moe_combine", &moe_combine);
  m.def("topk_pool", &topk_pool);
  m.def("mla_rope_latent", &mla_rope_latent);
  m.def("moe_route_fused", &moe_route_fused, py::arg("x"), py::arg("w_tiled"), py::arg("E"), py::arg("bias"),
        py::arg("k"), py::arg("mode"), py::arg("scale"), py::arg("e_lo"), py::arg("e_local"), py::arg("bn"),
        py::arg("partial"), py::arg("w_out"), py::arg("id_out"), py::arg("seg_offsets"), py::arg("tile_offsets"),
        py::arg("sorted_src"), py::arg("inv_map"), py::arg("q"), py::arg("sf"), py::arg("sync"), py::arg("status"),
        py::arg("k_chunks"));
  m.def("gemm_bf16", &gemm_bf16);
  m.def("gemm_bf16_grouped", &gemm_bf16_grouped);
  m.def("moe_gemm", &moe_gemm, py::arg("out"), py::arg("xq"), py::arg("sfb"), py::arg("w"), py::arg("sfa"),
        py::arg("bias"), py::arg("seg_offsets"), py::arg("tile_offsets"), py::arg("bn"), py::arg("epi"),
        py::arg("alpha"), py::arg("limit"), py::arg("num_sms"), py::arg("status"), py::arg("F"),
        py::arg("qout") = py::none(), py::arg("sfout") = py::none());
  m.def("silu_and_mul", &silu_and_mul);
  m.def("symm_alloc", &symm_alloc);
  m.def("symm_open", &symm_open);
  m.def("symm_close", &symm_close);
  m.def("one_shot_allreduce", &one_shot_allreduce, py::arg("out"), py::arg("inp"), py::arg("bufs"), py::arg("rank"),
        py::arg("capacity"), py::arg("num_ctas"), py::arg("status"), py::arg("residual") = py::none(), py::arg("weight") = py::none(), py::arg("eps") = 0.0,
        py::arg("wait_ns") = 0);
  m.def("moe_combine_allreduce", &moe_combine_allreduce, py::arg("out"), py::arg("y"), py::arg("inv_map"),
        py::arg("w"), py::arg("bufs"), py::arg("rank"), py::arg("capacity"), py::arg("num_ctas"), py::arg("status"),
        py::arg("residual") = py::none(), py::arg("weight") = py::none(), py::arg("eps") = 0.0,
        py::arg("wait_ns") = 0);
  m.def("gemm_bf16_allreduce", &gemm_bf16_allreduce);
  m.def("sp_allgather", &sp_allgather);
  m.def("sp_reducescatter", &sp_reducescatter);
  m.def("splitk_allreduce", &splitk_allreduce, py::arg("out"), py::arg("partial"), py::arg("splits"),
        py::arg("bias"), py::arg("bufs"), py::arg("rank"), py::arg("capacity"), py::arg("num_ctas"),
        py::arg("status"), py::arg("residual") = py::none(), py::arg("weight") = py::none(), py::arg("eps") = 0.0,
        py::arg("wait_ns") = 0);
  m.def("set_pdl", &set_pdl);
  m.def("set_decode_fp8_variant", &set_decode_fp8_variant, py::arg("variant"));
  m.def("mla_decode", &mla_decode);
  m.def("mla_extend", &mla_extend, py::arg("out"), py::arg("q"), py::arg("cache"), py::arg("block_table"),
        py::arg("seq_lens"), py::arg("qo_indptr"), py::arg("max_extend"), py::arg("page_size"), py::arg("sm_scale"),
        py::arg("dcp_size") = 1, py::arg("dcp_rank") = 0, py::arg("lse_out") = py::none());
  m.def("kv_page_copy", &kv_page_copy);
  m.def("kv_page_slice_copy", &kv_page_slice_copy);
  m.def("nvls_flag_bytes", &nvls_flag_bytes);
  m.def("nvls_allreduce", &nvls_allreduce);
  m.def("nvls_combine_allreduce", &nvls_combine_allreduce);
  m.def("nvls_splitk_allreduce", &nvls_splitk_allreduce);
  m.def("get_pdl", &get_pdl);
}
