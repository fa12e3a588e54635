// Python bindings of the cascadia_b200 sm_100a kernels (module `_C`).
#include <torch/extension.h>

#include <vector>

namespace cb {
// gemm_w4a16.cu
void w4a16_gemm(torch::Tensor x, torch::Tensor wblob, torch::Tensor out, int64_t N,
                int64_t group_size, int64_t epilogue, c10::optional<torch::Tensor> residual,
                torch::Tensor ws, torch::Tensor counters, torch::Tensor status,
                int64_t forced_splits);
int64_t w4a16_workspace_floats(int64_t M, int64_t N, int64_t K, int64_t forced_splits);
void set_pdl(bool on);
// gdn.cu
void gdn_conv(torch::Tensor x, int64_t C, torch::Tensor w, torch::Tensor state,
              torch::Tensor seq_start, torch::Tensor block_tables, torch::Tensor block_slot);
void gdn_recurrent(torch::Tensor qkv, torch::Tensor z, torch::Tensor ab, torch::Tensor a_log,
                   torch::Tensor dt_bias, torch::Tensor norm_w, torch::Tensor state,
                   torch::Tensor seq_start, torch::Tensor block_tables, torch::Tensor block_slot,
                   torch::Tensor out, int64_t Hk, int64_t Hv, double eps);
void sigmoid_gate(torch::Tensor x, torch::Tensor gate);
// ffn_sparse.cu
void ffn_sparse_forward(torch::Tensor x, torch::Tensor gate_packed, torch::Tensor gate_scales,
                        torch::Tensor up_packed, torch::Tensor up_scales,
                        torch::Tensor downT_packed, torch::Tensor downT_scales,
                        c10::optional<torch::Tensor> tau, double tau_all,
                        c10::optional<torch::Tensor> residual, torch::Tensor out,
                        torch::Tensor iwork, torch::Tensor fwork, int64_t group_size,
                        int64_t down_group_size);
bool pdl_enabled();
int64_t w4a16_counter_count(int64_t M, int64_t N);
void bf16_gemm(torch::Tensor x, torch::Tensor w, torch::Tensor out,
               c10::optional<torch::Tensor> residual, torch::Tensor ws, torch::Tensor counters,
               torch::Tensor status, int64_t splits);
std::vector<int64_t> bf16_gemm_plan(int64_t M, int64_t N, int64_t K, int64_t splits);
std::vector<torch::Tensor> hc_pre(torch::Tensor copies, torch::Tensor fn, torch::Tensor base,
                                  torch::Tensor scale, int64_t iters, double hc_eps,
                                  double norm_eps);
void w4a16_gemm_rope_kv(torch::Tensor x, torch::Tensor wblob, torch::Tensor out, int64_t N,
                        int64_t group_size, torch::Tensor ws, torch::Tensor counters,
                        torch::Tensor status, torch::Tensor positions, torch::Tensor cos_sin,
                        torch::Tensor slots, torch::Tensor k_cache, torch::Tensor v_cache,
                        int64_t layer, int64_t hq, int64_t hkv);
void w4a16_gemm_push(torch::Tensor x, torch::Tensor wblob, int64_t N, int64_t group_size,
                     torch::Tensor out_ptrs, int64_t ldo, torch::Tensor sig_ptrs, int64_t my_rank,
                     torch::Tensor push_done, torch::Tensor push_epoch, torch::Tensor ws,
                     torch::Tensor counters, torch::Tensor status);
void w4a16_set_trace(c10::optional<torch::Tensor> buf);
std::vector<int64_t> w4a16_plan(int64_t M, int64_t N, int64_t K, int64_t forced_splits);
void w4a16_gemm_grouped(torch::Tensor x, torch::Tensor wblob, torch::Tensor out, int64_t N,
                        int64_t group_size, int64_t epilogue, torch::Tensor group_offsets,
                        int64_t num_groups, int64_t max_rows_per_group, torch::Tensor status,
                        c10::optional<torch::Tensor> out_rows);
// mla.cu
void mla_rope_write(torch::Tensor ckv, torch::Tensor kr, torch::Tensor qrope,
                    int64_t q_head_stride, torch::Tensor q_out, torch::Tensor positions,
                    torch::Tensor cos_sin, torch::Tensor slots, torch::Tensor cache,
                    int64_t layer, int64_t heads);
void mla_decode(torch::Tensor q, torch::Tensor cache, torch::Tensor block_tables,
                torch::Tensor seq_lens, torch::Tensor out, int64_t layer, int64_t num_splits,
                int64_t blocks_per_split, torch::Tensor part_o, torch::Tensor part_ml,
                double scale, torch::Tensor status, c10::optional<torch::Tensor> sel,
                c10::optional<torch::Tensor> sel_thr);
void dsa_scores(torch::Tensor q, torch::Tensor w, torch::Tensor kcache, torch::Tensor block_tables,
                torch::Tensor lens, torch::Tensor out, int64_t layer);
// ep.cu
void ep_dispatch(torch::Tensor x, torch::Tensor ids, torch::Tensor dest, torch::Tensor pos,
                 torch::Tensor send_cnt, torch::Tensor xbuf_ptrs, torch::Tensor rbuf_ptrs,
                 torch::Tensor meta_ptrs, torch::Tensor sig_ptrs, torch::Tensor epoch,
                 torch::Tensor done, torch::Tensor status, int64_t rank, int64_t world,
                 int64_t cap, int64_t e_local);
void ep_receive(torch::Tensor xp, torch::Tensor offsets, torch::Tensor src_row,
                torch::Tensor out_rows, torch::Tensor total, torch::Tensor xbuf_ptrs,
                torch::Tensor rbuf_ptrs, torch::Tensor meta_ptrs, torch::Tensor sig_ptrs,
                torch::Tensor epoch, torch::Tensor done, torch::Tensor status, int64_t rank,
                int64_t world, int64_t cap, int64_t e_local);
void ep_combine(torch::Tensor w, torch::Tensor dest, torch::Tensor pos,
                c10::optional<torch::Tensor> add, torch::Tensor out, torch::Tensor xbuf_ptrs,
                torch::Tensor rbuf_ptrs, torch::Tensor meta_ptrs, torch::Tensor sig_ptrs,
                torch::Tensor epoch, torch::Tensor done, torch::Tensor status, int64_t rank,
                int64_t world, int64_t cap, int64_t e_local);
// gemv_w4a16.cu
void w4a16_gemv(torch::Tensor x, torch::Tensor wblob, torch::Tensor out, int64_t N,
                int64_t group_size, int64_t epilogue, c10::optional<torch::Tensor> residual,
                torch::Tensor ws, torch::Tensor counters, torch::Tensor status,
                int64_t forced_splits);
int64_t gemv_workspace_floats(int64_t M, int64_t N, int64_t K, int64_t forced_splits);
void moe_prep_fp16(torch::Tensor x, c10::optional<torch::Tensor> perm, int64_t topk,
                   int64_t rows, torch::Tensor x16, torch::Tensor xsum,
                   c10::optional<torch::Tensor> rows_dev);
std::vector<int64_t> moe_prep_shape(int64_t K);
void w4a16_gemv_grouped(torch::Tensor x16, torch::Tensor xsum, torch::Tensor wblob,
                        torch::Tensor out, int64_t N, int64_t epilogue, torch::Tensor offsets,
                        int64_t num_groups, torch::Tensor status,
                        c10::optional<torch::Tensor> out_rows,
                        c10::optional<torch::Tensor> sched);
// moe.cu
void moe_topk_gate(torch::Tensor x, torch::Tensor wg, c10::optional<torch::Tensor> bias,
                   int64_t k, int64_t scoring, bool norm_topk, double routed_scale,
                   torch::Tensor topk_ids, torch::Tensor topk_w, torch::Tensor logits,
                   torch::Tensor counters);
void moe_permute(torch::Tensor topk_ids, int64_t E, torch::Tensor offsets, torch::Tensor perm,
                 torch::Tensor inv, c10::optional<torch::Tensor> x,
                 c10::optional<torch::Tensor> xp);
void moe_combine(torch::Tensor y, torch::Tensor inv, torch::Tensor w,
                 c10::optional<torch::Tensor> add, torch::Tensor out,
                 c10::optional<torch::Tensor> shared, c10::optional<torch::Tensor> shared_gate);
// attention.cu
void attn_decode(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache,
                 torch::Tensor block_tables, torch::Tensor seq_lens, torch::Tensor out,
                 int64_t layer, int64_t num_splits, int64_t blocks_per_split,
                 torch::Tensor part_o, torch::Tensor part_ml, double scale, torch::Tensor status,
                 int64_t window, int64_t sinks);
void attn_prefill(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache,
                  torch::Tensor block_tables, torch::Tensor tiles, torch::Tensor out, int64_t layer,
                  double scale, torch::Tensor status, int64_t window, int64_t sinks);
// elementwise.cu
void embedding(torch::Tensor ids, torch::Tensor table, torch::Tensor out, int64_t vocab_lo);
void rmsnorm(torch::Tensor x, c10::optional<torch::Tensor> residual, torch::Tensor w,
             torch::Tensor out, double eps);
void rope_kv_write(torch::Tensor qkv, torch::Tensor positions, torch::Tensor cos_sin,
                   torch::Tensor slots, torch::Tensor k_cache, torch::Tensor v_cache, int64_t layer,
                   int64_t Hq, int64_t Hkv, int64_t D, int64_t rot, bool interleaved);
void argmax(torch::Tensor logits, torch::Tensor out_idx, c10::optional<torch::Tensor> out_val,
            int64_t idx_offset);
void sample(torch::Tensor logits, torch::Tensor params, c10::optional<torch::Tensor> history,
            c10::optional<torch::Tensor> hist_len, torch::Tensor work, torch::Tensor seeds,
            torch::Tensor offsets, torch::Tensor out);
void spec_verify_fused(torch::Tensor logits, torch::Tensor row_seq, torch::Tensor row_start,
                       torch::Tensor draft, torch::Tensor picks, torch::Tensor done,
                       torch::Tensor kv_len, torch::Tensor out);
void spec_verify(torch::Tensor target, torch::Tensor draft, torch::Tensor out);
void head_rmsnorm(torch::Tensor qkv, torch::Tensor q_w, torch::Tensor k_w, int64_t Hq,
                  int64_t Hkv, int64_t D, double eps);
// comm.cu
void ar_rmsnorm_pushed(torch::Tensor slot_ptrs, torch::Tensor sig_ptrs, torch::Tensor epoch,
                       torch::Tensor done, torch::Tensor status, int64_t rank, int64_t world,
                       int64_t M, int64_t H, c10::optional<torch::Tensor> residual,
                       c10::optional<torch::Tensor> w, torch::Tensor out, double eps);
void ar_rmsnorm(torch::Tensor buf_ptrs, int64_t buf_offset_bytes, torch::Tensor sig_ptrs,
                torch::Tensor epoch, torch::Tensor done, torch::Tensor status, int64_t rank,
                int64_t world, int64_t M, int64_t H, c10::optional<torch::Tensor> residual,
                c10::optional<torch::Tensor> w, torch::Tensor out, double eps, int64_t mc_ptr);
}  // namespace cb

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "cascadia_b200 sm_100a kernels";
  m.def("w4a16_gemm", &cb::w4a16_gemm);
  m.def("w4a16_workspace_floats", &cb::w4a16_workspace_floats);
  m.def("w4a16_counter_count", &cb::w4a16_counter_count);
  m.def("w4a16_gemm_push", &cb::w4a16_gemm_push);
  m.def("w4a16_gemm_rope_kv", &cb::w4a16_gemm_rope_kv);
  m.def("bf16_gemm", &cb::bf16_gemm);
  m.def("bf16_gemm_plan", &cb::bf16_gemm_plan);
  m.def("hc_pre", &cb::hc_pre);
  m.def("w4a16_plan", &cb::w4a16_plan);
  m.def("w4a16_set_trace", &cb::w4a16_set_trace);
  m.def("set_pdl", &cb::set_pdl);
  m.def("gdn_conv", &cb::gdn_conv);
  m.def("gdn_recurrent", &cb::gdn_recurrent);
  m.def("sigmoid_gate", &cb::sigmoid_gate);
  m.def("ffn_sparse_forward", &cb::ffn_sparse_forward);
  m.def("pdl_enabled", &cb::pdl_enabled);
  m.def("attn_decode", &cb::attn_decode, py::arg("q"), py::arg("k_cache"), py::arg("v_cache"),
        py::arg("block_tables"), py::arg("seq_lens"), py::arg("out"), py::arg("layer"),
        py::arg("num_splits"), py::arg("blocks_per_split"), py::arg("part_o"), py::arg("part_ml"),
        py::arg("scale"), py::arg("status"), py::arg("window") = 0, py::arg("sinks") = 0);
  m.def("attn_prefill", &cb::attn_prefill, py::arg("q"), py::arg("k_cache"), py::arg("v_cache"),
        py::arg("block_tables"), py::arg("tiles"), py::arg("out"), py::arg("layer"),
        py::arg("scale"), py::arg("status"), py::arg("window") = 0, py::arg("sinks") = 0);
  m.def("embedding", &cb::embedding);
  m.def("rmsnorm", &cb::rmsnorm);
  m.def("rope_kv_write", &cb::rope_kv_write);
  m.def("argmax", &cb::argmax);
  m.def("sample", &cb::sample);
  m.def("spec_verify", &cb::spec_verify);
  m.def("spec_verify_fused", &cb::spec_verify_fused);
  m.def("ar_rmsnorm", &cb::ar_rmsnorm);
  m.def("ar_rmsnorm_pushed", &cb::ar_rmsnorm_pushed);
  m.def("w4a16_gemm_grouped", &cb::w4a16_gemm_grouped);
  m.def("moe_topk_gate", &cb::moe_topk_gate);
  m.def("moe_permute", &cb::moe_permute);
  m.def("moe_combine", &cb::moe_combine, py::arg("y"), py::arg("inv"), py::arg("w"),
        py::arg("add"), py::arg("out"), py::arg("shared") = py::none(),
        py::arg("shared_gate") = py::none());
  m.def("ep_dispatch", &cb::ep_dispatch);
  m.def("mla_rope_write", &cb::mla_rope_write);
  m.def("mla_decode", &cb::mla_decode, py::arg("q"), py::arg("cache"), py::arg("block_tables"),
        py::arg("seq_lens"), py::arg("out"), py::arg("layer"), py::arg("num_splits"),
        py::arg("blocks_per_split"), py::arg("part_o"), py::arg("part_ml"), py::arg("scale"),
        py::arg("status"), py::arg("sel") = py::none(), py::arg("sel_thr") = py::none());
  m.def("dsa_scores", &cb::dsa_scores);
  m.def("ep_receive", &cb::ep_receive);
  m.def("ep_combine", &cb::ep_combine);
  m.def("head_rmsnorm", &cb::head_rmsnorm);
  m.def("w4a16_gemv", &cb::w4a16_gemv);
  m.def("gemv_workspace_floats", &cb::gemv_workspace_floats);
  m.def("moe_prep_fp16", &cb::moe_prep_fp16);
  m.def("moe_prep_shape", &cb::moe_prep_shape);
  m.def("w4a16_gemv_grouped", &cb::w4a16_gemv_grouped, py::arg("x16"), py::arg("xsum"),
        py::arg("wblob"), py::arg("out"), py::arg("N"), py::arg("epilogue"), py::arg("offsets"),
        py::arg("num_groups"), py::arg("status"), py::arg("out_rows") = py::none(),
        py::arg("sched") = py::none());
}
