// Python bindings for the sm_100a kernels (module fak_b200._C).
#include <torch/extension.h>

torch::Tensor quantize_blocks(torch::Tensor x, int64_t qtype);
torch::Tensor dequantize_rows(torch::Tensor w, int64_t qtype, int64_t rows, int64_t cols, int64_t pitch,
                              c10::ScalarType out_dtype);
void quant_act(torch::Tensor x, c10::optional<torch::Tensor> gamma, double eps, torch::Tensor qx, torch::Tensor ds);
void qgemv(torch::Tensor w, int64_t qtype, int64_t N, int64_t K, int64_t pitch, torch::Tensor qx, torch::Tensor ds,
           int64_t B, torch::Tensor y, c10::optional<torch::Tensor> bias, int64_t epi);
void decode_attention(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache, torch::Tensor block_table,
                      torch::Tensor ctx_len, int64_t n_split, int64_t pages_per_split,
                      c10::optional<torch::Tensor> out, c10::optional<torch::Tensor> qx,
                      c10::optional<torch::Tensor> ds, c10::optional<torch::Tensor> workspace, int64_t ldo,
                      c10::optional<torch::Tensor> tickets, c10::optional<torch::Tensor> prefetch, int64_t window,
                      c10::optional<torch::Tensor> shared_pages, int64_t prefix_splits, double scale, double softcap,
                      c10::optional<torch::Tensor> sinks);
void kv_move(torch::Tensor k_cache, torch::Tensor v_cache, torch::Tensor src_slot, torch::Tensor dst_slot,
             torch::Tensor rot, torch::Tensor cos_n, torch::Tensor sin_n);
torch::Tensor dsa_index_score(torch::Tensor iq, torch::Tensor ik, torch::Tensor w, int64_t qpos, double scale);
std::vector<torch::Tensor> dsa_topk(torch::Tensor score, int64_t qpos, int64_t topk);
torch::Tensor dsa_sparse_attend(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache, torch::Tensor sel,
                                torch::Tensor count, double scale);
void prefill_attention(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache, torch::Tensor block_table,
                       torch::Tensor tile_seq, torch::Tensor tile_q0, torch::Tensor seq_qoff, torch::Tensor seq_qlen,
                       torch::Tensor seq_pos0, int64_t n_tiles, torch::Tensor out, int64_t window, double scale,
                       double softcap,
                       c10::optional<torch::Tensor> sinks);
void embed(torch::Tensor table, int64_t qtype, int64_t pitch, int64_t V, int64_t d, torch::Tensor ids,
           c10::optional<torch::Tensor> out_f32, c10::optional<torch::Tensor> out_bf16,
           c10::optional<torch::Tensor> err, double scale);
void rmsnorm_add(torch::Tensor y, torch::Tensor w, double eps, torch::Tensor x);
void rope_kv(torch::Tensor qkv, torch::Tensor pos, torch::Tensor slot, torch::Tensor cos_t, torch::Tensor sin_t,
             int64_t H, int64_t Hkv, c10::optional<torch::Tensor> q_norm, c10::optional<torch::Tensor> k_norm, double eps,
             c10::optional<torch::Tensor> q_f32, c10::optional<torch::Tensor> q_bf16, torch::Tensor k_cache,
             torch::Tensor v_cache);
void rmsnorm_bf16(torch::Tensor x, torch::Tensor w, double eps, torch::Tensor y);
void argmax_rows(torch::Tensor logits, int64_t V, torch::Tensor out, c10::optional<torch::Tensor> keys,
                 c10::optional<torch::Tensor> tickets);
void qmmv(torch::Tensor w, int64_t qtype, int64_t N, int64_t K, int64_t pitch, torch::Tensor qx, torch::Tensor ds,
          int64_t B, torch::Tensor y, c10::optional<torch::Tensor> bias, int64_t epi, int64_t flags);
void quant_act_wide(torch::Tensor x, c10::optional<torch::Tensor> gamma, double eps, torch::Tensor qx,
                    torch::Tensor ds, c10::optional<torch::Tensor> prefetch, bool unit);
void p2p_allgather_cols(torch::Tensor peers, torch::Tensor src, int64_t src_ld, int64_t dst_off, int64_t dst_ld,
                        int64_t col0, int64_t ncols, int64_t B, int64_t flags_off, int64_t site, int64_t me,
                        torch::Tensor counters, torch::Tensor err, int64_t ctas, c10::optional<torch::Tensor> src2,
                        int64_t src2_ld, int64_t dst2_off, int64_t dst2_ld, int64_t col2, int64_t ncols2,
                        int64_t spin_limit);
void p2p_allreduce_add(torch::Tensor peers, int64_t part_off, torch::Tensor x, int64_t n, int64_t flags_off,
                       int64_t site, int64_t me, torch::Tensor counters, torch::Tensor err, int64_t ctas,
                       int64_t spin_limit);
void p2p_argmax(torch::Tensor peers, torch::Tensor logits, int64_t Vl, int64_t v_off, int64_t cand_off,
                torch::Tensor out, int64_t B, torch::Tensor keys, torch::Tensor tickets, torch::Tensor epochs,
                int64_t me, torch::Tensor err, int64_t spin_limit);
void p2p_moe_combine_ar(torch::Tensor peers, torch::Tensor out, torch::Tensor ids, torch::Tensor wts, int64_t k,
                        int64_t e0, int64_t E_local, torch::Tensor x, int64_t B, int64_t parts_off, int64_t parity,
                        int64_t flags_off, int64_t site, int64_t me, torch::Tensor counters, torch::Tensor err,
                        int64_t ctas, int64_t spin_limit);
void moe_route(torch::Tensor x, torch::Tensor gamma, double eps, torch::Tensor wr, int64_t k, bool norm_topk,
               torch::Tensor ids, torch::Tensor wts,
               c10::optional<torch::Tensor> rbias, int64_t kind);
void moe_group(torch::Tensor ids, int64_t P, int64_t e0, int64_t E_local, int64_t max_chunks, torch::Tensor chunk_expert,
               torch::Tensor chunk_pairs, torch::Tensor n_chunks);
void tgemv(torch::Tensor w, int64_t qtype, int64_t N, int64_t K, c10::optional<torch::Tensor> qx,
           c10::optional<torch::Tensor> ds, c10::optional<torch::Tensor> x, c10::optional<torch::Tensor> gamma,
           double eps, int64_t B, torch::Tensor y, c10::optional<torch::Tensor> bias, int64_t epi, torch::Tensor part,
           torch::Tensor cnt, c10::optional<torch::Tensor> err, int64_t flags, c10::optional<torch::Tensor> ar_peers,
           int64_t ar_me, int64_t ar_parts_off, c10::optional<torch::Tensor> ar_epochs,
           c10::optional<torch::Tensor> prefetch, int64_t ar_spin_limit, bool unit);
std::vector<int64_t> tgemv_workspace(int64_t qtype, int64_t N, int64_t K, int64_t device);
int64_t tgemv_unit_bytes(int64_t qtype);
std::vector<int64_t> tgemv_pair_plan(int64_t qa, int64_t Na, int64_t qb, int64_t Nb, int64_t K, int64_t B,
                                     int64_t device);
void tgemv_pair(torch::Tensor wa, int64_t qa, int64_t Na, torch::Tensor ya, c10::optional<torch::Tensor> bias_a,
                torch::Tensor wb, int64_t qb, int64_t Nb, torch::Tensor yb, c10::optional<torch::Tensor> bias_b,
                int64_t K, torch::Tensor qx, torch::Tensor ds, int64_t B, torch::Tensor part, torch::Tensor cnt,
                c10::optional<torch::Tensor> err, c10::optional<torch::Tensor> prefetch, bool unit);
void moe_tgemv(torch::Tensor w, int64_t qtype, int64_t rows_per_expert, int64_t K, torch::Tensor qx,
               torch::Tensor ds, int64_t topk, bool act_by_token, torch::Tensor chunk_expert, torch::Tensor chunk_pairs,
               torch::Tensor n_chunks, int64_t max_chunks, torch::Tensor y, int64_t epi, torch::Tensor err,
               c10::optional<torch::Tensor> bias);
void moe_qmmv(torch::Tensor w, int64_t qtype, int64_t rows_per_expert, int64_t K, int64_t pitch, torch::Tensor qx,
              torch::Tensor ds, int64_t topk, bool act_by_token, torch::Tensor chunk_expert, torch::Tensor chunk_pairs,
              torch::Tensor n_chunks, int64_t max_chunks, torch::Tensor y, int64_t epi, torch::Tensor err);
void moe_combine(torch::Tensor out, torch::Tensor ids, torch::Tensor wts, int64_t k, int64_t e0, int64_t E_local,
                 torch::Tensor x);
void gemm_bf16(torch::Tensor a, torch::Tensor b, torch::Tensor out, c10::optional<torch::Tensor> bias, int64_t epi,
               c10::optional<torch::Tensor> err);
void gemm_bf16_rs(torch::Tensor a, torch::Tensor b, torch::Tensor peers, int64_t me, int64_t parts_off,
                  int64_t flags_off, int64_t MR, int64_t epoch, c10::optional<torch::Tensor> err);
void p2p_rs_reduce(torch::Tensor peers, int64_t parts_off, int64_t flags_off, int64_t x_off, int64_t M, int64_t N,
                   int64_t MR, int64_t me, int64_t epoch, int64_t bar_off, int64_t site, torch::Tensor counters,
                   torch::Tensor err, int64_t ctas, int64_t spin_limit, c10::optional<torch::Tensor> x_local);
void sp_rmsnorm_shard(torch::Tensor peers, torch::Tensor x_local, torch::Tensor gamma, double eps, int64_t valid,
                      int64_t shard_off, int64_t flags_off, int64_t me, int64_t epoch);
void gemm_bf16_ag(int64_t M, torch::Tensor b, torch::Tensor out, torch::Tensor peers, int64_t me, int64_t shard_off,
                  int64_t MR, int64_t flags_off, int64_t epoch, int64_t spin, c10::optional<torch::Tensor> bias,
                  int64_t epi, c10::optional<torch::Tensor> err);
void p2p_rs_push(torch::Tensor peers, torch::Tensor part, int64_t MR, int64_t parts_off, int64_t flags_off, int64_t me,
                 int64_t epoch);
void decode_advance(torch::Tensor next, torch::Tensor ids, torch::Tensor pos, torch::Tensor slot, torch::Tensor ctx,
                    torch::Tensor bt, int64_t B);
void scatter_i32(torch::Tensor dst, torch::Tensor idx_val, int64_t n);
std::tuple<int64_t, torch::Tensor> ipc_alloc(int64_t nbytes, int64_t device);
int64_t ipc_open(torch::Tensor handle, int64_t device);
void ipc_close(int64_t ptr);
void ipc_free(int64_t ptr);
torch::Tensor ipc_view(int64_t ptr, int64_t nbytes, int64_t device);
void sample_rows(torch::Tensor logits, int64_t V, torch::Tensor params, torch::Tensor bias_tok, torch::Tensor bias_val,
                 c10::optional<torch::Tensor> counts, torch::Tensor out, int64_t B, double softcap);
torch::Tensor philox4x32_10_host(std::vector<int64_t> ctr, std::vector<int64_t> key);
void prefill_attention_tc(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache, int64_t layer,
                          torch::Tensor block_table, torch::Tensor tile_seq, torch::Tensor tile_q0, torch::Tensor seq_qoff,
                          torch::Tensor seq_qlen, torch::Tensor seq_pos0, int64_t n_tiles, torch::Tensor out,
                          c10::optional<torch::Tensor> err);

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "fak_b200 sm_100a kernels";
  m.def("quantize_blocks", &quantize_blocks);
  m.def("dequantize_rows", &dequantize_rows);
  m.def("quant_act", &quant_act);
  m.def("qgemv", &qgemv);
  m.def("decode_attention", &decode_attention, pybind11::arg("q"), pybind11::arg("k_cache"), pybind11::arg("v_cache"),
        pybind11::arg("block_table"), pybind11::arg("ctx_len"), pybind11::arg("n_split"),
        pybind11::arg("pages_per_split"), pybind11::arg("out"), pybind11::arg("qx"), pybind11::arg("ds"),
        pybind11::arg("workspace"), pybind11::arg("ldo") = 0, pybind11::arg("tickets") = pybind11::none(),
        pybind11::arg("prefetch") = pybind11::none(), pybind11::arg("window") = 0,
        pybind11::arg("shared_pages") = pybind11::none(), pybind11::arg("prefix_splits") = 0,
        pybind11::arg("scale") = 0.0, pybind11::arg("softcap") = 0.0, pybind11::arg("sinks") = pybind11::none());
  m.def("prefill_attention", &prefill_attention, pybind11::arg("q"), pybind11::arg("k_cache"),
        pybind11::arg("v_cache"), pybind11::arg("block_table"), pybind11::arg("tile_seq"), pybind11::arg("tile_q0"),
        pybind11::arg("seq_qoff"), pybind11::arg("seq_qlen"), pybind11::arg("seq_pos0"), pybind11::arg("n_tiles"),
        pybind11::arg("out"), pybind11::arg("window") = 0, pybind11::arg("scale") = 0.0,
        pybind11::arg("softcap") = 0.0, pybind11::arg("sinks") = pybind11::none());
  m.def("embed", &embed, pybind11::arg("table"), pybind11::arg("qtype"), pybind11::arg("pitch"), pybind11::arg("V"),
        pybind11::arg("d"), pybind11::arg("ids"), pybind11::arg("out_f32"), pybind11::arg("out_bf16"),
        pybind11::arg("err"), pybind11::arg("scale") = 1.0);
  m.def("rmsnorm_add", &rmsnorm_add);
  m.def("dsa_index_score", &dsa_index_score);
  m.def("dsa_topk", &dsa_topk);
  m.def("dsa_sparse_attend", &dsa_sparse_attend);
  m.def("kv_move", &kv_move, "move K/V rows between slots of all layers, re-rotating flagged keys back by n");
  m.def("rope_kv", &rope_kv);
  m.def("rmsnorm_bf16", &rmsnorm_bf16);
  m.def("argmax_rows", &argmax_rows, pybind11::arg("logits"), pybind11::arg("V"), pybind11::arg("out"),
        pybind11::arg("keys") = pybind11::none(), pybind11::arg("tickets") = pybind11::none());
  m.def("p2p_allgather_cols", &p2p_allgather_cols, pybind11::arg("peers"), pybind11::arg("src"), pybind11::arg("src_ld"),
        pybind11::arg("dst_off"), pybind11::arg("dst_ld"), pybind11::arg("col0"), pybind11::arg("ncols"), pybind11::arg("B"),
        pybind11::arg("flags_off"), pybind11::arg("site"), pybind11::arg("me"), pybind11::arg("counters"),
        pybind11::arg("err"), pybind11::arg("ctas"), pybind11::arg("src2") = pybind11::none(), pybind11::arg("src2_ld") = 0,
        pybind11::arg("dst2_off") = 0, pybind11::arg("dst2_ld") = 0, pybind11::arg("col2") = 0, pybind11::arg("ncols2") = 0,
        pybind11::arg("spin_limit") = 0);
  m.def("p2p_allreduce_add", &p2p_allreduce_add, pybind11::arg("peers"), pybind11::arg("part_off"), pybind11::arg("x"),
        pybind11::arg("n"), pybind11::arg("flags_off"), pybind11::arg("site"), pybind11::arg("me"),
        pybind11::arg("counters"), pybind11::arg("err"), pybind11::arg("ctas"), pybind11::arg("spin_limit") = 0);
  m.def("p2p_argmax", &p2p_argmax, pybind11::arg("peers"), pybind11::arg("logits"), pybind11::arg("Vl"),
        pybind11::arg("v_off"), pybind11::arg("cand_off"), pybind11::arg("out"), pybind11::arg("B"),
        pybind11::arg("keys"), pybind11::arg("tickets"), pybind11::arg("epochs"), pybind11::arg("me"),
        pybind11::arg("err"), pybind11::arg("spin_limit") = 0);
  m.def("p2p_moe_combine_ar", &p2p_moe_combine_ar, "MoE combine fused with the expert-parallel all-reduce");
  m.def("moe_route", &moe_route, pybind11::arg("x"), pybind11::arg("gamma"), pybind11::arg("eps"),
        pybind11::arg("wr"), pybind11::arg("k"), pybind11::arg("norm_topk"), pybind11::arg("ids"),
        pybind11::arg("wts"), pybind11::arg("rbias") = pybind11::none(), pybind11::arg("kind") = 0);
  m.def("moe_group", &moe_group);
  m.def("moe_qmmv", &moe_qmmv);
  m.def("moe_combine", &moe_combine);
  m.def("qmmv", &qmmv, pybind11::arg("w"), pybind11::arg("qtype"), pybind11::arg("N"), pybind11::arg("K"),
        pybind11::arg("pitch"), pybind11::arg("qx"), pybind11::arg("ds"), pybind11::arg("B"), pybind11::arg("y"),
        pybind11::arg("bias"), pybind11::arg("epi"), pybind11::arg("flags") = 0);
  m.def("quant_act_wide", &quant_act_wide, pybind11::arg("x"), pybind11::arg("gamma"), pybind11::arg("eps"),
        pybind11::arg("qx"), pybind11::arg("ds"), pybind11::arg("prefetch") = pybind11::none(),
        pybind11::arg("unit") = false);
  m.def("tgemv", &tgemv, pybind11::arg("w"), pybind11::arg("qtype"), pybind11::arg("N"), pybind11::arg("K"),
        pybind11::arg("qx"), pybind11::arg("ds"), pybind11::arg("x"), pybind11::arg("gamma"), pybind11::arg("eps"),
        pybind11::arg("B"), pybind11::arg("y"), pybind11::arg("bias"),
        pybind11::arg("epi"), pybind11::arg("part"), pybind11::arg("cnt"), pybind11::arg("err") = pybind11::none(),
        pybind11::arg("flags") = 0, pybind11::arg("ar_peers") = pybind11::none(), pybind11::arg("ar_me") = 0,
        pybind11::arg("ar_parts_off") = 0, pybind11::arg("ar_epochs") = pybind11::none(),
        pybind11::arg("prefetch") = pybind11::none(), pybind11::arg("ar_spin_limit") = 0,
        pybind11::arg("unit") = false);
  m.def("tgemv_workspace", &tgemv_workspace);
  m.def("tgemv_unit_bytes", &tgemv_unit_bytes);
  m.def("tgemv_pair_plan", &tgemv_pair_plan);
  m.def("tgemv_pair", &tgemv_pair, pybind11::arg("wa"), pybind11::arg("qa"), pybind11::arg("Na"), pybind11::arg("ya"),
        pybind11::arg("bias_a"), pybind11::arg("wb"), pybind11::arg("qb"), pybind11::arg("Nb"), pybind11::arg("yb"),
        pybind11::arg("bias_b"), pybind11::arg("K"), pybind11::arg("qx"), pybind11::arg("ds"), pybind11::arg("B"),
        pybind11::arg("part"), pybind11::arg("cnt"), pybind11::arg("err") = pybind11::none(),
        pybind11::arg("prefetch") = pybind11::none(), pybind11::arg("unit") = false);
  m.def("moe_tgemv", &moe_tgemv, pybind11::arg("w"), pybind11::arg("qtype"), pybind11::arg("rows_per_expert"),
        pybind11::arg("K"), pybind11::arg("qx"), pybind11::arg("ds"), pybind11::arg("topk"),
        pybind11::arg("act_by_token"), pybind11::arg("chunk_expert"), pybind11::arg("chunk_pairs"),
        pybind11::arg("n_chunks"), pybind11::arg("max_chunks"), pybind11::arg("y"), pybind11::arg("epi"),
        pybind11::arg("err"), pybind11::arg("bias") = pybind11::none());
  m.def("decode_advance", &decode_advance, "next step's lane inputs from this step's tokens (device-resident state)");
  m.def("scatter_i32", &scatter_i32, "dst.flatten()[idx] = val for (idx, val) pairs on the device");
  m.def("ipc_alloc", &ipc_alloc, "zeroed device buffer + its CUDA IPC handle");
  m.def("ipc_open", &ipc_open, "map a peer's IPC handle (lazy peer access)");
  m.def("ipc_close", &ipc_close);
  m.def("ipc_free", &ipc_free);
  m.def("ipc_view", &ipc_view, "non-owning uint8 tensor over a device buffer");
  m.def("sample_rows", &sample_rows, "bias / penalties / temperature / top-k / top-p draw per row (Philox RNG)",
        pybind11::arg("logits"), pybind11::arg("V"), pybind11::arg("params"), pybind11::arg("bias_tok"),
        pybind11::arg("bias_val"), pybind11::arg("counts"), pybind11::arg("out"), pybind11::arg("B"),
        pybind11::arg("softcap") = 0.0);
  m.def("philox4x32_10_host", &philox4x32_10_host);
  m.def("prefill_attention_tc", &prefill_attention_tc, "paged causal prefill attention on tcgen05 / TMEM (head dim 128)",
        pybind11::arg("q"), pybind11::arg("k_cache"), pybind11::arg("v_cache"), pybind11::arg("layer"),
        pybind11::arg("block_table"), pybind11::arg("tile_seq"), pybind11::arg("tile_q0"), pybind11::arg("seq_qoff"),
        pybind11::arg("seq_qlen"), pybind11::arg("seq_pos0"), pybind11::arg("n_tiles"), pybind11::arg("out"),
        pybind11::arg("err") = pybind11::none());
  m.def("gemm_bf16", &gemm_bf16, pybind11::arg("a"), pybind11::arg("b"), pybind11::arg("out"),
        pybind11::arg("bias") = pybind11::none(), pybind11::arg("epi") = 0, pybind11::arg("err") = pybind11::none());
  m.def("gemm_bf16_rs", &gemm_bf16_rs, pybind11::arg("a"), pybind11::arg("b"), pybind11::arg("peers"),
        pybind11::arg("me"), pybind11::arg("parts_off"), pybind11::arg("flags_off"), pybind11::arg("MR"),
        pybind11::arg("epoch"), pybind11::arg("err") = pybind11::none());
  m.def("p2p_rs_reduce", &p2p_rs_reduce, pybind11::arg("peers"), pybind11::arg("parts_off"),
        pybind11::arg("flags_off"), pybind11::arg("x_off"), pybind11::arg("M"), pybind11::arg("N"), pybind11::arg("MR"),
        pybind11::arg("me"), pybind11::arg("epoch"), pybind11::arg("bar_off"), pybind11::arg("site"),
        pybind11::arg("counters"), pybind11::arg("err"), pybind11::arg("ctas"), pybind11::arg("spin_limit") = 0,
        pybind11::arg("x_local") = pybind11::none());
  m.def("sp_rmsnorm_shard", &sp_rmsnorm_shard, pybind11::arg("peers"), pybind11::arg("x_local"),
        pybind11::arg("gamma"), pybind11::arg("eps"), pybind11::arg("valid"), pybind11::arg("shard_off"),
        pybind11::arg("flags_off"), pybind11::arg("me"), pybind11::arg("epoch"));
  m.def("gemm_bf16_ag", &gemm_bf16_ag, pybind11::arg("M"), pybind11::arg("b"), pybind11::arg("out"),
        pybind11::arg("peers"), pybind11::arg("me"), pybind11::arg("shard_off"), pybind11::arg("MR"),
        pybind11::arg("flags_off"), pybind11::arg("epoch"), pybind11::arg("spin") = 0,
        pybind11::arg("bias") = pybind11::none(), pybind11::arg("epi") = 0, pybind11::arg("err") = pybind11::none());
  m.def("p2p_rs_push", &p2p_rs_push, pybind11::arg("peers"), pybind11::arg("part"), pybind11::arg("MR"),
        pybind11::arg("parts_off"), pybind11::arg("flags_off"), pybind11::arg("me"), pybind11::arg("epoch"));
}
