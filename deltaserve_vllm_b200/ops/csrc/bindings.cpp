// Python bindings of the sm_100a kernels (module deltaserve_vllm_b200.ops._C).
#include <torch/extension.h>

void dsv_gemm(torch::Tensor a, torch::Tensor b, torch::Tensor out, bool b_mn, int64_t epi,
              c10::optional<torch::Tensor> z, c10::optional<torch::Tensor> b2, c10::optional<torch::Tensor> tile_slots,
              int64_t lora_seg, c10::optional<torch::Tensor> save, int64_t save_lo, int64_t save_hi,
              int64_t save_dst, int64_t force_bn, int64_t max_ctas, c10::optional<torch::Tensor> aux,
              c10::optional<torch::Tensor> aux_out, bool overlap_prev);
void dsv_rms_norm_bwd(torch::Tensor x, torch::Tensor dy, torch::Tensor w, c10::optional<torch::Tensor> add,
                      torch::Tensor dx, c10::optional<torch::Tensor> dx_bf, double eps);
void dsv_swiglu_bwd(torch::Tensor gu, torch::Tensor dact, torch::Tensor dgu, c10::optional<torch::Tensor> act);
torch::Tensor dsv_gemm_ar(torch::Tensor a, torch::Tensor b, c10::optional<torch::Tensor> z,
                          c10::optional<torch::Tensor> b2, c10::optional<torch::Tensor> tile_slots, int64_t lora_seg,
                          torch::Tensor peer, int64_t tile_cnt, int64_t rank, int64_t world, int64_t owned_cap,
                          int64_t out_rows, int64_t force_splits, int64_t force_reducers);
std::tuple<int64_t, std::string> dsv_peer_alloc(int64_t bytes);
int64_t dsv_peer_open(const std::string& handle);
void dsv_peer_close(int64_t addr);
void dsv_peer_free(int64_t addr);
void dsv_peer_zero(int64_t addr, int64_t bytes);
torch::Tensor dsv_peer_view(int64_t addr, std::vector<int64_t> shape, c10::ScalarType dtype, int64_t device);
int64_t dsv_gemm_ce_stats(torch::Tensor h, torch::Tensor w, torch::Tensor labels, int64_t v0, torch::Tensor stats,
                          torch::Tensor tgt, int64_t max_ctas);
void dsv_gemm_ce_grad(torch::Tensor h, torch::Tensor w, torch::Tensor labels, int64_t v0, torch::Tensor lse,
                      double scale, torch::Tensor dlog, int64_t max_ctas);
void dsv_gemm_push(torch::Tensor a, torch::Tensor b, c10::optional<torch::Tensor> z, c10::optional<torch::Tensor> b2,
                   c10::optional<torch::Tensor> tile_slots, int64_t lora_seg, torch::Tensor table, int64_t rank,
                   int64_t world, int64_t blocks_cap, int64_t ld, c10::optional<torch::Tensor> add,
                   int64_t max_ctas);
void dsv_gemm_wgrad(torch::Tensor a, torch::Tensor b, torch::Tensor out, int64_t kind, int64_t n_valid, int64_t R,
                    int64_t b1, int64_t b2, bool interleave, double scale, int64_t max_ctas);
void dsv_wait_counts(int64_t cnt, int64_t n, int64_t per_block, int64_t rows, int64_t skip_mod, int64_t skip_rem);
void dsv_reduce_norm_bcast(int64_t recv, int64_t rank, int64_t world, int64_t blocks_cap, int64_t ld, int64_t M,
                           int64_t D, c10::optional<torch::Tensor> x, c10::optional<torch::Tensor> w, double eps,
                           c10::optional<torch::Tensor> add, torch::Tensor out, torch::Tensor table);
void dsv_push_slices(torch::Tensor g, int64_t lo, int64_t hi, int64_t slice, int64_t rank, int64_t world,
                     torch::Tensor table);
void dsv_reduce_slice_sumsq(int64_t recv, int64_t world, int64_t slice, int64_t first, int64_t len, int64_t seg_len,
                            torch::Tensor g, torch::Tensor sq);
void dsv_exchange_rows(torch::Tensor a, c10::optional<torch::Tensor> b, int64_t rank, int64_t world,
                       torch::Tensor table);
void dsv_clip_coef(torch::Tensor rows, double max_norm, torch::Tensor coef, torch::Tensor total);
void dsv_adamw_slice_bcast(torch::Tensor p, torch::Tensor g, torch::Tensor m, torch::Tensor v, int64_t first,
                           int64_t len, int64_t seg_len, torch::Tensor coef, double lr, double b1, double b2,
                           double eps, double wd, int64_t step, int64_t rank, int64_t world, torch::Tensor table);
void dsv_ce_merge(torch::Tensor stats, int64_t n_tiles, torch::Tensor tgt, torch::Tensor part);
void dsv_ce_finalize(torch::Tensor parts, torch::Tensor labels, torch::Tensor lse, torch::Tensor loss);
int64_t dsv_read_error_gemm(bool clear);
int64_t dsv_read_error_attn_bwd(bool clear);
int64_t dsv_read_error_tp_bwd(bool clear);
int64_t dsv_read_error_attn_tc(bool clear);
int64_t dsv_read_error_attn_bwd_tc(bool clear);
static int64_t dsv_read_error(bool clear) {
  const int64_t codes[5] = {dsv_read_error_gemm(clear), dsv_read_error_attn_bwd(clear), dsv_read_error_tp_bwd(clear),
                            dsv_read_error_attn_tc(clear), dsv_read_error_attn_bwd_tc(clear)};
  for (int64_t c : codes)
    if (c != 0) return c;
  return 0;
}
void dsv_attn_bwd_tc(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor o, torch::Tensor d_o,
                     torch::Tensor tiles, torch::Tensor lse, torch::Tensor dd, c10::optional<torch::Tensor> dq,
                     c10::optional<torch::Tensor> dk, c10::optional<torch::Tensor> dv, double scale,
                     c10::optional<torch::Tensor> rope_cos, c10::optional<torch::Tensor> rope_sin,
                     c10::optional<torch::Tensor> dqkv, int64_t bf16_mask);
void dsv_attn_bwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor d_o, torch::Tensor tiles,
                  torch::Tensor lse, torch::Tensor dd, torch::Tensor do_bf, c10::optional<torch::Tensor> dq,
                  c10::optional<torch::Tensor> dk, c10::optional<torch::Tensor> dv, double scale,
                  c10::optional<torch::Tensor> rope_cos, c10::optional<torch::Tensor> rope_sin,
                  c10::optional<torch::Tensor> dqkv, int64_t bf16_mask);
void dsv_attn_fwd_dense(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor tiles, torch::Tensor o,
                        double scale);
void dsv_paged_prefill(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache, torch::Tensor block_tables,
                       torch::Tensor cu_q, torch::Tensor ctx_lens, torch::Tensor tile_info, torch::Tensor out,
                       int64_t num_heads, double scale, int64_t tile_rows);
void dsv_paged_prefill_tc(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache, torch::Tensor block_tables,
                          torch::Tensor cu_q, torch::Tensor ctx_lens, torch::Tensor tile_info, torch::Tensor out,
                          int64_t num_heads, double scale);
void dsv_attn_fwd_dense_tc(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor tiles, torch::Tensor out,
                           int64_t num_heads, int64_t num_kv_heads, double scale, c10::optional<torch::Tensor> lse,
                           c10::optional<torch::Tensor> d_o, c10::optional<torch::Tensor> dd);
void dsv_paged_decode(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache, torch::Tensor block_tables,
                      torch::Tensor ctx_lens, torch::Tensor out, torch::Tensor part_o, torch::Tensor part_ml,
                      int64_t num_heads, double scale, int64_t splits, int64_t keys_per_split);
void dsv_rms_norm(torch::Tensor x, c10::optional<torch::Tensor> residual, torch::Tensor w, torch::Tensor out,
                  double eps, c10::optional<torch::Tensor> save, int64_t save_lo, int64_t save_hi, int64_t save_dst);
void dsv_qk_norm_rope_cache(torch::Tensor qkv, torch::Tensor positions, torch::Tensor cos_sin,
                            c10::optional<torch::Tensor> q_norm, c10::optional<torch::Tensor> k_norm, double eps,
                            int64_t num_heads, int64_t num_kv_heads, c10::optional<torch::Tensor> k_cache,
                            c10::optional<torch::Tensor> v_cache, c10::optional<torch::Tensor> slot_mapping);
void dsv_lora_shrink(torch::Tensor x, torch::Tensor A, torch::Tensor slot_ids, torch::Tensor Z, int64_t seg);
torch::Tensor dsv_peer_tmaps(torch::Tensor ptrs, int64_t rows, int64_t cols, int64_t ld);
void dsv_gemm_ag(torch::Tensor maps, int64_t ag_rows, int64_t world, torch::Tensor a_local, torch::Tensor b,
                 torch::Tensor out, int64_t epi, c10::optional<torch::Tensor> z, c10::optional<torch::Tensor> b2,
                 c10::optional<torch::Tensor> tile_slots, int64_t lora_seg, c10::optional<torch::Tensor> gathered,
                 c10::optional<torch::Tensor> cnt, c10::optional<torch::Tensor> src, int64_t rank);
void dsv_lora_shrink_ag(torch::Tensor maps, int64_t ag_rows, int64_t world, torch::Tensor x_local, torch::Tensor A,
                        torch::Tensor slot_ids, torch::Tensor Z, int64_t pr, int64_t seg,
                        c10::optional<torch::Tensor> gathered, c10::optional<torch::Tensor> cnt,
                        c10::optional<torch::Tensor> src, int64_t rank);
void dsv_embedding_peer(torch::Tensor ids, torch::Tensor tables, int64_t v_local, int64_t vocab, torch::Tensor out);
void dsv_embedding(torch::Tensor ids, torch::Tensor table, torch::Tensor out, int64_t v0);
void dsv_ce_fwd_bwd(torch::Tensor logits, torch::Tensor targets, torch::Tensor loss,
                    c10::optional<torch::Tensor> grad, double gscale);
void dsv_seg_sumsq(torch::Tensor g, int64_t seg_len, torch::Tensor out);
void dsv_adamw(torch::Tensor p, torch::Tensor g, torch::Tensor m, torch::Tensor v, int64_t seg_len,
               c10::optional<torch::Tensor> seg_sumsq, double max_norm, double grad_scale, double lr, double b1,
               double b2, double eps, double wd, int64_t step);
void dsv_lora_publish(torch::Tensor A_src, torch::Tensor A_dst, torch::Tensor Bt_src, torch::Tensor B2_dst,
                      int64_t col0, int64_t b1, int64_t b2, bool interleave64, double scale);
void dsv_sample(torch::Tensor logits, torch::Tensor temps, torch::Tensor seeds, torch::Tensor out,
                c10::optional<torch::Tensor> topk, c10::optional<torch::Tensor> topp,
                c10::optional<torch::Tensor> logprobs);

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("gemm", &dsv_gemm, "tcgen05 GEMM with fused epilogues / LoRA expand");
  m.def("gemm_ar", &dsv_gemm_ar, "tcgen05 GEMM fused with an all-reduce over peer memory");
  m.def("gemm_ce_stats", &dsv_gemm_ce_stats, "LM-head GEMM whose epilogue keeps only softmax statistics");
  m.def("gemm_ce_grad", &dsv_gemm_ce_grad, "LM-head GEMM whose epilogue writes the cross-entropy gradient");
  m.def("gemm_push", &dsv_gemm_push, "MN-major GEMM pushing bf16 partial rows to their owner rank");
  m.def("gemm_wgrad", &dsv_gemm_wgrad, "LoRA factor-gradient GEMM over the token dimension");
  m.def("wait_counts", &dsv_wait_counts, "one-CTA bounded wait on this rank's arrival counters");
  m.def("reduce_norm_bcast", &dsv_reduce_norm_bcast, "owned-row reduce + RMSNorm backward + P2P all-gather");
  m.def("push_slices", &dsv_push_slices, "push fp32 partials to their slice owners over peer memory");
  m.def("reduce_slice_sumsq", &dsv_reduce_slice_sumsq, "sum an owned slice over the ranks + per-layer sum of squares");
  m.def("exchange_rows", &dsv_exchange_rows, "write a small row into every rank's table");
  m.def("clip_coef", &dsv_clip_coef, "per-layer clip coefficients from the ranks' sums of squares");
  m.def("adamw_slice_bcast", &dsv_adamw_slice_bcast, "AdamW on an owned slice, updated values to every rank");
  m.def("ce_merge", &dsv_ce_merge, "merge per-tile softmax statistics of one vocabulary slice");
  m.def("ce_finalize", &dsv_ce_finalize, "log-sum-exp and loss over the ranks' vocabulary slices");
  m.def("peer_alloc", [](int64_t bytes) {
    auto r = dsv_peer_alloc(bytes);
    return std::make_tuple(std::get<0>(r), pybind11::bytes(std::get<1>(r)));
  }, "cudaMalloc'd zeroed block + its CUDA IPC handle");
  m.def("peer_open", [](pybind11::bytes h) { return dsv_peer_open(std::string(h)); }, "open a peer's IPC block");
  m.def("peer_close", &dsv_peer_close, "unmap a peer block");
  m.def("peer_free", &dsv_peer_free, "free this rank's block");
  m.def("peer_zero", &dsv_peer_zero, "zero a range of this rank's block");
  m.def("peer_view", &dsv_peer_view, "tensor over a range of a peer workspace block");
  m.def("read_error", &dsv_read_error, "read (and optionally clear) the device error word");
  m.def("paged_prefill", &dsv_paged_prefill, "paged varlen causal attention (prefill), warp-level MMA");
  m.def("paged_prefill_tc", &dsv_paged_prefill_tc, "paged varlen causal attention (prefill), tcgen05 + TMA");
  m.def("attn_bwd_tc", &dsv_attn_bwd_tc,
        "varlen causal GQA attention backward, tcgen05 + TMA (dQ pass, then dK / dV pass)");
  m.def("attn_fwd_dense_tc", &dsv_attn_fwd_dense_tc,
        "varlen causal GQA attention forward on packed rows, tcgen05 + TMA (optional lse / rowsum(dO*O))");
  m.def("paged_decode", &dsv_paged_decode, "paged split-KV GQA decode attention");
  m.def("attn_bwd", &dsv_attn_bwd, "varlen causal GQA attention backward (dQ, dK, dV)");
  m.def("attn_fwd_dense", &dsv_attn_fwd_dense, "varlen causal GQA attention forward on packed rows");
  m.def("rms_norm", &dsv_rms_norm, "RMSNorm / fused residual add + RMSNorm (+ row capture)");
  m.def("qk_norm_rope_cache", &dsv_qk_norm_rope_cache, "q/k norm + RoPE + paged KV write");
  m.def("lora_shrink", &dsv_lora_shrink, "segmented multi-LoRA shrink");
  m.def("peer_tmaps", &dsv_peer_tmaps, "TMA tensor maps of the ranks' peer buffers (A operand of the all-gather GEMMs)");
  m.def("gemm_ag", &dsv_gemm_ag, "all-gather -> column-parallel GEMM: A row blocks read from their owner ranks by TMA");
  m.def("lora_shrink_ag", &dsv_lora_shrink_ag, "LoRA shrink of an all-gathered input (rows read from their owners)");
  m.def("embedding_peer", &dsv_embedding_peer, "vocab-parallel embedding read from every rank's shard over peer memory");
  m.def("embedding", &dsv_embedding, "vocab-parallel embedding gather");
  m.def("ce_fwd_bwd", &dsv_ce_fwd_bwd, "cross-entropy loss + gradient rows");
  m.def("seg_sumsq", &dsv_seg_sumsq, "per-segment sum of squares");
  m.def("adamw", &dsv_adamw, "flat AdamW with per-segment clipping");
  m.def("lora_publish", &dsv_lora_publish, "publish fp32 LoRA masters into a served slot");
  m.def("sample", &dsv_sample, "greedy / Gumbel-max sampling");
  m.def("rms_norm_bwd", &dsv_rms_norm_bwd, "RMSNorm backward (+ residual add)");
  m.def("swiglu_bwd", &dsv_swiglu_bwd, "SwiGLU backward over interleaved gate/up");
}
