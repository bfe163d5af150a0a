// Python bindings of the sm_100a kernels (torch extension module mesh_b200._C).
#include <torch/extension.h>

namespace mesh {
void gemm_tcgen05(const at::Tensor& A, const at::Tensor& B, at::Tensor& out, int64_t epi, bool trans, int64_t bn,
                  int64_t mode, at::Tensor& workspace, at::Tensor& counters, at::Tensor& err,
                  const c10::optional<at::Tensor>& trace, const std::vector<int64_t>& push);
void gemm_allreduce_norm(const at::Tensor& w, const at::Tensor& x, at::Tensor& part, const std::vector<int64_t>& push,
                         const std::vector<int64_t>& cfg, const at::Tensor& gamma, double eps, at::Tensor& epoch,
                         int64_t mode, at::Tensor& workspace, at::Tensor& counters, at::Tensor& err,
                         const c10::optional<at::Tensor>& trace);
std::vector<int64_t> gemm_plan(int64_t M, int64_t N, int64_t K, int64_t epi, bool trans, int64_t device);
void gemm_qkv_rope(const at::Tensor& w, const at::Tensor& x, at::Tensor& q_out, const at::Tensor& pos,
                   const at::Tensor& slot, const at::Tensor& cos_t, const at::Tensor& sin_t, at::Tensor& kcache,
                   at::Tensor& vcache, int64_t hq, int64_t hkv, int64_t mode, at::Tensor& workspace,
                   at::Tensor& counters, at::Tensor& err);
void add_rmsnorm(const c10::optional<at::Tensor>& delta, at::Tensor& resid, const at::Tensor& gamma, at::Tensor& normed,
                 double eps);
void rope_kv_write(const at::Tensor& qkv, const at::Tensor& pos, const at::Tensor& slot, const at::Tensor& cos_t,
                   const at::Tensor& sin_t, at::Tensor& q_out, at::Tensor& kcache, at::Tensor& vcache, int64_t hq,
                   int64_t hkv);
void embedding(const at::Tensor& ids, const at::Tensor& table, at::Tensor& out, at::Tensor& err);
void argmax_partial(const at::Tensor& logits, int64_t vocab_offset, at::Tensor& out);
void argmax_merge(const at::Tensor& cand, at::Tensor& ids);
void argmax_tiles(const at::Tensor& cand, int64_t vocab_offset, at::Tensor& out);
void attn_decode(const at::Tensor& q, const at::Tensor& kcache, const at::Tensor& vcache,
                 const at::Tensor& block_tables, const at::Tensor& seq_lens, at::Tensor& out, at::Tensor& ws,
                 int64_t splits, double scale, int64_t window);
int64_t attn_decode_pick_splits(int64_t B, int64_t hkv, int64_t max_len, int64_t num_sms);
void attn_decode_tc(const at::Tensor& q, const at::Tensor& kcache, const at::Tensor& vcache,
                    const at::Tensor& block_tables, const at::Tensor& seq_lens, at::Tensor& out, at::Tensor& ws,
                    at::Tensor& err, int64_t splits, double scale, int64_t window,
                    const c10::optional<at::Tensor>& counters);
void attn_prefill(const at::Tensor& q, const at::Tensor& kcache, const at::Tensor& vcache, const at::Tensor& cu_q,
                  const at::Tensor& k_lens, const at::Tensor& block_tables, at::Tensor& out, int64_t max_q_len,
                  double scale, int64_t window);
void attn_prefill_tc(const at::Tensor& q, const at::Tensor& kcache, const at::Tensor& vcache, const at::Tensor& cu_q,
                     const at::Tensor& k_lens, const at::Tensor& block_tables, at::Tensor& out, int64_t max_q_len,
                     double scale, int64_t window, at::Tensor& err);
bool attn_prefill_tc_supported(int64_t head_dim, int64_t page_size, int64_t group);
void gemm_2sm(const at::Tensor& A, const at::Tensor& B, at::Tensor& out, int64_t epi, at::Tensor& err,
              const c10::optional<at::Tensor>& trace, int64_t tn);
bool gemm_2sm_supported(int64_t M, int64_t N, int64_t K, int64_t epi);
void samp_stats(const at::Tensor& logits, const at::Tensor& inv_t, const at::Tensor& gmax, at::Tensor& out,
                int64_t step);
void samp_init(int64_t stage, int64_t world, int64_t rank, const at::Tensor& inv_t, const at::Tensor& top_p,
               const at::Tensor& thr, const at::Tensor& masses, at::Tensor& st, at::Tensor& active);
void samp_radix(const at::Tensor& logits, const at::Tensor& inv_t, const at::Tensor& gmax, at::Tensor& st,
                at::Tensor& active, at::Tensor& hist, int64_t shift, int64_t phase);
void samp_find(const at::Tensor& logits, const at::Tensor& inv_t, const at::Tensor& gmax, const at::Tensor& top_p,
               const at::Tensor& thr, at::Tensor& st, at::Tensor& active, int64_t vocab_offset, at::Tensor& cand);
void samp_merge(const at::Tensor& inv_t, const at::Tensor& top_p, const at::Tensor& cand, const at::Tensor& greedy,
                at::Tensor& ids);
void embed_peer_norm(const at::Tensor& bases, const at::Tensor& ids, int64_t V, const at::Tensor& gamma, double eps,
                     at::Tensor& resid, at::Tensor& normed, at::Tensor& err);
void kv_pages_copy(at::Tensor& k_pool, at::Tensor& v_pool, at::Tensor& buf, const at::Tensor& pages, bool to_buf);
void ar_fused_norm(const at::Tensor& bases, int64_t off_flags, int64_t off_p0, int64_t off_p1, int64_t off_resid,
                   int64_t off_normed, int64_t rank, int64_t world, int64_t T, int64_t H, int64_t parity,
                   const at::Tensor& gamma, double eps, at::Tensor& epoch, at::Tensor& err, int64_t nblocks,
                   bool two_shot, double timeout_s, int64_t mc_base, const at::Tensor& trace);
void ar_barrier(const at::Tensor& bases, int64_t off_flags, int64_t rank, int64_t world, at::Tensor& epoch,
                at::Tensor& err, double timeout_s, const at::Tensor& device_ref);
int64_t ar_flags_bytes();
void ar_push_reduce_norm(const at::Tensor& bases, int64_t off_flags, int64_t off_push, int64_t off_resid,
                         int64_t off_normed, int64_t rank, int64_t world, int64_t T, int64_t t_max, int64_t H,
                         const at::Tensor& gamma, double eps, at::Tensor& epoch, at::Tensor& err, int64_t nblocks,
                         bool two_shot, double timeout_s);
}  // namespace mesh

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "mesh_b200 sm_100a kernels";
  m.def("gemm_tcgen05", &mesh::gemm_tcgen05, "tcgen05 GEMM out = A @ B^T (or its transpose)", py::arg("A"),
        py::arg("B"), py::arg("out"), py::arg("epi"), py::arg("trans"), py::arg("bn"), py::arg("mode"),
        py::arg("workspace"), py::arg("counters"), py::arg("err"), py::arg("trace") = py::none(),
        py::arg("push") = std::vector<int64_t>{});
  m.def("gemm_qkv_rope", &mesh::gemm_qkv_rope, "decode qkv GEMM with RoPE and the paged KV write in the epilogue");
  m.def("gemm_allreduce_norm", &mesh::gemm_allreduce_norm,
        "decode GEMM with the tensor-parallel all-reduce, residual add, RMSNorm and all-gather fused in",
        py::arg("w"), py::arg("x"), py::arg("part"), py::arg("push"), py::arg("cfg"), py::arg("gamma"), py::arg("eps"),
        py::arg("epoch"), py::arg("mode"), py::arg("workspace"), py::arg("counters"), py::arg("err"),
        py::arg("trace") = py::none());
  m.def("gemm_plan", &mesh::gemm_plan, "tile plan [bn, workspace_floats, stream-K tiles, stages, grid, dp_tiles, sk_iters]");
  m.def("add_rmsnorm", &mesh::add_rmsnorm, "resid += delta; normed = rmsnorm(resid) * gamma");
  m.def("rope_kv_write", &mesh::rope_kv_write, "RoPE on q/k + paged KV write");
  m.def("embedding", &mesh::embedding, "embedding gather");
  m.def("argmax_partial", &mesh::argmax_partial, "per-row (max, global index) over local vocab");
  m.def("argmax_merge", &mesh::argmax_merge, "merge per-rank argmax candidates");
  m.def("argmax_tiles", &mesh::argmax_tiles, "reduce LM-head per-tile argmax candidates");
  m.def("attn_decode", &mesh::attn_decode, "paged GQA decode attention (split-KV)");
  m.def("attn_decode_tc", &mesh::attn_decode_tc, "paged GQA decode attention, TMA-streamed tensor-core variant",
        py::arg("q"), py::arg("kcache"), py::arg("vcache"), py::arg("block_tables"), py::arg("seq_lens"),
        py::arg("out"), py::arg("ws"), py::arg("err"), py::arg("splits"), py::arg("scale"), py::arg("window"),
        py::arg("counters") = py::none());
  m.def("attn_decode_pick_splits", &mesh::attn_decode_pick_splits, "split-KV heuristic");
  m.def("attn_prefill", &mesh::attn_prefill, "paged causal varlen GQA prefill attention");
  m.def("attn_prefill_tc", &mesh::attn_prefill_tc,
        "paged causal varlen GQA prefill attention on tcgen05 (TMEM scores and accumulator, TMA page loads)");
  m.def("attn_prefill_tc_supported", &mesh::attn_prefill_tc_supported, "shapes the tcgen05 prefill attention serves");
  m.def("gemm_2sm", &mesh::gemm_2sm, "prefill GEMM on SM pairs (tcgen05.mma.cta_group::2, 256x256 tiles)",
        py::arg("A"), py::arg("B"), py::arg("out"), py::arg("epi"), py::arg("err"), py::arg("trace") = py::none(),
        py::arg("tn") = 0);
  m.def("gemm_2sm_supported", &mesh::gemm_2sm_supported, "shapes the SM-pair GEMM serves");
  m.def("samp_stats", &mesh::samp_stats, "sampling: row max (step 0) / fixed-point mass (step 1)");
  m.def("samp_init", &mesh::samp_init, "sampling: per-row selection set-up");
  m.def("samp_radix", &mesh::samp_radix, "sampling: radix pass (phase 0 histogram, phase 1 select)");
  m.def("samp_find", &mesh::samp_find, "sampling: this rank's candidate token per row");
  m.def("samp_merge", &mesh::samp_merge, "sampling: merge sampled and greedy tokens");
  m.def("embed_peer_norm", &mesh::embed_peer_norm,
        "vocabulary-parallel embedding read from the owner rank's table over NVLink, fused with RMSNorm");
  m.def("kv_pages_copy", &mesh::kv_pages_copy,
        "gather a session's KV pages (every layer) into a contiguous buffer, or scatter one into pages");
  m.def("ar_fused_norm", &mesh::ar_fused_norm, "peer-memory all-reduce + residual + RMSNorm");
  m.def("ar_barrier", &mesh::ar_barrier, "bounded cross-rank barrier over peer flags");
  m.def("ar_flags_bytes", &mesh::ar_flags_bytes, "bytes of the flag region of the AR workspace");
  m.def("ar_push_reduce_norm", &mesh::ar_push_reduce_norm,
        "reduce the partial tiles peers pushed into this rank (+residual, RMSNorm, all-gather)");
}
