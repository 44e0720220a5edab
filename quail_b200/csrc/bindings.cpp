// Python bindings of the sm_100a kernels (module quail_b200._C).
#include <torch/extension.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_runtime.h>

#include <mutex>

#include "gemm_sm100.h"

namespace qb {

void embed_gather(const torch::Tensor& ids, const torch::Tensor& table, torch::Tensor& out);
void post_norm_add_norm(const torch::Tensor& y, torch::Tensor& h, const torch::Tensor& wpost,
                        const c10::optional<torch::Tensor>& wnext, const c10::optional<torch::Tensor>& x, double eps);
void kv_copy_rows(torch::Tensor& k_cache, torch::Tensor& v_cache, const torch::Tensor& src, const torch::Tensor& dst);
void attention_merge(const torch::Tensor& o_a, const torch::Tensor& lse_a, const torch::Tensor& o_b,
                     const torch::Tensor& lse_b, const torch::Tensor& source, int64_t QH, torch::Tensor& out,
                     const c10::optional<torch::Tensor>& out_sf);
void rmsnorm_quant(const torch::Tensor& x, const torch::Tensor& w, double eps, const c10::optional<torch::Tensor>& y8,
                   const c10::optional<torch::Tensor>& ys, const c10::optional<torch::Tensor>& ybf, int64_t T);
void quant_rows(const torch::Tensor& x, bool swiglu, const c10::optional<torch::Tensor>& y8,
                const c10::optional<torch::Tensor>& ys, const c10::optional<torch::Tensor>& ybf, int64_t T);
void qk_norm_rope_kv(const torch::Tensor& qkv, const torch::Tensor& positions, const torch::Tensor& qw,
                     const torch::Tensor& kw, const torch::Tensor& cos_sin, const torch::Tensor& slots,
                     torch::Tensor& q_out, torch::Tensor& k_cache, torch::Tensor& v_cache, int64_t QH, int64_t KH,
                     double eps, bool norm_qk, int64_t T);
void final_norm_readout(const torch::Tensor& x, const torch::Tensor& rows, const torch::Tensor& w, double eps,
                        const torch::Tensor& head, torch::Tensor& logits, const c10::optional<torch::Tensor>& normed);
void prefill_attention(const torch::Tensor& q, const torch::Tensor& k_cache, const torch::Tensor& v_cache,
                       const torch::Tensor& seqs, const torch::Tensor& tiles, const torch::Tensor& page_list,
                       double softmax_scale, torch::Tensor& out, const c10::optional<torch::Tensor>& out_scale);

void gemm_mx_qkv_rope(const torch::Tensor& a, const torch::Tensor& sfa, const torch::Tensor& b,
                      const torch::Tensor& sfb, const torch::Tensor& positions, const torch::Tensor& slots,
                      const torch::Tensor& qn, const torch::Tensor& kn, const torch::Tensor& cos_sin,
                      torch::Tensor& q_out, torch::Tensor& k_cache, torch::Tensor& v_cache, int64_t QH, int64_t KH,
                      double eps, bool norm_qk, const c10::optional<torch::Tensor>& row_ss);
void prefill_attention_tc2(const torch::Tensor& q, const torch::Tensor& k_cache, const torch::Tensor& v_cache,
                           const torch::Tensor& seqs, const torch::Tensor& blocks, const torch::Tensor& page_list,
                           double softmax_scale, torch::Tensor& out, const c10::optional<torch::Tensor>& out_sf,
                           const c10::optional<torch::Tensor>& lse);
void gemm_mx(const torch::Tensor& a, const torch::Tensor& sfa, const torch::Tensor& b, const torch::Tensor& sfb,
             int64_t epi, torch::Tensor& out, const c10::optional<torch::Tensor>& out_sf,
             const c10::optional<torch::Tensor>& residual, const c10::optional<torch::Tensor>& row_ss,
             double ss_eps, const c10::optional<torch::Tensor>& xq, const c10::optional<torch::Tensor>& xq_sf,
             const c10::optional<torch::Tensor>& ss_out);
void quant_mx_ss(const torch::Tensor& x, torch::Tensor& y8, torch::Tensor& sf, torch::Tensor& ss, int64_t T);
void row_rinv(const torch::Tensor& parts, int64_t K, double eps, torch::Tensor& out);
void gemm_nvfp4(const torch::Tensor& a, const torch::Tensor& sfa, const torch::Tensor& b, const torch::Tensor& sfb,
                double alpha, int64_t epi, torch::Tensor& out, const c10::optional<torch::Tensor>& residual,
                const c10::optional<torch::Tensor>& row_scale);
void nvfp4_quant_rows(const torch::Tensor& x, bool swiglu, torch::Tensor& q, torch::Tensor& sf,
                      torch::Tensor& row_scale);
void rmsnorm_quant_mx(const torch::Tensor& x, const torch::Tensor& w, double eps, torch::Tensor& y8,
                      torch::Tensor& sf, int64_t T);
void quant_rows_mx(const torch::Tensor& x, bool swiglu, torch::Tensor& y8, torch::Tensor& sf, int64_t T);

void row_argmax_lse(const torch::Tensor& logits, torch::Tensor& arg, torch::Tensor& lse);

void prefill_attention_tc(const torch::Tensor& q, const torch::Tensor& k_cache, const torch::Tensor& v_cache,
                          const torch::Tensor& seqs, const torch::Tensor& tiles, const torch::Tensor& page_list,
                          double softmax_scale, torch::Tensor& out, const c10::optional<torch::Tensor>& out_sf);

void tp_ag_gemm(const torch::Tensor& a_local, const torch::Tensor& sfa_local, const std::vector<int64_t>& a_peer,
                const std::vector<int64_t>& sfa_peer, const std::vector<int64_t>& flag_peer,
                const torch::Tensor& tile_ready, int64_t epoch, int64_t rank, int64_t rpr, const torch::Tensor& b,
                const torch::Tensor& sfb, int64_t mode, torch::Tensor& out, const c10::optional<torch::Tensor>& out_sf);
void tp_gemm_rs(const torch::Tensor& a, const torch::Tensor& sfa, const torch::Tensor& b, const torch::Tensor& sfb,
                const std::vector<int64_t>& slot_ptrs, int64_t ld_slot, const std::vector<int64_t>& counter_ptrs,
                int64_t rank, int64_t rpr);
void tp_reduce_norm(const torch::Tensor& slots, int64_t tp_slots, const torch::Tensor& counters, int64_t want,
                    torch::Tensor& resid, const torch::Tensor& w, double eps, torch::Tensor& a_sym,
                    torch::Tensor& sf_sym, int64_t row0, torch::Tensor& done_ctr, int64_t done_base,
                    torch::Tensor& flag, int64_t epoch);

void moe_route(const torch::Tensor& logits, int64_t E, int64_t topk, torch::Tensor& ids, torch::Tensor& wts,
               torch::Tensor& pos, torch::Tensor& counts);
int64_t moe_plan_ints(int64_t E, int64_t Epr, int64_t tcap);
void moe_plan(torch::Tensor& counts, const std::vector<int64_t>& counts_all_peer,
              const std::vector<int64_t>& cflag_peer, const torch::Tensor& counts_all_local,
              const torch::Tensor& cflag_local, torch::Tensor& plan, torch::Tensor& cum, int64_t rank, int64_t E,
              int64_t tcap, int64_t epoch);
void moe_sort(const torch::Tensor& ids, const torch::Tensor& pos, int64_t n, const torch::Tensor& plan, int64_t E,
              torch::Tensor& src_list);
void moe_gate_up(const torch::Tensor& x8, const torch::Tensor& xsf, const torch::Tensor& src_list,
                 const torch::Tensor& wts, const torch::Tensor& plan, int64_t rank, int64_t E, int64_t topk,
                 int64_t tcap, const std::vector<int64_t>& recv_a_peer, const std::vector<int64_t>& recv_sf_peer,
                 const std::vector<int64_t>& recv_meta_peer, const std::vector<int64_t>& recv_count_peer,
                 const torch::Tensor& recv_a, const torch::Tensor& recv_sf, const torch::Tensor& recv_count,
                 const torch::Tensor& w_gu, const torch::Tensor& s_gu, torch::Tensor& y, torch::Tensor& ysf,
                 int64_t act);
void moe_down(const torch::Tensor& y, const torch::Tensor& ysf, const torch::Tensor& plan, int64_t E, int64_t tcap,
              const torch::Tensor& recv_meta, const torch::Tensor& w_d, const torch::Tensor& s_d,
              const std::vector<int64_t>& comb_peer, const std::vector<int64_t>& comb_counter_peer);
void moe_combine(const torch::Tensor& comb, int64_t M, int64_t topk, const torch::Tensor& counter, int64_t want,
                 torch::Tensor& resid, const c10::optional<torch::Tensor>& w, double eps,
                 const c10::optional<torch::Tensor>& y8, const c10::optional<torch::Tensor>& ysf);
void decode_attention(const torch::Tensor& q, const torch::Tensor& k_cache, const torch::Tensor& v_cache,
                      const torch::Tensor& seqs, const torch::Tensor& dseqs, const torch::Tensor& page_list,
                      double softmax_scale, torch::Tensor& out, const c10::optional<torch::Tensor>& out_sf);
void sae_topk(const torch::Tensor& pre, const torch::Tensor& bias, int64_t keep, torch::Tensor& out);
void gdn_layer(const torch::Tensor& proj, const torch::Tensor& wconv, const torch::Tensor& A_log,
               const torch::Tensor& dt_bias, const torch::Tensor& norm_w, const torch::Tensor& seqs,
               const torch::Tensor& state_io, torch::Tensor& conv_state, torch::Tensor& ssm_state, int64_t gi,
               int64_t Hk, int64_t Hv, int64_t DK, int64_t DV, double eps, torch::Tensor& conv_out,
               torch::Tensor& o, torch::Tensor& y, int64_t mode);
void small_attention(const torch::Tensor& q, const torch::Tensor& k_cache, const torch::Tensor& v_cache,
                     const torch::Tensor& seqs, const torch::Tensor& tiles, const torch::Tensor& dseqs,
                     const torch::Tensor& page_list, double softmax_scale, torch::Tensor& out,
                     const c10::optional<torch::Tensor>& gate, int64_t gate_hstride);
void hybrid_qk_rope_kv(const torch::Tensor& proj, int64_t QH, int64_t KH, bool gated, const torch::Tensor& positions,
                       const torch::Tensor& qw, const torch::Tensor& kw, bool offset, const torch::Tensor& cos_sin,
                       const torch::Tensor& slots, torch::Tensor& k_cache, torch::Tensor& v_cache,
                       torch::Tensor& q_out, double eps, int64_t sec_h, int64_t sec_w);
void qkv_norm_rope_kv(const torch::Tensor& proj, int64_t QH, int64_t KH, const torch::Tensor& positions,
                      const torch::Tensor& qw, const torch::Tensor& kw, const torch::Tensor& cos_sin,
                      const torch::Tensor& slots, torch::Tensor& k_cache, torch::Tensor& v_cache,
                      torch::Tensor& q_out, double eps, int64_t vmode);
void short_conv(const torch::Tensor& bcx, const torch::Tensor& wconv, const torch::Tensor& seqs,
                const torch::Tensor& state_io, torch::Tensor& state, int64_t li, torch::Tensor& y);

static std::mutex g_err_mu;
static int* g_err[64] = {nullptr};

int* device_error_word(int dev) {
  std::lock_guard<std::mutex> lk(g_err_mu);
  if (!g_err[dev]) {
    c10::cuda::CUDAGuard guard(dev);
    // 16 bytes: the error code (int) and, at byte 8, the wait budget (int64, 0 = default)
    int* p = nullptr;
    C10_CUDA_CHECK(cudaMalloc(&p, 16));
    C10_CUDA_CHECK(cudaMemset(p, 0, 16));
    g_err[dev] = p;
  }
  return g_err[dev];
}

// Synchronizes the device, returns the error code kernels recorded since the
// last call (0 = none) and clears it.
int64_t read_and_clear_error(int64_t dev) {
  int* p = device_error_word((int)dev);
  c10::cuda::CUDAGuard guard((int)dev);
  int h = 0;
  C10_CUDA_CHECK(cudaDeviceSynchronize());
  C10_CUDA_CHECK(cudaMemcpy(&h, p, sizeof(int), cudaMemcpyDeviceToHost));
  if (h) C10_CUDA_CHECK(cudaMemset(p, 0, sizeof(int)));
  return h;
}

// Sets the spin budget (clock cycles) of every bounded wait on the device;
// 0 or below restores the default. Takes effect for kernels launched after it.
void set_wait_budget(int64_t dev, int64_t cycles) {
  int* p = device_error_word((int)dev);
  c10::cuda::CUDAGuard guard((int)dev);
  long long v = cycles > 0 ? cycles : 0;
  C10_CUDA_CHECK(cudaDeviceSynchronize());
  C10_CUDA_CHECK(cudaMemcpy(p + 2, &v, sizeof(v), cudaMemcpyHostToDevice));
}

}  // namespace qb

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "quail_b200 sm_100a kernels";
  m.def("gemm", &qb::gemm_sm100, "tcgen05 GEMM (bf16 or block-scaled e4m3) with fused epilogues", py::arg("a"),
        py::arg("b"), py::arg("sa"), py::arg("sb"), py::arg("sb_gran"), py::arg("epi"), py::arg("out"),
        py::arg("out_scale"), py::arg("residual"), py::arg("bn"));
  m.def("gemm_mx", &qb::gemm_mx, "tcgen05 fp8 GEMM with UE8M0 block scales (kind::mxf8f6f4.block_scale)");
  m.def("row_rinv", &qb::row_rinv, "1 / rms per row from partial sums of squares");
  m.def("quant_mx_ss", &qb::quant_mx_ss, "bf16 rows -> MX e4m3 (no normalization) + per-row sum of squares");
  m.def("prefill_attention_tc2", &qb::prefill_attention_tc2,
        "persistent tcgen05 prefill attention: TMA loader, MMA warp, two ping-pong softmax warpgroups");
  m.def("gemm_mx_qkv_rope", &qb::gemm_mx_qkv_rope,
        "MX fp8 QKV projection with q/k RMSNorm, NeoX RoPE and the paged KV write in the epilogue");
  m.def("gemm_nvfp4", &qb::gemm_nvfp4, "tcgen05 NVFP4 GEMM: E2M1 operands, UE4M3 16-element block scales");
  m.def("nvfp4_quant_rows", &qb::nvfp4_quant_rows, "bf16 rows (or SwiGLU of gate|up) -> NVFP4 + per-row scale");
  m.def("rmsnorm_quant_mx", &qb::rmsnorm_quant_mx);
  m.def("quant_rows_mx", &qb::quant_rows_mx);
  m.def("row_argmax_lse", &qb::row_argmax_lse);
  m.def("embed_gather", &qb::embed_gather);
  m.def("post_norm_add_norm", &qb::post_norm_add_norm, "LFM3 sandwich norm: h += norm(y) * w; x = norm(h) * w_next");
  m.def("kv_copy_rows", &qb::kv_copy_rows, "copy K and V rows between arena slots");
  m.def("attention_merge", &qb::attention_merge, "merge two attention reads of the same rows by log-sum-exp");
  m.def("rmsnorm_quant", &qb::rmsnorm_quant);
  m.def("quant_rows", &qb::quant_rows);
  m.def("qk_norm_rope_kv", &qb::qk_norm_rope_kv);
  m.def("final_norm_readout", &qb::final_norm_readout);
  m.def("prefill_attention", &qb::prefill_attention);
  m.def("prefill_attention_tc", &qb::prefill_attention_tc, "tcgen05/TMEM packed-prompt prefill attention");
  m.def("decode_attention", &qb::decode_attention, "split-KV decode attention, all q heads of a KV head per CTA");
  m.def("sae_topk", &qb::sae_topk, "SAE features: bias + per-row top-k (radix select), packed indices + strengths");
  m.def("gdn_layer", &qb::gdn_layer, "Gated DeltaNet: causal conv + L2 norm, delta-rule recurrence, gated RMSNorm");
  m.def("small_attention", &qb::small_attention, "paged attention for any head_dim <= 256, optional sigmoid gate");
  m.def("hybrid_qk_rope_kv", &qb::hybrid_qk_rope_kv, "q/k RMSNorm + partial RoPE + KV write of gated attention");
  m.def("qkv_norm_rope_kv", &qb::qkv_norm_rope_kv,
        "Gemma 4 attention inputs: q/k RMSNorm + RoPE, values RMS-normalized (own or the key projection), KV write");
  m.def("short_conv", &qb::short_conv, "LFM2 gated short convolution with per-key state slots");
  m.def("read_and_clear_error", &qb::read_and_clear_error);
  m.def("tp_ag_gemm", &qb::tp_ag_gemm, "all-gather -> MX GEMM fused over NVLink peer memory");
  m.def("tp_gemm_rs", &qb::tp_gemm_rs, "MX GEMM -> reduce-scatter fused: epilogue pushes tiles to owner ranks");
  m.def("set_wait_budget", &qb::set_wait_budget, "spin budget (cycles) of the kernels' bounded waits; 0 = default");
  m.def("tp_reduce_norm", &qb::tp_reduce_norm, "sum RS slots + residual, RMSNorm, MX quant into the AG buffer");
  m.def("moe_route", &qb::moe_route, "MoE router: softmax, top-k, renormalized weights, per-expert slots");
  m.def("moe_plan_ints", &qb::moe_plan_ints);
  m.def("moe_plan", &qb::moe_plan, "MoE count exchange over peers and dispatch / tile planning");
  m.def("moe_sort", &qb::moe_sort);
  m.def("moe_gate_up", &qb::moe_gate_up, "token dispatch (P2P) fused into the grouped MX gate_up GEMM + SwiGLU");
  m.def("moe_down", &qb::moe_down, "grouped MX down GEMM with the weighted combine pushed from the epilogue");
  m.def("moe_combine", &qb::moe_combine, "sum expert rows into the residual + next RMSNorm as MX");
  m.attr("EPI_BF16") = (int)qb::kEpiBf16;
  m.attr("EPI_RESIDUAL") = (int)qb::kEpiResidual;
  m.attr("EPI_SWIGLU_FP8") = (int)qb::kEpiSwigluFp8;
  m.attr("EPI_SWIGLU_BF16") = (int)qb::kEpiSwigluBf16;
}
