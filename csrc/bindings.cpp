// Python bindings for every helexa_b200 CUDA op (one function per kernel family).
#include <torch/extension.h>

void gemv(torch::Tensor W, torch::Tensor x, torch::Tensor y, int64_t mode, c10::optional<torch::Tensor> resid,
          c10::optional<torch::Tensor> norm_w, double eps);
void gemv_experts(torch::Tensor W, torch::Tensor x, torch::Tensor ids, torch::Tensor y, int64_t mode,
                  int64_t x_row_div, c10::optional<torch::Tensor> norm_w, double eps);
void moe_topk(torch::Tensor logits, int64_t E, int64_t k, bool has_shared, bool norm_topk, torch::Tensor ids,
              torch::Tensor wts);
void moe_down(torch::Tensor Wd, torch::Tensor act, torch::Tensor ids, torch::Tensor wts, torch::Tensor x,
              c10::optional<torch::Tensor> partial_out);
void gdn_decode(torch::Tensor proj, torch::Tensor conv_w, torch::Tensor conv_ring, torch::Tensor rec,
                torch::Tensor A_log, torch::Tensor dt_bias, torch::Tensor norm_w, torch::Tensor slots,
                torch::Tensor pos, torch::Tensor out, int64_t Hk, int64_t Hv, int64_t Dk, int64_t Dv, double eps);
void attn_decode(torch::Tensor proj, c10::optional<torch::Tensor> q_norm_w, c10::optional<torch::Tensor> k_norm_w,
                 torch::Tensor inv_freq, torch::Tensor kc, torch::Tensor vc, torch::Tensor slots, torch::Tensor pos,
                 torch::Tensor part_o, torch::Tensor part_ml, torch::Tensor counters, torch::Tensor out, int64_t Hq,
                 int64_t Hkv, int64_t D, int64_t rot, bool gated, double eps, c10::optional<torch::Tensor> rope_delta);
void gemv_ar(torch::Tensor W, torch::Tensor inp, torch::Tensor x, std::vector<int64_t> bases, int64_t rank,
             int64_t slot_elems, torch::Tensor epoch, torch::Tensor err, double timeout_s);
void moe_down_ar(torch::Tensor Wd, torch::Tensor act, torch::Tensor ids, torch::Tensor wts, torch::Tensor x,
                 std::vector<int64_t> bases, int64_t rank, int64_t slot_elems, torch::Tensor epoch, torch::Tensor err,
                 double timeout_s);
void attn_prefill(torch::Tensor q, torch::Tensor kc, torch::Tensor vc, torch::Tensor out, int64_t Hq, int64_t p0,
                  double scale, c10::optional<torch::Tensor> gate, int64_t gate_head_stride);
void add_rmsnorm(torch::Tensor x, c10::optional<torch::Tensor> o, torch::Tensor w, torch::Tensor h, double eps);
void qk_rope_kv(torch::Tensor qkv, int64_t Hq, int64_t Hkv, int64_t D, int64_t qw, c10::optional<torch::Tensor> q_norm,
                c10::optional<torch::Tensor> k_norm, torch::Tensor inv_freq, int64_t rot, torch::Tensor kc,
                torch::Tensor vc, int64_t p0, torch::Tensor q_out, double eps, c10::optional<torch::Tensor> pos3,
                c10::optional<torch::Tensor> axes, int64_t rope_off);
void conv_ring_update(torch::Tensor proj, torch::Tensor ring, int64_t p0);
void rs_norm_ag(std::vector<int64_t> bases, int64_t rank, int64_t stage_off, int64_t h_off, torch::Tensor x,
                torch::Tensor w, double eps, torch::Tensor ctr, torch::Tensor err, double timeout_s, int64_t ctas,
                int64_t mc);
int64_t rs_norm_ag_flag_bytes();
void gemv_tma(torch::Tensor W, torch::Tensor x, torch::Tensor y, int64_t mode, c10::optional<torch::Tensor> resid,
              c10::optional<torch::Tensor> norm_w, double eps, torch::Tensor err);
void gemv_tma_ar(torch::Tensor W, torch::Tensor inp, torch::Tensor x, std::vector<int64_t> bases, int64_t rank,
                 int64_t slot_elems, torch::Tensor ctr, torch::Tensor err, double timeout_s);
void gemv_tma_experts(torch::Tensor W, torch::Tensor x, torch::Tensor ids, torch::Tensor y, int64_t mode,
                      int64_t x_row_div, c10::optional<torch::Tensor> norm_w, double eps, int64_t e_base,
                      int64_t e_count, torch::Tensor err);
void moe_down_tma(torch::Tensor Wd, torch::Tensor act, torch::Tensor ids, torch::Tensor wts, torch::Tensor x,
                  c10::optional<torch::Tensor> partial_out, int64_t e_base, int64_t e_count, torch::Tensor err,
                  c10::optional<std::vector<int64_t>> bases, int64_t rank, int64_t slot_elems,
                  c10::optional<torch::Tensor> ctr, double timeout_s);
void gemv_tma_argmax(torch::Tensor W, torch::Tensor x, c10::optional<torch::Tensor> logits, torch::Tensor norm_w,
                     double eps, torch::Tensor best, torch::Tensor counter, torch::Tensor tok, torch::Tensor slots,
                     torch::Tensor pos, torch::Tensor out_tokens, torch::Tensor step, int64_t v_off, torch::Tensor err,
                     c10::optional<std::vector<int64_t>> bases, int64_t rank, int64_t slot_elems,
                     c10::optional<torch::Tensor> ctr, double timeout_s);
bool gemv_tma_ok(int64_t N, int64_t K, int64_t x_rows, int64_t groups_per_rb);
torch::Tensor gguf_pad_q6k(torch::Tensor W);
void sample_step(torch::Tensor logits, int64_t V, torch::Tensor slots, torch::Tensor temp, torch::Tensor top_k,
                 torch::Tensor top_p, torch::Tensor penalty, torch::Tensor seed, torch::Tensor ctr, torch::Tensor hist,
                 torch::Tensor hist_n, torch::Tensor hist_at, torch::Tensor hist_cap, torch::Tensor tok,
                 torch::Tensor pos, torch::Tensor out_tokens, torch::Tensor step);
void moe_fused(torch::Tensor x, torch::Tensor norm_w, double eps, torch::Tensor router, torch::Tensor w_gu,
               torch::Tensor w_d, int64_t E, int64_t topk, bool has_shared, bool norm_topk, torch::Tensor rlogits,
               torch::Tensor act, torch::Tensor bar, torch::Tensor err, int64_t e_base, int64_t e_count,
               c10::optional<std::vector<int64_t>> bases, int64_t rank, int64_t slot_elems,
               c10::optional<torch::Tensor> ctr, double timeout_s);
void attn_prefill_tc(torch::Tensor q, torch::Tensor kc, torch::Tensor vc, torch::Tensor out, int64_t Hq, int64_t p0,
                     double scale, c10::optional<torch::Tensor> gate, int64_t gate_head_stride, torch::Tensor err, bool causal);
void gemv_experts_ep(torch::Tensor W, torch::Tensor x, torch::Tensor ids, torch::Tensor y, int64_t mode,
                     int64_t x_row_div, c10::optional<torch::Tensor> norm_w, double eps, int64_t e_base);
void moe_down_ar_ep(torch::Tensor Wd, torch::Tensor act, torch::Tensor ids, torch::Tensor wts, torch::Tensor x,
                    std::vector<int64_t> bases, int64_t rank, int64_t slot_elems, torch::Tensor epoch,
                    torch::Tensor err, double timeout_s, int64_t e_base);
void moe_combine(torch::Tensor y, torch::Tensor rows, torch::Tensor wts, torch::Tensor x, bool accumulate);
void moe_route_prefill(torch::Tensor logits, int64_t E, int64_t k, bool has_shared, bool norm_topk, torch::Tensor hn,
                       torch::Tensor ids, torch::Tensor wts, torch::Tensor rows, torch::Tensor counts,
                       torch::Tensor offsets, torch::Tensor cursor, torch::Tensor tiles, torch::Tensor ntiles,
                       torch::Tensor A, int64_t e_base, int64_t e_count);
void gemm_grouped_dev(torch::Tensor A, torch::Tensor B, torch::Tensor C, torch::Tensor tiles, torch::Tensor ntiles,
                      int64_t n, int64_t epi, torch::Tensor err);
void embed(torch::Tensor E, torch::Tensor tok, torch::Tensor x);
void argmax_step(torch::Tensor logits, torch::Tensor tok, c10::optional<torch::Tensor> slots,
                 c10::optional<torch::Tensor> pos, c10::optional<torch::Tensor> out, c10::optional<torch::Tensor> step);

std::vector<torch::Tensor> ipc_alloc(int64_t bytes, int64_t device);
int64_t ipc_open(torch::Tensor handle, int64_t device);
void ipc_close(int64_t ptr);
void ar_oneshot(std::vector<int64_t> peer_bases, int64_t rank, torch::Tensor partial, torch::Tensor x,
                c10::optional<torch::Tensor> out_plain, int64_t data_bytes, torch::Tensor epoch, torch::Tensor err,
                int64_t ctas, double timeout_s);

void gemm(torch::Tensor A, torch::Tensor B, torch::Tensor C, int64_t epi, torch::Tensor err);
void gemm_grouped(torch::Tensor A, torch::Tensor B, torch::Tensor C, torch::Tensor tiles, int64_t n, int64_t epi,
                  torch::Tensor err);

void gemv_router(torch::Tensor W, torch::Tensor x, torch::Tensor logits, torch::Tensor norm_w, double eps,
                 int64_t E, int64_t topk, bool has_shared, bool norm_topk, torch::Tensor ids, torch::Tensor wts,
                 torch::Tensor counter);
void gemv_argmax(torch::Tensor W, torch::Tensor x, c10::optional<torch::Tensor> logits, torch::Tensor norm_w,
                 double eps, torch::Tensor best, torch::Tensor counter, torch::Tensor tok,
                 c10::optional<torch::Tensor> slots, c10::optional<torch::Tensor> pos,
                 c10::optional<torch::Tensor> out_tokens, c10::optional<torch::Tensor> step);
void gemv_argmax_tp(torch::Tensor W, torch::Tensor x, c10::optional<torch::Tensor> logits, torch::Tensor norm_w,
                    double eps, torch::Tensor best, torch::Tensor counter, torch::Tensor tok, torch::Tensor slots,
                    torch::Tensor pos, torch::Tensor out_tokens, torch::Tensor step, int64_t v_off,
                    std::vector<int64_t> bases, int64_t rank, int64_t slot_elems, torch::Tensor epoch,
                    torch::Tensor err, double timeout_s);

void gdn_prefill(torch::Tensor proj, torch::Tensor conv_w, torch::Tensor ring, torch::Tensor A_log,
                 torch::Tensor dt_bias, torch::Tensor norm_w, torch::Tensor state, torch::Tensor out, int64_t Hk,
                 int64_t Hv, int64_t D, int64_t p0, double eps);

#include "hx_runtime.h"

torch::Tensor gguf_dequant_host(torch::Tensor raw, int64_t type, int64_t n);
torch::Tensor gguf_quant_host(torch::Tensor x, int64_t type);
void gguf_gemv(torch::Tensor W, int64_t type, int64_t K, torch::Tensor x, torch::Tensor y, int64_t mode,
               c10::optional<torch::Tensor> resid, c10::optional<torch::Tensor> norm_w, double eps);
void gguf_dequant(torch::Tensor W, int64_t type, int64_t K, torch::Tensor out);
torch::Tensor gguf_quant(torch::Tensor W, int64_t type);
void gguf_experts(torch::Tensor W, int64_t type, int64_t K, torch::Tensor x, torch::Tensor ids, torch::Tensor act,
                  int64_t J, c10::optional<torch::Tensor> norm_w, double eps, int64_t e_base, int64_t e_count);
void gguf_moe_down(torch::Tensor W, int64_t type, int64_t I, torch::Tensor act, torch::Tensor ids, torch::Tensor wts,
                   torch::Tensor x, int64_t J, int64_t e_base, int64_t e_count);

void dit_norm_mod(torch::Tensor x, torch::Tensor w, c10::optional<torch::Tensor> scale, torch::Tensor y, double eps);
void dit_gate_res(torch::Tensor x, torch::Tensor y, torch::Tensor w, c10::optional<torch::Tensor> gate, double eps);
void dit_qk_rope(torch::Tensor qkv, c10::optional<torch::Tensor> qw, c10::optional<torch::Tensor> kw,
                 torch::Tensor ang, int64_t H, int64_t Dh, double eps, torch::Tensor q, torch::Tensor k,
                 torch::Tensor v);

void gemm_q(torch::Tensor A, torch::Tensor Wq, int64_t type, int64_t K, torch::Tensor C, int64_t epi,
            torch::Tensor err);

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("set_pdl", [](bool on) { hx_pdl_enabled() = on; });
  m.def("gemv", &gemv);
  m.def("gemv_experts", &gemv_experts);
  m.def("moe_topk", &moe_topk);
  m.def("moe_down", &moe_down);
  m.def("moe_combine", &moe_combine, py::arg("y"), py::arg("rows"), py::arg("wts"), py::arg("x"),
        py::arg("accumulate") = true);
  m.def("gemv_ar", &gemv_ar);
  m.def("moe_down_ar", &moe_down_ar);
  m.def("gemv_experts_ep", &gemv_experts_ep);
  m.def("moe_down_ar_ep", &moe_down_ar_ep);
  m.def("moe_route_prefill", &moe_route_prefill);
  m.def("gemm_grouped_dev", &gemm_grouped_dev);
  m.def("gdn_decode", &gdn_decode);
  m.def("attn_decode", &attn_decode, py::arg("proj"), py::arg("q_norm_w"), py::arg("k_norm_w"), py::arg("inv_freq"),
        py::arg("kc"), py::arg("vc"), py::arg("slots"), py::arg("pos"), py::arg("part_o"), py::arg("part_ml"),
        py::arg("counters"), py::arg("out"), py::arg("Hq"), py::arg("Hkv"), py::arg("D"), py::arg("rot"),
        py::arg("gated"), py::arg("eps"), py::arg("rope_delta") = py::none());
  m.def("attn_prefill", &attn_prefill, py::arg("q"), py::arg("kc"), py::arg("vc"), py::arg("out"), py::arg("Hq"),
        py::arg("p0"), py::arg("scale"), py::arg("gate") = py::none(), py::arg("gate_head_stride") = 0);
  m.def("add_rmsnorm", &add_rmsnorm);
  m.def("qk_rope_kv", &qk_rope_kv, py::arg("qkv"), py::arg("Hq"), py::arg("Hkv"), py::arg("D"), py::arg("qw"),
        py::arg("q_norm"), py::arg("k_norm"), py::arg("inv_freq"), py::arg("rot"), py::arg("kc"), py::arg("vc"),
        py::arg("p0"), py::arg("q_out"), py::arg("eps"), py::arg("pos3") = py::none(), py::arg("axes") = py::none(),
        py::arg("rope_off") = 0);
  m.def("conv_ring_update", &conv_ring_update);
  m.def("rs_norm_ag", &rs_norm_ag, py::arg("bases"), py::arg("rank"), py::arg("stage_off"), py::arg("h_off"),
        py::arg("x"), py::arg("w"), py::arg("eps"), py::arg("ctr"), py::arg("err"), py::arg("timeout_s"),
        py::arg("ctas"), py::arg("mc") = 0);
  m.def("rs_norm_ag_flag_bytes", &rs_norm_ag_flag_bytes);
  m.def("gemv_tma", &gemv_tma);
  m.def("gemv_tma_ar", &gemv_tma_ar);
  m.def("gemv_tma_experts", &gemv_tma_experts);
  m.def("moe_down_tma", &moe_down_tma, py::arg("Wd"), py::arg("act"), py::arg("ids"), py::arg("wts"), py::arg("x"),
        py::arg("partial_out"), py::arg("e_base"), py::arg("e_count"), py::arg("err"), py::arg("bases") = py::none(),
        py::arg("rank") = 0, py::arg("slot_elems") = 0, py::arg("ctr") = py::none(), py::arg("timeout_s") = 5.0);
  m.def("gemv_tma_argmax", &gemv_tma_argmax, py::arg("W"), py::arg("x"), py::arg("logits"), py::arg("norm_w"),
        py::arg("eps"), py::arg("best"), py::arg("counter"), py::arg("tok"), py::arg("slots"), py::arg("pos"),
        py::arg("out_tokens"), py::arg("step"), py::arg("v_off"), py::arg("err"), py::arg("bases") = py::none(),
        py::arg("rank") = 0, py::arg("slot_elems") = 0, py::arg("ctr") = py::none(), py::arg("timeout_s") = 5.0);
  m.def("gemv_tma_ok", &gemv_tma_ok);
  m.def("gguf_pad_q6k", &gguf_pad_q6k);
  m.def("attn_prefill_tc", &attn_prefill_tc, py::arg("q"), py::arg("kc"), py::arg("vc"), py::arg("out"), py::arg("Hq"),
        py::arg("p0"), py::arg("scale"), py::arg("gate"), py::arg("gate_head_stride"), py::arg("err"),
        py::arg("causal") = true);
  m.def("sample_step", &sample_step);
  m.def("moe_fused", &moe_fused, py::arg("x"), py::arg("norm_w"), py::arg("eps"), py::arg("router"), py::arg("w_gu"),
        py::arg("w_d"), py::arg("E"), py::arg("topk"), py::arg("has_shared"), py::arg("norm_topk"),
        py::arg("rlogits"), py::arg("act"), py::arg("bar"), py::arg("err"), py::arg("e_base") = 0,
        py::arg("e_count") = 0, py::arg("bases") = py::none(), py::arg("rank") = 0, py::arg("slot_elems") = 0,
        py::arg("ctr") = py::none(), py::arg("timeout_s") = 5.0);
  m.def("embed", &embed);
  m.def("dit_norm_mod", &dit_norm_mod);
  m.def("dit_gate_res", &dit_gate_res);
  m.def("dit_qk_rope", &dit_qk_rope);
  m.def("argmax_step", &argmax_step);
  m.def("ipc_alloc", &ipc_alloc);
  m.def("ipc_open", &ipc_open);
  m.def("ipc_close", &ipc_close);
  m.def("ar_oneshot", &ar_oneshot);
  m.def("gemm", &gemm);
  m.def("gemm_q", &gemm_q);
  m.def("gguf_dequant_host", &gguf_dequant_host);
  m.def("gguf_quant_host", &gguf_quant_host);
  m.def("gguf_gemv", &gguf_gemv);
  m.def("gguf_dequant", &gguf_dequant);
  m.def("gguf_quant", &gguf_quant);
  m.def("gguf_experts", &gguf_experts, py::arg("W"), py::arg("type"), py::arg("K"), py::arg("x"), py::arg("ids"),
        py::arg("act"), py::arg("J"), py::arg("norm_w") = py::none(), py::arg("eps") = 0.0, py::arg("e_base") = 0,
        py::arg("e_count") = 0);
  m.def("gguf_moe_down", &gguf_moe_down, py::arg("W"), py::arg("type"), py::arg("I"), py::arg("act"), py::arg("ids"),
        py::arg("wts"), py::arg("x"), py::arg("J"), py::arg("e_base") = 0, py::arg("e_count") = 0);
  m.def("gdn_prefill", &gdn_prefill);
  m.def("gemv_router", &gemv_router);
  m.def("gemv_argmax", &gemv_argmax);
  m.def("gemv_argmax_tp", &gemv_argmax_tp);
  m.def("gemm_grouped", &gemm_grouped);
}
