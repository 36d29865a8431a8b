// Python bindings of the zeroq_b200 native extension (zeroq_b200._C).
#include <torch/extension.h>

#include <vector>

// nf4.cu
void nf4_quantize(at::Tensor x, at::Tensor packed, at::Tensor absmax, int64_t blocksize, int64_t qtype);
void nf4_dequantize(at::Tensor packed, at::Tensor absmax, at::Tensor out, int64_t n, int64_t blocksize,
                    int64_t qtype);
// gemm_sm100.cu
void gemm_bf16_tn(at::Tensor a, at::Tensor b, at::Tensor c);
void attn_fwd_tc(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor o, at::Tensor lse, bool causal,
                 double scale, c10::optional<at::Tensor> trace, bool kv_bhsd);
void attn_bwd_tc(at::Tensor dout, at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor o,
                 at::Tensor lse, at::Tensor dq, at::Tensor dk, at::Tensor dv, bool causal,
                 double scale, c10::optional<at::Tensor> trace, c10::optional<at::Tensor> rope_cs);
void gemm_nf4(at::Tensor a, at::Tensor packed, at::Tensor absmax, int64_t rows, int64_t cols,
              int64_t blocksize, int64_t quant_type, bool w_is_kn, at::Tensor c,
              c10::optional<at::Tensor> a2, c10::optional<at::Tensor> b2);
void lora_pack(at::Tensor A, at::Tensor B, double scaling, at::Tensor a_pad, at::Tensor b_pad,
               c10::optional<at::Tensor> b_t);
void lora_pack_many(at::Tensor table, int64_t max_elems);
// lora_sm100.cu
void lora_down(at::Tensor p, at::Tensor w, at::Tensor u, c10::optional<at::Tensor> ut, int64_t cs,
               int64_t stages, int64_t kb);
void lora_wgrad(at::Tensor p, at::Tensor qt, int64_t nq, std::vector<int64_t> i_begin,
                std::vector<int64_t> i_count, std::vector<int64_t> q_row, std::vector<double> alpha,
                std::vector<at::Tensor> outs, int64_t gsz, int64_t rvalid, bool transposed,
                int64_t splits, int64_t stages, int64_t kb);
bool lora_vdb(at::Tensor g, at::Tensor bt, at::Tensor ut, at::Tensor v, at::Tensor vt, int64_t nqb,
              std::vector<int64_t> n_begin, std::vector<int64_t> n_count, std::vector<int64_t> q_row,
              std::vector<at::Tensor> outs, int64_t rvalid, int64_t cs, int64_t stages);
void matmul_accum_f32(at::Tensor A, at::Tensor B, at::Tensor C, double alpha, double beta);
void gemm_bf16_tn_extra(at::Tensor a, at::Tensor b, at::Tensor c, at::Tensor a2, at::Tensor b2);
void gemm_bf16_nn(at::Tensor a, at::Tensor b, at::Tensor c, c10::optional<at::Tensor> a2,
                  c10::optional<at::Tensor> b2);
std::vector<int64_t> gemm_status(int64_t device);
void set_gemm_pair_mode(int64_t mode);
void nf4_to_bf16_segments(std::vector<at::Tensor> packed, std::vector<at::Tensor> absmax,
                          std::vector<int64_t> numel, at::Tensor out, int64_t blocksize, int64_t qtype);
void nf4_to_bf16(at::Tensor packed, at::Tensor absmax, at::Tensor out, int64_t rows, int64_t cols,
                 int64_t blocksize, int64_t qtype, bool transpose);
// elementwise.cu
void add_rmsnorm_fwd(at::Tensor h, c10::optional<at::Tensor> d, at::Tensor w, at::Tensor hout,
                     at::Tensor y, at::Tensor rstd, double eps);
void rmsnorm_bwd(at::Tensor gy, at::Tensor x, at::Tensor w, at::Tensor rstd,
                 c10::optional<at::Tensor> gh, at::Tensor dx, at::Tensor dw_part);
void colsum_accum(at::Tensor part, at::Tensor out);
void rope(at::Tensor x, at::Tensor out, at::Tensor cs, double sign);
void rope_into(at::Tensor x, at::Tensor out, at::Tensor cs, double sign);
void rope_into2(at::Tensor x1, at::Tensor out1, at::Tensor x2, at::Tensor out2, at::Tensor cs, double sign);
void gelu_fwd(at::Tensor x, at::Tensor y);
void gelu_cdf_pdf(at::Tensor x, at::Tensor cdf, at::Tensor pdf);
void gelu_bwd(at::Tensor g, at::Tensor x, at::Tensor dx);
void swiglu_fwd(at::Tensor gate, at::Tensor up, at::Tensor y);
void swiglu_bwd(at::Tensor g, at::Tensor gate, at::Tensor up, at::Tensor dgate, at::Tensor dup);
void ce_fwd(at::Tensor logits, at::Tensor targets, at::Tensor loss, at::Tensor lse,
            c10::optional<at::Tensor> count, int64_t vocab, int64_t ignore_index, int64_t col0,
            int64_t vocab_total);
void ce_bwd(at::Tensor logits, at::Tensor targets, at::Tensor lse, at::Tensor scale, int64_t vocab,
            int64_t ignore_index, int64_t col0, int64_t vocab_total);
void adamw_step(at::Tensor p, at::Tensor g, at::Tensor m, at::Tensor v, c10::optional<at::Tensor> pbf16,
                double lr, double b1, double b2, double eps, double wd, double bc1, double bc2,
                double gscale, c10::optional<at::Tensor> bc, c10::optional<at::Tensor> clip_sq,
                double max_norm);
void opt_tick(at::Tensor clk, at::Tensor bc, double b1, double b2, bool bump_epoch);
void lion_step(at::Tensor master, at::Tensor grad, at::Tensor mom, double lr, double b1, double b2,
               double wd, int64_t seed);
// p2p.cu
std::vector<int64_t> peer_alloc(int64_t bytes);
at::Tensor peer_handle(int64_t ptr);
int64_t peer_open(at::Tensor handle);
void peer_close(int64_t ptr);
void peer_free(int64_t ptr);
at::Tensor tensor_from_ptr(int64_t ptr, int64_t numel, at::ScalarType dtype, int64_t device);
std::vector<int64_t> peer_status_read(int64_t flags_ptr);
int64_t peer_flag_words();
void rs_adamw(std::vector<int64_t> grads, std::vector<int64_t> params, std::vector<int64_t> flags,
              int64_t rank, int64_t epoch, int64_t lo, int64_t n, at::Tensor m, at::Tensor v,
              int64_t grad_is_bf16, double lr, double b1, double b2, double eps, double wd,
              double bc1, double bc2, double gscale, bool push, int64_t timeout_ms,
              c10::optional<at::Tensor> clk, c10::optional<at::Tensor> bc,
              c10::optional<at::Tensor> clip_sq, double max_norm, int64_t epoch_mul, int64_t epoch_add,
              int64_t max_ctas);
void rs_sumsq(std::vector<int64_t> grads, std::vector<int64_t> flags, int64_t rank, int64_t epoch, int64_t lo,
              int64_t n, at::Tensor sq, int64_t grad_is_bf16, double gscale, int64_t timeout_ms,
              c10::optional<at::Tensor> clk, int64_t epoch_mul, int64_t epoch_add);
void plan_gather(std::vector<int64_t> src, std::vector<int64_t> flags, int64_t rank, int64_t epoch,
                 std::vector<int64_t> offsets, std::vector<int64_t> lengths, at::Tensor out,
                 int64_t timeout_ms);
void ag_gemm_nf4(at::Tensor a, std::vector<int64_t> psrc, std::vector<int64_t> pstarts,
                 std::vector<int64_t> asrc, std::vector<int64_t> astarts, int64_t packed_total,
                 int64_t absmax_total, int64_t rank, int64_t N, int64_t K, int64_t blocksize,
                 int64_t quant_type, at::Tensor wbuf, at::Tensor c, c10::optional<at::Tensor> a2,
                 c10::optional<at::Tensor> b2, c10::optional<at::Tensor> swiglu_g,
                 c10::optional<at::Tensor> swiglu_out);
void ag_gemm_f32(at::Tensor a, std::vector<int64_t> src, std::vector<int64_t> starts, int64_t total,
                 int64_t rank, int64_t N, int64_t K, at::Tensor wbuf, at::Tensor c,
                 c10::optional<at::Tensor> a2, c10::optional<at::Tensor> b2);
void gemm_rope(at::Tensor a, at::Tensor b, at::Tensor c, at::Tensor cs,
               c10::optional<at::Tensor> a2, c10::optional<at::Tensor> b2, int64_t ncols);
void gemm_gelu(at::Tensor a, at::Tensor b, at::Tensor c, at::Tensor aux, bool b_mn,
               c10::optional<at::Tensor> a2, c10::optional<at::Tensor> b2);
void gemm_swiglu(at::Tensor a, at::Tensor b, at::Tensor c, at::Tensor c2, at::Tensor g,
                 c10::optional<at::Tensor> u, bool b_mn, c10::optional<at::Tensor> a2,
                 c10::optional<at::Tensor> b2);
void plan_gather_dequant(std::vector<int64_t> psrc, std::vector<int64_t> pstarts,
                         std::vector<int64_t> asrc, std::vector<int64_t> astarts, int64_t rows,
                         int64_t cols, int64_t row0, int64_t blocksize, int64_t qtype, bool transpose,
                         at::Tensor out);

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "zeroq_b200 sm_100a kernels";
  m.def("nf4_quantize", &nf4_quantize);
  m.def("nf4_dequantize", &nf4_dequantize);
  m.def("gemm_bf16_tn", &gemm_bf16_tn);
  m.def("gemm_bf16_tn_extra", &gemm_bf16_tn_extra);
  m.def("gemm_bf16_nn", &gemm_bf16_nn);
  m.def("gemm_nf4", &gemm_nf4);
  m.def("attn_bwd_tc", &attn_bwd_tc, "tcgen05 attention backward", pybind11::arg("dout"),
        pybind11::arg("q"), pybind11::arg("k"), pybind11::arg("v"), pybind11::arg("o"),
        pybind11::arg("lse"), pybind11::arg("dq"), pybind11::arg("dk"), pybind11::arg("dv"),
        pybind11::arg("causal"), pybind11::arg("scale"), pybind11::arg("trace") = pybind11::none(),
        pybind11::arg("rope_cs") = pybind11::none());
  m.def("attn_fwd_tc", &attn_fwd_tc, "tcgen05 attention forward", pybind11::arg("q"),
        pybind11::arg("k"), pybind11::arg("v"), pybind11::arg("o"), pybind11::arg("lse"),
        pybind11::arg("causal"), pybind11::arg("scale"), pybind11::arg("trace") = pybind11::none(),
        pybind11::arg("kv_bhsd") = false);
  m.def("lora_pack", &lora_pack, py::arg("A"), py::arg("B"), py::arg("scaling"), py::arg("a_pad"),
        py::arg("b_pad"), py::arg("b_t") = py::none());
  m.def("lora_pack_many", &lora_pack_many, "many LoRA operand packs in one launch (a table of jobs)");
  m.def("lora_down", &lora_down, py::arg("p"), py::arg("w"), py::arg("u"), py::arg("ut") = py::none(),
        py::arg("cs") = 0, py::arg("stages") = 0, py::arg("kb") = 0);
  m.def("lora_wgrad", &lora_wgrad, py::arg("p"), py::arg("qt"), py::arg("nq"), py::arg("i_begin"),
        py::arg("i_count"), py::arg("q_row"), py::arg("alpha"), py::arg("outs"), py::arg("gsz"),
        py::arg("rvalid"), py::arg("transposed"), py::arg("splits") = 0, py::arg("stages") = 0,
        py::arg("kb") = 0);
  m.def("lora_vdb", &lora_vdb, py::arg("g"), py::arg("bt"), py::arg("ut"), py::arg("v"), py::arg("vt"),
        py::arg("nqb"), py::arg("n_begin"), py::arg("n_count"), py::arg("q_row"), py::arg("outs"),
        py::arg("rvalid"), py::arg("cs") = 0, py::arg("stages") = 0);
  m.def("matmul_accum_f32", &matmul_accum_f32);
  m.def("gemm_status", &gemm_status);
  m.def("set_gemm_pair_mode", &set_gemm_pair_mode);
  m.def("nf4_to_bf16", &nf4_to_bf16);
  m.def("nf4_to_bf16_segments", &nf4_to_bf16_segments,
        "several 4-bit weights into consecutive ranges of one bf16 buffer, one launch");
  m.def("add_rmsnorm_fwd", &add_rmsnorm_fwd);
  m.def("rmsnorm_bwd", &rmsnorm_bwd);
  m.def("colsum_accum", &colsum_accum);
  m.def("rope", &rope);
  m.def("rope_into", &rope_into);
  m.def("rope_into2", &rope_into2, "rope_into for two (x, out) pairs in one launch");
  m.def("gelu_fwd", &gelu_fwd);
  m.def("gelu_bwd", &gelu_bwd);
  m.def("gelu_cdf_pdf", &gelu_cdf_pdf);
  m.def("swiglu_fwd", &swiglu_fwd);
  m.def("swiglu_bwd", &swiglu_bwd);
  // (col0, vocab_total): the logits buffer holds vocabulary columns [col0, col0 + vocab)
  m.def("ce_fwd", &ce_fwd, py::arg("logits"), py::arg("targets"), py::arg("loss"), py::arg("lse"),
        py::arg("count"), py::arg("vocab"), py::arg("ignore_index"), py::arg("col0") = 0,
        py::arg("vocab_total") = -1);
  m.def("ce_bwd", &ce_bwd, py::arg("logits"), py::arg("targets"), py::arg("lse"), py::arg("scale"),
        py::arg("vocab"), py::arg("ignore_index"), py::arg("col0") = 0, py::arg("vocab_total") = -1);
  m.def("adamw_step", [](at::Tensor p, at::Tensor g, at::Tensor m_, at::Tensor v,
                         c10::optional<at::Tensor> pbf16, double lr, double b1, double b2, double eps,
                         double wd, double bc1, double bc2, double gscale) {
    adamw_step(p, g, m_, v, pbf16, lr, b1, b2, eps, wd, bc1, bc2, gscale, c10::nullopt, c10::nullopt, 0.0);
  });
  // bias corrections read from the device-side optimizer clock (bc, see opt_tick);
  // optional device-side gradient clipping (clip_sq = squared global norm, max_norm)
  m.def("adamw_step_dev", &adamw_step, py::arg("p"), py::arg("g"), py::arg("m"), py::arg("v"),
        py::arg("pbf16"), py::arg("lr"), py::arg("b1"), py::arg("b2"), py::arg("eps"), py::arg("wd"),
        py::arg("bc1"), py::arg("bc2"), py::arg("gscale"), py::arg("bc") = py::none(),
        py::arg("clip_sq") = py::none(), py::arg("max_norm") = 0.0);
  m.def("opt_tick", &opt_tick, "advance the device-side optimizer clock");
  m.def("lion_step", &lion_step);
  m.def("peer_alloc", &peer_alloc);
  m.def("peer_handle", &peer_handle);
  m.def("peer_open", &peer_open);
  m.def("peer_close", &peer_close);
  m.def("peer_free", &peer_free);
  m.def("tensor_from_ptr", &tensor_from_ptr);
  m.def("peer_status_read", &peer_status_read);
  m.def("peer_flag_words", &peer_flag_words);
  m.def("rs_adamw", [](std::vector<int64_t> grads, std::vector<int64_t> params, std::vector<int64_t> flags,
                       int64_t rank, int64_t epoch, int64_t lo, int64_t n, at::Tensor m_, at::Tensor v,
                       int64_t grad_is_bf16, double lr, double b1, double b2, double eps, double wd,
                       double bc1, double bc2, double gscale, bool push, int64_t timeout_ms) {
    rs_adamw(grads, params, flags, rank, epoch, lo, n, m_, v, grad_is_bf16, lr, b1, b2, eps, wd, bc1,
             bc2, gscale, push, timeout_ms, c10::nullopt, c10::nullopt, c10::nullopt, 0.0, 1, 0, 0);
  });
  // epoch and bias corrections from the device-side optimizer clock (clk, bc);
  // optional device-side gradient clipping (clip_sq, max_norm)
  m.def("rs_adamw_dev", &rs_adamw, py::arg("grads"), py::arg("params"), py::arg("flags"), py::arg("rank"),
        py::arg("epoch"), py::arg("lo"), py::arg("n"), py::arg("m"), py::arg("v"), py::arg("grad_is_bf16"),
        py::arg("lr"), py::arg("b1"), py::arg("b2"), py::arg("eps"), py::arg("wd"), py::arg("bc1"),
        py::arg("bc2"), py::arg("gscale"), py::arg("push"), py::arg("timeout_ms"),
        py::arg("clk") = py::none(), py::arg("bc") = py::none(), py::arg("clip_sq") = py::none(),
        py::arg("max_norm") = 0.0, py::arg("epoch_mul") = 1, py::arg("epoch_add") = 0,
        py::arg("max_ctas") = 0);
  m.def("rs_sumsq", &rs_sumsq, py::arg("grads"), py::arg("flags"), py::arg("rank"), py::arg("epoch"),
        py::arg("lo"), py::arg("n"), py::arg("sq"), py::arg("grad_is_bf16"), py::arg("gscale"),
        py::arg("timeout_ms"), py::arg("clk") = py::none(), py::arg("epoch_mul") = 1,
        py::arg("epoch_add") = 0);
  m.def("plan_gather", &plan_gather);
  m.def("plan_gather_dequant", &plan_gather_dequant);
  m.def("ag_gemm_f32", &ag_gemm_f32, "gather of fp32 pieces + bf16 cast + tcgen05 GEMM in one kernel",
        pybind11::arg("a"), pybind11::arg("src"), pybind11::arg("starts"), pybind11::arg("total"),
        pybind11::arg("rank"), pybind11::arg("N"), pybind11::arg("K"), pybind11::arg("wbuf"),
        pybind11::arg("c"), pybind11::arg("a2") = pybind11::none(), pybind11::arg("b2") = pybind11::none());
  m.def("gemm_rope", &gemm_rope, "tcgen05 GEMM with the rotary-embedding epilogue",
        pybind11::arg("a"), pybind11::arg("b"), pybind11::arg("c"), pybind11::arg("cs"),
        pybind11::arg("a2") = pybind11::none(), pybind11::arg("b2") = pybind11::none(),
        pybind11::arg("ncols") = -1);
  m.def("gemm_gelu", &gemm_gelu, "tcgen05 GEMM with the GELU output / GELU-gradient epilogue",
        pybind11::arg("a"), pybind11::arg("b"), pybind11::arg("c"), pybind11::arg("aux"),
        pybind11::arg("b_mn"), pybind11::arg("a2") = pybind11::none(),
        pybind11::arg("b2") = pybind11::none());
  m.def("ag_gemm_nf4", &ag_gemm_nf4, "gather + dequantise + tcgen05 GEMM in one kernel",
        pybind11::arg("a"), pybind11::arg("psrc"), pybind11::arg("pstarts"), pybind11::arg("asrc"),
        pybind11::arg("astarts"), pybind11::arg("packed_total"), pybind11::arg("absmax_total"),
        pybind11::arg("rank"), pybind11::arg("N"), pybind11::arg("K"), pybind11::arg("blocksize"),
        pybind11::arg("quant_type"), pybind11::arg("wbuf"), pybind11::arg("c"),
        pybind11::arg("a2") = pybind11::none(), pybind11::arg("b2") = pybind11::none(),
        pybind11::arg("swiglu_g") = pybind11::none(), pybind11::arg("swiglu_out") = pybind11::none());
  m.def("gemm_swiglu", &gemm_swiglu,
        "tcgen05 GEMM with the SwiGLU output (b_mn=false) / SwiGLU-gradient (b_mn=true) epilogue",
        pybind11::arg("a"), pybind11::arg("b"), pybind11::arg("c"), pybind11::arg("c2"),
        pybind11::arg("g"), pybind11::arg("u"), pybind11::arg("b_mn"),
        pybind11::arg("a2") = pybind11::none(), pybind11::arg("b2") = pybind11::none());
}
