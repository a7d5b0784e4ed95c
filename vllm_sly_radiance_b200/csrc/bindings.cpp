// Python bindings of the sm_100a kernel library.
#include <torch/extension.h>

#include <vector>

namespace rad {
void mxfp4_gemm(torch::Tensor a, torch::Tensor a_scale, torch::Tensor wp, torch::Tensor sf,
                torch::Tensor out, int64_t splits_override, torch::Tensor status);
void mxfp4_grouped_gemm(torch::Tensor a, torch::Tensor a_scale, torch::Tensor wp, torch::Tensor sf,
                        torch::Tensor out, torch::Tensor items, int64_t bn, int64_t n_per_group,
                        torch::Tensor status);
void add_rms_quant(torch::Tensor x, torch::Tensor residual, torch::Tensor weight,
                   torch::Tensor res_out, torch::Tensor q, torch::Tensor scale, torch::Tensor nout,
                   double eps);
void silu_mul_quant(torch::Tensor gate_up, torch::Tensor q, torch::Tensor scale);
void gdn_norm_quant(torch::Tensor o, torch::Tensor z, torch::Tensor weight, int64_t head_dim,
                    double eps, torch::Tensor q, torch::Tensor scale, torch::Tensor nout);
void gate_mul_quant(torch::Tensor a, torch::Tensor gate, int64_t head_dim, int64_t gate_head_stride,
                    torch::Tensor q, torch::Tensor scale, torch::Tensor nout);
void quant_fp8_rows(torch::Tensor x, torch::Tensor q, torch::Tensor scale);
void gdn_conv(torch::Tensor x, torch::Tensor w, torch::Tensor conv_state, torch::Tensor qsl,
              torch::Tensor slots, torch::Tensor has_init, torch::Tensor tok_seq, int64_t qk_dim,
              int64_t head_dim, torch::Tensor y, double eps, bool update_state);
void gdn_conv_state_update(torch::Tensor x, torch::Tensor conv_state, torch::Tensor qsl,
                           torch::Tensor slots, torch::Tensor has_init, torch::Tensor commit_len);
void gdn_recurrent(torch::Tensor y, torch::Tensor ba, torch::Tensor A_log, torch::Tensor dt_bias,
                   torch::Tensor state, torch::Tensor qsl, torch::Tensor slots,
                   torch::Tensor has_init, torch::Tensor commit_len, int64_t Hk, double scale,
                   torch::Tensor out, bool write_out);
void gdn_decode_fused(torch::Tensor x, int64_t ba_off, torch::Tensor conv_w,
                      torch::Tensor conv_state, torch::Tensor A_log, torch::Tensor dt_bias,
                      torch::Tensor state, torch::Tensor slots, torch::Tensor has_init, int64_t Hk,
                      double scale, double eps, torch::Tensor out, int64_t split, int64_t z_off,
                      torch::Tensor norm_w, double norm_eps, torch::Tensor nout, torch::Tensor ws,
                      torch::Tensor q, torch::Tensor q_scale);
void gdn_chunked(torch::Tensor y, torch::Tensor ba, torch::Tensor A_log, torch::Tensor dt_bias,
                 torch::Tensor state, torch::Tensor qsl, torch::Tensor slots,
                 torch::Tensor has_init, int64_t Hk, double scale, torch::Tensor out,
                 int64_t split_override);
int64_t gdn_chunked2_ws_bytes(int64_t T, int64_t B, int64_t Hv);
void gdn_chunked2(torch::Tensor y, torch::Tensor ba, torch::Tensor A_log, torch::Tensor dt_bias,
                  torch::Tensor state, torch::Tensor qsl, torch::Tensor slots,
                  torch::Tensor has_init, int64_t Hk, double scale, torch::Tensor out,
                  torch::Tensor ws, int64_t split_override);
void qkv_prologue(torch::Tensor qkv, int64_t q_head_stride, int64_t k_off, int64_t v_off,
                  torch::Tensor positions, torch::Tensor qn_w, torch::Tensor kn_w,
                  torch::Tensor cos_sin, int64_t rot, int64_t Hq, int64_t Hkv, double eps,
                  torch::Tensor q_out, torch::Tensor k_cache, torch::Tensor v_cache,
                  torch::Tensor slot_mapping);
void paged_attention(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache,
                     torch::Tensor block_tables, torch::Tensor seq_lens, torch::Tensor qsl,
                     torch::Tensor tile_seq, torch::Tensor tile_row0, double scale, bool causal,
                     int64_t window, int64_t num_splits, torch::Tensor part_o,
                     torch::Tensor part_ml, torch::Tensor out, torch::Tensor counters,
                     bool decode, torch::Tensor gate, int64_t gate_head_stride,
                     torch::Tensor gate_cnt, torch::Tensor gq, torch::Tensor gq_scale);
int64_t mxfp4_gemm_push(torch::Tensor a, torch::Tensor a_scale, torch::Tensor wp, torch::Tensor sf,
                        std::vector<int64_t> peers, int64_t rank, int64_t half_words,
                        torch::Tensor status);
int64_t push_buffer_bytes(int64_t world, int64_t mmax, int64_t H);
void mxfp4_gemv(torch::Tensor a, torch::Tensor a_scale, torch::Tensor wp, torch::Tensor sf,
                torch::Tensor out, torch::Tensor ws, int64_t ctas_per_sm, int64_t fin_mode,
                torch::Tensor res, torch::Tensor w, torch::Tensor res_out, torch::Tensor q,
                torch::Tensor scale, double eps, torch::Tensor status);
int64_t mxfp4_gemv_push(torch::Tensor a, torch::Tensor a_scale, torch::Tensor wp, torch::Tensor sf,
                        torch::Tensor ws, int64_t ctas_per_sm, std::vector<int64_t> peers,
                        int64_t rank, int64_t half_words, torch::Tensor status);
int64_t mxfp4_gemm_rs(torch::Tensor a, torch::Tensor a_scale, torch::Tensor wp, torch::Tensor sf,
                      std::vector<int64_t> peers, int64_t rank, int64_t per, torch::Tensor status);
int64_t ts_header_bytes();
int64_t ts_buffer_bytes(int64_t mmax, int64_t H);
int64_t ts_rows_per_rank(int64_t M, int64_t world);
void ts_allreduce(std::vector<int64_t> peers, int64_t rank, int64_t M, int64_t H,
                  int64_t buf_bytes, torch::Tensor x, bool pushed, int64_t expected,
                  torch::Tensor out, torch::Tensor residual, torch::Tensor weight, double eps,
                  torch::Tensor res_out, torch::Tensor q, torch::Tensor scale,
                  torch::Tensor status);
void embed_gather(torch::Tensor codes, torch::Tensor scales, torch::Tensor ids, int64_t bits,
                  torch::Tensor out);
void mxfp4_gemm_fin(torch::Tensor a, torch::Tensor a_scale, torch::Tensor wp, torch::Tensor sf,
                    torch::Tensor out, int64_t fin_mode, torch::Tensor res, torch::Tensor w,
                    torch::Tensor res_out, torch::Tensor q, torch::Tensor scale, double eps,
                    torch::Tensor ws, torch::Tensor status);
void kv4_to_e4m3_pages(torch::Tensor k4, torch::Tensor v4, torch::Tensor block_tables,
                       torch::Tensor seq_lens, torch::Tensor k8, torch::Tensor v8,
                       torch::Tensor bt_out);
void fmha_prefill(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache,
                  torch::Tensor block_tables, torch::Tensor seq_lens, torch::Tensor qsl,
                  torch::Tensor tile_seq, torch::Tensor tile_row0, double scale, torch::Tensor out,
                  torch::Tensor status);
void mxfp4_gemm_act(int64_t mode, torch::Tensor x, torch::Tensor res, torch::Tensor w,
                    torch::Tensor res_out, double eps, torch::Tensor wp, torch::Tensor sf,
                    torch::Tensor out, torch::Tensor status);
void push_allreduce_recv(std::vector<int64_t> peers, int64_t rank, int64_t M, int64_t H,
                         int64_t half_words, torch::Tensor out, torch::Tensor residual,
                         torch::Tensor weight, double eps, torch::Tensor res_out, torch::Tensor q,
                         torch::Tensor scale, int64_t num_blocks, torch::Tensor status);
void rejection_sample_cuda(torch::Tensor draft, torch::Tensor t_ids, torch::Tensor t_probs,
                           torch::Tensor d_ids, torch::Tensor d_probs, torch::Tensor greedy,
                           torch::Tensor seq_lens, torch::Tensor forced, torch::Tensor seeds,
                           int64_t kind, double delta, int64_t fade_start, int64_t fade_end,
                           double cap_r, double escape, double theta, torch::Tensor out,
                           torch::Tensor n_acc);
void lookup_draft_cuda(torch::Tensor hist, torch::Tensor rows, torch::Tensor len, int64_t k,
                       int64_t max_ngram, int64_t min_ngram, torch::Tensor out,
                       torch::Tensor n_out);
void w4a16_gemv(torch::Tensor x, torch::Tensor wq, torch::Tensor sz, torch::Tensor out,
                torch::Tensor status);
void w4a16_dequant(torch::Tensor wq, torch::Tensor sz, int64_t n0, torch::Tensor out);
void segment_copy(torch::Tensor table, torch::Tensor offs, torch::Tensor idx, torch::Tensor stage,
                  int64_t item_bytes, bool gather);
int64_t ep_buffer_bytes(int64_t world, int64_t maxr, int64_t H, int64_t K, int64_t maxt);
std::vector<int64_t> ep_offsets(int64_t world, int64_t maxr, int64_t H, int64_t K, int64_t maxt);
void ep_dispatch(std::vector<int64_t> peers, int64_t rank, int64_t maxr, int64_t El,
                 int64_t maxt, torch::Tensor q, torch::Tensor s, torch::Tensor ids,
                 torch::Tensor status);
void ep_items(std::vector<int64_t> peers, int64_t rank, int64_t maxr, int64_t H, int64_t K,
              int64_t El, int64_t maxt, int64_t bn, torch::Tensor items, torch::Tensor status);
void ep_silu_items(torch::Tensor gu, torch::Tensor items, int64_t bn, torch::Tensor q,
                   torch::Tensor scale);
void ep_combine(std::vector<int64_t> peers, int64_t rank, int64_t maxr, int64_t El,
                int64_t maxt, torch::Tensor y, torch::Tensor w, torch::Tensor out,
                torch::Tensor status);
void dflash_conv(torch::Tensor h, torch::Tensor delta, torch::Tensor base, int64_t G,
                 int64_t block, torch::Tensor out);
void dflash_walk(torch::Tensor unary, torch::Tensor cand, torch::Tensor anchors, torch::Tensor hp,
                 torch::Tensor pred, torch::Tensor succ, torch::Tensor temps, torch::Tensor seeds,
                 torch::Tensor drafts, torch::Tensor winp, torch::Tensor status);
void argmax_rows(torch::Tensor x, torch::Tensor out_ids, torch::Tensor out_vals,
                 torch::Tensor workspace);
void topk_window(torch::Tensor x, torch::Tensor out_vals, torch::Tensor out_ids,
                 torch::Tensor workspace, torch::Tensor temperature, torch::Tensor top_k,
                 torch::Tensor top_p, torch::Tensor min_p, torch::Tensor seeds, int64_t step,
                 torch::Tensor out_tok, torch::Tensor probs_out);
void sample_from_topk(torch::Tensor vals, torch::Tensor ids, torch::Tensor temperature,
                      torch::Tensor top_k, torch::Tensor top_p, torch::Tensor min_p,
                      torch::Tensor seeds, int64_t step, torch::Tensor out,
                      torch::Tensor out_logprob, torch::Tensor probs_out);
torch::Tensor ipc_handle(torch::Tensor buf);
int64_t ipc_open(torch::Tensor handle);
void ipc_close(int64_t ptr);
int64_t symm_header_bytes();
void allreduce_oneshot(std::vector<int64_t> peers, int64_t rank, torch::Tensor inp,
                       int64_t slot_bytes, torch::Tensor out, torch::Tensor residual,
                       torch::Tensor weight, double eps, torch::Tensor res_out, torch::Tensor q,
                       torch::Tensor scale, int64_t num_blocks, torch::Tensor status);
}  // namespace rad

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "sm_100a kernels of the radiance B200 serving engine";
  m.def("mxfp4_gemm", &rad::mxfp4_gemm, "MXFP4 W4A8 block-scaled tcgen05 GEMM");
  m.def("mxfp4_grouped_gemm", &rad::mxfp4_grouped_gemm, "grouped (MoE) MXFP4 W4A8 tcgen05 GEMM");
  m.def("add_rms_quant", &rad::add_rms_quant, "fused residual add + Gemma RMSNorm (+ e4m3 quant)");
  m.def("silu_mul_quant", &rad::silu_mul_quant, "SiLU(gate)*up + e4m3 quant");
  m.def("gdn_norm_quant", &rad::gdn_norm_quant, "GDN gated RMSNorm (+ e4m3 quant)");
  m.def("gate_mul_quant", &rad::gate_mul_quant, "attention sigmoid gate (+ e4m3 quant)");
  m.def("quant_fp8_rows", &rad::quant_fp8_rows, "per-row e4m3 quant");
  m.def("gdn_conv", &rad::gdn_conv, "GDN varlen causal conv1d + SiLU + q/k L2 norm");
  m.def("gdn_conv_state_update", &rad::gdn_conv_state_update, "GDN conv state write-back");
  m.def("gdn_recurrent", &rad::gdn_recurrent, "GDN varlen recurrent delta rule");
  m.def("qkv_prologue", &rad::qkv_prologue, "QK RMSNorm + RoPE + paged KV write");
  m.def("paged_attention", &rad::paged_attention, "varlen paged attention (split-KV)");
  m.def("rejection_sample", &rad::rejection_sample_cuda,
        "speculative acceptance (Leviathan / Cactus / NSD / greedy / forced), one warp per request");
  m.def("lookup_draft", &rad::lookup_draft_cuda, "prompt-lookup drafts: longest suffix match");
  m.def("w4a16_gemv", &rad::w4a16_gemv, "int4 (g128) x bf16 linear for up to 8 rows");
  m.def("w4a16_dequant", &rad::w4a16_dequant, "int4 (g128) weight rows -> bf16");
  m.def("segment_copy", &rad::segment_copy, "cache segments <-> contiguous staging (KV offload)");
  m.def("ep_buffer_bytes", &rad::ep_buffer_bytes, "expert-parallel peer buffer size");
  m.def("ep_offsets", &rad::ep_offsets, "expert-parallel buffer offsets (rows, scales, meta, combine)");
  m.def("ep_dispatch", &rad::ep_dispatch, "MoE rows -> expert owners' receive buffers (NVLink)");
  m.def("ep_items", &rad::ep_items, "wait for every source; grouped GEMM work table in place");
  m.def("ep_silu_items", &rad::ep_silu_items, "SiLU*mul + e4m3 for the work table's rows");
  m.def("ep_combine", &rad::ep_combine, "expert outputs -> sources; weighted sum over top-k");
  m.def("dflash_walk", &rad::dflash_walk, "DFlash2 candidate path walk (one warp per request)");
  m.def("dflash_conv", &rad::dflash_conv, "DFlash2 block-causal grouped depthwise conv");
  m.def("gdn_chunked", &rad::gdn_chunked, "chunked (64-token) gated delta rule for prefill");
  m.def("gdn_chunked2_ws_bytes", &rad::gdn_chunked2_ws_bytes, "two-phase chunk scan workspace");
  m.def("gdn_chunked2", &rad::gdn_chunked2,
        "two-phase chunked gated delta rule: chunk-parallel solve, then the state scan");
  m.def("gdn_decode_fused", &rad::gdn_decode_fused,
        "one-token GDN step: conv update + SiLU + q/k L2 norm + gates + delta rule");
  m.def("mxfp4_gemm_push", &rad::mxfp4_gemm_push,
        "row-parallel W4A8 GEMM that pushes its tiles into every peer's receive buffer");
  m.def("push_buffer_bytes", &rad::push_buffer_bytes, "size of a GEMM-push receive buffer");
  m.def("mxfp4_gemv", &rad::mxfp4_gemv,
        "persistent stream-K decode W4A8 GEMM (<= 16 rows) with an optional fused row finisher");
  m.def("mxfp4_gemv_push", &rad::mxfp4_gemv_push,
        "persistent decode W4A8 GEMM pushing its tiles into every rank's receive buffer");
  m.def("mxfp4_gemm_rs", &rad::mxfp4_gemm_rs,
        "row-parallel W4A8 GEMM pushing its rows into their owners' two-shot slots");
  m.def("ts_header_bytes", &rad::ts_header_bytes, "two-shot all-reduce buffer header bytes");
  m.def("ts_buffer_bytes", &rad::ts_buffer_bytes, "two-shot all-reduce buffer bytes");
  m.def("ts_rows_per_rank", &rad::ts_rows_per_rank, "rows owned per rank by the two-shot all-reduce");
  m.def("ts_allreduce", &rad::ts_allreduce,
        "two-shot NVLink all-reduce (+ residual add + RMSNorm + e4m3) for prefill-sized messages");
  m.def("embed_gather", &rad::embed_gather, "int8 / int4-g128 embedding lookup into bf16 rows");
  m.def("mxfp4_gemm_fin", &rad::mxfp4_gemm_fin,
        "decode W4A8 GEMM whose last CTA also runs the next linear's producer over the rows");
  m.def("kv4_to_e4m3_pages", &rad::kv4_to_e4m3_pages,
        "dequantise the 4-bit KV pages a prefill chunk reaches into compact e4m3 pages");
  m.def("fmha_prefill", &rad::fmha_prefill,
        "causal prefill attention on tcgen05 (e4m3 QK and PV, TMEM accumulators, paged fp8 KV)");
  m.def("mxfp4_gemm_act", &rad::mxfp4_gemm_act,
        "decode W4A8 GEMM with its producer fused in (1: add + RMSNorm + e4m3, 2: SiLU*mul + e4m3)");
  m.def("push_allreduce_recv", &rad::push_allreduce_recv,
        "receiving half of the GEMM-fused all-reduce (+ add / RMSNorm / e4m3 quant)");
  m.def("ipc_handle", &rad::ipc_handle, "CUDA IPC handle of a device buffer");
  m.def("ipc_open", &rad::ipc_open, "open a peer's IPC handle -> device pointer");
  m.def("ipc_close", &rad::ipc_close, "close an opened IPC mapping");
  m.def("symm_header_bytes", &rad::symm_header_bytes, "flag/counter header size of a symmetric buffer");
  m.def("allreduce_oneshot", &rad::allreduce_oneshot, "one-shot NVLink all-reduce (+ fused add/RMSNorm/quant)");
  m.def("argmax_rows", &rad::argmax_rows, "greedy argmax per row");
  m.def("sample_from_topk", &rad::sample_from_topk, "temperature/top-k/top-p/min-p sampling");
  m.def("topk_window", &rad::topk_window, "top-64 window of each row (+ optional fused draw)");
}
