/*
 * oracle.h — CPU oracle for the Qwen3-ASR text-decoder step.  TEST INFRASTRUCTURE ONLY.
 *
 * A C++ restatement of the reference crate's host decoder `CpuTextDecoder`
 * (eclipse005/qwen3-asr-wgpu v0.3.0, src/cpu_decoder.rs:11-585), its INT8 dequant
 * (src/weights.rs:372-385) and its MRoPE tables (src/mrope.rs:5-80 rounded as
 * src/inference.rs:1037-1047).  Only tests/, __graft_entry__.smoke() and bench.py's
 * CPU-baseline / reference legs may load it, and only as the checker or the timed CPU
 * baseline; the B200 library never links or calls it.
 *
 * Pinning: the reference is Rust (no cargo/rustc here) and cannot be built, so this
 * restatement is pinned by the reference's own known-answer tests (dequant values,
 * int8 word layout, fused scale order, mrope quota map, gemm-vs-naive tolerance) —
 * see tests/test_oracle_kats.py.  Decode (rows == 1) is restated operation for
 * operation.  Prefill (rows >= 2) goes through the third-party `gemm 0.18.2` crate in
 * the reference, whose summation order is not restated: that boundary is pinned only
 * to |Δ| < 1e-3 (src/cpu_decoder.rs:591-617), i.e. "parity unpinned" at bit level.
 */
#ifndef QASR_ORACLE_H
#define QASR_ORACLE_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
  int32_t vocab_size, hidden_size, intermediate_size, num_hidden_layers;
  int32_t num_attention_heads, num_key_value_heads, head_dim;
  float rms_norm_eps;
} oracle_cfg; /* TextConfig, src/decoder.rs:166-175 */

typedef struct oracle_model oracle_model;
typedef struct oracle_seq oracle_seq;

oracle_model* oracle_model_create(const oracle_cfg* cfg);
void oracle_model_destroy(oracle_model* m);
int oracle_load_embed(oracle_model* m, const uint16_t* embed, const uint16_t* final_norm);
/* weight_format 0: f16 linears; 1: int8 linears + F32 per-row scales (the reference's
 * PackedInt8 / dequant_i8 format).  Order q,k,v,o,gate,up,down. */
int oracle_load_layer(oracle_model* m, int layer, int weight_format, const void* const lin[7],
                      const float* const scales[7], const uint16_t* iln, const uint16_t* pln,
                      const uint16_t* qn, const uint16_t* kn);
int oracle_set_rope_tables(oracle_model* m, const uint16_t* cos, const uint16_t* sin,
                           int positions);

oracle_seq* oracle_seq_create(oracle_model* m, int max_seq);
void oracle_seq_destroy(oracle_seq* s);
/* CpuTextDecoder::prefill / step; logits (f32 [vocab]) may be NULL. */
int oracle_prefill(oracle_seq* s, const uint16_t* hidden, int rows, int kv_start, int32_t* token,
                   float* logits);
int oracle_step(oracle_seq* s, int32_t* token, float* logits);
void oracle_set_last_token(oracle_seq* s, int32_t tok);
int oracle_pos(const oracle_seq* s);
void oracle_set_pos(oracle_seq* s, int pos);
/* Summation order of every f32 dot product (process-wide): 0 = the reference's, 1 = each
 * accumulator over k backwards -- the same sums in another valid order, to measure how much
 * the model's logits move with the order of f32 additions. */
void oracle_set_sum_order(int order);
/* Copy the f16 hidden state rows of the last forward (rows x hidden). */
int oracle_last_hidden(const oracle_seq* s, uint16_t* out, int rows);
/* K / V cache rows (f16-rounded values as f32) of one layer and kv head. */
int oracle_kv_rows(const oracle_seq* s, int layer, int kv_head, int pos0, int n, float* k,
                   float* v);

/* ---- operation-level restatements (kernel parity and known-answer tests) ---- */
uint16_t oracle_f32_to_f16(float f);
float oracle_f16_to_f32(uint16_t h);
void oracle_dequant_i8(const int8_t* q, const float* scale, int rows, int cols, uint16_t* out);
/* Mat::batch_dot with rows == 1 (dot_transposed, 4 accumulators): y = f16(W x). */
void oracle_gemv_f16(const uint16_t* w, int n_out, int cols, const uint16_t* x, uint16_t* y);
/* Mat::batch_dot_acc with rows == 1: h = f16(f32(h) + W x). */
void oracle_gemv_acc_f16(const uint16_t* w, int n_out, int cols, const uint16_t* x, uint16_t* h);
/* The oracle's rows >= 2 matmul (standing in for gemm_row_major): out[m, n] = x . w^T. */
void oracle_matmul_rows(const float* x, const float* w, int m, int n, int k, float* out);
/* gemm_row_major restated as the naive triple loop the reference test compares to. */
void oracle_gemm_naive(float* out, const float* x, const float* w, int m, int n, int k);
void oracle_rms_norm_row(const uint16_t* x, const float* w, int n, float eps, uint16_t* out);
void oracle_norm_rope_head(const uint16_t* raw, const float* nw, int hd, float eps,
                           const float* cos_row, const float* sin_row, uint16_t* out);
/* attention() for one (row, head): q f16 [hd], k/v f32 [valid, hd] -> f16 out [hd]. */
void oracle_attention_head(const uint16_t* q, const float* k, const float* v, int valid, int hd,
                           uint16_t* out);
int oracle_argmax(const float* logits, int n);
void oracle_build_dim_map(const int* section, int nsection, int half, int interleaved, int* out);
void oracle_mrope_cos_sin_f32(int positions, int head_dim, double theta, const int* section,
                              int nsection, int interleaved, float* cos, float* sin);

#ifdef __cplusplus
}
#endif
#endif
