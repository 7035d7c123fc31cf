/*
 * oracle.h — CPU restatement of the reference's quantized-Llama decode path.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the parity checker for the CUDA
 * path in arm_ai_b200/. Only tests/, __graft_entry__.smoke() and bench.py's
 * CPU-baseline leg may load it. The product never links or calls it.
 *
 * What it restates:
 *   - candle-core 0.8.4 k-quants (generic, non-SIMD paths — the ones an
 *     x86_64 build without target-cpu=native runs): BlockQ8K::from_float,
 *     BlockQ4K/BlockQ5K/BlockQ6K vec_dot_unopt and to_float, the legacy
 *     BlockQ4_0/BlockQ5_0/BlockQ8_0 (to_float, vec_dot with a Q8_0 lhs) and
 *     BlockQ8_0::from_float, and the CPU QMatMul driver (quantise each lhs
 *     row to the weight's VecDotType — Q8_K or Q8_0 — one vec_dot per output
 *     column). The crate is pinned in the reference at
 *     native/arm_ai_nif/Cargo.lock:175-178 (candle-core 0.8.4); it is not
 *     vendored under the reference tree.
 *   - candle-transformers 0.8.4 models::quantized_llama::ModelWeights
 *     (from_gguf + forward), candle-nn 0.8.4 rms_norm / softmax_last_dim /
 *     rope_i, and the greedy loop of native/arm_ai_nif/src/llama_candle.rs:69-176.
 *   - The reference's own x86 scalar primitive kernels in
 *     native/arm_ai_nif/src/shape_ops.rs (file:line cited per function in
 *     oracle.c).
 *
 * Parity status: the Q4_K / Q5_K / Q6_K / Q4_0 / Q5_0 / Q8_0 block layouts
 * and dequantisation, and Q8_0 quantisation, are pinned against gguf-py
 * 0.19.0's independent dequantize() / quantize(); the GGUF container is
 * read by gguf-py's GGUFReader. Q8_K quantisation rounding, the vec_dot
 * combine order and the forward-pass details are restated from candle's
 * published source and are NOT pinned by any reference-run output (no Rust
 * toolchain or crate sources exist here): parity for those is "unpinned".
 */
#ifndef ARMAI_ORACLE_H
#define ARMAI_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* GGML tensor type ids (GGUF spec). */
enum { ORC_F32 = 0, ORC_F16 = 1, ORC_Q4_0 = 2, ORC_Q5_0 = 6, ORC_Q8_0 = 8, ORC_Q4_K = 12, ORC_Q5_K = 13,
       ORC_Q6_K = 14 };

#define ORC_QK_K 256

typedef struct {
  uint16_t d;
  uint16_t dmin;
  uint8_t scales[12];
  uint8_t qs[128];
} orc_block_q4k; /* 144 bytes */

typedef struct {
  uint8_t ql[128];
  uint8_t qh[64];
  int8_t scales[16];
  uint16_t d;
} orc_block_q6k; /* 210 bytes */

typedef struct {
  float d;
  int8_t qs[256];
  int16_t bsums[16];
} orc_block_q8k; /* 292 bytes */

typedef struct {
  uint16_t d;
  uint16_t dmin;
  uint8_t scales[12];
  uint8_t qh[32];
  uint8_t qs[128];
} orc_block_q5k; /* 176 bytes */

/* 32-value blocks of the legacy types; their matmuls quantise the lhs to Q8_0. */
#define ORC_QK8_0 32
typedef struct {
  uint16_t d;
  uint8_t qs[16];
} orc_block_q4_0; /* 18 bytes */

typedef struct {
  uint16_t d;
  uint8_t qh[4];
  uint8_t qs[16];
} orc_block_q5_0; /* 22 bytes */

typedef struct {
  uint16_t d;
  int8_t qs[32];
} orc_block_q8_0; /* 34 bytes */

/* ---- k-quant block math (candle-core 0.8.4 k_quants.rs) ---- */
float orc_f16_to_f32(uint16_t h);
int orc_quantize_row_q8k(const float* x, int64_t k, orc_block_q8k* y);
float orc_vec_dot_q4k_q8k(int64_t n, const orc_block_q4k* x, const orc_block_q8k* y);
float orc_vec_dot_q6k_q8k(int64_t n, const orc_block_q6k* x, const orc_block_q8k* y);
float orc_vec_dot_q5k_q8k(int64_t n, const orc_block_q5k* x, const orc_block_q8k* y);
uint16_t orc_f32_to_f16(float f);
int orc_quantize_row_q8_0(const float* x, int64_t k, orc_block_q8_0* y);
float orc_vec_dot_q4_0_q8_0(int64_t n, const orc_block_q4_0* x, const orc_block_q8_0* y);
float orc_vec_dot_q5_0_q8_0(int64_t n, const orc_block_q5_0* x, const orc_block_q8_0* y);
float orc_vec_dot_q8_0_q8_0(int64_t n, const orc_block_q8_0* x, const orc_block_q8_0* y);
/* to_float of one row of k values of any type above (F32 and F16 too); -1 if unsupported. */
int orc_dequant_row(int type, const void* row, int64_t k, float* y);
void orc_dequant_row_q4k(const orc_block_q4k* x, int64_t k, float* y);
void orc_dequant_row_q6k(const orc_block_q6k* x, int64_t k, float* y);
/* Integer per-super-block dot products (the exact integers candle combines
 * in f32): isum = sum_j scale_j * <q_j, q8_j>, msum = sum_j min_j * bsums_j. */
void orc_q4k_block_ints(const orc_block_q4k* x, const orc_block_q8k* y, int64_t nb,
                        int32_t* isum, int32_t* msum);
void orc_q6k_block_ints(const orc_block_q6k* x, const orc_block_q8k* y, int64_t nb,
                        int32_t* isum);
/* QMatMul: out[m][n] = vec_dot(w row n, Q8_K(x row m)). */
int orc_qmatmul(const void* w, int wtype, int64_t n, int64_t k, const float* x, int64_t m,
                float* out);

/* ---- quantized_llama (candle-transformers 0.8.4) ---- */
typedef struct orc_llama orc_llama;
orc_llama* orc_llama_new(int n_layer, int n_embd, int n_head, int n_head_kv, int rope_dim,
                         int n_vocab, int n_ff, float eps, float rope_base, int max_seq);
int orc_llama_set_tensor(orc_llama* m, const char* role, int layer, const void* data,
                         int ggml_type, int64_t rows, int64_t cols);
int orc_llama_finalize(orc_llama* m);
/* Store K/V cache entries rounded to IEEE binary16 (round to nearest even)
 * and read them back as f32: the f16 KV cache of the long-context configuration. candle's
 * quantized_llama keeps an f32 cache; this mode is off by default. */
void orc_llama_set_kv_f16(orc_llama* m, int on);
void orc_llama_free(orc_llama* m);
/* ModelWeights::forward(tokens[1,n], index_pos) -> logits of last position. */
int orc_llama_forward(orc_llama* m, const uint32_t* tokens, int n, int index_pos,
                      float* logits);
/* llama_candle.rs generate_greedy_with, including the timers. */
int orc_llama_generate(orc_llama* m, const uint32_t* prompt, int n_prompt, int max_new,
                       const uint32_t* stop, int n_stop, uint32_t* out, int* n_out,
                       uint64_t* prefill_us, uint64_t* decode_us);
uint32_t orc_argmax(const float* v, int64_t n);
const char* orc_last_error(void);
void orc_set_threads(int n);
/* Test perturbation, not the reference's arithmetic: v = 1 accumulates
 * rms_norm's sum of squares in f64, v = 2 / 3 moves its rms scale one ulp
 * up / down, v = 4 sums the squares in reverse order.
 * The change either causes in a model's logits is the model's sensitivity to
 * last-bit f32 differences (activation quantisation rounds a value the other
 * way once in a while and the model carries that forward); parity tests size
 * their bound by it. v = 0 is the restatement of candle. Process-wide. */
void orc_set_norm_variant(int v);
int orc_get_threads(void);

/* ---- reference primitive kernels (shape_ops.rs, x86 scalar paths) ---- */
int orc_int8_matmul_f32(const int8_t* a, const int8_t* w, float act_scale, const float* w_scales,
                        int64_t m, int64_t n, int64_t k, float* out);
int orc_int8_matmul_f32_per_token(const int8_t* a, const int8_t* w, const float* act_scales,
                                  const float* w_scales, int64_t m, int64_t n, int64_t k,
                                  float* out);
int orc_int8_matmul_s32(const int8_t* a, const int8_t* w, int64_t m, int64_t n, int64_t k,
                        int32_t* out);
int orc_quantize_int8_per_token(const float* a, int64_t m, int64_t k, int8_t* q, float* scales);
int orc_int4_matmul_f32(const float* a, const uint8_t* w_packed, const float* w_scales, int64_t m,
                        int64_t n, int64_t k, float* out);
int orc_int4_matmul_q4_x_q8(const float* a, const uint8_t* w_packed, const float* w_scales,
                            int64_t n, int64_t k, float* out);
int orc_quantize_int4_q4_0(const float* w, int64_t n, int64_t k, uint8_t* packed, float* scales);
int orc_rmsnorm_f32(const float* x, const float* gamma, int64_t n_outer, int64_t inner, float eps,
                    float* out);
int orc_flash_attention_f32(const float* q, const float* k, const float* v, float scale,
                            int64_t b, int64_t h, int64_t sq, int64_t sk, int64_t d, int causal,
                            float* out);
int orc_dequant_matmul_int8_f32(const float* act, const int8_t* w, const float* scales, int64_t b,
                                int64_t m, int64_t n, int64_t k, float* out);
/* LLM helper primitives (lib.rs:147-354); lengths are the caller's to check. */
int orc_rope_f32(const float* x, const int64_t* positions, const float* inv_freq, int64_t n_rows,
                 int64_t head_dim, int64_t heads_per_token, float* out);
int orc_softmax_last_axis_f32(const float* x, int64_t outer, int64_t inner, float* out);
int orc_silu_gate_mul_up_f32(const float* gate, const float* up, int64_t n, float* out);
int orc_dequantize_q6_k(const uint8_t* in, int64_t n_blocks, float* out);
int orc_dequant_matmul_f16_f32(const float* act, const uint16_t* w, int64_t b, int64_t m, int64_t n,
                               int64_t k, float* out);

#ifdef __cplusplus
}
#endif
#endif
