/*
 * armai.h — C ABI of libarmai_cuda.so, the B200 (sm_100a) implementation of
 * arm_ai's quantized-Llama decode path and its int8/int4 primitive NIFs.
 *
 * A Rust NIF shim (native/arm_ai_nif, feature "cuda") binds these entry
 * points with `extern "C"` and keeps every NIF name and arity of the
 * reference. Each entry point cites the reference function it replaces.
 *
 * Conventions
 *   - Status: 0 = ok, negative = error (see ARMAI_E_*). The message of the
 *     last failing call on the calling thread is armai_last_error().
 *   - Host-pointer entry points take plain host buffers plus their lengths
 *     (in elements), exactly the binaries a NIF receives, and write into a
 *     caller-owned output buffer (the NIF's OwnedBinary). Length mismatches
 *     are errors with the reference's wording.
 *   - armai_dev_* entry points take device pointers and a cudaStream_t
 *     (passed as void*) and do not synchronise.
 *   - Every call sets its CUDA device on the calling thread first.
 */
#ifndef ARMAI_H
#define ARMAI_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define ARMAI_API __attribute__((visibility("default")))
#else
#define ARMAI_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define ARMAI_OK 0
#define ARMAI_E_INVALID -1     /* bad argument / length mismatch */
#define ARMAI_E_IO -2          /* file open / read failure */
#define ARMAI_E_FORMAT -3      /* malformed or unsupported GGUF content */
#define ARMAI_E_CUDA -4        /* CUDA runtime error */
#define ARMAI_E_NOMEM -5       /* device or host allocation failure */
#define ARMAI_E_DEVICE -6      /* kernel-side error flag (bounded wait expired) */
#define ARMAI_E_RANGE -7       /* position beyond the rotary table / KV capacity */

/* ------------------------------------------------------------------ */
/* Quantized Llama model                                                */
/* ------------------------------------------------------------------ */
typedef struct armai_llama armai_llama;

typedef struct armai_llama_opts {
  int32_t device;       /* CUDA device ordinal; default 0 */
  int32_t max_seq_len;  /* rotary table length = KV capacity; default 4096
                           (candle quantized_llama MAX_SEQ_LEN) */
  int32_t kv_f16;       /* 0: f32 KV cache (as candle); 1: f16 KV cache */
  int32_t max_batch;    /* sequences per batched decode step; default 1 */
  int32_t use_graph;    /* capture the decode step as a CUDA graph; default 1 */
  int32_t use_pdl;      /* programmatic dependent launch between kernels; default 1 */
  int32_t tp_size;      /* tensor-parallel degree; default 1 */
  int32_t tp_rank;      /* this process's rank in the TP group */
  const void* tp_unique_id; /* ncclUniqueId bytes (128), same on every rank */
  int32_t decode_kernel;/* 0: one persistent kernel per decode step (default);
                           1: one kernel per operation (PDL chain) */
  int32_t prefill_gemm; /* prompt matmuls: 0 = tensor-core GEMM for prompts of
                           at least 64 tokens, dp4a matvec below (default);
                           1 = always the dp4a matvec; 2 = always the GEMM */
  int32_t batch_gemm;   /* batched decode steps (armai_llama_generate_batch):
                           0 = tensor-core GEMM for Q4_K / Q6_K models (also
                           tensor parallel), integer matvec otherwise
                           (default); 1 = always the integer matvec (token for
                           token the single-sequence chain); 2 = the GEMM
                           where available */
  int32_t reserved[5];
} armai_llama_opts;

/* Tensor parallelism (tp_size > 1; 7B/8B-class models): every rank calls
 * armai_llama_load with the same path, its tp_rank and the same 128-byte
 * NCCL unique id, which rank 0 creates with armai_nccl_unique_id and shares
 * out of band (no reference counterpart: the reference runs on one CPU).
 * Query/KV heads, gate/up rows and vocab rows are split over the ranks;
 * attn_output and ffn_down are split along K. The persistent decode kernel
 * adds their partial sums through peer memory (CUDA IPC); the per-kernel
 * chain, prompts (tensor-core GEMM path) and batched decode use NCCL
 * all-reduces. Ranks must be on distinct GPUs and make the same calls in the
 * same order; host waits are bounded (the communicator is aborted after
 * 120 s without progress). */
ARMAI_API int armai_nccl_unique_id(void* out128);

/* Fill `o` with the defaults above. */
ARMAI_API void armai_llama_default_opts(armai_llama_opts* o);

/* Replaces llama_candle::load_model (native/arm_ai_nif/src/llama_candle.rs:35-48)
 * behind llama_candle_load_op (native/arm_ai_nif/src/lib.rs:1659-1665).
 * Parses the GGUF file, uploads the Q4_K / Q6_K super-blocks to HBM,
 * allocates the KV cache and prepares the decode step (the persistent
 * kernel's phase table, or the per-kernel chain captured as a CUDA graph).
 * Other weight types are rejected, naming the tensor. `opts` may be NULL. */
ARMAI_API int armai_llama_load(const char* path, const armai_llama_opts* opts, armai_llama** out);

/* Releases every device and host resource of the model (the NIF resource's
 * Drop; native/arm_ai_nif/src/lib.rs:2040-2043). NULL is a no-op. */
ARMAI_API void armai_llama_free(armai_llama* m);

typedef struct armai_llama_info {
  int32_t n_layer, n_embd, n_ff, n_head, n_head_kv, head_dim, n_vocab, max_seq_len;
  float rms_eps, rope_theta;
  int64_t weight_bytes;      /* bytes of weights streamed per decode token */
  int64_t device_bytes;      /* total device memory held by the model */
  int32_t n_kernels_per_step;/* kernels launched per decode step */
  int32_t kv_f16;
} armai_llama_info;
ARMAI_API int armai_llama_get_info(const armai_llama* m, armai_llama_info* info);

/* Per-token callback: called on the generating thread as soon as each
 * token's id has reached the host (llama_candle_stream_op sends
 * {:llama_token, id} from this point; native/arm_ai_nif/src/lib.rs:1682-1699). */
typedef void (*armai_token_cb)(void* user, uint32_t token);

/* Replaces llama_candle::generate_greedy_with (llama_candle.rs:69-137)
 * behind llama_candle_generate_op / llama_candle_stream_op
 * (native/arm_ai_nif/src/lib.rs:1667-1699). Greedy decode: prefill at offset
 * 0, then up to max_new-1 single-token steps, stopping after a token in
 * `stop` (the stop token is included in `out`). max_new == 0 or n_prompt == 0
 * yields no tokens and zero timings. `out` must hold max_new ids.
 * prefill_us / decode_us are the reference's two wall-clock timers. */
ARMAI_API int armai_llama_generate(armai_llama* m, const uint32_t* prompt, size_t n_prompt,
                         size_t max_new, const uint32_t* stop, size_t n_stop,
                         armai_token_cb on_token, void* user, uint32_t* out, size_t* n_out,
                         uint64_t* prefill_us, uint64_t* decode_us);

/* Batched greedy decode of n_seq independent sequences (e.g. 16 sequences per GPU):
 * prompts are concatenated in `prompts` with lengths in `n_prompt[n_seq]`.
 * Each sequence behaves exactly like one armai_llama_generate call; decode
 * steps of all live sequences run as one batched step. out is
 * [n_seq][max_new], n_out[n_seq]. No reference counterpart (the reference
 * holds one KV cache per handle, llama_candle.rs:27-29). */
ARMAI_API int armai_llama_generate_batch(armai_llama* m, const uint32_t* prompts, const size_t* n_prompt,
                               size_t n_seq, size_t max_new, const uint32_t* stop,
                               size_t n_stop, uint32_t* out, size_t* n_out,
                               uint64_t* prefill_us, uint64_t* decode_us);

/* ModelWeights::forward(tokens[1, n], index_pos) (candle-transformers 0.8.4
 * quantized_llama, called at llama_candle.rs:92-94 and :118-120): runs the
 * tokens at positions index_pos.. (index_pos == 0 resets the KV cache) and
 * writes the last position's f32 logits [n_vocab] to host `logits` (may be
 * NULL) and its first-max argmax (llama_candle.rs:145-176) to *token. */
ARMAI_API int armai_llama_forward(armai_llama* m, const uint32_t* tokens, size_t n, size_t index_pos,
                        float* logits, uint32_t* token);

/* Device-resident decode benchmark: runs `n_steps` greedy decode steps
 * back to back from the current state (token and position already on the
 * device after a forward/prefill), without host round trips, and returns the
 * device time (CUDA events on the model's stream) in *ms. */
ARMAI_API int armai_llama_bench_decode(armai_llama* m, int32_t n_steps, float* ms);

/* Kernel-level timing for roofline figures: launches one kind of decode
 * kernel (0 = gate/up matvec, 1 = q/k/v matvec, 2 = attn_output matvec,
 * 3 = ffn_down matvec, 4 = output head + argmax, 5 = attention) once per
 * layer, layer after layer, `rounds` times, back to back without PDL on the
 * model's stream, and returns the average device time per launch (CUDA
 * events) and the weight bytes one launch streams (layer average). The
 * launches read whatever activations are resident; results are discarded. */
ARMAI_API int armai_llama_bench_kernel(armai_llama* m, int32_t kind, int32_t rounds, float* ms_per_launch,
                                       int64_t* bytes_per_launch);

/* Phase timeline of one decode step of the persistent decode kernel (no
 * reference counterpart; the reference only times prefill and decode as a
 * whole, native/arm_ai_nif/src/llama_candle.rs:83-130). Runs one step from
 * the current state and writes, for phase p (in kernel order: per layer
 * q/k/v, attention, attn_output, gate/up, ffn_down; then the head) and CTA c,
 * ten globaltimer stamps in ns at out[(p * n_ctas + c) * 10 + s]:
 * s = 0 phase start, 1 activation built, 2 phase done, 3 weight producer
 * issued the phase's first copy, 4 first copy landed, 5 first chunk
 * computed, 6 activation loaded, 7 rms scale known, 8 / 9 first row unit's
 * dot products / epilogue done (0 where a phase has no such step). A last
 * row (p = number of phases) holds each CTA's kernel entry in s = 0 and, for
 * the CTA that wrote the step's token, that moment in s = 1. `cap` is the
 * capacity of `out` in stamps. */
ARMAI_API int armai_llama_trace_decode(armai_llama* m, uint64_t* out, size_t cap, int32_t* n_phases,
                                       int32_t* n_ctas);

/* Test-only error injection for the persistent decode kernel (no reference
 * counterpart). From the next decode step on, phase `phase` (numbered as in
 * armai_llama_trace_decode) publishes none of its outputs, and every wait on
 * another CTA's output gives up after `poll_limit` polls (0 keeps the
 * default): the consumers of that phase run out their bounded waits, the
 * launch ends with the device error word set, and the call returns
 * ARMAI_E_DEVICE; the model then answers every call with "reload the
 * model". No GPU fault is involved: the kernel only stops waiting. */
ARMAI_API int armai_llama_test_stall(armai_llama* m, int32_t phase, uint32_t poll_limit);

/* ------------------------------------------------------------------ */
/* Primitive NIFs (nx_arm building blocks). Host buffers in, caller-owned  */
/* host output buffer out; same argument order as the NIFs.                */
/* ------------------------------------------------------------------ */

/* int8_matmul_f32_op (native/arm_ai_nif/src/lib.rs:215-235 ->
 * shape_ops.rs:1169-1211): out[M,N] = (f32)(sum_k a[m,k] w[n,k]) * act_scale * w_scales[n]. */
ARMAI_API int armai_int8_matmul_f32(const int8_t* a, size_t a_len, const int8_t* w, size_t w_len,
                          const float* w_scales, size_t w_scales_len, double act_scale,
                          size_t m, size_t n, size_t k, float* out);

/* int8_matmul_f32_per_token_op (lib.rs:239-264 -> shape_ops.rs:1222-1264). */
ARMAI_API int armai_int8_matmul_f32_per_token(const int8_t* a, size_t a_len, const int8_t* w, size_t w_len,
                                    const float* act_scales, size_t act_scales_len,
                                    const float* w_scales, size_t w_scales_len, size_t m,
                                    size_t n, size_t k, float* out);

/* The s8 x s8 -> s32 GEMM underneath the two entry points above
 * (shape_ops.rs:1364-1370 int8_dot per output). out[M,N] int32. */
ARMAI_API int armai_int8_matmul_s32(const int8_t* a, size_t a_len, const int8_t* w, size_t w_len,
                          size_t m, size_t n, size_t k, int32_t* out);

/* quantize_int8_per_token_op (lib.rs:268-296 -> shape_ops.rs:1273-1292):
 * q[M,K] int8, scales[M] f32. */
ARMAI_API int armai_quantize_int8_per_token(const float* a, size_t a_len, size_t m, size_t k, int8_t* q,
                                  float* scales);

/* int4_matmul_f32_op (lib.rs:450-473 -> shape_ops.rs:3175-3236): a[M,K] f32,
 * w_packed[N,K/2] (low nibble = even k, value-8), w_scales[N,K/32] f32. */
ARMAI_API int armai_int4_matmul_f32(const float* a, size_t a_len, const uint8_t* w_packed,
                          size_t w_packed_len, const float* w_scales, size_t w_scales_len,
                          size_t m, size_t n, size_t k, float* out);

/* int4_matmul_gemv_neon_op (lib.rs:427-446 -> shape_ops.rs:3059-3166): M = 1. */
ARMAI_API int armai_int4_matmul_gemv(const float* a, size_t a_len, const uint8_t* w_packed,
                           size_t w_packed_len, const float* w_scales, size_t w_scales_len,
                           size_t n, size_t k, float* out);

/* int4_matmul_gemv_q4_x_q8_neon_op (lib.rs:403-422 -> shape_ops.rs:2923-3028):
 * activations quantised Q8_0-style per 32 values, integer group dots. */
ARMAI_API int armai_int4_matmul_gemv_q4_x_q8(const float* a, size_t a_len, const uint8_t* w_packed,
                                   size_t w_packed_len, const float* w_scales,
                                   size_t w_scales_len, size_t n, size_t k, float* out);

/* quantize_int4_q4_0_op (lib.rs:477-502 -> shape_ops.rs:3242-3275):
 * packed[N,K/2], scales[N,K/32]. */
ARMAI_API int armai_quantize_int4_q4_0(const float* w, size_t w_len, size_t n, size_t k, uint8_t* packed,
                             float* scales);

/* rmsnorm_f32_op (lib.rs:127-145 -> shape_ops.rs:976-1018). */
ARMAI_API int armai_rmsnorm_f32(const float* input, size_t input_len, const float* gamma, size_t gamma_len,
                      size_t n_outer, size_t inner, double epsilon, float* out);

/* flash_attention_f32_op (lib.rs:743-764 -> shape_ops.rs:464-558):
 * q[B,H,Sq,D], k/v[B,H,Sk,D] f32 -> out[B,H,Sq,D]. */
ARMAI_API int armai_flash_attention_f32(const float* q, size_t q_len, const float* k, size_t k_len,
                              const float* v, size_t v_len, double scale, size_t b, size_t h,
                              size_t sq, size_t sk, size_t d, int causal, float* out);

/* dequant_matmul_int8_f32_op (lib.rs:507-532 -> shape_ops.rs:1525-1582). */
ARMAI_API int armai_dequant_matmul_int8_f32(const float* act, size_t act_len, const int8_t* w, size_t w_len,
                                  const float* scales, size_t scales_len, size_t b, size_t m,
                                  size_t n, size_t k, float* out);

/* rope_f32_op (lib.rs:147-171 -> shape_ops.rs:1040-1100): input [n_rows, head_dim],
 * positions i64 per token (row r uses positions[r / heads_per_token]),
 * inv_freq [head_dim / 2]; interleaved pairs (2k, 2k + 1). */
ARMAI_API int armai_rope_f32(const float* input, size_t input_len, const int64_t* positions,
                             size_t n_positions, const float* inv_freq, size_t inv_freq_len,
                             size_t n_rows, size_t head_dim, size_t heads_per_token, float* out);

/* dequant_matmul_f16_f32_op (lib.rs:173-196 -> shape_ops.rs:1462-1490):
 * act [B,M,K] f32 x weights [N,K] f16 bits -> out [B,M,N]. */
ARMAI_API int armai_dequant_matmul_f16_f32(const float* act, size_t act_len, const uint16_t* weights,
                                           size_t weights_len, size_t b, size_t m, size_t n, size_t k,
                                           float* out);

/* softmax_last_axis_f32_op (lib.rs:298-318 -> shape_ops.rs:2719-2751). */
ARMAI_API int armai_softmax_last_axis_f32(const float* input, size_t input_len, size_t outer,
                                          size_t inner, float* out);

/* silu_gate_mul_up_f32_op (lib.rs:320-342 -> shape_ops.rs:2755-2770). */
ARMAI_API int armai_silu_gate_mul_up_f32(const float* gate, size_t gate_len, const float* up,
                                         size_t up_len, float* out);

/* dequantize_q6_k_op (lib.rs:344-354 -> shape_ops.rs:2848-2899): 210-byte
 * blocks -> n_elements f32 (n_elements = 256 * whole blocks in input). */
ARMAI_API int armai_dequantize_q6_k(const uint8_t* input, size_t input_len, size_t n_elements,
                                    float* out);

/* ------------------------------------------------------------------ */
/* Device-pointer variants (benchmarks, and callers that keep tensors     */
/* resident). `stream` is a cudaStream_t.                                   */
/* ------------------------------------------------------------------ */
ARMAI_API int armai_dev_int8_matmul_s32(const int8_t* a, const int8_t* w, int32_t* out, int64_t m,
                              int64_t n, int64_t k, void* stream);
ARMAI_API int armai_dev_int8_matmul_f32(const int8_t* a, const int8_t* w, const float* act_scales,
                              int per_token, float act_scale, const float* w_scales, float* out,
                              int64_t m, int64_t n, int64_t k, void* stream);
ARMAI_API int armai_dev_int4_matmul_f32(const float* a, const uint8_t* w_packed, const float* w_scales,
                              float* out, int64_t m, int64_t n, int64_t k, void* stream);
ARMAI_API int armai_dev_int4_gemv_q4_x_q8(const float* a, const uint8_t* w_packed, const float* w_scales,
                                float* out, int64_t n, int64_t k, void* stream);
/* No-allocation variant of armai_dev_int4_gemv_q4_x_q8 (no reference
 * counterpart: the reference's NIF allocates its Vec scratch on the CPU
 * heap, native/arm_ai_nif/src/shape_ops.rs:2923-3028). For callers that must
 * not allocate device memory on the call path, e.g. a serving loop that has
 * reserved the device's memory up front and cannot afford an allocation's
 * latency or its failure in mid-step. Same arguments and results as
 * armai_dev_int4_gemv_q4_x_q8; the stage-1 scratch is a static device array
 * sized for K <= 16384 (ARMAI_E_RANGE above that). Calls on one device share
 * that scratch: they must not overlap (use one stream, or order them). Each
 * call looks up the current device's scratch address (so a device reset
 * between calls is harmless); the first call on a device may load the
 * module, so make it before any stream capture. */
ARMAI_API int armai_dev_int4_gemv_q4_x_q8_noalloc(const float* a, const uint8_t* w_packed,
                                                  const float* w_scales, float* out, int64_t n, int64_t k,
                                                  void* stream);
/* The int4 gemv with per-32-group f16 scales [N,K/32] (instead of f32). */
ARMAI_API int armai_dev_int4_gemv_f16s(const float* a, const uint8_t* w_packed, const uint16_t* w_scales,
                             float* out, int64_t n, int64_t k, void* stream);
ARMAI_API int armai_dev_rmsnorm_f32(const float* x, const float* gamma, float* out, int64_t n_outer,
                          int64_t inner, float eps, void* stream);
/* Causal/non-causal attention, f16 q/k/v [B,H,S,D] -> f32 out. */
ARMAI_API int armai_dev_flash_attention_f16(const uint16_t* q, const uint16_t* k, const uint16_t* v,
                                  float* out, float scale, int64_t b, int64_t h, int64_t sq,
                                  int64_t sk, int64_t d, int causal, void* stream);
ARMAI_API int armai_dev_flash_attention_f32(const float* q, const float* k, const float* v, float* out,
                                  float scale, int64_t b, int64_t h, int64_t sq, int64_t sk,
                                  int64_t d, int causal, void* stream);
ARMAI_API int armai_dev_rope_f32(const float* x, const int64_t* positions, const float* inv_freq,
                                 float* out, int64_t n_rows, int64_t head_dim, int64_t heads_per_token,
                                 void* stream);
ARMAI_API int armai_dev_softmax_last_axis_f32(const float* x, float* out, int64_t outer, int64_t inner,
                                              void* stream);
ARMAI_API int armai_dev_silu_gate_mul_up_f32(const float* gate, const float* up, float* out, int64_t n,
                                             void* stream);
/* n_blocks 210-byte Q6_K blocks -> 256 * n_blocks f32. */
ARMAI_API int armai_dev_dequantize_q6_k(const uint8_t* in, float* out, int64_t n_blocks, void* stream);
/* act [rows, K] f32 x weights [N, K] f16 bits -> out [rows, N]. */
ARMAI_API int armai_dev_dequant_matmul_f16_f32(const float* act, const uint16_t* w, float* out,
                                               int64_t rows, int64_t n, int64_t k, void* stream);

/* ------------------------------------------------------------------ */
/* k-quant building blocks, exposed for bit-exact parity tests.           */
/* ------------------------------------------------------------------ */
/* Q8_K quantisation of x[m, k] (candle BlockQ8K::from_float): writes
 * blocks of {f32 d, int8 qs[256], int16 bsums[16]} (292 B) to host `out`. */
ARMAI_API int armai_quantize_q8k(const float* x, size_t m, size_t k, void* out);
/* Integer per-super-block dot products of weight rows w[n, k] (GGML type
 * 12 = Q4_K or 14 = Q6_K, raw GGUF bytes) with Q8_K rows q8[m, k]:
 * isum[m][n][k/256] = sum_j scale_j*<q_j, q8_j>; msum (Q4_K only) =
 * sum_j min_j * bsum_j. The same device code the decode kernels use. */
ARMAI_API int armai_kquant_block_dots(const void* w, int type, size_t n, size_t k, const void* q8,
                            size_t m, int32_t* isum, int32_t* msum);
/* QMatMul: out[m][n] = vec_dot(w row n, Q8_K(x row m)) through the decode
 * (m == 1) or prefill (m > 1) matvec kernels. */
ARMAI_API int armai_qmatmul(const void* w, int type, size_t n, size_t k, const float* x, size_t m,
                  float* out);

/* Test entry (no reference counterpart): the prefill tensor-core GEMM on
 * host buffers. x [m][k] f32 (rms-normalised with gamma when not null),
 * quantised per token to Q8_K and expanded to f16; w [n] rows of GGML
 * Q4_K/Q6_K blocks dequantised to f16; out [m][n] = A W^T with f32
 * accumulation (tcgen05). The reference computes the same product through
 * QMatMul (llama_candle.rs:92-94) with integer Q8_K dots. */
ARMAI_API int armai_qgemm(const void* w, int type, size_t n, size_t k, const float* x, size_t m,
                          const float* gamma, float eps, float* out);

/* Thread-local message of the last failing call on this thread. */
ARMAI_API const char* armai_last_error(void);
/* Library version string. */
ARMAI_API const char* armai_version(void);

#ifdef __cplusplus
}
#endif
#endif
