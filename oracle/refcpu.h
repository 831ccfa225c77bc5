/*
 * refcpu — CPU restatement of the Cactus reference kernels (TEST INFRASTRUCTURE).
 *
 * This library is the parity oracle and the timed CPU baseline. It is never
 * linked into, loaded by, or called from the product library (libcactus_b200).
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
 * arm may load it.
 *
 * Every function restates the arithmetic of one reference function (path:line
 * relative to the Ayan9074/cactus tree) with the same rounding points:
 *   - fp16 storage is uint16_t (IEEE binary16); conversions round to nearest even;
 *   - NEON fp16 vector ops (vaddq_f16, vmulq_f16, vfmaq_f16) round once per op;
 *   - vfmaq_f32 and the compiler-contracted `acc += a * b` are fused (fmaf);
 *   - vcvtnq_s32_f32 rounds half to even, vcvtq_s32_f32 truncates;
 *   - NEON lane orders of the fp32 reductions are reproduced where they
 *     determine the result bits (rms norm, softmax, attention scores).
 * The reference NEON code does not build on x86 (arm_neon.h / __fp16), so this
 * restatement stands in for it; parity is pinned by the reference's own tests
 * (tests/test_kernel.cpp, tests/test_graph.cpp, tests/test_kv_cache.cpp) and by
 * fixtures generated with the reference's Python quantizer (python/src/tensor_io.py).
 */
#ifndef CACTUS_REFCPU_H
#define CACTUS_REFCPU_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

void ref_set_threads(int n);
int ref_get_threads(void);

/* fp16 helpers (exposed for tests) */
float ref_f16_to_f32(uint16_t h);
uint16_t ref_f32_to_f16(float f);

/* kernel_quants.cpp:196-221 */
float ref_fp16_max_abs(const uint16_t* src, size_t count);
/* kernel_quants.cpp:158-194 (single-chunk semantics: elements past the last multiple of 8 use round-half-away) */
void ref_fp16_to_int8(const uint16_t* src, int8_t* dst, size_t count, float scale);
/* graph_ops_nn.cpp:35-66 */
void ref_quantize_activations(const uint16_t* x, int8_t* q, float* scales, size_t M, size_t K);
/* kernel_gemm.cpp:128-327 */
void ref_matmul_int8(const int8_t* A, const float* As, const int8_t* B, const uint16_t* Bs,
                     uint16_t* C, size_t M, size_t K, size_t N, size_t group_size);
/* kernel_gemm.cpp:329-529 (B packed two int4 per byte, low nibble = even k) */
void ref_matmul_int4(const int8_t* A, const float* As, const uint8_t* Bp, const uint16_t* Bs,
                     uint16_t* C, size_t M, size_t K, size_t N, size_t group_size);
/* kernel_gemm.cpp:17-126 (fp16 accumulation in 8 lanes) */
void ref_matmul_f16(const uint16_t* A, const uint16_t* Bt, uint16_t* C, size_t M, size_t K, size_t N);
/* kernel_attention.cpp:484-563 */
void ref_rms_norm_f16(const uint16_t* x, const uint16_t* w, uint16_t* y, size_t rows, size_t dims, float eps);
/* kernel_attention.cpp:565-612: fp16 cos/sin tables [n_pos, head_dim/2] */
void ref_rope_tables(uint16_t* cos_t, uint16_t* sin_t, size_t n_pos, size_t head_dim, float theta);
/* kernel_attention.cpp:614-676 */
void ref_rope_f16(const uint16_t* in, uint16_t* out, size_t batch, size_t seq_len, size_t num_heads,
                  size_t head_dim, size_t start_pos, float theta);
/* kernel_attention.cpp:10-255 (mask == NULL) */
void ref_attention_f16(const uint16_t* q, const uint16_t* k, const uint16_t* v, uint16_t* o,
                       size_t batch, size_t seq_len, size_t kv_seq_len, size_t num_q_heads,
                       size_t num_kv_heads, size_t head_dim, float scale, size_t position_offset,
                       size_t window_size, int is_causal);
/* kernel_attention.cpp:257-482 */
void ref_attention_hybrid_int8_fp16(const uint16_t* q, const int8_t* k_cache, const int8_t* v_cache,
                                    const float* k_scales, const float* v_scales,
                                    const uint16_t* k_new, const uint16_t* v_new, uint16_t* o,
                                    size_t batch, size_t seq_len, size_t cache_len, size_t new_len,
                                    size_t num_q_heads, size_t num_kv_heads, size_t head_dim,
                                    float scale, size_t position_offset, int is_causal,
                                    size_t quant_group_size);
/* kernel_quants.cpp:223-293 */
void ref_quantize_kv(const uint16_t* src, int8_t* dst, float* scales, size_t seq_len, size_t kv_heads,
                     size_t head_dim, size_t group_size);
/* kernel_utils.h:108-141 */
float ref_fast_exp(float x);
/* kernel_utils.h:143-163 */
float ref_fast_tanh(float x);
/* kernel_nn.cpp:12-44 */
void ref_set_chunk_pool(int workers);
void ref_silu_f16(const uint16_t* x, uint16_t* y, size_t n);
/* kernel_nn.cpp:46-91 */
void ref_gelu_f16(const uint16_t* x, uint16_t* y, size_t n);
/* kernel_blas.cpp:187-222, 224-262, 291-318 */
void ref_add_f16(const uint16_t* a, const uint16_t* b, uint16_t* y, size_t n);
void ref_add_f16_clipped(const uint16_t* a, const uint16_t* b, uint16_t* y, size_t n);
void ref_multiply_f16(const uint16_t* a, const uint16_t* b, uint16_t* y, size_t n);
/* kernel_scalar.cpp:7 (MULTIPLY branch): fp16 scalar, fp16 product */
void ref_scalar_multiply_f16(const uint16_t* x, uint16_t* y, size_t n, float s);
/* kernel_nn.cpp:152-251 */
void ref_softmax_f16(const uint16_t* x, uint16_t* y, size_t rows, size_t vocab);
/* graph_ops_tensor.cpp:226-331 */
void ref_embedding_int8(const int8_t* table, const uint16_t* scales, size_t group_size, size_t num_groups,
                        const uint32_t* ids, size_t n_ids, size_t hidden, uint16_t* out);
void ref_embedding_f16(const uint16_t* table, const uint32_t* ids, size_t n_ids, size_t hidden, uint16_t* out);
/* kernel_nn.cpp:451-467 */
uint32_t ref_argmax_f16(const uint16_t* logits, size_t vocab);
/* kernel_quants.cpp:295-351 */
void ref_unpack_int4(const uint8_t* packed, int8_t* out, size_t count);
/* restatement of python/src/tensor_io.py:82-197 (INT8) and :199-282 (INT4) on float32 input */
void ref_quantize_weights_int8(const float* w, int8_t* q, uint16_t* scales, size_t N, size_t K, size_t G);
void ref_quantize_weights_int4(const float* w, uint8_t* packed, uint16_t* scales, size_t N, size_t K, size_t G);

/* other families' kernels: LFM2 causal depthwise conv, Whisper conv1d k=3, layernorm */
void ref_conv1d_causal_depthwise_f16(const uint16_t* x, const uint16_t* w, uint16_t* y, size_t N, size_t L, size_t C,
                                     size_t K, size_t dil);
void ref_conv1d_f16_k3(const uint16_t* x, const uint16_t* w, uint16_t* y, size_t N, size_t L, size_t Cin, size_t Cout,
                       size_t stride);
void ref_layernorm_f16(const uint16_t* x, const uint16_t* w, const uint16_t* b, uint16_t* y, size_t rows, size_t F,
                       float eps);

#ifdef __cplusplus
}
#endif
#endif

