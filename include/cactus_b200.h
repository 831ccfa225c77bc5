/*
 * cactus_b200.h — C ABI of the B200 (sm_100a) kernels behind the Cactus hot path.
 *
 * Each entry point is the device counterpart of one reference kernel function
 * (Ayan9074/cactus, path:line given per function) or of one graph-node executor
 * that the reference runs around such a kernel. All tensor arguments are DEVICE
 * pointers (cudaMalloc'd or views into such allocations), 16-byte aligned where
 * marked; fp16 tensors are passed as uint16_t* holding IEEE binary16 bits.
 * `stream` is a cudaStream_t (NULL = legacy default stream). Calls are
 * asynchronous on `stream`; they return 0 on success or a negative code on an
 * argument / launch error, with a message in cactus_cuda_last_error().
 * Nothing here allocates per call except the RoPE table cache (grown once per
 * (theta, head_dim) up to the largest position seen).
 */
#ifndef CACTUS_B200_H
#define CACTUS_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define CB_API __attribute__((visibility("default")))
#else
#define CB_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum {
    CB_OK = 0,
    CB_ERR_ARG = -1,      /* invalid shape / size / alignment */
    CB_ERR_LAUNCH = -2,   /* CUDA launch or runtime error */
    CB_ERR_UNSUPPORTED = -3
};

CB_API const char* cactus_cuda_last_error(void);
/* Device error word set by kernels that gave up a bounded wait (0 = none); reading clears it. */
CB_API unsigned cactus_cuda_device_error(void* stream);
CB_API int cactus_cuda_version(void);

/* ---- activation quantization: graph_ops_nn.cpp:35-66 (cactus_fp16_max_abs
 *      kernel_quants.cpp:196-221 + cactus_fp16_to_int8 kernel_quants.cpp:158-194) */
CB_API int cactus_cuda_quantize_activations(const uint16_t* x, int8_t* q, float* scales,
                                            size_t M, size_t K, void* stream);

/* ---- grouped INT8 matmul: cactus_matmul_int8, kernel_gemm.cpp:128-327.
 *      A int8 [M,K], A_scales fp32 [M], B int8 [N,K] (16B aligned), B_scales fp16 [N,K/G]
 *      (16B aligned), C fp16 [M,N]. */
CB_API int cactus_cuda_matmul_int8(const int8_t* A, const float* A_scales, const int8_t* B,
                                   const uint16_t* B_scales, uint16_t* C, size_t M, size_t K,
                                   size_t N, size_t group_size, void* stream);
/* ---- grouped INT4 matmul: cactus_matmul_int4, kernel_gemm.cpp:329-529. B packed [N,K/2],
 *      byte i of a row holds k=2i in the low nibble and k=2i+1 in the high nibble. */
CB_API int cactus_cuda_matmul_int4(const int8_t* A, const float* A_scales, const uint8_t* B_packed,
                                   const uint16_t* B_scales, uint16_t* C, size_t M, size_t K,
                                   size_t N, size_t group_size, void* stream);
/* ---- compute_matmul_node with FP16 activations (graph_ops_nn.cpp:150-209): the activation
 *      quantization fused into the INT8 / INT4 matmul. */
CB_API int cactus_cuda_linear_int8(const uint16_t* X, const int8_t* B, const uint16_t* B_scales,
                                   uint16_t* C, size_t M, size_t K, size_t N, size_t group_size,
                                   void* stream);
CB_API int cactus_cuda_linear_int4(const uint16_t* X, const uint8_t* B_packed, const uint16_t* B_scales,
                                   uint16_t* C, size_t M, size_t K, size_t N, size_t group_size,
                                   void* stream);
/* ---- FP16 matmul with fp16 accumulation: cactus_matmul_f16, kernel_gemm.cpp:17-126.
 *      A [M,K], B_transposed [N,K], C [M,N]. */
CB_API int cactus_cuda_matmul_f16(const uint16_t* A, const uint16_t* B_transposed, uint16_t* C,
                                  size_t M, size_t K, size_t N, void* stream);

/* ---- RMSNorm: cactus_rms_norm_f16, kernel_attention.cpp:484-563 */
CB_API int cactus_cuda_rms_norm_f16(const uint16_t* input, const uint16_t* weight, uint16_t* output,
                                    size_t batch_size, size_t dims, float eps, void* stream);
/* ---- Causal depthwise conv1d (LFM2): cactus_conv1d_causal_depthwise_f16, kernel_conv.cpp:15-110.
 *      input/output [N, L, C], weight [C, K]; output t of channel c sums weight[c][K-1-k] *
 *      input[t - k*dilation][c] over taps k (positions before 0 are zero). */
CB_API int cactus_cuda_conv1d_causal_depthwise_f16(const uint16_t* input, const uint16_t* weight, uint16_t* output,
                                                   size_t N, size_t L, size_t C, size_t K, size_t dilation,
                                                   void* stream);
/* ---- Conv1d, kernel size 3, zero padding 1 (Whisper front end): cactus_conv1d_f16_k3,
 *      kernel_conv.cpp:112-227. input [N, C_in, L], weight [C_out, C_in, 3],
 *      output [N, C_out, (L - 1) / stride + 1]. */
CB_API int cactus_cuda_conv1d_f16_k3(const uint16_t* input, const uint16_t* weight, uint16_t* output, size_t N,
                                     size_t L, size_t C_in, size_t C_out, size_t stride, void* stream);
/* ---- LayerNorm over the last dimension, fp16 in / out: compute_layernorm_node,
 *      graph_ops_nn.cpp:373-457. input/output [rows, features], weight and bias [features];
 *      features up to 14528 (shared-memory staging of the row). */
CB_API int cactus_cuda_layernorm_f16(const uint16_t* input, const uint16_t* weight, const uint16_t* bias,
                                     uint16_t* output, size_t rows, size_t features, float eps, void* stream);
/* ---- RoPE (NeoX half rotation, fp16 cos/sin tables): cactus_rope_f16, kernel_attention.cpp:565-676.
 *      input/output [B, S, H, D]; position of token s is start_pos + s. */
CB_API int cactus_cuda_rope_f16(const uint16_t* input, uint16_t* output, size_t batch_size,
                                size_t seq_len, size_t num_heads, size_t head_dim, size_t start_pos,
                                float theta, void* stream);

/* ---- no-cache attention: cactus_attention_f16, kernel_attention.cpp:10-255 (mask = NULL).
 *      Q [B,S,Hq,D], K/V [B,Skv,Hkv,D], O [B,S,Hq,D]; head_dim % 32 == 0, <= 256. */
CB_API int cactus_cuda_attention_f16(const uint16_t* queries, const uint16_t* keys, const uint16_t* values,
                                     uint16_t* output, size_t batch_size, size_t seq_len,
                                     size_t kv_seq_len, size_t num_q_heads, size_t num_kv_heads,
                                     size_t head_dim, float scale, size_t position_offset,
                                     size_t window_size, int is_causal, void* stream);
/* ---- INT8-cache + FP16-new attention: cactus_attention_hybrid_int8_fp16,
 *      kernel_attention.cpp:257-482. Cache int8 [B, cache_len, Hkv, D] with fp32 scales
 *      [cache_len, Hkv, ceil(D/group)] indexed without a batch offset, as the reference does. */
CB_API int cactus_cuda_attention_hybrid_int8_fp16(const uint16_t* queries, const int8_t* keys_cached,
                                                  const int8_t* values_cached, const float* k_scales,
                                                  const float* v_scales, const uint16_t* keys_new,
                                                  const uint16_t* values_new, uint16_t* output,
                                                  size_t batch_size, size_t seq_len, size_t cache_len,
                                                  size_t new_len, size_t num_q_heads, size_t num_kv_heads,
                                                  size_t head_dim, float scale, size_t position_offset,
                                                  int is_causal, size_t quant_group_size, void* stream);

/* ---- KV quantization: cactus_quantize_kv_fp16_to_int8, kernel_quants.cpp:266-293 */
CB_API int cactus_cuda_quantize_kv_fp16_to_int8(const uint16_t* src, int8_t* dst, float* scales,
                                                size_t seq_len, size_t kv_heads, size_t head_dim,
                                                size_t group_size, void* stream);

/* ---- activations / elementwise: kernel_nn.cpp:12-91, kernel_blas.cpp:187-343, kernel_scalar.cpp:7 */
CB_API int cactus_cuda_silu_f16(const uint16_t* input, uint16_t* output, size_t n, void* stream);
CB_API int cactus_cuda_gelu_f16(const uint16_t* input, uint16_t* output, size_t n, void* stream);
CB_API int cactus_cuda_add_f16(const uint16_t* a, const uint16_t* b, uint16_t* out, size_t n, void* stream);
CB_API int cactus_cuda_add_f16_clipped(const uint16_t* a, const uint16_t* b, uint16_t* out, size_t n,
                                       void* stream);
CB_API int cactus_cuda_multiply_f16(const uint16_t* a, const uint16_t* b, uint16_t* out, size_t n,
                                    void* stream);
CB_API int cactus_cuda_scalar_multiply_f16(const uint16_t* input, uint16_t* output, size_t n, float scalar,
                                           void* stream);
/* ---- row softmax: cactus_softmax_f16, kernel_nn.cpp:152-251 */
CB_API int cactus_cuda_softmax_f16(const uint16_t* input, uint16_t* output, size_t rows, size_t vocab,
                                   void* stream);

/* ---- embedding gather (+ grouped INT8 dequant): compute_embedding_node, graph_ops_tensor.cpp:226-331 */
CB_API int cactus_cuda_embedding_int8(const int8_t* table, const uint16_t* scales, size_t group_size,
                                      size_t vocab, size_t hidden, const uint32_t* ids, size_t n_ids,
                                      uint16_t* out, void* stream);
CB_API int cactus_cuda_embedding_f16(const uint16_t* table, size_t vocab, size_t hidden, const uint32_t* ids,
                                     size_t n_ids, uint16_t* out, void* stream);

/* ---- greedy sampling: cactus_sample_f16 with temperature 0, top_p <= 0, top_k 0
 *      (kernel_nn.cpp:451-467): first index of the maximum of row `rows-1`. */
CB_API int cactus_cuda_argmax_f16(const uint16_t* logits, size_t rows, size_t vocab, uint32_t* out_index,
                                  void* stream);

/* ---- non-greedy sampling: cactus_sample_f16 (kernel_nn.cpp:469-651) on row `rows-1`:
 *      temperature (fp16 multiply), repetition penalty 1.1 over `history`, top-k, top-p
 *      (any top_k, including 0 = no top-k, and any number of surviving candidates), then the
 *      first index whose in-order cumulative probability reaches `uniform` (the reference
 *      draws it from std::mt19937).
 *      `work` is caller-provided fp16 scratch of `vocab` elements. Greedy arguments
 *      (temperature 0, top_p <= 0, top_k 0) give the first-max argmax. */
CB_API int cactus_cuda_sample_f16(const uint16_t* logits, size_t rows, size_t vocab, float temperature, float top_p,
                                  size_t top_k, float uniform, const uint32_t* history, size_t n_history,
                                  uint16_t* work, uint32_t* out_index, void* stream);
/* ---- cactus_cuda_sample_f16 without the `work` argument; no counterpart in the reference.
 *      For callers that must not allocate device memory (code running inside CUDA stream
 *      capture, or under an allocator they do not control). The scratch is a fixed array
 *      inside this library holding up to 262144 fp16 entries per device; larger vocabularies
 *      are rejected with CB_ERR_ARG. Nothing in it needs to start at zero (every entry used is
 *      written before it is read). The first call on each device resolves the array's address
 *      (cudaGetSymbolAddress); make it before any stream capture. After a device reset the
 *      next call resolves it again in the new context (so make one call before capturing there too). Calls that overlap in time
 *      on one device (different streams or host threads) share the array and race: serialise
 *      them. Results equal cactus_cuda_sample_f16's. */
CB_API int cactus_cuda_sample_f16_noalloc(const uint16_t* logits, size_t rows, size_t vocab, float temperature,
                                          float top_p, size_t top_k, float uniform, const uint32_t* history,
                                          size_t n_history, uint32_t* out_index, void* stream);
/* ---- normalised entropy of softmax(logits[rows-1]) (engine_model.cpp:255-290), fp32 out */
CB_API int cactus_cuda_entropy_f16(const uint16_t* logits, size_t rows, size_t vocab, float* out, void* stream);

/* ---- INT4 unpack: cactus_unpack_int4_to_int8, kernel_quants.cpp:295-351 */
CB_API int cactus_cuda_unpack_int4_to_int8(const uint8_t* packed, int8_t* unpacked, size_t count,
                                           void* stream);

/* ---- 2-D transpose: cactus_transpose_2d_f16, kernel_blas.cpp:407-493 (whole matrix).
 *      source [num_rows, num_cols] -> destination [num_cols, num_rows]. */
CB_API int cactus_cuda_transpose_2d_f16(const uint16_t* source, uint16_t* destination, size_t num_rows,
                                        size_t num_cols, void* stream);

#ifdef __cplusplus
}
#endif
#endif
