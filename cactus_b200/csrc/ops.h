// Internal launcher declarations shared by the C ABI (abi.cu) and the engine.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "kv_paging.h"

namespace cb {

// ---- grouped GEMV (gemv.cu)
enum GemvPro { kProPreq = 0, kProQuant = 1, kProRmsNormQuant = 2 };
enum GemvEpi { kEpiStore = 0, kEpiResidual = 1, kEpiGluSilu = 2, kEpiGluGelu = 3 };
struct GemvCall {
    int int4;  // 0: int8 weights [N,K]; 1: packed int4 [N,K/2]
    int pro, epi;
    const __half* x;       // fp16 activations [M,K] (kProQuant / kProRmsNormQuant)
    const __half* norm_w;  // [K] (kProRmsNormQuant)
    float eps;
    const int8_t* aq;  // kProPreq
    const float* as;   // kProPreq
    const void* w;
    const __half* ws;
    __half* out;
    const __half* resid;
    int8_t* aq_out;
    float* as_out;
    int M, K, N, G;
    bool pdl;  // launch with programmatic stream serialization
};
int launch_gemv(const GemvCall& c, cudaStream_t st);
void gemv_prepare();  // set kernel attributes of all variants (call before graph capture)
const char* gemv_check(const GemvCall& c);  // nullptr when the shape is supported
// Largest number of activation rows (8, 4, 2 or 1) one GEMV launch takes for this weight
// format / prologue / K / G within the shared-memory limit (0: not even one row fits).
int gemv_rows_per_launch(int int4, int pro, int K, int G);

// ---- grouped INT8 / INT4 GEMM for M >= 16 on the tensor cores (gemm.cu); A pre-quantised
const char* gemm_check(int M, int K, int N, int G, int int4);  // nullptr when supported
int launch_gemm(const int8_t* aq, const float* as, const void* w, const __half* ws, __half* out, const __half* resid,
                int M, int K, int N, int G, int int4, int epi, cudaStream_t st);
constexpr int kGemmMinRows = 16;  // below this the GEMV is faster

// ---- misc (misc.cu)
int launch_quantize_act(const __half* x, int8_t* q, float* s, int M, int K, cudaStream_t st);
int launch_rms_norm(const __half* x, const __half* w, __half* y, int rows, int dims, float eps, cudaStream_t st);
// other families' kernels (conv_norm.cu)
int launch_conv1d_causal_depthwise(const __half* x, const __half* w, __half* y, int N, int L, int C, int K, int dil,
                                   cudaStream_t st);
int launch_conv1d_k3(const __half* x, const __half* w, __half* y, int N, int L, int Cin, int Cout, int stride,
                     cudaStream_t st);
int layernorm_max_features();
int launch_layernorm(const __half* x, const __half* w, const __half* b, __half* y, int rows, int F, float eps,
                     cudaStream_t st);
int launch_rope(const __half* in, __half* out, const __half* ct, const __half* stab, long long rows, int seq_len,
                int heads, int head_dim, long long start_pos, cudaStream_t st);
int launch_quantize_kv(const __half* src, int8_t* dst, float* scales, long long rows, int head_dim, int G,
                       cudaStream_t st);
int launch_silu(const __half* x, __half* y, long long n, cudaStream_t st);
int launch_gelu(const __half* x, __half* y, long long n, cudaStream_t st);
int launch_binary(const __half* a, const __half* b, __half* y, long long n, int op, cudaStream_t st);
int launch_scalar_mul(const __half* x, __half* y, long long n, float s, cudaStream_t st);
int launch_softmax(const __half* x, __half* y, int rows, int V, cudaStream_t st);
int launch_embedding_int8(const int8_t* t, const __half* s, int G, int hidden, const uint32_t* ids, int n,
                          __half* out, cudaStream_t st);
int launch_embedding_f16(const __half* t, int hidden, const uint32_t* ids, int n, __half* out, cudaStream_t st);
int launch_argmax(const __half* logits, int V, uint32_t* out, cudaStream_t st);
int launch_unpack_int4(const uint8_t* p, int8_t* o, long long count, cudaStream_t st);
int launch_transpose_2d(const uint16_t* src, uint16_t* dst, long long rows, long long cols, cudaStream_t st);
int launch_matmul_f16(const __half* A, const __half* Bt, __half* C, int M, int K, int N, cudaStream_t st);

// ---- attention (attention.cu)
int launch_attention_f16(const __half* q, const __half* k, const __half* v, __half* o, int B, int S, int Skv, int Hq,
                         int Hkv, int D, float scale, long long pos_off, long long window, int causal,
                         cudaStream_t st);
int launch_attention_hybrid(const __half* q, const int8_t* kc, const int8_t* vc, const float* ks, const float* vs,
                            const __half* kn, const __half* vn, __half* o, int B, int S, int cache_len, int new_len,
                            int Hq, int Hkv, int D, float scale, long long pos_off, int causal, int qgs,
                            long long kc_bstride, long long sc_bstride, cudaStream_t st,
                            const int* dstate = nullptr);
int launch_attention_hybrid_exact(const __half* q, const int8_t* kc, const int8_t* vc, const float* ks,
                                  const float* vs, const __half* kn, const __half* vn, __half* o, int B, int S,
                                  int cache_len, int new_len, int Hq, int Hkv, int D, float scale, long long pos_off,
                                  int causal, int qgs, long long kc_bstride, long long sc_bstride, cudaStream_t st,
                                  const int* dstate = nullptr, KvPaging pg = KvPaging());
void attention_prepare();  // kernel attributes, called before any graph capture
// Exact hybrid attention split over the keys for long caches (attention_split.cu): same
// result bits as launch_attention_hybrid_exact; -1 when the shape or the scratch size is
// outside its limits (the caller then uses the one-CTA-per-query kernel).
constexpr long long kSplitMinKeys = 512;
constexpr size_t kSplitMaxSmem = 227 * 1024;
constexpr size_t kSplitMaxScratch = size_t(4) << 30;
int launch_attention_split(const __half* q, const int8_t* kc, const int8_t* vc, const float* ks, const float* vs,
                           const __half* kn, const __half* vn, __half* o, int B, int S, int cache_len, int new_len,
                           int Hq, int Hkv, int D, float scale, long long pos_off, int causal, int qgs,
                           long long kc_bstride, long long sc_bstride, cudaStream_t st, KvPaging pg = KvPaging());
// The same split with the lengths read on the device from dstate = [cache_len, total_len]
// (CUDA-graph decode: one captured launch serves every step). The grid and the caller-owned
// scratch (attention_split_scratch_bytes(B*S*Hq, max_keys) bytes) are sized for max_keys keys;
// blocks past the live length return at once. attention_split_prepare sets the kernels'
// shared-memory limits for max_keys (call it before any stream capture).
size_t attention_split_scratch_bytes(long long items, long long max_keys);
int attention_split_prepare(int D, int Hq, int Hkv, long long max_keys);
int launch_attention_split_dev(const __half* q, const int8_t* kc, const int8_t* vc, const float* ks, const float* vs,
                               const __half* kn, const __half* vn, __half* o, int B, int S, int new_len, int Hq,
                               int Hkv, int D, float scale, int causal, int qgs, long long kc_bstride,
                               long long sc_bstride, long long max_keys, const int* dstate, float* scratch,
                               size_t scratch_bytes, cudaStream_t st, KvPaging pg = KvPaging());

// ---- sampling (sample.cu)
int launch_sample(const __half* logits, int V, float temperature, float top_p, int top_k, float uniform,
                  const uint32_t* history, int n_history, __half* work, uint32_t* out, cudaStream_t st);
int launch_entropy(const __half* logits, int V, float* out, cudaStream_t st);

// ---- RoPE tables (abi.cu): fp16 cos/sin [n_pos, head_dim/2] built on the host with the
// reference formula and cached on the current device.
bool rope_tables(float theta, int head_dim, long long n_pos, const __half** ct, const __half** st);

}  // namespace cb
