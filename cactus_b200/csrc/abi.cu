// extern "C" entry points declared in include/cactus_b200.h: argument checks, then the
// launchers of gemv.cu / misc.cu / attention.cu. No entry point throws; failures return a
// negative code and leave a message for cactus_cuda_last_error().
#include <cmath>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/cactus_b200.h"
#include "common.cuh"
#include "ops.h"

namespace {
thread_local std::string g_last_error;

int fail(int code, const std::string& msg) {
    g_last_error = msg;
    return code;
}
int check_launch(const char* what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(CB_ERR_LAUNCH, std::string(what) + ": " + cudaGetErrorString(e));
    return CB_OK;
}
inline cudaStream_t S(void* s) { return reinterpret_cast<cudaStream_t>(s); }
inline const __half* H(const uint16_t* p) { return reinterpret_cast<const __half*>(p); }
inline __half* H(uint16_t* p) { return reinterpret_cast<__half*>(p); }
inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }
constexpr size_t kIntMax = 0x7fffffff;

// fp16 bits of a float, round to nearest even (host side)
uint16_t host_f2h(float f) { return __half_as_ushort(__float2half_rn(f)); }

struct RopeTable {
    long long n_pos = 0;
    __half* cos_t = nullptr;
    __half* sin_t = nullptr;
};
std::mutex g_rope_mu;
std::map<std::tuple<int, uint32_t, int>, RopeTable> g_rope;  // (device, theta bits, head_dim)
}  // namespace

namespace cb {
bool& pdl_flag() {
    static thread_local bool f = false;
    return f;
}

// Tables are built with the reference formula (kernel_attention.cpp:580-610):
// freq_i = 1 / powf(theta, (2i)/head_dim), angle = pos * freq_i, cos/sin rounded to fp16.
// They only grow (old tables stay allocated) so pointers handed to queued kernels stay valid.
bool rope_tables(float theta, int head_dim, long long n_pos, const __half** ct, const __half** st) {
    int dev = 0;
    cudaGetDevice(&dev);
    uint32_t tb;
    std::memcpy(&tb, &theta, 4);
    std::lock_guard<std::mutex> lk(g_rope_mu);
    RopeTable& t = g_rope[std::make_tuple(dev, tb, head_dim)];
    if (t.n_pos < n_pos) {
        long long np = n_pos < 4096 ? 4096 : n_pos;
        if (t.n_pos > 0 && np < 2 * t.n_pos) np = 2 * t.n_pos;
        const int half = head_dim / 2;
        std::vector<uint16_t> hc((size_t)np * half), hs((size_t)np * half);
        for (long long pos = 0; pos < np; ++pos) {
            const float pf = (float)pos;
            for (int i = 0; i < half; ++i) {
                const float freq = 1.0f / powf(theta, (2.0f * (float)i) / (float)head_dim);
                const float angle = pf * freq;
                hc[(size_t)pos * half + i] = host_f2h(cosf(angle));
                hs[(size_t)pos * half + i] = host_f2h(sinf(angle));
            }
        }
        __half *dc = nullptr, *ds = nullptr;
        if (cudaMalloc(&dc, hc.size() * 2) != cudaSuccess) return false;
        if (cudaMalloc(&ds, hs.size() * 2) != cudaSuccess) return false;
        if (cudaMemcpy(dc, hc.data(), hc.size() * 2, cudaMemcpyHostToDevice) != cudaSuccess) return false;
        if (cudaMemcpy(ds, hs.data(), hs.size() * 2, cudaMemcpyHostToDevice) != cudaSuccess) return false;
        t.n_pos = np;
        t.cos_t = dc;
        t.sin_t = ds;
    }
    *ct = t.cos_t;
    *st = t.sin_t;
    return true;
}
}  // namespace cb

extern "C" {

CB_API const char* cactus_cuda_last_error(void) { return g_last_error.c_str(); }

CB_API unsigned cactus_cuda_device_error(void* stream) {
    unsigned v = 0, zero = 0;
    cudaStreamSynchronize(S(stream));
    cudaMemcpyFromSymbol(&v, cb::g_dev_error, sizeof(v));
    cudaMemcpyToSymbol(cb::g_dev_error, &zero, sizeof(zero));
    return v;
}

CB_API int cactus_cuda_version(void) { return 1; }

CB_API int cactus_cuda_quantize_activations(const uint16_t* x, int8_t* q, float* scales, size_t M, size_t K,
                                            void* stream) {
    if (M == 0 || K == 0) return CB_OK;
    if (M > kIntMax || K > kIntMax) return fail(CB_ERR_ARG, "quantize_activations: size too large");
    cb::launch_quantize_act(H(x), q, scales, (int)M, (int)K, S(stream));
    return check_launch("quantize_activations");
}

static int gemv_or_chunks(cb::GemvCall c, size_t M, size_t K, size_t N, size_t G, const char* name,
                          cudaStream_t st) {
    if (M == 0 || K == 0 || N == 0) return CB_OK;
    if (G == 0) return fail(CB_ERR_ARG, std::string(name) + ": group_size must be > 0");
    if (K > kIntMax || N > kIntMax || M > kIntMax) return fail(CB_ERR_ARG, std::string(name) + ": size too large");
    c.K = (int)K;
    c.N = (int)N;
    c.G = (int)G;
    // rows beyond one launch's limit (8, fewer for very large K) are processed in chunks
    // (the weights are re-read from L2)
    const size_t per = (size_t)cb::gemv_rows_per_launch(c.int4, c.pro, c.K, c.G);
    if (per == 0) return fail(CB_ERR_ARG, std::string(name) + ": gemv: K too large for the shared-memory tile");
    for (size_t m0 = 0; m0 < M; m0 += per) {
        cb::GemvCall cc = c;
        cc.M = (int)((M - m0) < per ? (M - m0) : per);
        if (cc.x) cc.x = c.x + m0 * K;
        if (cc.aq) cc.aq = c.aq + m0 * K;
        if (cc.as) cc.as = c.as + m0;
        cc.out = c.out + m0 * N;
        if (const char* why = cb::gemv_check(cc)) return fail(CB_ERR_ARG, std::string(name) + ": " + why);
        if (cb::launch_gemv(cc, st) != 0) {
            const int e = check_launch(name);
            return e ? e : fail(CB_ERR_LAUNCH, std::string(name) + ": launch failed");
        }
    }
    return check_launch(name);
}

// ---- M >= 16 rows: the tensor-core GEMM (gemm.cu), same result bits as the GEMV
// Grow-only per-device scratch for the quantised activations of linear_* calls (old buffers
// stay allocated so kernels already queued on other streams keep valid pointers).
namespace {
std::mutex g_gemm_mu;
std::map<int, std::pair<void*, size_t>> g_gemm_scratch;
void* gemm_scratch(size_t bytes) {
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lk(g_gemm_mu);
    auto& e = g_gemm_scratch[dev];
    if (e.second < bytes) {
        void* p = nullptr;
        if (cudaMalloc(&p, bytes) != cudaSuccess) {
            cudaGetLastError();
            return nullptr;
        }
        e = {p, bytes};
    }
    return e.first;
}

// the GEMM stages rows with 16-byte copies and the scales with 8-byte copies
bool use_gemm(size_t M, size_t K, size_t N, size_t G, int int4, const void* A, const void* B, const void* Bs) {
    return M >= (size_t)cb::kGemmMinRows && M <= kIntMax && K <= kIntMax && N <= kIntMax && G <= kIntMax &&
           cb::gemm_check((int)M, (int)K, (int)N, (int)G, int4) == nullptr && (!A || aligned16(A)) &&
           aligned16(B) && (reinterpret_cast<uintptr_t>(Bs) & 7) == 0;
}

int gemm_preq(const int8_t* A, const float* As, const void* B, const uint16_t* Bs, uint16_t* C, size_t M, size_t K,
              size_t N, size_t G, int int4, const char* name, cudaStream_t st) {
    if (cb::launch_gemm(A, As, B, H(Bs), H(C), nullptr, (int)M, (int)K, (int)N, (int)G, int4, cb::kEpiStore, st) != 0)
        return fail(CB_ERR_LAUNCH, std::string(name) + ": gemm launch failed");
    return check_launch(name);
}

int gemm_linear(const uint16_t* X, const void* B, const uint16_t* Bs, uint16_t* C, size_t M, size_t K, size_t N,
                size_t G, int int4, const char* name, cudaStream_t st) {
    const size_t qbytes = (M * K + 255) / 256 * 256;
    uint8_t* scratch = static_cast<uint8_t*>(gemm_scratch(qbytes + M * 4));
    if (!scratch) return fail(CB_ERR_LAUNCH, std::string(name) + ": scratch allocation failed");
    int8_t* aq = reinterpret_cast<int8_t*>(scratch);
    float* as = reinterpret_cast<float*>(scratch + qbytes);
    cb::launch_quantize_act(H(X), aq, as, (int)M, (int)K, st);
    return gemm_preq(aq, as, B, Bs, C, M, K, N, G, int4, name, st);
}
}  // namespace

CB_API int cactus_cuda_matmul_int8(const int8_t* A, const float* A_scales, const int8_t* B, const uint16_t* B_scales,
                                   uint16_t* C, size_t M, size_t K, size_t N, size_t group_size, void* stream) {
    if (use_gemm(M, K, N, group_size, 0, A, B, B_scales))
        return gemm_preq(A, A_scales, B, B_scales, C, M, K, N, group_size, 0, "matmul_int8", S(stream));
    cb::GemvCall c = {};
    c.int4 = 0;
    c.pro = cb::kProPreq;
    c.epi = cb::kEpiStore;
    c.aq = A;
    c.as = A_scales;
    c.w = B;
    c.ws = H(B_scales);
    c.out = H(C);
    return gemv_or_chunks(c, M, K, N, group_size, "matmul_int8", S(stream));
}

CB_API int cactus_cuda_matmul_int4(const int8_t* A, const float* A_scales, const uint8_t* B_packed,
                                   const uint16_t* B_scales, uint16_t* C, size_t M, size_t K, size_t N,
                                   size_t group_size, void* stream) {
    if (use_gemm(M, K, N, group_size, 1, A, B_packed, B_scales))
        return gemm_preq(A, A_scales, B_packed, B_scales, C, M, K, N, group_size, 1, "matmul_int4", S(stream));
    cb::GemvCall c = {};
    c.int4 = 1;
    c.pro = cb::kProPreq;
    c.epi = cb::kEpiStore;
    c.aq = A;
    c.as = A_scales;
    c.w = B_packed;
    c.ws = H(B_scales);
    c.out = H(C);
    return gemv_or_chunks(c, M, K, N, group_size, "matmul_int4", S(stream));
}

CB_API int cactus_cuda_linear_int8(const uint16_t* X, const int8_t* B, const uint16_t* B_scales, uint16_t* C, size_t M,
                                   size_t K, size_t N, size_t group_size, void* stream) {
    if (use_gemm(M, K, N, group_size, 0, nullptr, B, B_scales))
        return gemm_linear(X, B, B_scales, C, M, K, N, group_size, 0, "linear_int8", S(stream));
    cb::GemvCall c = {};
    c.int4 = 0;
    c.pro = cb::kProQuant;
    c.epi = cb::kEpiStore;
    c.x = H(X);
    c.w = B;
    c.ws = H(B_scales);
    c.out = H(C);
    return gemv_or_chunks(c, M, K, N, group_size, "linear_int8", S(stream));
}

CB_API int cactus_cuda_linear_int4(const uint16_t* X, const uint8_t* B_packed, const uint16_t* B_scales, uint16_t* C,
                                   size_t M, size_t K, size_t N, size_t group_size, void* stream) {
    if (use_gemm(M, K, N, group_size, 1, nullptr, B_packed, B_scales))
        return gemm_linear(X, B_packed, B_scales, C, M, K, N, group_size, 1, "linear_int4", S(stream));
    cb::GemvCall c = {};
    c.int4 = 1;
    c.pro = cb::kProQuant;
    c.epi = cb::kEpiStore;
    c.x = H(X);
    c.w = B_packed;
    c.ws = H(B_scales);
    c.out = H(C);
    return gemv_or_chunks(c, M, K, N, group_size, "linear_int4", S(stream));
}

CB_API int cactus_cuda_matmul_f16(const uint16_t* A, const uint16_t* B_transposed, uint16_t* C, size_t M, size_t K,
                                  size_t N, void* stream) {
    if (M == 0 || K == 0 || N == 0) return CB_OK;
    if (M > kIntMax || K > kIntMax || N > kIntMax) return fail(CB_ERR_ARG, "matmul_f16: size too large");
    cb::launch_matmul_f16(H(A), H(B_transposed), H(C), (int)M, (int)K, (int)N, S(stream));
    return check_launch("matmul_f16");
}

CB_API int cactus_cuda_rms_norm_f16(const uint16_t* input, const uint16_t* weight, uint16_t* output, size_t batch_size,
                                    size_t dims, float eps, void* stream) {
    if (batch_size == 0 || dims == 0) return CB_OK;
    if (dims * 2 > 200 * 1024) return fail(CB_ERR_ARG, "rms_norm: dims too large");
    cb::launch_rms_norm(H(input), H(weight), H(output), (int)batch_size, (int)dims, eps, S(stream));
    return check_launch("rms_norm_f16");
}

CB_API int cactus_cuda_conv1d_causal_depthwise_f16(const uint16_t* input, const uint16_t* weight, uint16_t* output,
                                                   size_t N, size_t L, size_t C, size_t K, size_t dilation,
                                                   void* stream) {
    if (N == 0 || L == 0 || C == 0) return CB_OK;
    if (K == 0 || dilation == 0) return fail(CB_ERR_ARG, "conv1d_causal_depthwise: kernel size and dilation must be >= 1");
    if (N * L * C > (size_t)1 << 40 || L > kIntMax || C > kIntMax || K > kIntMax || (K - 1) * dilation > kIntMax)
        return fail(CB_ERR_ARG, "conv1d_causal_depthwise: size too large");
    cb::launch_conv1d_causal_depthwise(H(input), H(weight), H(output), (int)N, (int)L, (int)C, (int)K, (int)dilation,
                                       S(stream));
    return check_launch("conv1d_causal_depthwise_f16");
}

CB_API int cactus_cuda_conv1d_f16_k3(const uint16_t* input, const uint16_t* weight, uint16_t* output, size_t N,
                                     size_t L, size_t C_in, size_t C_out, size_t stride, void* stream) {
    if (N == 0 || L == 0 || C_out == 0) return CB_OK;
    if (stride == 0) return fail(CB_ERR_ARG, "conv1d_k3: stride must be >= 1");
    if (L > kIntMax || C_in > kIntMax || C_out > kIntMax || N * C_out * L > (size_t)1 << 40)
        return fail(CB_ERR_ARG, "conv1d_k3: size too large");
    cb::launch_conv1d_k3(H(input), H(weight), H(output), (int)N, (int)L, (int)C_in, (int)C_out, (int)stride, S(stream));
    return check_launch("conv1d_f16_k3");
}

CB_API int cactus_cuda_layernorm_f16(const uint16_t* input, const uint16_t* weight, const uint16_t* bias,
                                     uint16_t* output, size_t rows, size_t features, float eps, void* stream) {
    if (rows == 0) return CB_OK;
    if (features == 0 || features > (size_t)cb::layernorm_max_features())
        return fail(CB_ERR_ARG, "layernorm: feature count out of range");
    if (rows > kIntMax) return fail(CB_ERR_ARG, "layernorm: too many rows");
    cb::launch_layernorm(H(input), H(weight), H(bias), H(output), (int)rows, (int)features, eps, S(stream));
    return check_launch("layernorm_f16");
}

CB_API int cactus_cuda_rope_f16(const uint16_t* input, uint16_t* output, size_t batch_size, size_t seq_len,
                                size_t num_heads, size_t head_dim, size_t start_pos, float theta, void* stream) {
    if (batch_size == 0 || seq_len == 0 || num_heads == 0) return CB_OK;
    if (head_dim == 0 || (head_dim & 1)) return fail(CB_ERR_ARG, "rope: head_dim must be even");
    const __half *ct = nullptr, *st = nullptr;
    if (!cb::rope_tables(theta, (int)head_dim, (long long)(start_pos + seq_len), &ct, &st))
        return fail(CB_ERR_LAUNCH, "rope: table allocation failed");
    cb::launch_rope(H(input), H(output), ct, st, (long long)(batch_size * seq_len * num_heads), (int)seq_len,
                    (int)num_heads, (int)head_dim, (long long)start_pos, S(stream));
    return check_launch("rope_f16");
}

static const char* attn_dims_check(size_t Hq, size_t Hkv, size_t D) {
    if (Hq == 0 || Hkv == 0 || Hq % Hkv) return "num_q_heads must be a positive multiple of num_kv_heads";
    if (D == 0 || D > 256) return "head_dim must be in [1, 256]";
    return nullptr;
}

CB_API int cactus_cuda_attention_f16(const uint16_t* queries, const uint16_t* keys, const uint16_t* values,
                                     uint16_t* output, size_t batch_size, size_t seq_len, size_t kv_seq_len,
                                     size_t num_q_heads, size_t num_kv_heads, size_t head_dim, float scale,
                                     size_t position_offset, size_t window_size, int is_causal, void* stream) {
    if (batch_size == 0 || seq_len == 0) return CB_OK;
    if (const char* why = attn_dims_check(num_q_heads, num_kv_heads, head_dim))
        return fail(CB_ERR_ARG, std::string("attention_f16: ") + why);
    if (!aligned16(keys) || !aligned16(values)) return fail(CB_ERR_ARG, "attention_f16: K/V must be 16-byte aligned");
    if (scale == 0.0f) scale = 1.0f / sqrtf((float)head_dim);
    cb::launch_attention_f16(H(queries), H(keys), H(values), H(output), (int)batch_size, (int)seq_len, (int)kv_seq_len,
                             (int)num_q_heads, (int)num_kv_heads, (int)head_dim, scale, (long long)position_offset,
                             (long long)window_size, is_causal, S(stream));
    return check_launch("attention_f16");
}

CB_API int cactus_cuda_attention_hybrid_int8_fp16(const uint16_t* queries, const int8_t* keys_cached,
                                                  const int8_t* values_cached, const float* k_scales,
                                                  const float* v_scales, const uint16_t* keys_new,
                                                  const uint16_t* values_new, uint16_t* output, size_t batch_size,
                                                  size_t seq_len, size_t cache_len, size_t new_len,
                                                  size_t num_q_heads, size_t num_kv_heads, size_t head_dim,
                                                  float scale, size_t position_offset, int is_causal,
                                                  size_t quant_group_size, void* stream) {
    if (batch_size == 0 || seq_len == 0) return CB_OK;
    if (const char* why = attn_dims_check(num_q_heads, num_kv_heads, head_dim))
        return fail(CB_ERR_ARG, std::string("attention_hybrid: ") + why);
    if (head_dim % 32) return fail(CB_ERR_UNSUPPORTED, "attention_hybrid: head_dim must be a multiple of 32");
    if (quant_group_size == 0 || quant_group_size % 8) return fail(CB_ERR_ARG, "attention_hybrid: bad quant group");
    if (!aligned16(keys_new) || !aligned16(values_new) || (reinterpret_cast<uintptr_t>(keys_cached) & 7) ||
        (reinterpret_cast<uintptr_t>(values_cached) & 7))
        return fail(CB_ERR_ARG, "attention_hybrid: misaligned K/V");
    if (scale == 0.0f) scale = 1.0f / sqrtf((float)head_dim);
    // The reference order (bit-exact): long caches split over the keys inside
    // launch_attention_hybrid_exact; the non-exact kernel only when neither exact path takes
    // the shape.
    const long long kc_bs = (long long)(cache_len * num_kv_heads * head_dim);
    // the exact kernels stage cached rows with 16-byte copies
    const bool rows16 = aligned16(keys_cached) && aligned16(values_cached);
    if (!rows16 || cb::launch_attention_hybrid_exact(H(queries), keys_cached, values_cached, k_scales, v_scales,
                                                     H(keys_new), H(values_new), H(output), (int)batch_size,
                                                     (int)seq_len, (int)cache_len, (int)new_len, (int)num_q_heads,
                                                     (int)num_kv_heads, (int)head_dim, scale,
                                                     (long long)position_offset, is_causal, (int)quant_group_size,
                                                     kc_bs, 0, S(stream)) != 0)
        cb::launch_attention_hybrid(H(queries), keys_cached, values_cached, k_scales, v_scales, H(keys_new),
                                    H(values_new), H(output), (int)batch_size, (int)seq_len, (int)cache_len,
                                    (int)new_len, (int)num_q_heads, (int)num_kv_heads, (int)head_dim, scale,
                                    (long long)position_offset, is_causal, (int)quant_group_size, kc_bs, 0,
                                    S(stream));
    return check_launch("attention_hybrid_int8_fp16");
}

CB_API int cactus_cuda_quantize_kv_fp16_to_int8(const uint16_t* src, int8_t* dst, float* scales, size_t seq_len,
                                                size_t kv_heads, size_t head_dim, size_t group_size, void* stream) {
    if (seq_len == 0 || kv_heads == 0 || head_dim == 0) return CB_OK;
    if (group_size == 0) return fail(CB_ERR_ARG, "quantize_kv: group_size must be > 0");
    cb::launch_quantize_kv(H(src), dst, scales, (long long)(seq_len * kv_heads), (int)head_dim, (int)group_size,
                           S(stream));
    return check_launch("quantize_kv");
}

CB_API int cactus_cuda_silu_f16(const uint16_t* input, uint16_t* output, size_t n, void* stream) {
    if (!n) return CB_OK;
    cb::launch_silu(H(input), H(output), (long long)n, S(stream));
    return check_launch("silu_f16");
}
CB_API int cactus_cuda_gelu_f16(const uint16_t* input, uint16_t* output, size_t n, void* stream) {
    if (!n) return CB_OK;
    cb::launch_gelu(H(input), H(output), (long long)n, S(stream));
    return check_launch("gelu_f16");
}
CB_API int cactus_cuda_add_f16(const uint16_t* a, const uint16_t* b, uint16_t* out, size_t n, void* stream) {
    if (!n) return CB_OK;
    cb::launch_binary(H(a), H(b), H(out), (long long)n, 0, S(stream));
    return check_launch("add_f16");
}
CB_API int cactus_cuda_add_f16_clipped(const uint16_t* a, const uint16_t* b, uint16_t* out, size_t n, void* stream) {
    if (!n) return CB_OK;
    cb::launch_binary(H(a), H(b), H(out), (long long)n, 1, S(stream));
    return check_launch("add_f16_clipped");
}
CB_API int cactus_cuda_multiply_f16(const uint16_t* a, const uint16_t* b, uint16_t* out, size_t n, void* stream) {
    if (!n) return CB_OK;
    cb::launch_binary(H(a), H(b), H(out), (long long)n, 2, S(stream));
    return check_launch("multiply_f16");
}
CB_API int cactus_cuda_scalar_multiply_f16(const uint16_t* input, uint16_t* output, size_t n, float scalar,
                                           void* stream) {
    if (!n) return CB_OK;
    cb::launch_scalar_mul(H(input), H(output), (long long)n, scalar, S(stream));
    return check_launch("scalar_multiply_f16");
}
CB_API int cactus_cuda_softmax_f16(const uint16_t* input, uint16_t* output, size_t rows, size_t vocab, void* stream) {
    if (!rows || !vocab) return CB_OK;
    cb::launch_softmax(H(input), H(output), (int)rows, (int)vocab, S(stream));
    return check_launch("softmax_f16");
}
CB_API int cactus_cuda_embedding_int8(const int8_t* table, const uint16_t* scales, size_t group_size, size_t vocab,
                                      size_t hidden, const uint32_t* ids, size_t n_ids, uint16_t* out, void* stream) {
    (void)vocab;
    if (!n_ids) return CB_OK;
    if (group_size == 0 || hidden % group_size) return fail(CB_ERR_ARG, "embedding_int8: hidden % group_size != 0");
    cb::launch_embedding_int8(table, H(scales), (int)group_size, (int)hidden, ids, (int)n_ids, H(out), S(stream));
    return check_launch("embedding_int8");
}
CB_API int cactus_cuda_embedding_f16(const uint16_t* table, size_t vocab, size_t hidden, const uint32_t* ids,
                                     size_t n_ids, uint16_t* out, void* stream) {
    (void)vocab;
    if (!n_ids) return CB_OK;
    cb::launch_embedding_f16(H(table), (int)hidden, ids, (int)n_ids, H(out), S(stream));
    return check_launch("embedding_f16");
}
CB_API int cactus_cuda_argmax_f16(const uint16_t* logits, size_t rows, size_t vocab, uint32_t* out_index,
                                  void* stream) {
    if (rows == 0) return fail(CB_ERR_ARG, "argmax: no rows");
    if (vocab == 0) {
        cudaMemsetAsync(out_index, 0, 4, S(stream));
        return check_launch("argmax_f16");
    }
    cb::launch_argmax(H(logits) + (rows - 1) * vocab, (int)vocab, out_index, S(stream));
    return check_launch("argmax_f16");
}
CB_API int cactus_cuda_sample_f16(const uint16_t* logits, size_t rows, size_t vocab, float temperature, float top_p,
                                  size_t top_k, float uniform, const uint32_t* history, size_t n_history,
                                  uint16_t* work, uint32_t* out_index, void* stream) {
    if (rows == 0 || vocab == 0) return fail(CB_ERR_ARG, "sample: empty logits");
    const uint16_t* last = logits + (rows - 1) * vocab;
    if (temperature == 0.0f && top_p <= 0.0f && top_k == 0) {
        cb::launch_argmax(H(last), (int)vocab, out_index, S(stream));
        return check_launch("sample_f16");
    }
    if (!work) return fail(CB_ERR_ARG, "sample: scratch buffer required");
    cb::launch_sample(H(last), (int)vocab, temperature, top_p, (int)top_k, uniform, history, (int)n_history, H(work),
                      out_index, S(stream));
    return check_launch("sample_f16");
}

// ---- sampling without caller scratch: the filtered-logits buffer is a fixed file-scope
// device array (one per device and per loaded copy of this library); nothing is allocated.
namespace {
constexpr size_t kStaticSampleVocab = 262144;  // largest vocabulary of the supported models
__device__ __align__(256) uint16_t g_sample_scratch[kStaticSampleVocab];
constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
void* g_scratch_ptr[kMaxDevices] = {};
unsigned long long g_scratch_ctx[kMaxDevices] = {};  // id of the context the address belongs to

// Unique id of the calling thread's current context (cuCtxGetId, reached through the
// runtime's driver entry points so the library does not link libcuda). A device reset
// creates a new context with a new id, which invalidates a resolved symbol address.
bool current_context_id(unsigned long long* id) {
    using get_cur_t = int (*)(void**);
    using get_id_t = int (*)(void*, unsigned long long*);
    static get_cur_t get_cur = nullptr;
    static get_id_t get_id = nullptr;
    if (!get_cur || !get_id) {
        void* f1 = nullptr;
        void* f2 = nullptr;
        cudaDriverEntryPointQueryResult q1, q2;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f1, cudaEnableDefault, &q1) != cudaSuccess ||
            cudaGetDriverEntryPoint("cuCtxGetId", &f2, cudaEnableDefault, &q2) != cudaSuccess || !f1 || !f2) {
            cudaGetLastError();
            return false;
        }
        get_cur = reinterpret_cast<get_cur_t>(f1);
        get_id = reinterpret_cast<get_id_t>(f2);
    }
    void* ctx = nullptr;
    if (get_cur(&ctx) != 0 || !ctx) return false;
    return get_id(ctx, id) == 0;
}
}  // namespace

CB_API int cactus_cuda_sample_f16_noalloc(const uint16_t* logits, size_t rows, size_t vocab, float temperature,
                                          float top_p, size_t top_k, float uniform, const uint32_t* history,
                                          size_t n_history, uint32_t* out_index, void* stream) {
    if (rows == 0 || vocab == 0) return fail(CB_ERR_ARG, "sample_noalloc: empty logits");
    if (vocab > kStaticSampleVocab)
        return fail(CB_ERR_ARG, "sample_noalloc: vocab " + std::to_string(vocab) + " exceeds the static scratch of " +
                                    std::to_string(kStaticSampleVocab) + " entries");
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        cudaGetLastError();
        return fail(CB_ERR_LAUNCH, "sample_noalloc: no usable current device");
    }
    void* scratch = nullptr;
    {
        // set-up on the first call per device (and again after a device reset replaced the
        // context): resolve the array's address with the device current
        std::lock_guard<std::mutex> lk(g_scratch_mu);
        if (g_scratch_ptr[dev]) {
            unsigned long long ctx = 0;
            if (!current_context_id(&ctx) || ctx != g_scratch_ctx[dev]) g_scratch_ptr[dev] = nullptr;
        }
        if (!g_scratch_ptr[dev]) {
            void* p = nullptr;
            const cudaError_t e = cudaGetSymbolAddress(&p, g_sample_scratch);
            if (e != cudaSuccess || !p) {
                cudaGetLastError();
                return fail(CB_ERR_LAUNCH, std::string("sample_noalloc: cudaGetSymbolAddress failed: ") +
                                               cudaGetErrorString(e));
            }
            unsigned long long ctx = 0;
            if (!current_context_id(&ctx))
                return fail(CB_ERR_LAUNCH, "sample_noalloc: cannot identify the current CUDA context");
            g_scratch_ptr[dev] = p;
            g_scratch_ctx[dev] = ctx;
        }
        scratch = g_scratch_ptr[dev];
    }
    return cactus_cuda_sample_f16(logits, rows, vocab, temperature, top_p, top_k, uniform, history, n_history,
                                  static_cast<uint16_t*>(scratch), out_index, stream);
}

CB_API int cactus_cuda_entropy_f16(const uint16_t* logits, size_t rows, size_t vocab, float* out, void* stream) {
    if (rows == 0 || vocab == 0) return fail(CB_ERR_ARG, "entropy: empty logits");
    cb::launch_entropy(H(logits) + (rows - 1) * vocab, (int)vocab, out, S(stream));
    return check_launch("entropy_f16");
}

CB_API int cactus_cuda_unpack_int4_to_int8(const uint8_t* packed, int8_t* unpacked, size_t count, void* stream) {
    if (!count) return CB_OK;
    cb::launch_unpack_int4(packed, unpacked, (long long)count, S(stream));
    return check_launch("unpack_int4");
}

CB_API int cactus_cuda_transpose_2d_f16(const uint16_t* source, uint16_t* destination, size_t num_rows,
                                        size_t num_cols, void* stream) {
    if (!source || !destination) return fail(CB_ERR_ARG, "transpose_2d: null pointer");
    cb::launch_transpose_2d(source, destination, (long long)num_rows, (long long)num_cols, S(stream));
    return check_launch("transpose_2d_f16");
}

}  // extern "C"
