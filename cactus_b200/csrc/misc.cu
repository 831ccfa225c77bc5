// Elementwise, normalisation, RoPE, KV-quantisation, softmax, embedding and argmax
// kernels (sm_100a). Each kernel states the reference function whose arithmetic it
// reproduces; see common.cuh for the rounding conventions.
#include "common.cuh"
#include "gemv.cuh"
#include "ops.h"

namespace cb {

__device__ unsigned g_dev_error = 0;

unsigned* dev_error_ptr() {
    static unsigned* p = [] {
        void* a = nullptr;
        return cudaGetSymbolAddress(&a, g_dev_error) == cudaSuccess ? static_cast<unsigned*>(a) : nullptr;
    }();
    return p;
}

// ------------------------------------------------------------------ activation quantization
// graph_ops_nn.cpp:35-66: per row absmax -> scale = max(absmax/127, 1e-10) -> int8 (RNE).
__global__ void quantize_act_kernel(const __half* __restrict__ x, int8_t* __restrict__ q, float* __restrict__ scales,
                                    int K) {
    pdl_launch_dependents();
    pdl_wait();
    const int m = blockIdx.x;
    const __half* xm = x + (size_t)m * K;
    __shared__ float red[33];
    float mx = 0.0f;
    for (int k = threadIdx.x; k < K; k += blockDim.x) mx = fmaxf(mx, fabsf(h2f(xm[k])));
    mx = warp_max(mx);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
    __syncthreads();
    if (threadIdx.x < 32) {
        float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0f;
        v = warp_max(v);
        if (threadIdx.x == 0) red[32] = v;
    }
    __syncthreads();
    float scale = __fdiv_rn(red[32], 127.0f);
    if (scale < 1e-10f) scale = 1e-10f;
    const float inv = __fdiv_rn(1.0f, scale);
    const int vec_end = (K / 8) * 8;
    for (int k = threadIdx.x; k < K; k += blockDim.x) q[(size_t)m * K + k] = quant_act(h2f(xm[k]), inv, k < vec_end);
    if (threadIdx.x == 0) scales[m] = scale;
}

// ------------------------------------------------------------------ RMSNorm (kernel_attention.cpp:484-563)
__global__ void rms_norm_kernel(const __half* __restrict__ x, const __half* __restrict__ w, __half* __restrict__ y,
                                int dims, float eps) {
    pdl_launch_dependents();
    pdl_wait();
    extern __shared__ __align__(16) uint8_t sm[];
    __half* xs = reinterpret_cast<__half*>(sm);
    __shared__ float ssum;
    const size_t r = blockIdx.x;
    for (int k = threadIdx.x; k < dims; k += blockDim.x) xs[k] = x[r * dims + k];
    __syncthreads();
    if (threadIdx.x < 32) {
        float ss = rms_sumsq_warp(xs, dims);
        if (threadIdx.x == 0) ssum = ss;
    }
    __syncthreads();
    const float rms = __fsqrt_rn(__fadd_rn(__fdiv_rn(ssum, (float)dims), eps));
    const float inv = __fdiv_rn(1.0f, rms);
    const __half inv16 = __float2half_rn(inv);
    const int vec_end = dims >= 8 ? (dims / 8) * 8 : 0;
    for (int k = threadIdx.x; k < dims; k += blockDim.x) {
        __half v = xs[k];
        y[r * dims + k] = (k < vec_end) ? __hmul(__hmul(v, inv16), w[k])
                                        : __float2half_rn(__fmul_rn(__fmul_rn(h2f(v), inv), h2f(w[k])));
    }
}

// ------------------------------------------------------------------ RoPE (kernel_attention.cpp:614-676)
// One thread per (token, head, i < D/2) rotation pair; cos/sin come from the fp16 tables
// that the host builds with the reference's formula (cactus_rope_tables()).
__global__ void rope_kernel(const __half* __restrict__ in, __half* __restrict__ out, const __half* __restrict__ ct,
                            const __half* __restrict__ st, long long total_pairs, int seq_len, int num_heads,
                            int head_dim, long long start_pos) {
    pdl_launch_dependents();
    pdl_wait();
    const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= total_pairs) return;
    const int half = head_dim / 2;
    const int i = (int)(idx % half);
    const long long row = idx / half;  // (b*S + s)*H + h
    const int s = (int)((row / num_heads) % seq_len);
    const long long pos = start_pos + s;
    const __half* xr = in + row * head_dim;
    __half* yr = out + row * head_dim;
    const __half c = ct[pos * half + i], sn = st[pos * half + i];
    const __half x1 = xr[i], x2 = xr[i + half];
    const int vec_half = (half / 8) * 8;
    if (i < vec_half) {
        yr[i] = __hfma(__hneg(x2), sn, __hmul(x1, c));
        yr[i + half] = __hfma(x1, sn, __hmul(x2, c));
    } else {
        const float f1 = h2f(x1), f2 = h2f(x2), fc = h2f(c), fs = h2f(sn);
        yr[i] = f2h(__fsub_rn(__fmul_rn(f1, fc), __fmul_rn(f2, fs)));
        yr[i + half] = f2h(__fadd_rn(__fmul_rn(f2, fc), __fmul_rn(f1, fs)));
    }
}

// ------------------------------------------------------------------ KV quantisation (kernel_quants.cpp:223-293)
// One warp per (token*head, group): absmax -> scale -> RNE quantisation of the vector part.
__global__ void quantize_kv_kernel(const __half* __restrict__ src, int8_t* __restrict__ dst, float* __restrict__ scales,
                                   long long rows, int head_dim, int G) {
    pdl_launch_dependents();
    pdl_wait();
    const int ng = (head_dim + G - 1) / G;
    const long long wid = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (wid >= rows * ng) return;
    const long long row = wid / ng;
    const int g = (int)(wid % ng);
    const int g0 = g * G;
    const int cnt = min(G, head_dim - g0);
    const __half* hs = src + row * head_dim + g0;
    float mx = 0.0f;
    for (int k = lane; k < cnt; k += 32) mx = fmaxf(mx, fabsf(h2f(hs[k])));
    mx = warp_max(mx);
    float scale = __fdiv_rn(mx, 127.0f);
    if (scale < 1e-10f) scale = 1e-10f;
    const float inv = __fdiv_rn(1.0f, scale);
    const int vec = (cnt / 8) * 8;
    for (int k = lane; k < cnt; k += 32) {
        const float v = __fmul_rn(h2f(hs[k]), inv);
        dst[row * head_dim + g0 + k] = (int8_t)sat8(k < vec ? cvt_rne_sat(v) : (int)roundf(v));
    }
    if (lane == 0) scales[row * ng + g] = scale;
}

// ------------------------------------------------------------------ elementwise
// Vector-path semantics for the first (n/8)*8 elements, scalar-tail semantics after.
__global__ void silu_kernel(const __half* __restrict__ x, __half* __restrict__ y, long long n) {
    pdl_launch_dependents();
    pdl_wait();
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    if (i < (n / 8) * 8) {
        y[i] = ref_silu(x[i]);
    } else {
        const float v = h2f(x[i]);
        y[i] = f2h(__fmul_rn(v, __fdiv_rn(1.0f, __fadd_rn(1.0f, expf_cr(-v)))));
    }
}
__global__ void gelu_kernel(const __half* __restrict__ x, __half* __restrict__ y, long long n) {
    pdl_launch_dependents();
    pdl_wait();
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    if (i < (n / 8) * 8) {
        y[i] = ref_gelu(x[i]);
    } else {
        const float v = h2f(x[i]);
        const float inner = __fmul_rn(0.7978845608028654f, fmaf(__fmul_rn(__fmul_rn(0.044715f, v), v), v, v));
        y[i] = f2h(__fmul_rn(__fmul_rn(0.5f, v), __fadd_rn(1.0f, tanhf_cr(inner))));
    }
}
// op: 0 add, 1 add clipped (fp32 add, clamp +-65500), 2 multiply
__global__ void binary_kernel(const __half* __restrict__ a, const __half* __restrict__ b, __half* __restrict__ y,
                              long long n, int op) {
    pdl_launch_dependents();
    pdl_wait();
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    if (op == 0) {
        y[i] = __hadd(a[i], b[i]);
    } else if (op == 1) {
        float r = __fadd_rn(h2f(a[i]), h2f(b[i]));
        r = fminf(fmaxf(r, -65500.0f), 65500.0f);
        y[i] = f2h(r);
    } else {
        y[i] = __hmul(a[i], b[i]);
    }
}
__global__ void scalar_mul_kernel(const __half* __restrict__ x, __half* __restrict__ y, long long n, __half s) {
    pdl_launch_dependents();
    pdl_wait();
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) y[i] = __hmul(x[i], s);
}

// ------------------------------------------------------------------ softmax (kernel_nn.cpp:152-251)
// One warp per row. Lane e owns the reference's accumulator for offset e of every 32-wide
// chunk, so the fp32 sum follows the NEON lane order exactly.
__global__ void softmax_kernel(const __half* __restrict__ x, __half* __restrict__ y, int rows, int V) {
    pdl_launch_dependents();
    pdl_wait();
    const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    const __half* in = x + (size_t)row * V;
    __half* out = y + (size_t)row * V;
    float mx = -INFINITY;
    for (int i = lane; i < V; i += 32) mx = fmaxf(mx, h2f(in[i]));
    mx = warp_max(mx);
    const int vv = (V / 32) * 32;
    float acc = 0.0f;
    for (int i = lane; i < vv; i += 32) {
        const float e = ref_fast_exp(__fsub_rn(h2f(in[i]), mx));
        out[i] = f2h(e);
        acc = __fadd_rn(acc, e);
    }
    // lane l (0..3): acc[l] + acc[4+l] + ... + acc[28+l], sequentially
    float s = __shfl_sync(0xffffffffu, acc, lane & 3);
    for (int u = 1; u < 8; ++u) s = __fadd_rn(s, __shfl_sync(0xffffffffu, acc, 4 * u + (lane & 3)));
    const float l0 = __shfl_sync(0xffffffffu, s, 0), l1 = __shfl_sync(0xffffffffu, s, 1);
    const float l2 = __shfl_sync(0xffffffffu, s, 2), l3 = __shfl_sync(0xffffffffu, s, 3);
    float sum = __fadd_rn(__fadd_rn(l0, l1), __fadd_rn(l2, l3));
    for (int i = vv; i < V; ++i) {  // scalar tail, in order (identical on all lanes)
        const float e = expf_cr(__fsub_rn(h2f(in[i]), mx));
        if (lane == 0) out[i] = f2h(e);
        sum = __fadd_rn(sum, e);
    }
    __syncwarp();
    const float inv = __fdiv_rn(1.0f, sum);
    const __half inv16 = __float2half_rn(inv);
    for (int i = lane; i < vv; i += 32) out[i] = __hmul(out[i], inv16);
    for (int i = vv + lane; i < V; i += 32) out[i] = f2h(__fmul_rn(h2f(out[i]), inv));
}

// ------------------------------------------------------------------ embedding (graph_ops_tensor.cpp:226-331)
__global__ void embedding_int8_kernel(const int8_t* __restrict__ table, const __half* __restrict__ scales, int G,
                                      int ng, int hidden, const uint32_t* __restrict__ ids, int n_ids,
                                      __half* __restrict__ out) {
    pdl_launch_dependents();
    pdl_wait();
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)n_ids * hidden) return;
    const int t = (int)(i / hidden), k = (int)(i % hidden);
    const size_t row = ids[t];
    out[i] = f2h(__fmul_rn((float)table[row * hidden + k], h2f(scales[row * ng + k / G])));
}
__global__ void embedding_f16_kernel(const __half* __restrict__ table, int hidden, const uint32_t* __restrict__ ids,
                                     int n_ids, __half* __restrict__ out) {
    pdl_launch_dependents();
    pdl_wait();
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)n_ids * hidden) return;
    const int t = (int)(i / hidden), k = (int)(i % hidden);
    out[i] = table[(size_t)ids[t] * hidden + k];
}

// ------------------------------------------------------------------ argmax (kernel_nn.cpp:451-467)
// Keys order by (value, then lower index): the first maximum wins as with the strict '>'.
__device__ __forceinline__ unsigned long long argmax_key(float v, unsigned idx) {
    if (v != v) return 0ull;  // NaN never compares greater
    unsigned u = __float_as_uint(v);
    u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((unsigned long long)u << 32) | (0xFFFFFFFFu - idx);
}
__global__ void argmax_kernel(const __half* __restrict__ logits, int V, uint32_t* __restrict__ out) {
    pdl_launch_dependents();
    pdl_wait();
    __shared__ unsigned long long red[32];
    unsigned long long best = 0ull;
    int i0 = 0;
    if ((reinterpret_cast<uintptr_t>(logits) & 15) == 0) {
        // 16-byte loads of 8 logits, four in flight per thread; the maximum key is the first
        // maximum whatever the scan order
        const int n8 = V / 8;
        const int4* l8 = reinterpret_cast<const int4*>(logits);
#pragma unroll 4
        for (int c = threadIdx.x; c < n8; c += blockDim.x) {
            const int4 q = __ldg(l8 + c);
            const __half* h = reinterpret_cast<const __half*>(&q);
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const unsigned long long k = argmax_key(h2f(h[e]), (unsigned)(8 * c + e));
                best = k > best ? k : best;
            }
        }
        i0 = n8 * 8;
    }
    for (int i = i0 + threadIdx.x; i < V; i += blockDim.x) {
        const unsigned long long k = argmax_key(h2f(logits[i]), (unsigned)i);
        best = k > best ? k : best;
    }
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long k = __shfl_xor_sync(0xffffffffu, best, o);
        best = k > best ? k : best;
    }
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = best;
    __syncthreads();
    if (threadIdx.x < 32) {
        best = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0ull;
        for (int o = 16; o > 0; o >>= 1) {
            const unsigned long long k = __shfl_xor_sync(0xffffffffu, best, o);
            best = k > best ? k : best;
        }
        if (threadIdx.x == 0) out[0] = best == 0ull ? 0u : 0xFFFFFFFFu - (unsigned)(best & 0xFFFFFFFFull);
    }
}

// ------------------------------------------------------------------ INT4 unpack (kernel_quants.cpp:295-351)
__global__ void unpack_int4_kernel(const uint8_t* __restrict__ p, int8_t* __restrict__ o, long long count) {
    pdl_launch_dependents();
    pdl_wait();
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= count) return;
    const uint8_t b = p[i >> 1];
    int v = (i & 1) ? (b >> 4) : (b & 0x0F);
    o[i] = (int8_t)((v & 8) ? v - 16 : v);
}

// ------------------------------------------------------------------ 2-D transpose (kernel_blas.cpp:407-493)
// 32x32 tiles through shared memory (one padding column against bank conflicts); rows and
// columns both read and written coalesced.
__global__ void transpose_2d_kernel(const uint16_t* __restrict__ src, uint16_t* __restrict__ dst, long long rows,
                                    long long cols) {
    pdl_launch_dependents();
    pdl_wait();
    __shared__ uint16_t tile[32][33];
    const long long r0 = (long long)blockIdx.y * 32, c0 = (long long)blockIdx.x * 32;
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
        const long long r = r0 + i, c = c0 + threadIdx.x;
        if (r < rows && c < cols) tile[i][threadIdx.x] = src[r * cols + c];
    }
    __syncthreads();
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
        const long long c = c0 + i, r = r0 + threadIdx.x;
        if (r < rows && c < cols) dst[c * rows + r] = tile[threadIdx.x][i];
    }
}

// ------------------------------------------------------------------ FP16 matmul (kernel_gemm.cpp:17-126)
// fp16 accumulation in the reference's 8 lanes: thread j of an 8-thread group owns lane j of
// one output and performs the same sequence of fp16 FMAs; the lanes are folded with the
// reference's fp16 horizontal-sum tree (kernel_gemm.cpp:8-15).
__global__ void matmul_f16_kernel(const __half* __restrict__ A, const __half* __restrict__ Bt, __half* __restrict__ C,
                                  int M, int K, int N) {
    pdl_launch_dependents();
    pdl_wait();
    const int j = threadIdx.x & 7;
    const long long n = (long long)blockIdx.x * (blockDim.x >> 3) + (threadIdx.x >> 3);
    const bool valid = n < N;
    const int K16 = (K / 16) * 16, K8 = (K / 8) * 8;
    const __half* b = Bt + (valid ? n : 0) * (long long)K;
    for (int m = 0; m < M; ++m) {
        const __half* a = A + (size_t)m * K;
        __half acc = __float2half_rn(0.0f);
        if (valid) {
            for (int k = 0; k < K16; k += 16) {
                acc = __hfma(a[k + j], b[k + j], acc);
                acc = __hfma(a[k + 8 + j], b[k + 8 + j], acc);
            }
            for (int k = K16; k < K8; k += 8) acc = __hfma(a[k + j], b[k + j], acc);
            if (j == 0)
                for (int k = K8; k < K; ++k) acc = f2h(fmaf(h2f(a[k]), h2f(b[k]), h2f(acc)));
        }
        // hsum: lo+hi, then (0+2),(1+3), then (0)+(1)
        __half t = __hadd(acc, __shfl_down_sync(0xffffffffu, acc, 4, 8));
        __half u = __hadd(t, __shfl_down_sync(0xffffffffu, t, 2, 8));
        __half v = __hadd(u, __shfl_down_sync(0xffffffffu, u, 1, 8));
        if (valid && j == 0) C[(size_t)m * N + n] = v;
    }
}

// Few-row variant (M <= 8, K % 8 == 0): one thread per output column n computes all 8 fp16
// lanes of the reference's accumulators itself, as four half2 FMAs per 8-element chunk (each
// lane one fp16 fused multiply-add with a single rounding, in the reference's k order), so
// the weight row streams as 16-byte loads. Lanes fold with the same hsum tree. The A rows
// sit in shared memory and every thread reads them as broadcasts.
template <int MR>
__global__ void __launch_bounds__(256) matmul_f16_rows_kernel(const __half* __restrict__ A,
                                                              const __half* __restrict__ Bt, __half* __restrict__ C,
                                                              int M, int K, int N) {
    pdl_launch_dependents();
    extern __shared__ __align__(16) uint8_t smem_f16[];
    __half* sa = reinterpret_cast<__half*>(smem_f16);
    pdl_wait();
    {
        const int4* a4 = reinterpret_cast<const int4*>(A);
        int4* s4 = reinterpret_cast<int4*>(sa);
        for (int i = threadIdx.x; i < M * K / 8; i += blockDim.x) s4[i] = __ldg(a4 + i);
    }
    __syncthreads();
    const long long n = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (n >= N) return;
    const __half* b = Bt + n * (long long)K;
    const int K16 = (K / 16) * 16, K8 = (K / 8) * 8;
    __half2 acc[MR][4];
#pragma unroll
    for (int m = 0; m < MR; ++m)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[m][i] = __float2half2_rn(0.0f);
#pragma unroll 4
    for (int k = 0; k < K16; k += 16) {
        const int4 blo = __ldg(reinterpret_cast<const int4*>(b + k));
        const int4 bhi = __ldg(reinterpret_cast<const int4*>(b + k + 8));
        const __half2* bl = reinterpret_cast<const __half2*>(&blo);
        const __half2* bh = reinterpret_cast<const __half2*>(&bhi);
#pragma unroll
        for (int m = 0; m < MR; ++m) {
            if (m < M) {
                const int4 alo = *reinterpret_cast<const int4*>(sa + m * K + k);
                const int4 ahi = *reinterpret_cast<const int4*>(sa + m * K + k + 8);
                const __half2* al = reinterpret_cast<const __half2*>(&alo);
                const __half2* ah = reinterpret_cast<const __half2*>(&ahi);
#pragma unroll
                for (int i = 0; i < 4; ++i) acc[m][i] = __hfma2(al[i], bl[i], acc[m][i]);
#pragma unroll
                for (int i = 0; i < 4; ++i) acc[m][i] = __hfma2(ah[i], bh[i], acc[m][i]);
            }
        }
    }
    if (K8 > K16) {
        const int4 bv = __ldg(reinterpret_cast<const int4*>(b + K16));
        const __half2* bp = reinterpret_cast<const __half2*>(&bv);
#pragma unroll
        for (int m = 0; m < MR; ++m) {
            if (m < M) {
                const int4 av = *reinterpret_cast<const int4*>(sa + m * K + K16);
                const __half2* ap = reinterpret_cast<const __half2*>(&av);
#pragma unroll
                for (int i = 0; i < 4; ++i) acc[m][i] = __hfma2(ap[i], bp[i], acc[m][i]);
            }
        }
    }
#pragma unroll
    for (int m = 0; m < MR; ++m) {
        if (m < M) {
            // hsum_f16x8 (kernel_gemm.cpp:8-15): lanes (i, i+4), then (0+2, 1+3), then 0+1
            const __half2 s01 = __hadd2(acc[m][0], acc[m][2]);  // (l0+l4, l1+l5)
            const __half2 s23 = __hadd2(acc[m][1], acc[m][3]);  // (l2+l6, l3+l7)
            const __half2 u = __hadd2(s01, s23);
            C[(size_t)m * N + n] = __hadd(__low2half(u), __high2half(u));
        }
    }
}

}  // namespace cb

// ==================================================================== host launchers
namespace cb {

static inline unsigned nblocks(long long n, int t) { return (unsigned)((n + t - 1) / t); }

int launch_quantize_act(const __half* x, int8_t* q, float* s, int M, int K, cudaStream_t st) {
    launch_k(quantize_act_kernel, dim3(M), dim3(256), 0, st, x, q, s, K);
    return 0;
}
int launch_rms_norm(const __half* x, const __half* w, __half* y, int rows, int dims, float eps, cudaStream_t st) {
    const size_t sm = (size_t)dims * 2;
    if (sm > 48 * 1024) cudaFuncSetAttribute(rms_norm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
    launch_k(rms_norm_kernel, dim3(rows), dim3(256), sm, st, x, w, y, dims, eps);
    return 0;
}
int launch_rope(const __half* in, __half* out, const __half* ct, const __half* stab, long long rows, int seq_len,
                int heads, int head_dim, long long start_pos, cudaStream_t st) {
    const long long pairs = rows * (head_dim / 2);
    launch_k(rope_kernel, dim3(nblocks(pairs, 256)), dim3(256), 0, st, in, out, ct, stab, pairs, seq_len, heads, head_dim, start_pos);
    return 0;
}
int launch_quantize_kv(const __half* src, int8_t* dst, float* scales, long long rows, int head_dim, int G,
                       cudaStream_t st) {
    const int ng = (head_dim + G - 1) / G;
    launch_k(quantize_kv_kernel, dim3(nblocks(rows * ng * 32, 256)), dim3(256), 0, st, src, dst, scales, rows, head_dim, G);
    return 0;
}
int launch_silu(const __half* x, __half* y, long long n, cudaStream_t st) {
    launch_k(silu_kernel, dim3(nblocks(n, 256)), dim3(256), 0, st, x, y, n);
    return 0;
}
int launch_gelu(const __half* x, __half* y, long long n, cudaStream_t st) {
    launch_k(gelu_kernel, dim3(nblocks(n, 256)), dim3(256), 0, st, x, y, n);
    return 0;
}
int launch_binary(const __half* a, const __half* b, __half* y, long long n, int op, cudaStream_t st) {
    launch_k(binary_kernel, dim3(nblocks(n, 256)), dim3(256), 0, st, a, b, y, n, op);
    return 0;
}
int launch_scalar_mul(const __half* x, __half* y, long long n, float s, cudaStream_t st) {
    launch_k(scalar_mul_kernel, dim3(nblocks(n, 256)), dim3(256), 0, st, x, y, n, __float2half_rn(s));
    return 0;
}
int launch_softmax(const __half* x, __half* y, int rows, int V, cudaStream_t st) {
    launch_k(softmax_kernel, dim3(nblocks((long long)rows * 32, 128)), dim3(128), 0, st, x, y, rows, V);
    return 0;
}
int launch_embedding_int8(const int8_t* t, const __half* s, int G, int hidden, const uint32_t* ids, int n,
                          __half* out, cudaStream_t st) {
    launch_k(embedding_int8_kernel, dim3(nblocks((long long)n * hidden, 256)), dim3(256), 0, st, t, s, G, hidden / G, hidden, ids, n, out);
    return 0;
}
int launch_embedding_f16(const __half* t, int hidden, const uint32_t* ids, int n, __half* out, cudaStream_t st) {
    launch_k(embedding_f16_kernel, dim3(nblocks((long long)n * hidden, 256)), dim3(256), 0, st, t, hidden, ids, n, out);
    return 0;
}
int launch_argmax(const __half* logits, int V, uint32_t* out, cudaStream_t st) {
    launch_k(argmax_kernel, dim3(1), dim3(1024), 0, st, logits, V, out);
    return 0;
}
int launch_transpose_2d(const uint16_t* src, uint16_t* dst, long long rows, long long cols, cudaStream_t st) {
    if (rows == 0 || cols == 0) return 0;
    launch_k(transpose_2d_kernel, dim3((unsigned)((cols + 31) / 32), (unsigned)((rows + 31) / 32)), dim3(32, 8), 0, st,
             src, dst, rows, cols);
    return 0;
}

int launch_unpack_int4(const uint8_t* p, int8_t* o, long long count, cudaStream_t st) {
    launch_k(unpack_int4_kernel, dim3(nblocks(count, 256)), dim3(256), 0, st, p, o, count);
    return 0;
}
int launch_matmul_f16(const __half* A, const __half* Bt, __half* C, int M, int K, int N, cudaStream_t st) {
    // few rows with 16-byte aligned weight rows and no scalar K tail: the row-streaming kernel
    if (M <= 8 && K % 8 == 0 && (size_t)M * K * 2 <= 48 * 1024) {
        const dim3 grid(nblocks(N, 256)), block(256);
        const size_t sm = (size_t)M * K * 2;
        if (M == 1) launch_k(matmul_f16_rows_kernel<1>, grid, block, sm, st, A, Bt, C, M, K, N);
        else if (M <= 2) launch_k(matmul_f16_rows_kernel<2>, grid, block, sm, st, A, Bt, C, M, K, N);
        else if (M <= 4) launch_k(matmul_f16_rows_kernel<4>, grid, block, sm, st, A, Bt, C, M, K, N);
        else launch_k(matmul_f16_rows_kernel<8>, grid, block, sm, st, A, Bt, C, M, K, N);
        return 0;
    }
    launch_k(matmul_f16_kernel, dim3(nblocks((long long)N * 8, 256)), dim3(256), 0, st, A, Bt, C, M, K, N);
    return 0;
}

}  // namespace cb
