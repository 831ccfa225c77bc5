// Kernels of the other model families on the reference's path: the LFM2 causal depthwise
// convolution, the Whisper front-end conv1d with kernel size 3, and layernorm. Each output
// element keeps the reference's operation order, so results are bit-identical to it:
//  * cactus_conv1d_causal_depthwise_f16 (kernel_conv.cpp:15-110): four fp32 lane
//    accumulators take the taps of every 8-tap block (lane j: taps k+j then k+4+j, as two
//    vfmaq_f32), the lanes fold as vaddvq_f32 ((l0 + l1) + (l2 + l3)), the remaining taps are
//    added one at a time as fused multiply-adds, skipping positions before the sequence start;
//  * cactus_conv1d_f16_k3 (kernel_conv.cpp:112-227): three lane chains (taps t-1, t, t+1)
//    over the input channels in order, folded as (l0 + l2) + (l1 + l3) with lane 3 zero;
//  * compute_layernorm_node (graph_ops_nn.cpp:373-457): in-order fp32 sums for the mean and
//    the variance (diff*diff fused, as the reference's compilers contract it), then
//    fp16(fma((x - mean) * inv, w, b)) with inv = 1 / sqrt(var + eps).
// One thread per output element for the convolutions (the channel index is the fastest one in
// memory, so neighbouring threads read neighbouring inputs). Layernorm: one warp per row; the
// row is staged in shared memory with 16-byte loads, lane 0 runs the two sequential sums and
// all lanes write the normalised row.
#include "common.cuh"
#include "ops.h"

namespace cb {

namespace {

// output [N, L, C], element index e = (n * L + t) * C + c
__global__ void conv1d_causal_depthwise_kernel(const __half* __restrict__ x, const __half* __restrict__ w,
                                               __half* __restrict__ y, long long total, int L, int C, int K,
                                               int dil) {
    pdl_launch_dependents();
    pdl_wait();
    const long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= total) return;
    const int c = (int)(e % C);
    const long long nt = e / C;
    const int t = (int)(nt % L);
    const __half* xb = x + (nt - t) * C + c;  // sequence n, channel c: element t' at xb[t' * C]
    const __half* wc = w + (size_t)c * K;     // tap k uses wc[K - 1 - k]
    float lane[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    int k = 0;
    for (; k + 8 <= K; k += 8) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int kk = k + 4 * h + j;
                const int a = t - kk * dil;
                const float xv = a >= 0 ? h2f(xb[(size_t)a * C]) : 0.0f;
                lane[j] = fmaf(xv, h2f(wc[K - 1 - kk]), lane[j]);
            }
        }
    }
    float acc = __fadd_rn(__fadd_rn(lane[0], lane[1]), __fadd_rn(lane[2], lane[3]));
    for (; k < K; ++k) {
        const int a = t - k * dil;
        if (a >= 0) acc = fmaf(h2f(wc[K - 1 - k]), h2f(xb[(size_t)a * C]), acc);
    }
    y[e] = __float2half_rn(acc);
}

// input [N, C_in, L], weight [C_out, C_in, 3], output [N, C_out, out_len]; e = (n * C_out + oc) * out_len + o
__global__ void conv1d_k3_kernel(const __half* __restrict__ x, const __half* __restrict__ w, __half* __restrict__ y,
                                 long long total, int L, int Cin, int Cout, int stride, int out_len) {
    pdl_launch_dependents();
    pdl_wait();
    const long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= total) return;
    const int o = (int)(e % out_len);
    const long long noc = e / out_len;
    const int oc = (int)(noc % Cout);
    const long long n = noc / Cout;
    const int t = o * stride;
    const __half* xn = x + (size_t)n * Cin * L;
    const __half* wo = w + (size_t)oc * Cin * 3;
    float l0 = 0.0f, l1 = 0.0f, l2 = 0.0f;  // lane 3 multiplies zeros and stays +0
    for (int ic = 0; ic < Cin; ++ic) {
        const __half* xc = xn + (size_t)ic * L;
        const float xm = t >= 1 ? h2f(xc[t - 1]) : 0.0f;
        const float x0 = h2f(xc[t]);
        const float xp = t + 1 < L ? h2f(xc[t + 1]) : 0.0f;
        l0 = fmaf(xm, h2f(wo[3 * ic]), l0);
        l1 = fmaf(x0, h2f(wo[3 * ic + 1]), l1);
        l2 = fmaf(xp, h2f(wo[3 * ic + 2]), l2);
    }
    y[e] = __float2half_rn(__fadd_rn(__fadd_rn(l0, l2), __fadd_rn(l1, 0.0f)));
}

constexpr int kLnWarps = 4;  // rows per block

// one warp per row; smem: kLnWarps rows of F floats
__global__ void __launch_bounds__(kLnWarps * 32) layernorm_kernel(const __half* __restrict__ x,
                                                                  const __half* __restrict__ w,
                                                                  const __half* __restrict__ b,
                                                                  __half* __restrict__ y, int rows, int F,
                                                                  float eps) {
    pdl_launch_dependents();
    pdl_wait();
    extern __shared__ float lnrow[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long long r = (long long)blockIdx.x * kLnWarps + warp;
    if (r >= rows) return;
    float* xs = lnrow + (size_t)warp * F;
    const __half* xr = x + r * F;
    if ((F & 7) == 0 && (reinterpret_cast<uintptr_t>(xr) & 15) == 0) {
        for (int i = lane; i < F / 8; i += 32) {
            const int4 v = __ldg(reinterpret_cast<const int4*>(xr) + i);
            const __half* h = reinterpret_cast<const __half*>(&v);
#pragma unroll
            for (int j = 0; j < 8; ++j) xs[8 * i + j] = h2f(h[j]);
        }
    } else {
        for (int i = lane; i < F; i += 32) xs[i] = h2f(xr[i]);
    }
    __syncwarp();
    float mean = 0.0f, inv = 0.0f;
    if (lane == 0) {
        float s = 0.0f;
        for (int i = 0; i < F; ++i) s = __fadd_rn(s, xs[i]);
        mean = __fdiv_rn(s, (float)F);
        float var = 0.0f;
        for (int i = 0; i < F; ++i) {
            const float d = __fsub_rn(xs[i], mean);
            var = fmaf(d, d, var);
        }
        var = __fdiv_rn(var, (float)F);
        inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
    }
    mean = __shfl_sync(0xffffffffu, mean, 0);
    inv = __shfl_sync(0xffffffffu, inv, 0);
    __half* yr = y + r * F;
    for (int i = lane; i < F; i += 32)
        yr[i] = __float2half_rn(fmaf(__fmul_rn(__fsub_rn(xs[i], mean), inv), h2f(w[i]), h2f(b[i])));
}

inline unsigned nblk(long long n, int t) { return (unsigned)((n + t - 1) / t); }

}  // namespace

int launch_conv1d_causal_depthwise(const __half* x, const __half* w, __half* y, int N, int L, int C, int K, int dil,
                                   cudaStream_t st) {
    const long long total = (long long)N * L * C;
    return launch_k(conv1d_causal_depthwise_kernel, dim3(nblk(total, 256)), dim3(256), 0, st, x, w, y, total, L, C, K,
                    dil) == cudaSuccess ? 0 : -1;
}

int launch_conv1d_k3(const __half* x, const __half* w, __half* y, int N, int L, int Cin, int Cout, int stride,
                     cudaStream_t st) {
    const int out_len = (L - 1) / stride + 1;
    const long long total = (long long)N * Cout * out_len;
    return launch_k(conv1d_k3_kernel, dim3(nblk(total, 256)), dim3(256), 0, st, x, w, y, total, L, Cin, Cout, stride,
                    out_len) == cudaSuccess ? 0 : -1;
}

int layernorm_max_features() { return 227 * 1024 / (kLnWarps * 4); }

int launch_layernorm(const __half* x, const __half* w, const __half* b, __half* y, int rows, int F, float eps,
                     cudaStream_t st) {
    const size_t smem = (size_t)kLnWarps * F * sizeof(float);
    if (smem > 48 * 1024) {
        static size_t enabled = 0;
        if (smem > enabled) {
            if (cudaFuncSetAttribute(layernorm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
                cudaSuccess)
                return -1;
            enabled = smem;
        }
    }
    return launch_k(layernorm_kernel, dim3(nblk(rows, kLnWarps)), dim3(kLnWarps * 32), smem, st, x, w, b, y, rows, F,
                    eps) == cudaSuccess ? 0 : -1;
}

}  // namespace cb
