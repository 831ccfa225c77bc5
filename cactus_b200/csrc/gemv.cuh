// Grouped INT8 / INT4 weight GEMV for small M (decode), sm_100a.
//
// Replaces cactus_matmul_int8 (kernel_gemm.cpp:128-327) and cactus_matmul_int4
// (kernel_gemm.cpp:329-529) together with the activation quantization that
// compute_matmul_node runs first (graph_ops_nn.cpp:35-66, 150-209).
//
// Arithmetic (bit-exact with the reference semantics):
//   A_q[m,:] = sat8(rne(x[m,:] * (1 / s_m))),  s_m = max(absmax(x[m,:]) / 127, 1e-10)
//   C[m,n]   = fp16( fma-chain_g( float(sum_{k in g} A_q[m,k] * B[n,k]), float(Bs[n,g]) ) * s_m )
// with the group sums exact in int32 and the fp32 chain over groups in ascending g.
//
// Data path: weights are row-major [N, K] (int8) or [N, K/2] (int4, low nibble = even k)
// with fp16 scales [N, K/G]. A CTA owns tiles of R = 8*RPW consecutive rows; each tile's
// weight bytes and scales are contiguous in HBM and arrive in shared memory through one
// 1-D TMA bulk copy each (cp.async.bulk, no multicast) into an S-stage mbarrier ring.
// Weight copies are issued before griddepcontrol.wait, so under programmatic dependent
// launch they stream while the producer of the activations is still finishing.
#pragma once
#include "common.cuh"

namespace cb {

enum class WFmt : int { I8 = 0, I4 = 1 };
enum class Pro : int { PREQ = 0, QUANT = 1, RMSNORM_QUANT = 2 };
enum class Epi : int { STORE = 0, RESIDUAL = 1, GLU_SILU = 2, GLU_GELU = 3 };

struct GemvArgs {
    const __half* x;       // QUANT / RMSNORM_QUANT: fp16 activations [M, K]
    const __half* norm_w;  // RMSNORM_QUANT: [K]
    float eps;
    const int8_t* aq;  // PREQ: int8 activations [M, K]
    const float* as;   // PREQ: per-row scales [M]
    const void* w;     // [N, K] int8 or [N, K/2] uint8
    const __half* ws;  // [N, K/G]
    __half* out;       // STORE/RESIDUAL: [M, N]; GLU: [M, N/2]
    const __half* resid;  // RESIDUAL: [M, N] (may alias out)
    int8_t* aq_out;    // optional: block 0 writes the quantized activations here
    float* as_out;     // optional
    int M, K, N, G;
    int S;  // pipeline stages (>= 2)
};

constexpr int kGemvThreads = 256;
constexpr int kGemvWarps = kGemvThreads / 32;
constexpr int kGemvRedSq = 64;  // prologue scratch: per-warp maxima below, sums of squares from here

struct GemvLayout {
    int R, wrow, ng, stage_w, stage_s, stage_bytes, S, gpj, pairs;
    int off_act, off_asum, off_as, off_xs, off_stage, off_bar, off_gs, off_out, total;
};

__host__ __device__ inline int align_up(int v, int a) { return (v + a - 1) / a * a; }

__host__ __device__ inline GemvLayout gemv_layout(int wf, int MT, int RPW, int S, int pro, int K, int G) {
    GemvLayout L;
    L.R = 8 * RPW;
    L.wrow = wf == 0 ? K : K / 2;
    L.ng = K / G;
    L.stage_w = L.R * L.wrow;
    L.stage_s = L.R * L.ng * 2;
    L.stage_bytes = align_up(L.stage_w + align_up(L.stage_s, 16), 128);
    L.S = S;
    L.gpj = wf == 0 ? 512 / G : 1024 / G;  // groups covered by one 32-lane pass
    if (L.gpj < 1) L.gpj = 1;
    L.pairs = RPW * MT;
    int off = 0;
    L.off_act = off;   off += align_up(MT * K, 128);
    L.off_asum = off;  off += align_up(MT * L.ng * 4, 128);
    L.off_as = off;    off += align_up(MT * 4, 16) + 112;
    L.off_xs = off;    off += (pro != 0) ? align_up(MT * K * 2, 128) : 0;
    L.off_stage = off; off += S * L.stage_bytes;
    L.off_bar = off;   off += align_up(S * 8, 16) + 16;
    L.off_gs = off;    off += align_up(L.R * MT * 33 * 4, 16) > 512 ? align_up(L.R * MT * 33 * 4, 16) : 512;
    off = align_up(off, 16);
    L.off_out = off;   off += 2 * L.R * MT * 2;
    L.total = align_up(off, 128);
    return L;
}

// ------------------------------------------------------------------ prologue helpers
// Bit-exact restatement of cactus_rms_norm_f16's reduction (kernel_attention.cpp:496-540):
// 16 lane accumulators over 16-element tiles, an 8-element tail tile into lanes 0..7, the
// fixed combine tree and a scalar tail. Runs on one warp; result broadcast to all lanes.
__device__ __forceinline__ float rms_sumsq_warp(const __half* xs, int K) {
    const int lane = threadIdx.x & 31, l16 = lane & 15;
    float acc = 0.0f;
    // lane l (< 16) accumulates elements l, l + 16, ... of the full 16-element tiles in
    // order; loads are batched 8 tiles at a time so only the FMA chain is sequential (lanes
    // 16..31 mirror lanes 0..15 and are ignored by the fold below)
    const int ntiles = K / 16;
    int tt = 0;
    for (; tt + 8 <= ntiles; tt += 8) {
        float v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = h2f(xs[(tt + j) * 16 + l16]);
#pragma unroll
        for (int j = 0; j < 8; ++j) acc = fmaf(v[j], v[j], acc);
    }
    for (; tt < ntiles; ++tt) {
        const float v = h2f(xs[tt * 16 + l16]);
        acc = fmaf(v, v, acc);
    }
    int i = ntiles * 16;
    const int simd_end = K >= 8 ? K - 8 + 1 : 0;
    if (i < simd_end) {
        if (lane < 8) { float v = h2f(xs[i + lane]); acc = fmaf(v, v, acc); }
        i += 8;
    }
    float a4 = __shfl_sync(0xffffffffu, acc, (lane & 3) + 4);
    float a8 = __shfl_sync(0xffffffffu, acc, (lane & 3) + 8);
    float a12 = __shfl_sync(0xffffffffu, acc, (lane & 3) + 12);
    float a0 = __shfl_sync(0xffffffffu, acc, lane & 3);
    float t = __fadd_rn(__fadd_rn(__fadd_rn(a0, a4), a8), a12);
    float t0 = __shfl_sync(0xffffffffu, t, 0), t1 = __shfl_sync(0xffffffffu, t, 1);
    float t2 = __shfl_sync(0xffffffffu, t, 2), t3 = __shfl_sync(0xffffffffu, t, 3);
    float ss = __fadd_rn(__fadd_rn(t0, t1), __fadd_rn(t2, t3));
    for (; i < K; ++i) { float v = h2f(xs[i]); ss = fmaf(v, v, ss); }
    return ss;
}

// Shared-memory load helpers: explicit ld.shared (the compiler cannot always prove a pointer
// is shared inside large kernels and then emits slower generic loads).
__device__ __forceinline__ float lds_h2f(uint32_t saddr) {
    unsigned short u;
    asm volatile("ld.shared.b16 %0, [%1];" : "=h"(u) : "r"(saddr));
    return __half2float(__ushort_as_half(u));
}

// rms_sumsq_warp on a shared-memory address (same operation order).
__device__ __forceinline__ float rms_sumsq_warp_sh(uint32_t xs, int K) {
    const int lane = threadIdx.x & 31, l16 = lane & 15;
    float acc = 0.0f;
    const int ntiles = K / 16;
    int tt = 0;
    for (; tt + 8 <= ntiles; tt += 8) {
        float v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = lds_h2f(xs + 2u * ((tt + j) * 16 + l16));
#pragma unroll
        for (int j = 0; j < 8; ++j) acc = fmaf(v[j], v[j], acc);
    }
    for (; tt < ntiles; ++tt) {
        const float v = lds_h2f(xs + 2u * (tt * 16 + l16));
        acc = fmaf(v, v, acc);
    }
    int i = ntiles * 16;
    const int simd_end = K >= 8 ? K - 8 + 1 : 0;
    if (i < simd_end) {
        if (lane < 8) { float v = lds_h2f(xs + 2u * (i + lane)); acc = fmaf(v, v, acc); }
        i += 8;
    }
    float a4 = __shfl_sync(0xffffffffu, acc, (lane & 3) + 4);
    float a8 = __shfl_sync(0xffffffffu, acc, (lane & 3) + 8);
    float a12 = __shfl_sync(0xffffffffu, acc, (lane & 3) + 12);
    float a0 = __shfl_sync(0xffffffffu, acc, lane & 3);
    float t = __fadd_rn(__fadd_rn(__fadd_rn(a0, a4), a8), a12);
    float t0 = __shfl_sync(0xffffffffu, t, 0), t1 = __shfl_sync(0xffffffffu, t, 1);
    float t2 = __shfl_sync(0xffffffffu, t, 2), t3 = __shfl_sync(0xffffffffu, t, 3);
    float ss = __fadd_rn(__fadd_rn(t0, t1), __fadd_rn(t2, t3));
    for (; i < K; ++i) { float v = lds_h2f(xs + 2u * i); ss = fmaf(v, v, ss); }
    return ss;
}

// Quantize one fp16 value with the reference's activation rule; `vec` selects the
// NEON vector path (RNE after clamping) versus the scalar tail (round half away).
__device__ __forceinline__ int8_t quant_act(float v, float inv, bool vec) {
    float s = __fmul_rn(v, inv);
    s = fmaxf(fminf(s, 127.0f), -128.0f);
    return vec ? (int8_t)sat8(cvt_rne_sat(s)) : (int8_t)(int)roundf(s);
}

// Activation prologue of both GEMV kernels: the M rows of x (or the pre-quantised rows) into
// `act` (int8, [MT][K]; INT4 weights: each 8-element block permuted so that dp4a pairs the even
// and the odd k with the low and the high nibbles), the per-row scales into `as`, and for INT4
// the per-group activation sums into `asum`. `xs` holds MT * K halves, `red` kGemvRedSq + 8
// floats (the per-warp maxima of the NT / 32 warps (MT * NT / 32 <= kGemvRedSq), then the sums
// of squares). Ends with a block barrier.
template <int WF, int MT, int PRO, int NT = kGemvThreads>
__device__ __forceinline__ void gemv_prologue(const GemvArgs& a, int8_t* act, int* asum, float* as, __half* xs,
                                              float* red) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int K = a.K, G = a.G, M = a.M;
    const int ng = K / G;
    if constexpr (PRO == (int)Pro::PREQ) {
        for (int i = tid; i < M * K; i += NT) {
            const int m = i / K, k = i % K;
            int8_t v = a.aq[i];
            if constexpr (WF == 1) {
                const int blk = k >> 3, e = k & 7;
                act[m * K + blk * 8 + ((e & 1) ? 4 + (e >> 1) : (e >> 1))] = v;
            } else {
                act[i] = v;
            }
        }
        if (tid < M) as[tid] = a.as[tid];
        __syncthreads();
    } else {
        // Latency-oriented: one global round trip stages the M rows, warp m reduces row m's
        // sum of squares, then one pass normalises + takes per-warp maxima and one pass
        // quantises (3 block barriers for RMSNorm, 2 otherwise).
        const int vec_end = (K / 8) * 8;
        if ((K & 7) == 0 && (reinterpret_cast<uintptr_t>(a.x) & 15) == 0) {
            const int4* src = reinterpret_cast<const int4*>(a.x);
            int4* dst = reinterpret_cast<int4*>(xs);
            for (int i = tid; i < M * K / 8; i += NT) dst[i] = src[i];
        } else {
            for (int i = tid; i < M * K; i += NT) xs[i] = a.x[i];
        }
        __syncthreads();
        if constexpr (PRO == (int)Pro::RMSNORM_QUANT) {
            if (warp < M) {
                const float ss = rms_sumsq_warp(xs + warp * K, K);
                if (lane == 0) red[kGemvRedSq + warp] = ss;
            }
            __syncthreads();
        }
        for (int m = 0; m < M; ++m) {
            float inv_rms = 0.0f;
            __half inv16 = __float2half_rn(0.0f);
            if constexpr (PRO == (int)Pro::RMSNORM_QUANT) {
                const float rms = __fsqrt_rn(__fadd_rn(__fdiv_rn(red[kGemvRedSq + m], (float)K), a.eps));
                inv_rms = __fdiv_rn(1.0f, rms);
                inv16 = __float2half_rn(inv_rms);
            }
            float mx = 0.0f;
            for (int k = tid; k < K; k += NT) {
                __half v = xs[m * K + k];
                if constexpr (PRO == (int)Pro::RMSNORM_QUANT) {
                    v = (k < vec_end) ? __hmul(__hmul(v, inv16), a.norm_w[k])
                                      : __float2half_rn(__fmul_rn(__fmul_rn(h2f(v), inv_rms), h2f(a.norm_w[k])));
                    xs[m * K + k] = v;
                }
                mx = fmaxf(mx, fabsf(h2f(v)));
            }
            mx = warp_max(mx);
            if (lane == 0) red[m * (NT / 32) + warp] = mx;
        }
        __syncthreads();
        for (int m = 0; m < M; ++m) {
            float mx = red[m * (NT / 32)];
#pragma unroll
            for (int w = 1; w < NT / 32; ++w) mx = fmaxf(mx, red[m * (NT / 32) + w]);
            float scale = __fdiv_rn(mx, 127.0f);
            if (scale < 1e-10f) scale = 1e-10f;
            const float inv = __fdiv_rn(1.0f, scale);
            if (tid == 0) as[m] = scale;
            for (int k = tid; k < K; k += NT) {
                const int8_t q = quant_act(h2f(xs[m * K + k]), inv, k < vec_end);
                if constexpr (WF == 1) {
                    const int blk = k >> 3, e = k & 7;
                    act[m * K + blk * 8 + ((e & 1) ? 4 + (e >> 1) : (e >> 1))] = q;
                } else {
                    act[m * K + k] = q;
                }
                if (a.aq_out && blockIdx.x == 0) a.aq_out[(size_t)m * K + k] = q;
            }
            if (a.as_out && blockIdx.x == 0 && tid == 0) a.as_out[m] = scale;
        }
        __syncthreads();
    }
    if constexpr (WF == 1) {  // per-group activation sums for the unsigned-nibble dot product
        for (int i = tid; i < M * ng; i += NT) {
            const int m = i / ng, g = i % ng;
            int s = 0;
            for (int k = 0; k < G; ++k) s += act[m * K + g * G + k];  // permutation stays inside 8-blocks
            asum[i] = s;
        }
        __syncthreads();
    }

}

template <int WF, int MT, int RPW, int PRO, int EPI>
__global__ void __launch_bounds__(kGemvThreads) qgemv_kernel(GemvArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int S = a.S;
    const GemvLayout L = gemv_layout(WF, MT, RPW, S, PRO, a.K, a.G);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int K = a.K, N = a.N, G = a.G, M = a.M;
    const int R = L.R, ng = L.ng;
    const int ntiles = (N + R - 1) / R;

    int8_t* act = reinterpret_cast<int8_t*>(smem + L.off_act);
    int* asum = reinterpret_cast<int*>(smem + L.off_asum);
    float* as = reinterpret_cast<float*>(smem + L.off_as);
    int* s_abort = reinterpret_cast<int*>(smem + L.off_as + align_up(MT * 4, 16));
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem + L.off_bar);
    int* gsbuf = reinterpret_cast<int*>(smem + L.off_gs) + warp * L.pairs * L.gpj;
    uint16_t* outt = reinterpret_cast<uint16_t*>(smem + L.off_out);

    const uint8_t* wbase = reinterpret_cast<const uint8_t*>(a.w);
    auto issue = [&](int t, int s) {
        uint8_t* st = smem + L.off_stage + s * L.stage_bytes;
        const int rows = min(R, N - t * R);
        const unsigned wb = (unsigned)(rows * L.wrow);
        const unsigned sb_all = (unsigned)(rows * ng * 2);
        const unsigned sb = sb_all & ~15u;
        mbar_arrive_expect_tx(&bar[s], wb + sb);
        tma_load_1d(st, wbase + (size_t)t * R * L.wrow, wb, &bar[s]);
        const uint16_t* sc = reinterpret_cast<const uint16_t*>(a.ws) + (size_t)t * R * ng;
        if (sb) tma_load_1d(st + L.stage_w, sc, sb, &bar[s]);
        for (unsigned i = sb / 2; i < sb_all / 2; ++i)  // sub-16-byte remainder of a partial tile
            reinterpret_cast<uint16_t*>(st + L.stage_w)[i] = sc[i];
    };

    if (tid == 0) {
        *s_abort = 0;
        for (int s = 0; s < S; ++s) mbar_init(&bar[s], 1);
        fence_mbar_init();
    }
    __syncthreads();
    if (tid == 0)
        for (int s = 0; s < S; ++s) {
            const int t = blockIdx.x + s * gridDim.x;
            if (t < ntiles) issue(t, s);
        }
    // Weights are constant: their copies above may overlap the previous kernel.
    pdl_launch_dependents();
    pdl_wait();

    // ---------------------------------------------------------- prologue: activations -> smem int8
    gemv_prologue<WF, MT, PRO>(a, act, asum, as, reinterpret_cast<__half*>(smem + L.off_xs),
                               reinterpret_cast<float*>(smem + L.off_gs));

    // ---------------------------------------------------------- main loop over tiles
    // Per tile and per slice of 32 groups: (1) warps form the exact int32 group sums of their
    // rows (lanes split a row's 16-byte chunks, lanes of one group are folded by shuffles)
    // into gsm[(row*MT + m)*33 + group]; (2) thread t = row*MT + m continues the reference's
    // sequential fp32 chain over those groups. The padded stride 33 keeps both phases free of
    // shared-memory bank conflicts.
    const int cpg = WF == 0 ? G / 16 : G / 32;            // 16-byte weight chunks per group
    const int chunks = K / 16 / (WF == 1 ? 2 : 1);        // 16-byte chunks per row
    const int spc = 32 * cpg;                              // chunks per slice of 32 groups
    const int nslice = (ng + 31) / 32;
    const int npass = (spc + 31) / 32;
    int* gsm = reinterpret_cast<int*>(smem + L.off_gs);
    const int pr = tid / MT, pm = tid % MT;  // chain owner: pair (row pr, activation row pm)
    const bool chain_thread = tid < R * MT && pm < M;
    int it = 0;
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++it) {
        const int s = it % S;
        const unsigned par = (unsigned)((it / S) & 1);
        // one thread polls the stage (a block of spinning threads takes issue slots from the
        // co-resident block); after the barrier every thread checks the completed phase once,
        // which orders its reads of the copied bytes
        if (tid == 0 && !mbar_wait_bounded(&bar[s], par)) {
            report_dev_error(kDevTmaTimeout);
            atomicExch(s_abort, 1);
        }
        __syncthreads();
        if (*s_abort) return;  // uniform across the block
        mbar_wait_bounded(&bar[s], par);
        const uint8_t* st = smem + L.off_stage + s * L.stage_bytes;
        const uint16_t* sc = reinterpret_cast<const uint16_t*>(st + L.stage_w);
        uint16_t* ob = outt + (it & 1) * R * MT;
        const int rows_valid = min(R, N - t * R);

        float run = 0.0f;
        for (int sl = 0; sl < nslice; ++sl) {
            const int c0 = sl * spc;
            const int c1 = min(chunks, c0 + spc);
#pragma unroll
            for (int r = 0; r < RPW; ++r) {
                const int row = warp * RPW + r;
                for (int p = 0; p < npass; ++p) {
                    const int c = c0 + p * 32 + lane;
                    const bool cval = c < c1;
                    int4 wv = make_int4(0, 0, 0, 0);
                    if (cval && row < rows_valid) wv = *reinterpret_cast<const int4*>(st + row * L.wrow + c * 16);
#pragma unroll
                    for (int m = 0; m < MT; ++m) {
                        int acc = 0;
                        if (cval && m < M) {
                            if constexpr (WF == 0) {
                                const int4 av = *reinterpret_cast<const int4*>(act + m * K + c * 16);
                                acc = dp4a_ss(av.x, wv.x, acc);
                                acc = dp4a_ss(av.y, wv.y, acc);
                                acc = dp4a_ss(av.z, wv.z, acc);
                                acc = dp4a_ss(av.w, wv.w, acc);
                            } else {
                                const int4 a0 = *reinterpret_cast<const int4*>(act + m * K + c * 32);
                                const int4 a1 = *reinterpret_cast<const int4*>(act + m * K + c * 32 + 16);
                                const unsigned ww[4] = {(unsigned)wv.x, (unsigned)wv.y, (unsigned)wv.z,
                                                        (unsigned)wv.w};
                                const int ae[4] = {a0.x, a0.z, a1.x, a1.z};
                                const int ao[4] = {a0.y, a0.w, a1.y, a1.w};
#pragma unroll
                                for (int q = 0; q < 4; ++q) {
                                    const unsigned lo = (ww[q] & 0x0F0F0F0Fu) ^ 0x08080808u;
                                    const unsigned hi = ((ww[q] >> 4) & 0x0F0F0F0Fu) ^ 0x08080808u;
                                    acc = dp4a_su(ae[q], lo, acc);
                                    acc = dp4a_su(ao[q], hi, acc);
                                }
                            }
                        }
                        for (int o = 1; o < cpg; o <<= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
                        if ((lane % cpg) == 0 && cval) {
                            const int gl = (c - c0) / cpg;
                            if constexpr (WF == 1) acc -= 8 * asum[m * ng + sl * 32 + gl];
                            gsm[(row * MT + m) * 33 + gl] = acc;
                        }
                    }
                }
            }
            __syncthreads();
            if (chain_thread) {
                const int gcount = min(32, ng - sl * 32);
                const int* gp = gsm + tid * 33;
                const uint16_t* sp = sc + pr * ng + sl * 32;
                if ((ng & 7) == 0 && gcount == 32) {
                    // a row's scales are contiguous: 16-byte loads (one-at-a-time 2-byte loads
                    // across rows ng * 2 bytes apart hit the same banks)
                    const int4* sp4 = reinterpret_cast<const int4*>(sp);
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const int4 sv = sp4[q];
                        const uint16_t* s8 = reinterpret_cast<const uint16_t*>(&sv);
#pragma unroll
                        for (int e = 0; e < 8; ++e) run = fmaf((float)gp[q * 8 + e], h2f_bits(s8[e]), run);
                    }
                } else {
#pragma unroll 8
                    for (int gl = 0; gl < gcount; ++gl) run = fmaf((float)gp[gl], h2f_bits(sp[gl]), run);
                }
            }
            __syncthreads();
        }
        if (chain_thread) ob[pr * MT + pm] = f2h_bits(__fmul_rn(run, as[pm]));
        __syncthreads();
        if (tid == 0) {
            const int tn = t + S * (int)gridDim.x;
            if (tn < ntiles) issue(tn, s);
        }
        // ------------------------------------------------------ epilogue from the smem tile
        if constexpr (EPI == (int)Epi::STORE || EPI == (int)Epi::RESIDUAL) {
            for (int i = tid; i < rows_valid * M; i += kGemvThreads) {
                const int m = i / rows_valid, row = i % rows_valid;
                const int n = t * R + row;
                __half v = __ushort_as_half(ob[row * MT + m]);
                if constexpr (EPI == (int)Epi::RESIDUAL) v = __hadd(a.resid[(size_t)m * N + n], v);
                a.out[(size_t)m * N + n] = v;
            }
        } else {
            const int half_rows = rows_valid / 2;
            for (int i = tid; i < half_rows * M; i += kGemvThreads) {
                const int m = i / half_rows, hr = i % half_rows;
                const __half gate = __ushort_as_half(ob[(2 * hr) * MT + m]);
                const __half up = __ushort_as_half(ob[(2 * hr + 1) * MT + m]);
                const __half act_g = (EPI == (int)Epi::GLU_SILU) ? ref_silu(gate) : ref_gelu(gate);
                a.out[(size_t)m * (N / 2) + (t * R) / 2 + hr] = __hmul(act_g, up);
            }
        }
    }
}

// ------------------------------------------------------------------ row-streaming variant
// Same arithmetic, another data path, for group sizes whose 16-byte weight chunks per group
// (cpg = G/16 for INT8, G/32 for INT4) divide 32. After the shared prologue every warp works
// alone on its own row groups (RW consecutive rows): a per-warp ring of kRowsStages shared-
// memory stages is filled with cp.async (8 (row, pass) items of 32 lanes x 16 bytes = 4 KB
// per stage, plus the slice's group scales), so every warp keeps 12 KB of weights in flight
// while it forms the exact group sums with dp4a and a shuffle fold over the cpg lanes of a
// group; lanes (row, m) of the same warp then continue the fp32 chains. No block barrier
// after the prologue: warps never wait for one another.
constexpr int kRowsItems = 8;   // (row, pass) items per stage: 8 x 32 lanes x 16 bytes
constexpr int kRowsStages = 4;

struct GemvRowsLayout {
    int RW, stage_bytes, warp_bytes, off_act, off_asum, off_as, off_xs, off_red, off_warps, total;
};

__host__ __device__ inline int gemv_rows_per_warp(int wf, int MT, int G, int epi) {
    const int cpg = wf == 0 ? G / 16 : G / 32;
    int rw = kRowsItems / cpg;
    if (rw > 8) rw = 8;
    while (rw > 1 && rw * MT > 32) rw >>= 1;  // one chain lane per (row, activation row)
    if (rw < 1) rw = 1;
    if ((epi == (int)Epi::GLU_SILU || epi == (int)Epi::GLU_GELU) && rw < 2) rw = 2;
    return rw;
}

__host__ __device__ inline GemvRowsLayout gemv_rows_layout(int wf, int MT, int pro, int epi, int K, int G) {
    GemvRowsLayout L;
    L.RW = gemv_rows_per_warp(wf, MT, G, epi);
    const int ng = K / G;
    L.stage_bytes = kRowsItems * 512 + L.RW * 64;  // weights | RW rows x 32 fp16 scales
    L.warp_bytes = kRowsStages * L.stage_bytes + align_up(L.RW * MT * 33 * 4, 16);
    int off = 0;
    L.off_act = off;   off += align_up(MT * K, 128);
    L.off_asum = off;  off += align_up(MT * ng * 4, 128);
    L.off_as = off;    off += 128;
    L.off_xs = off;    off += (pro != 0) ? align_up(MT * K * 2, 128) : 0;
    L.off_red = off;   off += 128 * 4;
    L.off_warps = off; off += kGemvWarps * L.warp_bytes;
    L.total = align_up(off, 128);
    return L;
}

__host__ __device__ inline bool gemv_rows_ok(int wf, int G) {
    const int cpg = wf == 0 ? G / 16 : G / 32;
    return cpg >= 1 && cpg <= 32 && (32 % cpg) == 0;
}

template <int WF, int MT, int PRO, int EPI>
__global__ void __launch_bounds__(kGemvThreads) qgemv_rows_kernel(GemvArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const GemvRowsLayout L = gemv_rows_layout(WF, MT, PRO, EPI, a.K, a.G);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int K = a.K, N = a.N, G = a.G, M = a.M;
    const int ng = K / G, RW = L.RW;
    const int cpg = WF == 0 ? G / 16 : G / 32;     // 16-byte weight chunks per group (divides 32)
    const int chunks = WF == 0 ? K / 16 : K / 32;  // 16-byte weight chunks per row
    const int wrow = WF == 0 ? K : K / 2;
    const int nslice = (ng + 31) / 32;
    const int items = RW * cpg;                        // (row, pass) items of one slice
    const int nbps = (items + kRowsItems - 1) / kRowsItems;  // stages per slice
    const int NB = nslice * nbps;                      // stages per row group
    const bool vec_s = (ng & 7) == 0;                  // scales move as 16-byte chunks
    const int nwarps = gridDim.x * kGemvWarps;
    const int first_rg = warp * gridDim.x + blockIdx.x;  // consecutive row groups on different SMs
    const int nrg = (N + RW - 1) / RW;
    int8_t* act = reinterpret_cast<int8_t*>(smem + L.off_act);
    int* asum = reinterpret_cast<int*>(smem + L.off_asum);
    float* as = reinterpret_cast<float*>(smem + L.off_as);
    uint8_t* wsm = smem + L.off_warps + warp * L.warp_bytes;
    int* gs = reinterpret_cast<int*>(wsm + kRowsStages * L.stage_bytes);
    const uint8_t* wbase = reinterpret_cast<const uint8_t*>(a.w);
    const uint16_t* sbase = reinterpret_cast<const uint16_t*>(a.ws);

    // stage j of this warp: row group first_rg + (j / NB) * nwarps, slice, batch
    auto issue = [&](int j) {
        const int k = j / NB, rem = j % NB, sl = rem / nbps, b = rem % nbps;
        const int rg = first_rg + k * nwarps;
        if (rg < nrg) {
            uint8_t* st = wsm + (j % kRowsStages) * L.stage_bytes;
            const int row0 = rg * RW;
#pragma unroll
            for (int q = 0; q < kRowsItems; ++q) {
                const int it = b * kRowsItems + q;
                const int r = it / cpg, p = it % cpg;
                const int c = (sl * cpg + p) * 32 + lane;
                if (it < items && row0 + r < N && c < chunks)
                    cp_async16(st + q * 512 + lane * 16, wbase + (size_t)(row0 + r) * wrow + (size_t)c * 16);
            }
            if (b == 0 && vec_s && lane < RW * 4 && sl * 32 + 32 <= ng) {
                const int r = lane >> 2, qq = lane & 3;
                if (row0 + r < N)
                    cp_async16(st + kRowsItems * 512 + r * 64 + qq * 16, sbase + (size_t)(row0 + r) * ng + sl * 32 + qq * 8);
            }
        }
        cp_async_commit();  // possibly empty: keeps the group count uniform
    };

    // weights do not depend on the previous kernel: the first stages stream while it finishes
    for (int j = 0; j < kRowsStages - 1; ++j) issue(j);
    pdl_launch_dependents();
    pdl_wait();
    gemv_prologue<WF, MT, PRO>(a, act, asum, as, reinterpret_cast<__half*>(smem + L.off_xs),
                               reinterpret_cast<float*>(smem + L.off_red));

    const int cr = lane / MT, cm = lane % MT;  // chain lane (row cr of the group, activation row cm)
    const bool chain_lane = lane < RW * MT && cm < M;
    float run = 0.0f;
    int4 sv[4];
    for (int j = 0;; ++j) {
        const int k = j / NB, rem = j % NB, sl = rem / nbps, b = rem % nbps;
        const int rg = first_rg + k * nwarps;
        if (rg >= nrg) break;
        cp_async_wait<kRowsStages - 2>();
        __syncwarp();
        issue(j + kRowsStages - 1);  // into the stage consumed by the previous iteration
        const uint8_t* st = wsm + (j % kRowsStages) * L.stage_bytes;
        const int row0 = rg * RW;
        const int gcount = min(32, ng - sl * 32);
        const int crow = row0 + cr;
        const bool crow_ok = chain_lane && crow < N;
        const bool vs_slice = vec_s && gcount == 32;
        if (b == 0 && crow_ok && vs_slice) {
            const int4* sp = reinterpret_cast<const int4*>(st + kRowsItems * 512 + cr * 64);
#pragma unroll
            for (int q = 0; q < 4; ++q) sv[q] = sp[q];
        }
#pragma unroll
        for (int q = 0; q < kRowsItems; ++q) {
            const int it = b * kRowsItems + q;
            if (it >= items) break;  // uniform across the warp
            const int r = it / cpg, p = it % cpg;
            const int c = (sl * cpg + p) * 32 + lane;
            const bool cval = c < chunks;
            const int gl = (p * 32 + lane) / cpg;  // group within the slice
            const int4 wv = *reinterpret_cast<const int4*>(st + q * 512 + lane * 16);
#pragma unroll
            for (int m = 0; m < MT; ++m) {
                int acc = 0;
                if (cval && m < M) {
                    if constexpr (WF == 0) {
                        const int4 av = *reinterpret_cast<const int4*>(act + m * K + c * 16);
                        acc = dp4a_ss(av.x, wv.x, acc);
                        acc = dp4a_ss(av.y, wv.y, acc);
                        acc = dp4a_ss(av.z, wv.z, acc);
                        acc = dp4a_ss(av.w, wv.w, acc);
                    } else {
                        const int4 a0 = *reinterpret_cast<const int4*>(act + m * K + c * 32);
                        const int4 a1 = *reinterpret_cast<const int4*>(act + m * K + c * 32 + 16);
                        const unsigned ww[4] = {(unsigned)wv.x, (unsigned)wv.y, (unsigned)wv.z, (unsigned)wv.w};
                        const int ae[4] = {a0.x, a0.z, a1.x, a1.z};
                        const int ao[4] = {a0.y, a0.w, a1.y, a1.w};
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const unsigned lo = (ww[e] & 0x0F0F0F0Fu) ^ 0x08080808u;
                            const unsigned hi = ((ww[e] >> 4) & 0x0F0F0F0Fu) ^ 0x08080808u;
                            acc = dp4a_su(ae[e], lo, acc);
                            acc = dp4a_su(ao[e], hi, acc);
                        }
                    }
                }
                for (int o = 1; o < cpg; o <<= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
                if ((lane % cpg) == 0 && cval) {
                    if constexpr (WF == 1) acc -= 8 * asum[m * ng + sl * 32 + gl];
                    gs[(r * MT + m) * 33 + gl] = acc;
                }
            }
        }
        if (b == nbps - 1) {  // slice complete: continue the chains over its groups
            __syncwarp();
            if (crow_ok) {
                const int* gp = gs + lane * 33;  // lane == cr * MT + cm
                if (vs_slice) {
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const uint16_t* s8 = reinterpret_cast<const uint16_t*>(&sv[q]);
#pragma unroll
                        for (int e = 0; e < 8; ++e) run = fmaf((float)gp[q * 8 + e], h2f_bits(s8[e]), run);
                    }
                } else {
                    const uint16_t* sp = sbase + (size_t)crow * ng + sl * 32;
                    for (int g = 0; g < gcount; ++g) run = fmaf((float)gp[g], h2f_bits(__ldg(sp + g)), run);
                }
            }
            if (sl == nslice - 1) {  // row group complete: chain lanes hold C[cm, crow]
                const __half v = __float2half_rn(__fmul_rn(run, as[cm < M ? cm : 0]));
                if constexpr (EPI == (int)Epi::STORE || EPI == (int)Epi::RESIDUAL) {
                    if (crow_ok) {
                        __half o = v;
                        if constexpr (EPI == (int)Epi::RESIDUAL) o = __hadd(a.resid[(size_t)cm * N + crow], v);
                        a.out[(size_t)cm * N + crow] = o;
                    }
                } else {
                    // rows come in (gate, up) pairs: RW is even and row groups start at even rows
                    const __half up = __shfl_down_sync(0xffffffffu, v, MT);
                    if (crow_ok && (cr & 1) == 0 && crow + 1 < N) {
                        const __half g = (EPI == (int)Epi::GLU_SILU) ? ref_silu(v) : ref_gelu(v);
                        a.out[(size_t)cm * (N / 2) + crow / 2] = __hmul(g, up);
                    }
                }
                run = 0.0f;
            }
        }
        __syncwarp();  // the stage and the group sums are free for the next iteration
    }
    cp_async_wait<0>();
}

}  // namespace cb
