// Attention kernels (sm_100a).
//
//  * attn_f16_kernel — cactus_attention_f16 (kernel_attention.cpp:10-255): no-cache
//    attention with causal / sliding-window masks, GQA, online softmax over 32-key blocks
//    that start at the window start, and the reference's quadratic 2^x approximation for
//    the first floor(block/4)*4 keys of each block (expf for the rest).
//  * attn_hybrid_kernel — cactus_attention_hybrid_int8_fp16 (kernel_attention.cpp:257-482):
//    keys/values below cache_len come from the INT8 cache (x fp32 scale per 128-group),
//    the rest from the fp16 new tokens; expf throughout, so the 32-key block partition
//    only changes fp32 rounding and the keys can be split across warps.
//
// Scores use the reference's 8-lane fp32 dot-product order (accumulator j sums dims
// d = j mod 8 with FMAs, folded as ((a0+a4)+(a1+a5))+((a2+a6)+(a3+a7))).
#include "attention_core.cuh"
#include "common.cuh"
#include "ops.h"

namespace cb {

constexpr int kMaxHeadDim = 256;


// One warp per (batch, q head, query). Lane i scores key i of each 32-key block; lane l owns
// output dims l, l+32, ... for the value accumulation. As in the reference, dims past the last
// multiple of 8 (head_dim_aligned) only enter the scores; their outputs are zero.
__global__ void __launch_bounds__(128) attn_f16_kernel(const __half* __restrict__ Q, const __half* __restrict__ Kt,
                                                       const __half* __restrict__ Vt, __half* __restrict__ O, int B,
                                                       int S, int Skv, int Hq, int Hkv, int D, float scale,
                                                       long long pos_off, long long window, int causal) {
    pdl_launch_dependents();
    pdl_wait();
    __shared__ float qs[4][kMaxHeadDim];
    extern __shared__ __align__(16) __half vstage_all[];  // per warp: the block's 32 value rows [32][D]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __half* vstage = vstage_all + (size_t)warp * 32 * D;
    const long long item = (long long)blockIdx.x * 4 + warp;  // ((b*Hq + h)*S + q)
    if (item >= (long long)B * Hq * S) return;
    const int qp = (int)(item % S);
    const int h = (int)((item / S) % Hq);
    const int b = (int)(item / ((long long)S * Hq));
    const int kvh = h / (Hq / Hkv);
    const __half* q16 = Q + (((size_t)b * S + qp) * Hq + h) * D;
    __half* o = O + (((size_t)b * S + qp) * Hq + h) * D;
    for (int d = lane; d < D; d += 32) qs[warp][d] = h2f(q16[d]);
    __syncwarp();
    const int dpl = (D + 31) / 32;  // dims per lane
    const int hda = (D / 8) * 8;
    float acc[kMaxHeadDim / 32];
#pragma unroll
    for (int i = 0; i < kMaxHeadDim / 32; ++i) acc[i] = 0.0f;
    float run_max = -INFINITY, run_sum = 0.0f;
    const bool is_decode = (qp == S - 1) && S > 1;
    const long long aq = pos_off + qp;
    long long kv_start = 0, kv_end = Skv;
    if (window > 0 && window < Skv) {
        if (aq > window) kv_start = aq - window;
        if (causal && aq + 1 < kv_end) kv_end = aq + 1;
    } else if (causal && aq + 1 < kv_end) {
        kv_end = aq + 1;
    }
    const size_t kv_row = (size_t)Hkv * D;
    const __half* Kb = Kt + (size_t)b * Skv * kv_row + (size_t)kvh * D;
    const __half* Vb = Vt + (size_t)b * Skv * kv_row + (size_t)kvh * D;
    for (long long b0 = kv_start; b0 < kv_end; b0 += 32) {
        const int bs = (int)(min(b0 + 32, (long long)Skv) - b0);
        if (!is_decode && causal && b0 > aq) continue;
        float s = -INFINITY;
        const long long kp = b0 + lane;
        if (lane < bs && !(!is_decode && causal && kp > aq)) {
            const __half* kr = Kb + (size_t)kp * kv_row;
            float a8[8] = {0, 0, 0, 0, 0, 0, 0, 0};
            if ((D & 7) == 0) {
                for (int d = 0; d < D; d += 8) {
                    const int4 kv4 = *reinterpret_cast<const int4*>(kr + d);
                    const __half* kh = reinterpret_cast<const __half*>(&kv4);
#pragma unroll
                    for (int j = 0; j < 8; ++j) a8[j] = fmaf(qs[warp][d + j], h2f(kh[j]), a8[j]);
                }
            } else {
                for (int d = 0; d < hda; d += 8)
#pragma unroll
                    for (int j = 0; j < 8; ++j) a8[j] = fmaf(qs[warp][d + j], h2f(kr[d + j]), a8[j]);
            }
            float dot = fold8(a8);
            for (int d = hda; d < D; ++d) dot = fmaf(qs[warp][d], h2f(kr[d]), dot);
            s = __fmul_rn(dot, scale);
            if (causal && kp > aq) s = -INFINITY;
            else if (window > 0 && kp < aq && (aq - kp) > window) s = -INFINITY;
        }
        const float bmax = warp_max(s);
        if (bmax > -INFINITY) {
            const float corr = expf_cr(__fsub_rn(run_max, bmax));
            run_sum = __fmul_rn(run_sum, corr);
            for (int i = 0; i < dpl; ++i) acc[i] = __fmul_rn(acc[i], corr);
            run_max = bmax;
        }
        const int vec = (bs / 4) * 4;
        float y = 0.0f;
        if (lane < vec) y = (s == -INFINITY) ? 0.0f : attn_quad_exp(s, bmax);
        else if (lane < bs) y = (s == -INFINITY) ? 0.0f : expf_cr(__fsub_rn(s, bmax));
        // block sum in the reference order: quads ((y0+y1)+(y2+y3)) in sequence, then the tail
        const float y1 = __shfl_down_sync(0xffffffffu, y, 1), y2 = __shfl_down_sync(0xffffffffu, y, 2),
                    y3 = __shfl_down_sync(0xffffffffu, y, 3);
        const float quad = __fadd_rn(__fadd_rn(y, y1), __fadd_rn(y2, y3));
        float bsum = 0.0f;
        for (int qd = 0; qd < vec; qd += 4) bsum = __fadd_rn(bsum, __shfl_sync(0xffffffffu, quad, qd));
        for (int i = vec; i < bs; ++i) bsum = __fadd_rn(bsum, __shfl_sync(0xffffffffu, y, i));
        // stage the block's value rows with the warp's loads (16 bytes a lane where the rows
        // allow), so the in-order accumulation below reads shared memory instead of waiting
        // on a global load per key
        __syncwarp();
        if ((D & 7) == 0 && (kv_row & 7) == 0 && (reinterpret_cast<uintptr_t>(Vb) & 15) == 0) {
            const int cpr = D / 8;  // 16-byte chunks per row
            for (int c = lane; c < bs * cpr; c += 32) {
                const int i = c / cpr, j = c - i * cpr;
                reinterpret_cast<int4*>(vstage + (size_t)i * D)[j] =
                    __ldg(reinterpret_cast<const int4*>(Vb + (size_t)(b0 + i) * kv_row) + j);
            }
        } else {
            for (int c = lane; c < bs * D; c += 32) {
                const int i = c / D, d = c - i * D;
                vstage[(size_t)i * D + d] = Vb[(size_t)(b0 + i) * kv_row + d];
            }
        }
        __syncwarp();
        for (int i = 0; i < bs; ++i) {
            const float w = __shfl_sync(0xffffffffu, y, i);
            if (w == 0.0f) continue;
            const __half* vr = vstage + (size_t)i * D;
            for (int t = 0; t < dpl; ++t)
                if (lane + 32 * t < hda) acc[t] = fmaf(h2f(vr[lane + 32 * t]), w, acc[t]);
        }
        run_sum = __fadd_rn(run_sum, bsum);
    }
    const float inv = run_sum > 0.0f ? __fdiv_rn(1.0f, run_sum) : 0.0f;
    for (int t = 0; t < dpl; ++t) {
        const int d = lane + 32 * t;
        if (d < D) o[d] = (run_sum > 0.0f && d < hda) ? f2h(__fmul_rn(acc[t], inv)) : __float2half_rn(0.0f);
    }
}

// Hybrid INT8-cache / FP16-new attention. One CTA (4 warps) per (batch, q head, query);
// the warps take 32-key blocks round-robin, each keeps its own online-softmax state, and
// the four states are merged at the end. kc_bstride / sc_bstride are the per-batch strides
// (in elements) of the int8 cache and of its fp32 scales (the reference uses
// cache_len*Hkv*D and 0 respectively).
__global__ void __launch_bounds__(128) attn_hybrid_kernel(
    const __half* __restrict__ Q, const int8_t* __restrict__ Kc, const int8_t* __restrict__ Vc,
    const float* __restrict__ ks, const float* __restrict__ vs, const __half* __restrict__ Kn,
    const __half* __restrict__ Vn, __half* __restrict__ O, int B, int S, int cache_len, int new_len, int Hq, int Hkv,
    int D, float scale, long long pos_off, int causal, int qgs, long long kc_bstride, long long sc_bstride,
    const int* __restrict__ dstate) {
    pdl_launch_dependents();
    pdl_wait();
    if (dstate) {  // engine decode graphs keep {cache_len, total_len} in device memory
        cache_len = dstate[0];
        pos_off = dstate[1];
    }
    __shared__ float qs[kMaxHeadDim];
    __shared__ float wmax[4], wsum[4];
    __shared__ float wacc[4][kMaxHeadDim];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long long item = blockIdx.x;  // ((b*Hq + h)*S + q)
    const int qp = (int)(item % S);
    const int h = (int)((item / S) % Hq);
    const int b = (int)(item / ((long long)S * Hq));
    const int kvh = h / (Hq / Hkv);
    const int nqg = (D + qgs - 1) / qgs;
    const __half* q16 = Q + (((size_t)b * S + qp) * Hq + h) * D;
    for (int d = threadIdx.x; d < D; d += blockDim.x) qs[d] = h2f(q16[d]);
    __syncthreads();
    const int dpl = D / 32;
    float acc[kMaxHeadDim / 32];
#pragma unroll
    for (int i = 0; i < kMaxHeadDim / 32; ++i) acc[i] = 0.0f;
    float run_max = -INFINITY, run_sum = 0.0f;
    const long long kv_seq_len = (long long)cache_len + new_len;
    const long long aq = pos_off + qp;
    const long long kv_end = causal ? min(kv_seq_len, aq + 1) : kv_seq_len;
    const size_t kv_row = (size_t)Hkv * D;
    const int8_t* Kcb = Kc + b * kc_bstride + (size_t)kvh * D;
    const int8_t* Vcb = Vc + b * kc_bstride + (size_t)kvh * D;
    const float* ksb = ks + b * sc_bstride + (size_t)kvh * nqg;
    const float* vsb = vs + b * sc_bstride + (size_t)kvh * nqg;
    const __half* Knb = Kn + (size_t)b * new_len * kv_row + (size_t)kvh * D;
    const __half* Vnb = Vn + (size_t)b * new_len * kv_row + (size_t)kvh * D;
    for (long long b0 = (long long)warp * 32; b0 < kv_end; b0 += 128) {
        const int bs = (int)(min(b0 + 32, kv_end) - b0);
        const long long kp = b0 + lane;
        float s = -INFINITY;
        if (lane < bs && !(causal && kp > aq)) {
            float a8[8] = {0, 0, 0, 0, 0, 0, 0, 0};
            if (kp < cache_len) {
                const int8_t* kr = Kcb + (size_t)kp * kv_row;
                const float* sr = ksb + (size_t)kp * Hkv * nqg;
                for (int d = 0; d < D; d += 8) {
                    const int2 k8 = *reinterpret_cast<const int2*>(kr + d);
                    const int8_t* kb = reinterpret_cast<const int8_t*>(&k8);
                    const float sc = sr[d / qgs];
#pragma unroll
                    for (int j = 0; j < 8; ++j) a8[j] = fmaf(qs[d + j], __fmul_rn((float)kb[j], sc), a8[j]);
                }
            } else {
                const __half* kr = Knb + (size_t)(kp - cache_len) * kv_row;
                for (int d = 0; d < D; d += 8) {
                    const int4 kv4 = *reinterpret_cast<const int4*>(kr + d);
                    const __half* kh = reinterpret_cast<const __half*>(&kv4);
#pragma unroll
                    for (int j = 0; j < 8; ++j) a8[j] = fmaf(qs[d + j], h2f(kh[j]), a8[j]);
                }
            }
            s = __fmul_rn(fold8(a8), scale);
        }
        const float bmax = warp_max(s);
        if (bmax > -INFINITY) {
            const float corr = expf_cr(__fsub_rn(run_max, bmax));
            run_sum = __fmul_rn(run_sum, corr);
            for (int i = 0; i < dpl; ++i) acc[i] = __fmul_rn(acc[i], corr);
            run_max = bmax;
        }
        const float y = (lane < bs && s != -INFINITY) ? expf_cr(__fsub_rn(s, bmax)) : 0.0f;
        float bsum = 0.0f;
        for (int i = 0; i < bs; ++i) {
            const float w = __shfl_sync(0xffffffffu, y, i);
            bsum = __fadd_rn(bsum, w);
            if (w == 0.0f) continue;
            const long long kpi = b0 + i;
            if (kpi < cache_len) {
                const int8_t* vr = Vcb + (size_t)kpi * kv_row;
                const float* sr = vsb + (size_t)kpi * Hkv * nqg;
                for (int t = 0; t < dpl; ++t) {
                    const int d = lane + 32 * t;
                    acc[t] = fmaf(__fmul_rn((float)vr[d], sr[d / qgs]), w, acc[t]);
                }
            } else {
                const __half* vr = Vnb + (size_t)(kpi - cache_len) * kv_row;
                for (int t = 0; t < dpl; ++t) acc[t] = fmaf(h2f(vr[lane + 32 * t]), w, acc[t]);
            }
        }
        run_sum = __fadd_rn(run_sum, bsum);
    }
    // merge the four warp states
    if (lane == 0) { wmax[warp] = run_max; wsum[warp] = run_sum; }
    for (int t = 0; t < dpl; ++t) wacc[warp][lane + 32 * t] = acc[t];
    __syncthreads();
    if (warp == 0) {
        float m = fmaxf(fmaxf(wmax[0], wmax[1]), fmaxf(wmax[2], wmax[3]));
        float tot = 0.0f;
        float f[4];
        for (int w = 0; w < 4; ++w) {
            f[w] = (wmax[w] == -INFINITY) ? 0.0f : expf_cr(__fsub_rn(wmax[w], m));
            tot = fmaf(wsum[w], f[w], tot);
        }
        __half* o = O + (((size_t)b * S + qp) * Hq + h) * D;
        if (tot > 0.0f) {
            const float inv = __fdiv_rn(1.0f, tot);
            for (int t = 0; t < dpl; ++t) {
                const int d = lane + 32 * t;
                float v = 0.0f;
                for (int w = 0; w < 4; ++w) v = fmaf(wacc[w][d], f[w], v);
                o[d] = f2h(__fmul_rn(v, inv));
            }
        } else {
            for (int t = 0; t < dpl; ++t) o[lane + 32 * t] = __float2half_rn(0.0f);
        }
    }
}


// ------------------------------------------------------------------ exact hybrid attention
// Bit-for-bit restatement of cactus_attention_hybrid_int8_fp16's arithmetic: one CTA of 256
// threads per (batch, q head, query) walks the 32-key blocks in order with the same online
// softmax (corrections, block sums, fused V accumulation per dim) as the reference.
// Thread (i = t/8, j = t%8) forms lane j of key i's 8-lane dot product; threads t < D own
// output dim t. Raw INT8 K/V of the next blocks stream into shared memory with cp.async
// (three buffers) while the current block is computed.
// One CTA of 256 threads per (batch, q head, query) runs the reference-order core
// (attention_core.cuh) over chunks of 256 keys.
template <int D>
__global__ void __launch_bounds__(256) attn_hybrid_exact_kernel(
    const __half* __restrict__ Q, const int8_t* __restrict__ Kc, const int8_t* __restrict__ Vc,
    const float* __restrict__ ks, const float* __restrict__ vs, const __half* __restrict__ Kn,
    const __half* __restrict__ Vn, __half* __restrict__ O, int S, int cache_len, int new_len, int Hq, int Hkv,
    float scale, long long pos_off, int causal, int qgs, long long kc_bstride, long long sc_bstride,
    const int* __restrict__ dstate, KvPaging pg) {
    pdl_launch_dependents();
    pdl_wait();
    if (dstate) {
        cache_len = dstate[0];
        pos_off = dstate[1];
    }
    constexpr int CH = 256;
    extern __shared__ __align__(16) uint8_t smem[];
    float* qs = reinterpret_cast<float*>(smem + attn_core_smem<D, CH>());
    const int t = threadIdx.x;
    const long long item = blockIdx.x;
    const int qp = (int)(item % S);
    const int h = (int)((item / S) % Hq);
    const int b = (int)(item / ((long long)S * Hq));
    const int kvh = h / (Hq / Hkv);
    const int nqg = (D + qgs - 1) / qgs;
    const size_t kv_row = (size_t)Hkv * D;
    const __half* q16 = Q + (((size_t)b * S + qp) * Hq + h) * D;
    for (int d = t; d < D; d += 256) qs[d] = h2f(q16[d]);

    AttnCoreArgs c;
    c.qs = qs;
    const long long kb = pg.table ? 0 : b * kc_bstride, sb = pg.table ? 0 : b * sc_bstride;
    c.Kc = Kc + kb + (size_t)kvh * D;
    c.Vc = Vc + kb + (size_t)kvh * D;
    c.ks = ks + sb + (size_t)kvh * nqg;
    c.vs = vs + sb + (size_t)kvh * nqg;
    c.pages = pg.table ? pg.table + (size_t)b * pg.pps : nullptr;
    c.page_shift = pg.shift;
    c.Kn = Kn + (size_t)b * new_len * kv_row + (size_t)kvh * D;
    c.Vn = Vn + (size_t)b * new_len * kv_row + (size_t)kvh * D;
    c.kv_row = (long long)kv_row;
    c.sc_row = (long long)Hkv * nqg;
    c.kn_row = (long long)kv_row;
    c.cache_len = cache_len;
    c.new_len = new_len;
    c.qgs = qgs;
    const long long kv_seq_len = (long long)cache_len + new_len;
    c.aq = pos_off + qp;
    c.kv_end = causal ? min(kv_seq_len, c.aq + 1) : kv_seq_len;
    c.causal = causal;
    c.scale = scale;
    c.prestaged = 0;
    __syncthreads();
    const __half r = attn_exact_core<D, 256, CH>(c, smem, SyncBlock{});
    if (t < D) O[(((size_t)b * S + qp) * Hq + h) * D + t] = r;
}

template <int D>
static size_t exact_smem() {
    return (size_t)attn_core_smem<D, 256>() + (size_t)D * 4;
}

int launch_attention_hybrid_exact(const __half* q, const int8_t* kc, const int8_t* vc, const float* ks,
                                  const float* vs, const __half* kn, const __half* vn, __half* o, int B, int S,
                                  int cache_len, int new_len, int Hq, int Hkv, int D, float scale, long long pos_off,
                                  int causal, int qgs, long long kc_bstride, long long sc_bstride, cudaStream_t st,
                                  const int* dstate, KvPaging pg) {
    const unsigned items = (unsigned)((long long)B * Hq * S);
    // long caches: the same arithmetic split over the keys (not while the lengths live on the
    // device or the stream is being captured: the split path sizes a scratch buffer on the host)
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    if (!dstate && (long long)cache_len + new_len >= kSplitMinKeys && cudaStreamIsCapturing(st, &cap) == cudaSuccess &&
        cap == cudaStreamCaptureStatusNone &&
        launch_attention_split(q, kc, vc, ks, vs, kn, vn, o, B, S, cache_len, new_len, Hq, Hkv, D, scale, pos_off,
                               causal, qgs, kc_bstride, sc_bstride, st, pg) == 0)
        return 0;
#define CB_EXACT(DD)                                                                                          \
    {                                                                                                         \
        static bool attr = false;                                                                             \
        const size_t sm = exact_smem<DD>();                                                                   \
        if (!attr) {                                                                                          \
            cudaFuncSetAttribute(attn_hybrid_exact_kernel<DD>, cudaFuncAttributeMaxDynamicSharedMemorySize,   \
                                 (int)sm);                                                                    \
            attr = true;                                                                                      \
        }                                                                                                     \
        launch_k(attn_hybrid_exact_kernel<DD>, dim3(items), dim3(256), sm, st, q, kc, vc, ks, vs, kn, vn, o, S, cache_len,    \
                                                             new_len, Hq, Hkv, scale, pos_off, causal, qgs,    \
                                                             kc_bstride, sc_bstride, dstate, pg);              \
        return 0;                                                                                             \
    }
    if (qgs % 8 || (D + qgs - 1) / qgs > 2) return -1;
    switch (D) {
        case 64: CB_EXACT(64)
        case 128: CB_EXACT(128)
        case 256: CB_EXACT(256)
    }
#undef CB_EXACT
    return -1;
}

void attention_prepare() {
    cudaFuncSetAttribute(attn_hybrid_exact_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)exact_smem<64>());
    cudaFuncSetAttribute(attn_hybrid_exact_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)exact_smem<128>());
    cudaFuncSetAttribute(attn_hybrid_exact_kernel<256>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)exact_smem<256>());
}

int launch_attention_f16(const __half* q, const __half* k, const __half* v, __half* o, int B, int S, int Skv, int Hq,
                         int Hkv, int D, float scale, long long pos_off, long long window, int causal,
                         cudaStream_t st) {
    const long long items = (long long)B * Hq * S;
    const size_t smem = (size_t)4 * 32 * D * sizeof(__half);  // per warp, one 32-key block of value rows
    if (smem > 48 * 1024) {
        static size_t enabled = 0;
        if (smem > enabled) {
            if (cudaFuncSetAttribute(attn_f16_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
                cudaSuccess)
                return -1;
            enabled = smem;
        }
    }
    launch_k(attn_f16_kernel, dim3((unsigned)((items + 3) / 4)), dim3(128), smem, st, q, k, v, o, B, S, Skv, Hq, Hkv, D,
             scale, pos_off, window, causal);
    return 0;
}

int launch_attention_hybrid(const __half* q, const int8_t* kc, const int8_t* vc, const float* ks, const float* vs,
                            const __half* kn, const __half* vn, __half* o, int B, int S, int cache_len, int new_len,
                            int Hq, int Hkv, int D, float scale, long long pos_off, int causal, int qgs,
                            long long kc_bstride, long long sc_bstride, cudaStream_t st, const int* dstate) {
    const long long items = (long long)B * Hq * S;
    launch_k(attn_hybrid_kernel, dim3((unsigned)items), dim3(128), 0, st, q, kc, vc, ks, vs, kn, vn, o, B, S, cache_len, new_len, Hq,
                                                        Hkv, D, scale, pos_off, causal, qgs, kc_bstride, sc_bstride,
                                                        dstate);
    return 0;
}

}  // namespace cb
