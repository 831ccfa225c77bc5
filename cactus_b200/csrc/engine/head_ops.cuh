// Per-head device routines shared by the engine's kernels and the persistent decode kernel.
#pragma once
#include "../common.cuh"
#include "../gemv.cuh"

namespace cb {
namespace eng {

// One warp: optional per-head RMSNorm of xs (shared memory, fp16 [D], normalised in place) —
// QwenModel::build_attention's rms_norm over [seq*heads, head_dim] (model_qwen.cpp:63-70) —
// then RoPE at position `pos` from the fp16 tables (cactus_rope_f16, kernel_attention.cpp:
// 614-676) into dst. ct == nullptr disables RoPE (rope_theta <= 0).
// Same with the RoPE rows of the position given directly (crow/srow = ct/st + pos * D/2;
// null crow: no RoPE).
__device__ __forceinline__ void head_norm_rope_rows(__half* xs, int D, const __half* nw, float eps,
                                                    const __half* crow, const __half* srow, __half* dst) {
    const int lane = threadIdx.x & 31, half = D / 2;
    if (nw) {
        const float ss = rms_sumsq_warp(xs, D);
        const float rms = __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)D), eps));
        const float inv = __fdiv_rn(1.0f, rms);
        const __half inv16 = __float2half_rn(inv);
        const int vec_end = (D / 8) * 8;
        __syncwarp();
        for (int d = lane; d < D; d += 32) {
            const __half v = xs[d];
            xs[d] = d < vec_end ? __hmul(__hmul(v, inv16), nw[d])
                                : __float2half_rn(__fmul_rn(__fmul_rn(h2f(v), inv), h2f(nw[d])));
        }
        __syncwarp();
    }
    if (crow == nullptr) {
        for (int d = lane; d < D; d += 32) dst[d] = xs[d];
        return;
    }
    const __half* c = crow;
    const __half* sn = srow;
    const int vec_half = (half / 8) * 8;
    for (int i = lane; i < half; i += 32) {
        const __half x1 = xs[i], x2 = xs[i + half];
        if (i < vec_half) {
            dst[i] = __hfma(__hneg(x2), sn[i], __hmul(x1, c[i]));
            dst[i + half] = __hfma(x1, sn[i], __hmul(x2, c[i]));
        } else {
            const float f1 = h2f(x1), f2 = h2f(x2), fc = h2f(c[i]), fs = h2f(sn[i]);
            dst[i] = f2h(__fsub_rn(__fmul_rn(f1, fc), __fmul_rn(f2, fs)));
            dst[i + half] = f2h(__fadd_rn(__fmul_rn(f2, fc), __fmul_rn(f1, fs)));
        }
    }
}

__device__ __forceinline__ void head_norm_rope_warp(__half* xs, int D, const __half* nw, float eps,
                                                    const __half* ct, const __half* st, long long pos,
                                                    __half* dst) {
    const long long off = pos * (D / 2);
    head_norm_rope_rows(xs, D, nw, eps, ct ? ct + off : nullptr, ct ? st + off : nullptr, dst);
}

// One warp: the KV-cache quantisation of one (token, head, group) of `cnt` values
// (cactus_quantize_kv_fp16_to_int8, kernel_quants.cpp:223-264): scale = max(absmax/127,
// 1e-10), RNE over the 8-wide vector part and round-half-away on the tail.
__device__ __forceinline__ void kv_quant_group_warp(const __half* src, int cnt, int8_t* dst, float* sdst) {
    const int lane = threadIdx.x & 31;
    float mx = 0.0f;
    for (int k = lane; k < cnt; k += 32) mx = fmaxf(mx, fabsf(h2f(src[k])));
    mx = warp_max(mx);
    float scale = __fdiv_rn(mx, 127.0f);
    if (scale < 1e-10f) scale = 1e-10f;
    const float inv = __fdiv_rn(1.0f, scale);
    const int vec = (cnt / 8) * 8;
    for (int k = lane; k < cnt; k += 32) {
        const float v = __fmul_rn(h2f(src[k]), inv);
        dst[k] = (int8_t)sat8(k < vec ? cvt_rne_sat(v) : (int)roundf(v));
    }
    if (lane == 0) *sdst = scale;
}

}  // namespace eng
}  // namespace cb
