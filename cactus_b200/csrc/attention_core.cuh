// Reference-order attention of one (query, head) against an INT8 cache plus FP16 new keys —
// the arithmetic of cactus_attention_hybrid_int8_fp16 (kernel_attention.cpp:257-482):
// 32-key blocks from key 0, scores as 8-lane dot products folded by a fixed tree, online
// softmax whose running max is replaced by each block's max, exp() correctly rounded
// (expf_cr) and the V accumulation per dim in key order.
//
// The recurrence only chains the per-block (max, sum) pair and the per-dim accumulator;
// scores, block maxima, weights and block sums of a block depend on that block alone. So a
// chunk of CH keys is processed in phases:
//   1. all scores in parallel (8-lane dot products in the reference lane order),
//   2. per 32-key block (one warp each): max, weights expf(s - max), in-order block sum and
//      the block's correction (from the max of the last non-empty block before it),
//   3. per output dim (one thread each): walk the blocks in order applying the correction
//      expf(run_max - block_max) and the in-order V FMAs — the same operation sequence, so
//      the result is bit-identical, with only the V chain left sequential.
// Shared by the standalone attention kernel and the persistent decode kernel.
#pragma once
#include "common.cuh"

namespace cb {

__device__ __forceinline__ float fold8(const float* a) {
    return __fadd_rn(__fadd_rn(__fadd_rn(a[0], a[4]), __fadd_rn(a[1], a[5])),
                     __fadd_rn(__fadd_rn(a[2], a[6]), __fadd_rn(a[3], a[7])));
}


// Row stride of the staged INT8 keys (16 bytes of padding: consecutive keys start in
// different banks).
template <int D>
__host__ __device__ constexpr int attn_krow() {
    return D + 16;
}

// shared-memory footprint of attn_exact_core<D, CH> (a multiple of 16 bytes)
template <int D, int CH>
__host__ __device__ constexpr int attn_core_smem() {
    return CH * attn_krow<D>() + CH * D + (CH * 2 * 2 + 2 * CH + 3 * (CH / 32)) * 4;
}

struct SyncBlock {
    __device__ __forceinline__ void operator()() const { __syncthreads(); }
};

struct AttnCoreArgs {
    const float* qs;      // [D] query as float (shared memory)
    const int8_t* Kc;     // cache row 0 of this kv head: key i at Kc + i * kv_row
    const int8_t* Vc;
    const float* ks;      // scales of key i at ks + i * sc_row (nqg floats)
    const float* vs;
    const __half* Kn;     // new key j at Kn + j * kn_row (global or shared memory)
    const __half* Vn;
    long long kv_row, sc_row, kn_row;
    int cache_len, new_len, qgs;
    long long kv_end;     // keys [0, kv_end) are attended
    long long aq;         // absolute query position (causal mask)
    int causal;
    float scale;
    int prestaged;        // the caller already issued (and committed) chunk 0's cp.async copies
    const int* pages = nullptr;  // paged cache: this sequence's page table (Kc/Vc/ks/vs = pool row 0)
    int page_shift = 0;
};

// Issues the cp.async copies of the cached INT8 rows and scales of chunk [c0, c0 + CH) and
// commits them as one group (all NT threads call it).
template <int D, int NT, int CH>
__device__ __forceinline__ void attn_stage_chunk(const AttnCoreArgs& a, uint8_t* smem, long long c0) {
    constexpr int KR = attn_krow<D>();
    int8_t* kraw = reinterpret_cast<int8_t*>(smem);
    int8_t* vraw = kraw + CH * KR;
    float* ksc = reinterpret_cast<float*>(vraw + CH * D);
    float* vsc = ksc + CH * 2;
    const int t = threadIdx.x;
    const int nqg = (D + a.qgs - 1) / a.qgs;
    const int n = (int)min((long long)CH, a.kv_end - c0);
    const int ncached = (int)max(0LL, min((long long)n, (long long)a.cache_len - c0));
    for (int c = t; c < ncached * (D / 16); c += NT) {
        const int i = c / (D / 16), off = (c % (D / 16)) * 16;
        const long long row = a.pages ? kv_page_row(a.pages, a.page_shift, c0 + i) : c0 + i;
        const size_t src = (size_t)row * a.kv_row + off;
        cp_async16(kraw + i * KR + off, a.Kc + src);
        cp_async16(vraw + i * D + off, a.Vc + src);
    }
    for (int c = t; c < ncached * nqg; c += NT) {
        const int i = c / nqg, g = c % nqg;
        const long long row = a.pages ? kv_page_row(a.pages, a.page_shift, c0 + i) : c0 + i;
        cp_async4(ksc + i * 2 + g, a.ks + (size_t)row * a.sc_row + g);
        cp_async4(vsc + i * 2 + g, a.vs + (size_t)row * a.sc_row + g);
    }
    cp_async_commit();
}

// Runs on NT threads that all call it; `bar` synchronises exactly those threads. Thread t < D
// returns output dim t (fp16 bits); other threads return 0.
template <int D, int NT, int CH, class Bar>
__device__ __forceinline__ __half attn_exact_core(const AttnCoreArgs& a, uint8_t* smem, Bar bar) {
    static_assert(NT % 32 == 0 && NT >= D && NT >= 32 * (CH / 32), "thread count");
    constexpr int KR = attn_krow<D>();
    int8_t* kraw = reinterpret_cast<int8_t*>(smem);   // [CH][KR]
    int8_t* vraw = kraw + CH * KR;                      // [CH][D]
    float* ksc = reinterpret_cast<float*>(vraw + CH * D);  // [CH][2]
    float* vsc = ksc + CH * 2;                          // [CH][2]
    float* sc = vsc + CH * 2;                           // [CH] scores
    float* sw = sc + CH;                                // [CH] weights
    float* bmx = sw + CH;                               // [CH/32] block maxima
    float* bsm = bmx + CH / 32;                         // [CH/32] block sums
    float* bcorr = bsm + CH / 32;                       // [CH/32] running-max corrections
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const float* qs = a.qs;
    const int vg = t < D ? t / a.qgs : 0;  // V scale group of this thread's dim
    float acc = 0.0f, run_max = -INFINITY, run_sum = 0.0f;

    for (long long c0 = 0; c0 < a.kv_end; c0 += CH) {
        const int n = (int)min((long long)CH, a.kv_end - c0);
        const int ncached = (int)max(0LL, min((long long)n, (long long)a.cache_len - c0));
        // stage the cached INT8 rows and scales of this chunk
        if (!(c0 == 0 && a.prestaged)) attn_stage_chunk<D, NT, CH>(a, smem, c0);
        cp_async_wait<0>();
        bar();
        // phase 1: scores (thread = lane kj of key ki's 8-lane dot product: lane kj sums dims
        // kj, kj + 8, ... in order, then the fixed fold of the 8 lanes)
        constexpr int KPR = NT / 8;  // keys per scoring round
        const int kj = t & 7;
        const int rounds = (n + KPR - 1) / KPR;
        for (int r = 0; r < rounds; ++r) {
            const int i = (t >> 3) + KPR * r;
            float acc8 = 0.0f;
            if (i < n) {
                if (i < ncached) {
                    const int8_t* kr = kraw + i * KR;
                    const float s0 = ksc[i * 2], s1 = ksc[i * 2 + 1];
                    // at most two scale groups per row (checked by the launchers)
#pragma unroll
                    for (int d = kj; d < D; d += 8)
                        acc8 = fmaf(qs[d], __fmul_rn(i2f_small(kr[d]), d >= a.qgs ? s1 : s0), acc8);
                } else {
                    const __half* kr = a.Kn + (size_t)(c0 + i - a.cache_len) * a.kn_row;
#pragma unroll
                    for (int d = kj; d < D; d += 8) acc8 = fmaf(qs[d], h2f(kr[d]), acc8);
                }
            }
            // fold8's tree as a butterfly on the 8 lanes of the key: ((l0 + l4) + (l1 + l5)) +
            // ((l2 + l6) + (l3 + l7)), complete in lane kj = 0
            const float f4 = __fadd_rn(acc8, __shfl_down_sync(0xffffffffu, acc8, 4));
            const float f1 = __fadd_rn(f4, __shfl_down_sync(0xffffffffu, f4, 1));
            const float f2 = __fadd_rn(f1, __shfl_down_sync(0xffffffffu, f1, 2));
            float s = __fmul_rn(f2, a.scale);
            if (i >= n || (a.causal && c0 + i > a.aq)) s = -INFINITY;
            if (kj == 0 && i < CH) sc[i] = s;
        }
        bar();
        // phase 2: warp w owns block w of the chunk
        const int nb = (n + 31) / 32;
        if (warp < nb) {
            const int i = warp * 32 + lane;
            const int bs = min(32, n - warp * 32);
            const float s = lane < bs ? sc[i] : -INFINITY;
            const float m = warp_max(s);
            const float w = (lane < bs && s != -INFINITY) ? expf_cr(__fsub_rn(s, m)) : 0.0f;
            if (lane < bs) sw[i] = w;
            // the correction of this block, expf(running max before it - its max): the running
            // max is the max of the last non-empty block before it in the chunk, else that of
            // the earlier chunks; a maximum is exact in any order, so the warp recomputes it from
            // the scores (blocks before the last one of a chunk are full)
            float pm = run_max;
            for (int j = warp - 1; j >= 0; --j) {
                const float mj = warp_max(sc[j * 32 + lane]);
                if (mj > -INFINITY) {
                    pm = mj;
                    break;
                }
            }
            const float corr = expf_cr(__fsub_rn(pm, m));
            __syncwarp();
            if (lane == 0) {
                // the block's in-order weight sum from shared memory (16-byte loads)
                const float4* w4 = reinterpret_cast<const float4*>(sw + warp * 32);
                float sum = 0.0f;
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    const float4 x = w4[q];
                    if (4 * q < bs) sum = __fadd_rn(sum, x.x);
                    if (4 * q + 1 < bs) sum = __fadd_rn(sum, x.y);
                    if (4 * q + 2 < bs) sum = __fadd_rn(sum, x.z);
                    if (4 * q + 3 < bs) sum = __fadd_rn(sum, x.w);
                }
                bmx[warp] = m;
                bsm[warp] = sum;
                bcorr[warp] = corr;
            }
        }
        bar();
        // phase 3: the reference's sequential recurrence, one output dim per thread
        for (int blk = 0; blk < nb; ++blk) {
            const float m = bmx[blk];
            if (m > -INFINITY) {
                const float corr = bcorr[blk];
                run_sum = __fmul_rn(run_sum, corr);
                acc = __fmul_rn(acc, corr);
                run_max = m;
            }
            if (t < D) {
                // keys with weight 0 leave acc untouched (the reference skips them). A plain fmaf
                // does the same: v is finite, so v * (+0) is a signed zero, and acc is never -0
                // (it starts at +0, a product of zero adds +0 or -0 to +0 giving +0, an exact
                // cancellation rounds to +0, and scaling keeps the sign), so acc + (+-0) == acc.
                const int i0 = blk * 32, i1 = min(n, i0 + 32);
                const int nc = min(i1, max(i0, ncached)) - i0;  // [i0, i0 + nc) cached, then new keys
                // 16-byte weight / scale loads, the values of 16 keys dequantised ahead, then the
                // fmaf chain in key order (rows past the cached ones are staged memory, unused)
                const float4* w4 = reinterpret_cast<const float4*>(sw + i0);
                const float4* s4 = reinterpret_cast<const float4*>(vsc + i0 * 2);
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    float v[16], w[16];
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const float4 q = w4[4 * h + j];
                        w[4 * j] = q.x;
                        w[4 * j + 1] = q.y;
                        w[4 * j + 2] = q.z;
                        w[4 * j + 3] = q.w;
                    }
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        const float4 q = s4[8 * h + j];  // scales of keys 2j, 2j + 1: [key][2]
                        const int i = i0 + 16 * h + 2 * j;
                        v[2 * j] = __fmul_rn(i2f_small(vraw[i * D + t]), vg ? q.y : q.x);
                        v[2 * j + 1] = __fmul_rn(i2f_small(vraw[(i + 1) * D + t]), vg ? q.w : q.z);
                    }
#pragma unroll
                    for (int j = 0; j < 16; ++j)
                        if (16 * h + j < nc) acc = fmaf(v[j], w[j], acc);
                }
                for (int i = i0 + nc; i < i1; ++i)
                    acc = fmaf(h2f(a.Vn[(size_t)(c0 + i - a.cache_len) * a.kn_row + t]), sw[i], acc);
            }
            run_sum = __fadd_rn(run_sum, bsm[blk]);
        }
        bar();
    }
    if (t >= D) return __float2half_rn(0.0f);
    return run_sum > 0.0f ? f2h(__fmul_rn(acc, __fdiv_rn(1.0f, run_sum))) : __float2half_rn(0.0f);
}

}  // namespace cb
