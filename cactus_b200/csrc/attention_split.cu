// Long-context attention against an INT8 cache, in the reference order, split over the keys.
//
// cactus_attention_hybrid_int8_fp16 (kernel_attention.cpp:257-482) walks 32-key blocks in
// order; per block it takes the block maximum, the weights expf(s - block max) and their
// in-order sum, rescales the running sum and the per-dim accumulator by expf(previous block
// max - block max), then adds the block's keys to the accumulator one fmaf at a time. Only
// that last step is a recurrence over keys; everything else of a block depends on the block
// alone (attention_core.cuh states the same decomposition for one CTA). So with one query
// and tens of thousands of keys the work splits exactly:
//   1. attn_split_scores_kernel — one CTA per (sequence, query, kv head, 256 keys): scores
//      of every q head of the group (8-lane dot products folded in the reference tree),
//      block maxima, weights and in-order block sums, written to a scratch buffer;
//   2. attn_split_chain_kernel — one CTA per (sequence, query, q head, 64 dims), thread = dim:
//      the corrections of all blocks in parallel, then the in-order V recurrence over a
//      4-stage cp.async ring of 128-key V chunks (the only serial part: one fmaf per key).
// The result bits equal those of attn_exact_core (and of the reference) for every length.
#include <map>
#include <mutex>

#include "attention_core.cuh"
#include "common.cuh"
#include "ops.h"

namespace cb {

namespace {

constexpr int kS1Keys = 256;     // keys per scoring CTA (multiple of 32)
constexpr int kS1Threads = 256;
constexpr int kS2Keys = 128;     // keys per staged chunk of the recurrence (multiple of 32)
constexpr int kS2Stages = 4;

// int8 -> fp32, exact: 1.5 * 2^23 + x holds x in its low mantissa bits (|x| <= 128); an integer
// add and a float subtract instead of a conversion instruction
__device__ __forceinline__ float i8_to_f(int8_t x) {
    return __fsub_rn(__int_as_float(0x4B400000 + (int)x), 12582912.0f);
}

struct SplitArgs {
    const __half* q;
    const int8_t* kc;
    const int8_t* vc;
    const float* ks;
    const float* vs;
    const __half* kn;
    const __half* vn;
    __half* o;
    float* w;    // [items][lw] weights
    float* bmx;  // [items][nbw] block maxima
    float* bsm;  // [items][nbw] block sums
    int* bz;     // [items][nbw] 1: some weight of the block is 0
    long long kc_bstride, sc_bstride, pos_off, lw, nbw;
    int S, cache_len, new_len, Hq, Hkv, causal, qgs;
    float scale;
    const int* dstate;  // non-null: cache_len = dstate[0], pos_off = dstate[1] (read on the device)
    KvPaging pg;        // paged cache (table non-null): kc/vc/ks/vs are the pools, no batch stride
};

// Lengths that live on the device (CUDA-graph decode): read after griddepcontrol.wait, since
// the previous kernels of the step may still be advancing them.
__device__ __forceinline__ void split_lengths(SplitArgs& a) {
    if (a.dstate) {
        a.cache_len = __ldcg(a.dstate);
        a.pos_off = __ldcg(a.dstate + 1);
    }
}

__device__ __forceinline__ long long split_kv_end(const SplitArgs& a, int qp) {
    const long long kv_seq_len = (long long)a.cache_len + a.new_len;
    return a.causal ? min(kv_seq_len, a.pos_off + qp + 1) : kv_seq_len;
}

template <int D>
__host__ __device__ constexpr int s1_row() {  // padded K row: the keys of a warp's load hit different banks
    return D + 16;
}
template <int D>
__host__ __device__ constexpr int s1_smem(int grp) {
    return kS1Keys * s1_row<D>() + kS1Keys * 2 * 4 + grp * D * 4 + grp * kS1Keys * 4;
}
// dims of one chain CTA: up to 64 (two warps), so a head's dims spread over D / 64 CTAs and a
// single query keeps several SMs busy
template <int D>
__host__ __device__ constexpr int s2_dims() {
    return D < 64 ? D : 64;
}
template <int D>
__host__ __device__ constexpr int s2_stage_bytes() {  // V rows (this CTA's dims) | weights | V scales [2][keys]
    return kS2Keys * s2_dims<D>() + kS2Keys * 4 + kS2Keys * 2 * 4;
}

// grid (B * S * Hkv, ceil(kv_seq_len / kS1Keys)), kS1Threads threads
template <int D>
__global__ void __launch_bounds__(kS1Threads) attn_split_scores_kernel(SplitArgs a) {
    pdl_launch_dependents();
    pdl_wait();
    split_lengths(a);
    extern __shared__ __align__(16) uint8_t smem[];
    const int grp = a.Hq / a.Hkv;
    const long long gi = blockIdx.x;
    const int kvh = (int)(gi % a.Hkv);
    const int qp = (int)((gi / a.Hkv) % a.S);
    const int b = (int)(gi / ((long long)a.Hkv * a.S));
    const long long kv_end = split_kv_end(a, qp);
    const long long c0 = (long long)blockIdx.y * kS1Keys;
    if (c0 >= kv_end) return;
    const int n = (int)min((long long)kS1Keys, kv_end - c0);
    const int ncached = (int)max(0LL, min((long long)n, (long long)a.cache_len - c0));
    const int nqg = (D + a.qgs - 1) / a.qgs;
    const size_t kv_row = (size_t)a.Hkv * D;
    const long long sc_row = (long long)a.Hkv * nqg;
    constexpr int KR = s1_row<D>();
    int8_t* kraw = reinterpret_cast<int8_t*>(smem);                 // [kS1Keys][KR]
    float* ksc = reinterpret_cast<float*>(kraw + kS1Keys * KR);     // [kS1Keys][2]
    float* qs = ksc + kS1Keys * 2;                                  // [grp][D]
    float* sc = qs + grp * D;                                       // [grp][kS1Keys]
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const int* pt = a.pg.table ? a.pg.table + (size_t)b * a.pg.pps : nullptr;
    const int8_t* Kc = a.kc + (pt ? 0 : b * a.kc_bstride) + (size_t)kvh * D;
    const float* ks = a.ks + (pt ? 0 : b * a.sc_bstride) + (size_t)kvh * nqg;
    if (pt) {  // paged: rows through the block table (the branch is uniform, outside the loops)
        for (int c = t; c < ncached * (D / 16); c += kS1Threads) {
            const int i = c / (D / 16), off = (c % (D / 16)) * 16;
            cp_async16(kraw + i * KR + off, Kc + (size_t)kv_page_row(pt, a.pg.shift, c0 + i) * kv_row + off);
        }
        for (int c = t; c < ncached * nqg; c += kS1Threads) {
            const int i = c / nqg, g = c % nqg;
            cp_async4(ksc + i * 2 + g, ks + (size_t)kv_page_row(pt, a.pg.shift, c0 + i) * sc_row + g);
        }
    } else {
        for (int c = t; c < ncached * (D / 16); c += kS1Threads) {
            const int i = c / (D / 16), off = (c % (D / 16)) * 16;
            cp_async16(kraw + i * KR + off, Kc + (size_t)(c0 + i) * kv_row + off);
        }
        for (int c = t; c < ncached * nqg; c += kS1Threads) {
            const int i = c / nqg, g = c % nqg;
            cp_async4(ksc + i * 2 + g, ks + (size_t)(c0 + i) * sc_row + g);
        }
    }
    cp_async_commit();
    const int h0 = kvh * grp;
    for (int c = t; c < grp * D; c += kS1Threads) {
        const int qh = c / D, d = c % D;
        qs[c] = h2f(a.q[(((size_t)b * a.S + qp) * a.Hq + h0 + qh) * D + d]);
    }
    cp_async_wait<0>();
    __syncthreads();
    const __half* Kn = a.kn + (size_t)b * a.new_len * kv_row + (size_t)kvh * D;
    const long long aq = a.pos_off + qp;
    constexpr int KPR = kS1Threads / 8;  // keys per round
    const int kj = t & 7;
    for (int qh = 0; qh < grp; ++qh) {
        const float* qv = qs + qh * D;
        for (int r = 0; r < kS1Keys / KPR; ++r) {
            const int i = (t >> 3) + KPR * r;
            float acc8 = 0.0f;
            if (i < n) {
                if (i < ncached) {
                    const int8_t* kr = kraw + i * KR;
#pragma unroll
                    for (int d = kj; d < D; d += 8)
                        acc8 = fmaf(qv[d], __fmul_rn((float)kr[d], ksc[i * 2 + (d >= a.qgs ? 1 : 0)]), acc8);
                } else {
                    const __half* kr = Kn + (size_t)(c0 + i - a.cache_len) * kv_row;
#pragma unroll
                    for (int d = kj; d < D; d += 8) acc8 = fmaf(qv[d], h2f(kr[d]), acc8);
                }
            }
            const int base = lane & ~7;
            float p[8];
#pragma unroll
            for (int m = 0; m < 8; ++m) p[m] = __shfl_sync(0xffffffffu, acc8, base + m);
            float s = __fmul_rn(fold8(p), a.scale);
            if (i >= n || (a.causal && c0 + i > aq)) s = -INFINITY;
            if (kj == 0) sc[qh * kS1Keys + i] = s;
        }
    }
    __syncthreads();
    // one warp per (q head, 32-key block): maximum, weights, in-order sum
    const int nbk = (n + 31) / 32;
    for (int pb = warp; pb < grp * nbk; pb += kS1Threads / 32) {
        const int qh = pb / nbk, blk = pb % nbk;
        const int i = blk * 32 + lane;
        const int bs = min(32, n - blk * 32);
        const float s = lane < bs ? sc[qh * kS1Keys + i] : -INFINITY;
        const float m = warp_max(s);
        const float w = (lane < bs && s != -INFINITY) ? expf_cr(__fsub_rn(s, m)) : 0.0f;
        float sum = 0.0f;
#pragma unroll
        for (int l = 0; l < 32; ++l) {
            const float x = __shfl_sync(0xffffffffu, w, l);
            if (l < bs) sum = __fadd_rn(sum, x);
        }
        const long long item = ((long long)b * a.S + qp) * a.Hq + h0 + qh;
        if (lane < bs) a.w[item * a.lw + c0 + i] = w;
        const unsigned zero = __ballot_sync(0xffffffffu, lane < bs && w == 0.0f);
        if (lane == 0) {
            const long long gb = c0 / 32 + blk;
            a.bmx[item * a.nbw + gb] = m;
            a.bsm[item * a.nbw + gb] = sum;
            a.bz[item * a.nbw + gb] = zero ? 1 : 0;
        }
    }
}

// grid (B * S * Hq, D / DC), DC = s2_dims<D>() threads: thread t owns output dim blockIdx.y * DC + t
template <int D>
__global__ void __launch_bounds__(s2_dims<D>()) attn_split_chain_kernel(SplitArgs a) {
    pdl_launch_dependents();
    pdl_wait();
    split_lengths(a);
    extern __shared__ __align__(16) uint8_t smem[];
    constexpr int SB = s2_stage_bytes<D>();
    constexpr int DC = s2_dims<D>();
    const int dim0 = blockIdx.y * DC;
    const long long item = blockIdx.x;
    const int h = (int)(item % a.Hq);
    const int qp = (int)((item / a.Hq) % a.S);
    const int b = (int)(item / ((long long)a.Hq * a.S));
    const int kvh = h / (a.Hq / a.Hkv);
    const long long kv_end = split_kv_end(a, qp);
    const int nb = (int)((kv_end + 31) / 32);
    const int nqg = (D + a.qgs - 1) / a.qgs;
    const size_t kv_row = (size_t)a.Hkv * D;
    const long long sc_row = (long long)a.Hkv * nqg;
    const int t = threadIdx.x;
    float* bmx = reinterpret_cast<float*>(smem + kS2Stages * SB);
    float* bsm = bmx + a.nbw;
    float* corr = bsm + a.nbw;
    int* bz = reinterpret_cast<int*>(corr + a.nbw);
    for (int j = t; j < nb; j += DC) {
        bmx[j] = a.bmx[item * a.nbw + j];
        bsm[j] = a.bsm[item * a.nbw + j];
        bz[j] = a.bz[item * a.nbw + j];
    }
    __syncthreads();
    // correction of block j: expf(max of the last non-empty block before j - max of j)
    for (int j = t; j < nb; j += DC) {
        float pm = -INFINITY;
        for (int k = j - 1; k >= 0; --k) {
            if (bmx[k] > -INFINITY) {
                pm = bmx[k];
                break;
            }
        }
        corr[j] = expf_cr(__fsub_rn(pm, bmx[j]));
    }
    const int* pt = a.pg.table ? a.pg.table + (size_t)b * a.pg.pps : nullptr;
    const int8_t* Vc = a.vc + (pt ? 0 : b * a.kc_bstride) + (size_t)kvh * D;
    const float* vs = a.vs + (pt ? 0 : b * a.sc_bstride) + (size_t)kvh * nqg;
    const __half* Vn = a.vn + (size_t)b * a.new_len * kv_row + (size_t)kvh * D;
    const float* W = a.w + item * a.lw;
    const long long nch = (kv_end + kS2Keys - 1) / kS2Keys;
    auto stage = [&](long long c) {
        uint8_t* st = smem + (int)(c % kS2Stages) * SB;
        int8_t* vraw = reinterpret_cast<int8_t*>(st);
        float* wst = reinterpret_cast<float*>(st + kS2Keys * DC);
        float* vsc = wst + kS2Keys;
        const long long c0 = c * kS2Keys;
        const int n = (int)min((long long)kS2Keys, kv_end - c0);
        const int ncached = (int)max(0LL, min((long long)n, (long long)a.cache_len - c0));
        if (pt) {  // paged: rows through the block table (uniform branch, outside the loops)
            for (int x = t; x < ncached * (DC / 16); x += DC) {
                const int i = x / (DC / 16), off = (x % (DC / 16)) * 16;
                cp_async16(vraw + i * DC + off, Vc + (size_t)kv_page_row(pt, a.pg.shift, c0 + i) * kv_row + dim0 + off);
            }
            for (int x = t; x < ncached * nqg; x += DC) {
                const int i = x / nqg, g = x % nqg;
                cp_async4(vsc + g * kS2Keys + i, vs + (size_t)kv_page_row(pt, a.pg.shift, c0 + i) * sc_row + g);
            }
        } else {
            for (int x = t; x < ncached * (DC / 16); x += DC) {
                const int i = x / (DC / 16), off = (x % (DC / 16)) * 16;
                cp_async16(vraw + i * DC + off, Vc + (size_t)(c0 + i) * kv_row + dim0 + off);
            }
            for (int x = t; x < ncached * nqg; x += DC) {
                const int i = x / nqg, g = x % nqg;
                cp_async4(vsc + g * kS2Keys + i, vs + (size_t)(c0 + i) * sc_row + g);
            }
        }
        for (int x = t; x < n; x += DC) cp_async4(wst + x, W + c0 + x);
        cp_async_commit();
    };
    for (int c = 0; c < kS2Stages - 1; ++c) {
        if (c < nch) stage(c);
        else cp_async_commit();
    }
    const int vg = (dim0 + t) / a.qgs;
    float acc = 0.0f, run_sum = 0.0f;
    for (long long c = 0; c < nch; ++c) {
        cp_async_wait<kS2Stages - 2>();
        __syncthreads();
        const uint8_t* st = smem + (int)(c % kS2Stages) * SB;
        const int8_t* vraw = reinterpret_cast<const int8_t*>(st);
        const float* wst = reinterpret_cast<const float*>(st + kS2Keys * DC);
        const float* vs_t = wst + kS2Keys + vg * kS2Keys;
        const long long c0 = c * kS2Keys;
        const int n = (int)min((long long)kS2Keys, kv_end - c0);
        const int ncached = (int)max(0LL, min((long long)n, (long long)a.cache_len - c0));
        const int blk0 = (int)(c0 / 32);
        // full chunk of cached keys, every block non-empty and without a zero weight: straight-
        // line code in which the values of block b + 1 are dequantised ahead of block b's fmaf
        // chain, so the scheduler overlaps the two (the same operations per dim, in order)
        bool fast = n == kS2Keys && ncached == n;
#pragma unroll
        for (int bl = 0; bl < kS2Keys / 32; ++bl) fast = fast && bmx[blk0 + bl] > -INFINITY && !bz[blk0 + bl];
        if (fast) {
            auto deq = [&](float (&v)[32], int i0) {
                const float4* s4 = reinterpret_cast<const float4*>(vs_t + i0);
#pragma unroll
                for (int j4 = 0; j4 < 8; ++j4) {
                    const float4 sv = s4[j4];
                    const int i = i0 + 4 * j4;
                    v[4 * j4 + 0] = __fmul_rn(i8_to_f(vraw[i * DC + t]), sv.x);
                    v[4 * j4 + 1] = __fmul_rn(i8_to_f(vraw[(i + 1) * DC + t]), sv.y);
                    v[4 * j4 + 2] = __fmul_rn(i8_to_f(vraw[(i + 2) * DC + t]), sv.z);
                    v[4 * j4 + 3] = __fmul_rn(i8_to_f(vraw[(i + 3) * DC + t]), sv.w);
                }
            };
            auto step = [&](const float (&v)[32], int bl) {
                const float cr = corr[blk0 + bl];
                run_sum = __fmul_rn(run_sum, cr);
                acc = __fmul_rn(acc, cr);
                const float4* w4 = reinterpret_cast<const float4*>(wst + bl * 32);
#pragma unroll
                for (int j4 = 0; j4 < 8; ++j4) {
                    const float4 wq = w4[j4];
                    acc = fmaf(v[4 * j4 + 0], wq.x, acc);
                    acc = fmaf(v[4 * j4 + 1], wq.y, acc);
                    acc = fmaf(v[4 * j4 + 2], wq.z, acc);
                    acc = fmaf(v[4 * j4 + 3], wq.w, acc);
                }
                run_sum = __fadd_rn(run_sum, bsm[blk0 + bl]);
            };
            static_assert(kS2Keys == 128, "four 32-key blocks per chunk");
            float va[32], vb[32];
            deq(va, 0);
            deq(vb, 32);
            step(va, 0);
            deq(va, 64);
            step(vb, 1);
            deq(vb, 96);
            step(va, 2);
            step(vb, 3);
        }
        for (int bl = 0; !fast && bl < (n + 31) / 32; ++bl) {
            const int blk = blk0 + bl;
            if (bmx[blk] > -INFINITY) {
                const float cr = corr[blk];
                run_sum = __fmul_rn(run_sum, cr);
                acc = __fmul_rn(acc, cr);
            }
            // keys with weight 0 leave acc untouched (the reference skips them)
            const int i0 = bl * 32, i1 = min(n, i0 + 32);
            const int ic = min(i1, max(i0, ncached));  // [i0, ic) cached, [ic, i1) new keys
            if (ic - i0 == 32 && !bz[blk]) {
                // no zero weight in the block: dequantise the block's 32 values first (independent
                // loads and conversions), then the plain fmaf chain
                const float4* w4 = reinterpret_cast<const float4*>(wst + i0);
                const float4* s4 = reinterpret_cast<const float4*>(vs_t + i0);
                float v[32], w[32];
#pragma unroll
                for (int j4 = 0; j4 < 8; ++j4) {
                    const float4 wq = w4[j4], sv = s4[j4];
                    const int i = i0 + 4 * j4;
                    v[4 * j4 + 0] = __fmul_rn(i8_to_f(vraw[i * DC + t]), sv.x);
                    v[4 * j4 + 1] = __fmul_rn(i8_to_f(vraw[(i + 1) * DC + t]), sv.y);
                    v[4 * j4 + 2] = __fmul_rn(i8_to_f(vraw[(i + 2) * DC + t]), sv.z);
                    v[4 * j4 + 3] = __fmul_rn(i8_to_f(vraw[(i + 3) * DC + t]), sv.w);
                    w[4 * j4 + 0] = wq.x;
                    w[4 * j4 + 1] = wq.y;
                    w[4 * j4 + 2] = wq.z;
                    w[4 * j4 + 3] = wq.w;
                }
#pragma unroll
                for (int j = 0; j < 32; ++j) acc = fmaf(v[j], w[j], acc);
            } else if (ic - i0 == 32) {
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    const int i = i0 + j;
                    const float w = wst[i];
                    const float v = __fmul_rn((float)vraw[i * DC + t], vs_t[i]);
                    const float nacc = fmaf(v, w, acc);
                    acc = (w == 0.0f) ? acc : nacc;
                }
            } else {
                for (int i = i0; i < ic; ++i) {
                    const float w = wst[i];
                    const float v = __fmul_rn((float)vraw[i * DC + t], vs_t[i]);
                    const float nacc = fmaf(v, w, acc);
                    acc = (w == 0.0f) ? acc : nacc;
                }
            }
            for (int i = ic; i < i1; ++i) {
                const float w = wst[i];
                const float v = h2f(Vn[(size_t)(c0 + i - a.cache_len) * kv_row + dim0 + t]);
                const float nacc = fmaf(v, w, acc);
                acc = (w == 0.0f) ? acc : nacc;
            }
            run_sum = __fadd_rn(run_sum, bsm[blk]);
        }
        __syncthreads();  // every thread is done with this stage before it is refilled
        if (c + kS2Stages - 1 < nch) stage(c + kS2Stages - 1);
        else cp_async_commit();
    }
    cp_async_wait<0>();
    a.o[item * D + dim0 + t] = run_sum > 0.0f ? f2h(__fmul_rn(acc, __fdiv_rn(1.0f, run_sum))) : __float2half_rn(0.0f);
}

// Grow-only per-device scratch (old buffers stay allocated: kernels queued earlier on other
// streams may still read them).
std::mutex g_split_mu;
std::map<int, std::pair<void*, size_t>> g_split_scratch;
float* split_scratch(size_t bytes) {
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lk(g_split_mu);
    auto& e = g_split_scratch[dev];
    if (e.second < bytes) {
        void* p = nullptr;
        if (cudaMalloc(&p, bytes) != cudaSuccess) {
            cudaGetLastError();
            return nullptr;
        }
        e = {p, bytes};
    }
    return static_cast<float*>(e.first);
}

template <int D>
bool split_attrs(size_t sm1, size_t sm2) {
    static std::mutex mu;
    static size_t attr1 = 0, attr2 = 0;
    std::lock_guard<std::mutex> lk(mu);
    if (sm1 > attr1) {
        if (cudaFuncSetAttribute(attn_split_scores_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm1) !=
            cudaSuccess)
            return false;
        attr1 = sm1;
    }
    if (sm2 > attr2) {
        if (cudaFuncSetAttribute(attn_split_chain_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm2) !=
            cudaSuccess)
            return false;
        attr2 = sm2;
    }
    return true;
}

template <int D>
size_t split_sm1(int grp) { return (size_t)s1_smem<D>(grp); }
template <int D>
size_t split_sm2(long long nbw) { return (size_t)kS2Stages * s2_stage_bytes<D>() + (size_t)4 * nbw * 4; }

// size_keys: keys the grid and the scratch rows are sized for (the live length, or with
// device-side lengths the largest one the launch may see)
template <int D>
int launch_split(SplitArgs a, long long items, long long size_keys, int B, cudaStream_t st) {
    const int grp = a.Hq / a.Hkv;
    const size_t sm1 = split_sm1<D>(grp), sm2 = split_sm2<D>(a.nbw);
    if (sm1 > kSplitMaxSmem || sm2 > kSplitMaxSmem) return -1;
    if (!split_attrs<D>(sm1, sm2)) return -1;
    const long long kv_items = (long long)B * a.S * a.Hkv;
    const long long nchunk = (size_keys + kS1Keys - 1) / kS1Keys;
    if (kv_items > 0x7FFFFFFFLL || nchunk > 65535 || items > 0x7FFFFFFFLL) return -1;
    launch_k(attn_split_scores_kernel<D>, dim3((unsigned)kv_items, (unsigned)nchunk), dim3(kS1Threads), sm1, st, a);
    launch_k(attn_split_chain_kernel<D>, dim3((unsigned)items, D / s2_dims<D>()), dim3(s2_dims<D>()), sm2, st, a);
    return 0;
}

long long split_lw(long long keys) { return (keys + kS2Keys - 1) / kS2Keys * kS2Keys; }

int split_common(const __half* q, const int8_t* kc, const int8_t* vc, const float* ks, const float* vs,
                 const __half* kn, const __half* vn, __half* o, int B, int S, int cache_len, int new_len, int Hq,
                 int Hkv, int D, float scale, long long pos_off, int causal, int qgs, long long kc_bstride,
                 long long sc_bstride, long long size_keys, const int* dstate, float* scr, size_t scr_bytes,
                 cudaStream_t st, KvPaging pg) {
    if (B < 1 || S < 1 || Hkv < 1 || Hq % Hkv || qgs % 8 || (D + qgs - 1) / qgs > 2) return -1;
    const long long lw = split_lw(size_keys);
    const long long nbw = lw / 32;
    const long long items = (long long)B * S * Hq;
    const size_t bytes = (size_t)items * (size_t)(lw + 3 * nbw) * 4;
    if (bytes > kSplitMaxScratch) return -1;
    if (!scr) scr = split_scratch(bytes);
    else if (bytes > scr_bytes) return -1;
    if (!scr) return -1;
    SplitArgs a;
    a.q = q;
    a.kc = kc;
    a.vc = vc;
    a.ks = ks;
    a.vs = vs;
    a.kn = kn;
    a.vn = vn;
    a.o = o;
    a.w = scr;
    a.bmx = scr + items * lw;
    a.bsm = a.bmx + items * nbw;
    a.bz = reinterpret_cast<int*>(a.bsm + items * nbw);
    a.kc_bstride = kc_bstride;
    a.sc_bstride = sc_bstride;
    a.pos_off = pos_off;
    a.lw = lw;
    a.nbw = nbw;
    a.S = S;
    a.cache_len = cache_len;
    a.new_len = new_len;
    a.Hq = Hq;
    a.Hkv = Hkv;
    a.causal = causal;
    a.qgs = qgs;
    a.scale = scale;
    a.dstate = dstate;
    a.pg = pg;
    switch (D) {
        case 64: return launch_split<64>(a, items, size_keys, B, st);
        case 128: return launch_split<128>(a, items, size_keys, B, st);
        case 256: return launch_split<256>(a, items, size_keys, B, st);
    }
    return -1;
}

}  // namespace

int launch_attention_split(const __half* q, const int8_t* kc, const int8_t* vc, const float* ks, const float* vs,
                           const __half* kn, const __half* vn, __half* o, int B, int S, int cache_len, int new_len,
                           int Hq, int Hkv, int D, float scale, long long pos_off, int causal, int qgs,
                           long long kc_bstride, long long sc_bstride, cudaStream_t st, KvPaging pg) {
    return split_common(q, kc, vc, ks, vs, kn, vn, o, B, S, cache_len, new_len, Hq, Hkv, D, scale, pos_off, causal,
                        qgs, kc_bstride, sc_bstride, (long long)cache_len + new_len, nullptr, nullptr, 0, st, pg);
}

size_t attention_split_scratch_bytes(long long items, long long max_keys) {
    const long long lw = split_lw(max_keys);
    return (size_t)items * (size_t)(lw + 3 * (lw / 32)) * 4;
}

int attention_split_prepare(int D, int Hq, int Hkv, long long max_keys) {
    if (Hkv < 1 || Hq % Hkv) return -1;
    const long long nbw = split_lw(max_keys) / 32;
    const int grp = Hq / Hkv;
    bool ok = false;
    switch (D) {
        case 64: ok = split_sm1<64>(grp) <= kSplitMaxSmem && split_sm2<64>(nbw) <= kSplitMaxSmem &&
                      split_attrs<64>(split_sm1<64>(grp), split_sm2<64>(nbw)); break;
        case 128: ok = split_sm1<128>(grp) <= kSplitMaxSmem && split_sm2<128>(nbw) <= kSplitMaxSmem &&
                       split_attrs<128>(split_sm1<128>(grp), split_sm2<128>(nbw)); break;
        case 256: ok = split_sm1<256>(grp) <= kSplitMaxSmem && split_sm2<256>(nbw) <= kSplitMaxSmem &&
                       split_attrs<256>(split_sm1<256>(grp), split_sm2<256>(nbw)); break;
    }
    return ok ? 0 : -1;
}

int launch_attention_split_dev(const __half* q, const int8_t* kc, const int8_t* vc, const float* ks, const float* vs,
                               const __half* kn, const __half* vn, __half* o, int B, int S, int new_len, int Hq,
                               int Hkv, int D, float scale, int causal, int qgs, long long kc_bstride,
                               long long sc_bstride, long long max_keys, const int* dstate, float* scratch,
                               size_t scratch_bytes, cudaStream_t st, KvPaging pg) {
    if (!dstate || !scratch) return -1;
    return split_common(q, kc, vc, ks, vs, kn, vn, o, B, S, 0, new_len, Hq, Hkv, D, scale, 0, causal, qgs, kc_bstride,
                        sc_bstride, max_keys, dstate, scratch, scratch_bytes, st, pg);
}

}  // namespace cb
