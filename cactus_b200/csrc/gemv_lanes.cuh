// Grouped INT8 / INT4 GEMV for 1-4 activation rows, one weight row per lane.
//
// Same arithmetic and result bits as qgemv_kernel (cactus_matmul_int8 / _int4,
// kernel_gemm.cpp:128-529): exact int32 sums of each (row, group), an fp32 FMA chain over the
// groups in order, times the activation row scale, to fp16; the same prologues (activation
// quantisation, optionally RMSNorm) and epilogues (store, residual, SiLU / GELU GLU).
//
// Layout of the work: lane l of a warp owns output row 32 * b + l of the warp's row blocks b
// and walks that row's K in chunks of 128 weight bytes, the whole fp32 chain of the row in its
// own register — so the chain needs no cross-lane step and a chunk costs a lane about one
// instruction per 2 weight bytes. Each warp feeds itself: a slot of its own S-deep ring holds
// nb consecutive chunks of its 32 rows, loaded by nb 2-D TMA tile copies (cp.async.bulk.tensor,
// box of 128 bytes x 32 rows, 128-byte swizzle, no multicast, L2 evict-first) on one mbarrier;
// the swizzle puts the lanes' 16-byte shared loads of 8 consecutive rows into different banks.
// The warp re-issues a slot once it has read it, so no block barrier is needed after the
// activation prologue. Each lane also prefetches its row's group scales for the next chunk
// with plain 4- or 2-byte loads.
#pragma once
#include "gemv.cuh"

namespace cb {

constexpr int kLaneMaxSlots = 16;
constexpr int kLanesThreads = 384;  // 12 row-owning warps: more independent streams per SM
constexpr int kLanesWarps = kLanesThreads / 32;

struct GemvLanesLayout {
    int kc, kcb, slot;  // k per chunk, weight bytes per row chunk (128), slot bytes (32 rows)
    int off_act, off_asum, off_as, off_xs, off_red, off_bars, off_warps, fixed;
};

__host__ __device__ inline GemvLanesLayout gemv_lanes_layout(int wf, int mt, int K, int G) {
    GemvLanesLayout L;
    L.kcb = 128;
    L.kc = wf ? 256 : 128;
    L.slot = 32 * L.kcb;
    (void)K;
    int off = 0;
    L.off_act = off;   off += align_up(mt * K, 128);
    L.off_asum = off;  off += align_up(mt * (K / G) * 4, 128);
    L.off_as = off;    off += 128;
    L.off_xs = off;    off += align_up(mt * K * 2, 128);
    L.off_red = off;   off += align_up(72 * 4, 128);
    L.off_bars = off;  off += align_up(kLanesWarps * kLaneMaxSlots * 8, 128);
    L.off_warps = align_up(off, 1024);  // swizzled TMA destinations: 1024-byte aligned slots
    L.fixed = L.off_warps + 1024;       // + slack for the runtime alignment of the window
    return L;
}

template <int WF, int MT, int GT, int PRO, int EPI>
__global__ void __launch_bounds__(kLanesThreads, 1)
    qgemv_lanes_kernel(const __grid_constant__ CUtensorMap wmap, GemvArgs a, int S, int wpc, int nb) {
    extern __shared__ __align__(128) uint8_t smem[];
    const GemvLanesLayout L = gemv_lanes_layout(WF, MT, a.K, a.G);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    constexpr int G = GT;  // the group size is a template parameter: the chunk loops unroll
    const int K = a.K, N = a.N, M = a.M;
    constexpr int kc = WF ? 256 : 128, gpc = kc / G;
    const int ng = K / G, kcb = L.kcb, nch = K / kc;
    int8_t* act = reinterpret_cast<int8_t*>(smem + L.off_act);
    int* asum = reinterpret_cast<int*>(smem + L.off_asum);
    float* as = reinterpret_cast<float*>(smem + L.off_as);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.off_bars) + warp * kLaneMaxSlots;
    uint8_t* const ring0 = smem + L.off_warps;
    uint8_t* wsm = ring0 + ((1024u - (smem_u32(ring0) & 1023u)) & 1023u) + (size_t)warp * S * nb * L.slot;
    const uint16_t* sbase = reinterpret_cast<const uint16_t*>(a.ws);
    const uint64_t policy = l2_policy_evict_first();

    // row blocks of this warp: first_rb, first_rb + nw, ... (consecutive blocks on different SMs)
    const int nw = gridDim.x * wpc;
    const int first_rb = warp * gridDim.x + blockIdx.x;
    const int nrb = (N + 31) / 32;
    const int my_rb = (warp < wpc && first_rb < nrb) ? (nrb - first_rb + nw - 1) / nw : 0;
    const int T = my_rb * nch;  // (row block, chunk) tasks of this warp, in order
    const int slot = nb * L.slot;  // a ring slot holds nb consecutive chunks (nch % nb == 0)

    if (lane == 0)
        for (int s = 0; s < S; ++s) mbar_init(&bars[s], 1);
    fence_mbar_init();
    __syncwarp();
    // slot task v: chunks v * nb .. v * nb + nb - 1 (one row block) into slot v % S
    auto issue = [&](int v) {
        if (v * nb >= T) return;
        const int u = v * nb, rb = first_rb + (u / nch) * nw, c = u % nch, s = v % S;
        if (lane == 0) {  // rows past N read as zeros and still count in the transaction
            mbar_arrive_expect_tx(&bars[s], (unsigned)slot);
            for (int b = 0; b < nb; ++b)
                tma_load_2d_tile(wsm + (size_t)s * slot + b * L.slot, &wmap, (c + b) * kcb, rb * 32, &bars[s],
                                 policy);
        }
    };
    // weights do not depend on the previous kernel: the first chunks stream while it finishes
    for (int v = 0; v < S; ++v) issue(v);
    pdl_launch_dependents();
    pdl_wait();
    gemv_prologue<WF, MT, PRO, kLanesThreads>(a, act, asum, as, reinterpret_cast<__half*>(smem + L.off_xs),
                               reinterpret_cast<float*>(smem + L.off_red));

    // the lane's row scales of chunk t: gpc consecutive fp16 values (4-byte loads when gpc is
    // even: the offset (row * ng + c * gpc) * 2 is then a multiple of 4)
    auto load_scales = [&](int t, uint32_t (&r)[4]) {
        if (t >= T) return;
        const int rb = first_rb + (t / nch) * nw, c = t % nch, row = rb * 32 + lane;
        if (row >= N) return;
        const uint16_t* sp = sbase + (size_t)row * ng + (size_t)c * gpc;
        if (gpc >= 2) {
#pragma unroll
            for (int i = 0; i < 4; ++i)
                if (2 * i < gpc) r[i] = __ldg(reinterpret_cast<const uint32_t*>(sp) + i);
        } else {
            r[0] = __ldg(sp);
        }
    };
    uint32_t sc[4] = {0, 0, 0, 0}, scn[4] = {0, 0, 0, 0};
    load_scales(0, sc);
    float run[MT];
#pragma unroll
    for (int m = 0; m < MT; ++m) run[m] = 0.0f;
    bool ok = true;
    int t = 0;
    for (; t < T; ++t) {
        const int v = t / nb, b = t - v * nb, s = v % S, c = t % nch;
        const int row = (first_rb + (t / nch) * nw) * 32 + lane;
        load_scales(t + 1, scn);
        if (b == 0 && !mbar_wait_bounded(&bars[s], (unsigned)((v / S) & 1))) {
            ok = false;
            break;
        }
        // row `lane` of the chunk: 16-byte piece j at (j ^ (lane & 7)) * 16 (128-byte swizzle)
        const uint8_t* wr = wsm + (size_t)s * slot + b * L.slot + lane * 128;
        const int sw = lane & 7;
#pragma unroll
        for (int gi = 0; gi < gpc; ++gi) {
            // integer group sums are exact in any order: two independent dp4a chains per row
            int acc[MT][2];
#pragma unroll
            for (int m = 0; m < MT; ++m) acc[m][0] = acc[m][1] = 0;
            const int kb = c * kc + gi * G;  // first k of the group
            if constexpr (WF == 0) {
#pragma unroll
                for (int q = 0; q < G / 16; ++q) {
                    const int4 wv = *reinterpret_cast<const int4*>(wr + ((((gi * G) >> 4) + q) ^ sw) * 16);
#pragma unroll
                    for (int m = 0; m < MT; ++m) {
                        if (m < M) {
                            const int4 av = *reinterpret_cast<const int4*>(act + m * K + kb + q * 16);
                            acc[m][q & 1] = dp4a_ss(av.x, wv.x, acc[m][q & 1]);
                            acc[m][q & 1] = dp4a_ss(av.y, wv.y, acc[m][q & 1]);
                            acc[m][q & 1] = dp4a_ss(av.z, wv.z, acc[m][q & 1]);
                            acc[m][q & 1] = dp4a_ss(av.w, wv.w, acc[m][q & 1]);
                        }
                    }
                }
            } else {
                // 16 packed bytes = 32 k; activations permuted inside 8-blocks by the prologue so
                // that even k pair with low nibbles and odd k with high nibbles (nibble ^ 8 is
                // the value + 8, corrected with 8 * the group's activation sum)
#pragma unroll
                for (int q = 0; q < G / 32; ++q) {
                    const int4 wv = *reinterpret_cast<const int4*>(wr + ((((gi * (G / 2)) >> 4) + q) ^ sw) * 16);
                    const unsigned ww[4] = {(unsigned)wv.x, (unsigned)wv.y, (unsigned)wv.z, (unsigned)wv.w};
#pragma unroll
                    for (int m = 0; m < MT; ++m) {
                        if (m < M) {
                            const int4 a0 = *reinterpret_cast<const int4*>(act + m * K + kb + q * 32);
                            const int4 a1 = *reinterpret_cast<const int4*>(act + m * K + kb + q * 32 + 16);
                            const int ae[4] = {a0.x, a0.z, a1.x, a1.z};
                            const int ao[4] = {a0.y, a0.w, a1.y, a1.w};
#pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                const unsigned lo = (ww[e] & 0x0F0F0F0Fu) ^ 0x08080808u;
                                const unsigned hi = ((ww[e] >> 4) & 0x0F0F0F0Fu) ^ 0x08080808u;
                                acc[m][0] = dp4a_su(ae[e], lo, acc[m][0]);
                                acc[m][1] = dp4a_su(ao[e], hi, acc[m][1]);
                            }
                        }
                    }
                }
#pragma unroll
                for (int m = 0; m < MT; ++m)
                    if (m < M) acc[m][0] -= 8 * asum[m * ng + c * gpc + gi];
            }
            const int wi = (gi >> 1) & 3;  // register selects, not an indexed (local-memory) array
            const uint32_t swd = wi == 0 ? sc[0] : wi == 1 ? sc[1] : wi == 2 ? sc[2] : sc[3];
            const float scale = h2f_bits((uint16_t)(gpc >= 2 ? ((gi & 1) ? (swd >> 16) : (swd & 0xFFFFu)) : swd));
#pragma unroll
            for (int m = 0; m < MT; ++m)
                if (m < M) run[m] = fmaf(i2f_small(acc[m][0] + acc[m][1]), scale, run[m]);
        }
        // the slot is read: hand it to the slot task S ahead (after the generic-proxy reads,
        // before the bulk copy writes it)
        if (b == nb - 1) {
            __syncwarp();
            fence_proxy_async_shared();
            issue(v + S);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) sc[i] = scn[i];
        if (c == nch - 1) {  // row complete: C[m, row]
#pragma unroll
            for (int m = 0; m < MT; ++m) {
                if (m >= M) break;
                const __half v = __float2half_rn(__fmul_rn(run[m], as[m]));
                if constexpr (EPI == (int)Epi::STORE || EPI == (int)Epi::RESIDUAL) {
                    if (row < N) {
                        __half o = v;
                        if constexpr (EPI == (int)Epi::RESIDUAL) o = __hadd(a.resid[(size_t)m * N + row], v);
                        a.out[(size_t)m * N + row] = o;
                    }
                } else {
                    // rows come in (gate, up) pairs on neighbouring lanes (row blocks start even)
                    const __half up = __shfl_down_sync(0xffffffffu, v, 1);
                    if (row + 1 < N && (lane & 1) == 0) {
                        const __half g = (EPI == (int)Epi::GLU_SILU) ? ref_silu(v) : ref_gelu(v);
                        a.out[(size_t)m * (N / 2) + row / 2] = __hmul(g, up);
                    }
                }
                run[m] = 0.0f;
            }
        }
    }
    if (!ok) {
        if (lane == 0) report_dev_error(kDevTmaTimeout);
        // no copy may land after the block leaves: wait (bounded) for the ones issued
        for (int v = t / nb; v < t / nb + S && v * nb < T; ++v) mbar_wait_bounded(&bars[v % S], (unsigned)((v / S) & 1));
    }
}

}  // namespace cb
