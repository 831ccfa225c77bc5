// Persistent decode step: one cooperative launch runs a whole batch-1 decode token —
// embedding, every transformer layer (Qwen/Llama block: RMSNorm -> fused QKV -> per-head
// q/k norm + RoPE -> KV append -> attention -> O + residual -> RMSNorm -> gate/up + SiLU-GLU
// -> down + residual), the final norm, the lm head and the greedy argmax — with the same
// arithmetic as the multi-kernel path (gemv.cuh, attention_core.cuh, head_ops.cuh), so the
// tokens are bit-identical to it and to the reference order.
//
// Why: at batch 1 each projection is a few MB, so a kernel per op is bound by launch and
// dependency latency, not by HBM. Here one block per SM stays resident for the token:
//  * warp 11 of every block is a producer that streams the block's share of every weight
//    matrix of the token (a fixed row range per matrix, 8-row units) through a ring of
//    shared-memory slots with 1-D TMA bulk copies (no multicast), full/empty mbarriers per
//    slot. Weights do not depend on activations, so the stream runs ahead of the layer
//    dependency chain by the ring's depth and HBM stays busy across phase boundaries;
//  * warps 0-10 consume: per phase they rebuild the quantised activations in shared memory
//    (every block redundantly, which is cheaper than another exchange), reduce their rows and
//    write outputs. Phases (QKV | attention | O | gate-up | down, five per layer) hand data
//    over as tagged words (fp16 bits + the writer's version tag, see PArgs): a block polls
//    the words it needs until they carry the expected version, so there is no grid barrier
//    and a phase starts as soon as its own inputs exist (the attention blocks wait for their
//    head's rows only). Reuse of a buffer is ordered by the data flow: every block writes
//    QKV and gate-up rows (the grid is sized so), and every reader waits for whole vectors,
//    so a block can only overwrite a version once every block has read it. Per buffer:
//    - hidden (O / down outputs, read whole by the next RMSNorm prologue): a down writer has
//      read all of `gated`, which every block wrote after reading the O version; an O writer
//      has read all of `attn`, whose heads needed every QKV row, which every block wrote
//      after reading the down version. The residual reads are the writer's own rows.
//    - qkv: a writer has read the whole hidden state of the previous down phase, whose
//      writers read all of `gated`, written by every block after its attention work.
//    - attn: a head's writer read its QKV rows, written after their blocks read the whole
//      hidden state, i.e. after all of `gated` of the previous layer, which every block
//      wrote after its O prologue had read `attn`.
//    - gated: a writer read the whole O output, whose writers read all of `attn`, whose
//      heads waited for QKV rows that every block wrote after its down prologue of the
//      previous layer had read `gated`.
//  * blocks 0..Hq-1 run one attention head each (the reference-order core).
//  * the lm head keeps a per-block first-max key; the last block to finish combines them,
//    writes the next token, advances the device state and re-arms the sync words.
// Every wait is bounded; a timeout sets the abort word and the device error, every block
// leaves at its next wait, and producers first wait for their copies in flight.
#include <algorithm>
#include <cstdlib>

#include "../attention_core.cuh"
#include "../common.cuh"
#include "../gemv.cuh"
#include "decode_persistent.h"
#include "head_ops.cuh"

namespace cb {
namespace eng {

namespace {

constexpr int kPCW = 11;       // consumer warps
constexpr int kPC = kPCW * 32; // consumer threads
constexpr int kPT = kPC + 32;  // + one producer warp; 384 threads leave ~170 registers a thread
constexpr int kACH = 256;      // attention keys per staged chunk
constexpr int kStaticSmem = 1024;

enum : int { kEpiStore = 0, kEpiResid = 1, kEpiGlu = 2, kEpiLm = 3 };

__device__ __forceinline__ void cbar() { asm volatile("bar.sync 1, %0;" ::"n"(kPC) : "memory"); }
struct SyncConsumers {
    __device__ __forceinline__ void operator()() const { cbar(); }
};

__host__ __device__ inline int a128(int v) { return (v + 127) / 128 * 128; }

// rows of an [N, K] matrix owned by block c of P: 8-row units split evenly. 32-bit unsigned
// arithmetic (persistent_plan checks (N / 8) * (P + 1) < 2^31): a 64-bit division is a long
// software sequence, and this runs at the start of every projection.
__host__ __device__ inline void rows_of(int N, int c, int P, int& r0, int& r1) {
    const unsigned U = (unsigned)N >> 3;
    r0 = (int)((U * (unsigned)c) / (unsigned)P) * 8;
    r1 = (int)((U * (unsigned)(c + 1)) / (unsigned)P) * 8;
}

struct JobW {
    const int8_t* w;
    const __half* s;
    int N, K;
};

// job j = 4*layer + {0 qkv, 1 o, 2 gate-up, 3 down}; j = 4*L is the lm head
__device__ __forceinline__ JobW job_w(const PArgs& a, int j) {
    if (j == 4 * a.L) return {a.lm_w, a.lm_s, a.V, a.H};
    const PLayer& ly = a.layers[j >> 2];
    switch (j & 3) {
        case 0: return {ly.wqkv, ly.sqkv, a.QKVN, a.H};
        case 1: return {ly.wo, ly.so, a.H, a.Hq * a.D};
        case 2: return {ly.wgu, ly.sgu, 2 * a.F, a.H};
        default: return {ly.wd, ly.sd, a.H, a.F};
    }
}
__host__ __device__ inline int rows_per_slot(int slot_w, int K) { return (slot_w / K) & ~7; }

// Bounded mbarrier wait with back-off: a thread spinning on try_wait keeps the SM's shared
// memory pipe busy and slows every other warp of the block, so failed polls sleep `ns`.
__device__ __forceinline__ bool wait_abortable(uint64_t* bar, unsigned par, const unsigned* abort, unsigned ns,
                                               unsigned limit) {
    for (uint32_t i = 0; i < limit; ++i) {
        if (mbar_try_wait(bar, par)) return true;
        __nanosleep(ns);
        if ((i & 15) == 15 && ld_volatile_u32(abort)) return false;
    }
    return false;
}

__device__ __forceinline__ void set_abort(const PArgs& a, unsigned code) {
    atomicExch(&a.sync->abort, 1u);
    report_dev_error(code);
}

// ------------------------------------------------------------------ tagged activation words
__device__ __forceinline__ unsigned vtag(const PArgs& a, int v) { return 1u + (a.tag_base + (unsigned)v) % 65535u; }
__device__ __forceinline__ void st_tagged(uint32_t* p, __half h, unsigned tag) {
    const uint32_t w = (tag << 16) | (uint32_t)__half_as_ushort(h);
    asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(w) : "memory");
}
__device__ __forceinline__ uint4 ld_relaxed_v4(const uint32_t* p) {
    uint4 v;
    asm volatile("ld.relaxed.gpu.global.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p)
                 : "memory");
    return v;
}
__device__ __forceinline__ bool tagged4(const uint4& v, unsigned tag) {
    return ((v.x >> 16) == tag) & ((v.y >> 16) == tag) & ((v.z >> 16) == tag) & ((v.w >> 16) == tag);
}
__device__ __forceinline__ __half word_h(uint32_t w) { return __ushort_as_half((unsigned short)(w & 0xFFFFu)); }

// Bounded poll of the next attempt: false once `it` passes the spin limit (the abort word and
// the device error are set) or, checked every 64 attempts, once another block aborted.
__device__ __forceinline__ bool poll_go_on(const PArgs& a, uint32_t it) {
    if (it > a.spin_limit) {
        set_abort(a, kDevFlagTimeout);
        return false;
    }
    return (it & 63) != 63 || !ld_volatile_u32(&a.sync->abort);
}

// Polls one tagged word until it carries `tag`.
__device__ __forceinline__ bool poll_word(const PArgs& a, const uint32_t* p, unsigned tag, uint32_t& w) {
    w = ld_relaxed_gpu(p);
    for (uint32_t it = 0; (w >> 16) != tag; ++it) {
        if (!poll_go_on(a, it)) return false;
        w = ld_relaxed_gpu(p);
    }
    return true;
}

// ------------------------------------------------------------------ producer (one thread)
__device__ void producer(const PArgs& a, uint8_t* ring, uint64_t* full, uint64_t* empty) {
    const int NS = a.nslots, sb = a.slot_w + a.slot_s;
    unsigned k = 0;
    bool ok = true;
    const int J = 4 * a.L + 1;
    const uint64_t stream_policy = l2_policy_evict_first();
    for (int j = 0; j < J && ok; ++j) {
        const JobW jw = job_w(a, j);
        int r0, r1;
        rows_of(jw.N, blockIdx.x, gridDim.x, r0, r1);
        const int spr = rows_per_slot(a.slot_w, jw.K), ng = jw.K / a.G;
        for (int r = r0; r < r1; r += spr) {
            const int s = (int)(k % NS);
            if (k >= (unsigned)NS && !wait_abortable(&empty[s], ((k / NS) - 1) & 1, &a.sync->abort, 256, a.spin_limit)) {
                ok = false;
                break;
            }
            const int rows = min(spr, r1 - r);
            const unsigned wb = (unsigned)(rows * jw.K), sbytes = (unsigned)(rows * ng * 2);
            uint8_t* dst = ring + (size_t)s * sb;
            mbar_arrive_expect_tx(&full[s], wb + sbytes);
            tma_load_1d_hint(dst, jw.w + (size_t)r * jw.K, wb, &full[s], stream_policy);
            tma_load_1d_hint(dst + a.slot_w, jw.s + (size_t)r * ng, sbytes, &full[s], stream_policy);
            ++k;
        }
    }
    if (!ok) {
        set_abort(a, kDevTmaTimeout);
        // wait (bounded) for the copies already issued so none lands after the block exits
        for (unsigned kk = k > (unsigned)NS ? k - NS : 0; kk < k; ++kk) mbar_wait_bounded(&full[kk % NS], (kk / NS) & 1);
    }
}

// ------------------------------------------------------------------ consumer helpers
struct Cs {  // consumer shared memory
    int8_t* act;
    __half* xs;
    __half* xsT;  // lane-major copy for the RMS chain
    int* gsm;
    float* gsf;
    __half* ob;
    float* red;   // [64]
    float* as;    // activation scale of the current job
    int* flag;
    int* fail;    // set (never cleared) by a thread whose poll gave up
    unsigned long long* best;  // [16]
};

constexpr int kMaxCpg = 8;  // 16-byte chunks per quantisation group (G <= 128)

// Shared-memory work in these phases is latency-bound (one warp at a time on a dependent
// chain), so activations move as 16-byte chunks: one thread per 8 consecutive elements.

// Row stride (halves) of the lane-major copy of a K-element vector: K/16 rounded up to 8,
// plus 8 of padding (rows stay 16-byte aligned and fall into different banks).
__host__ __device__ constexpr int lanemajor_stride(int K) { return ((K / 16 + 7) & ~7) + 8; }

// Stages K fp16 activations written by other blocks (L2 loads) into xs (src == null: xs is
// filled already). With `transposed`, also writes xsT, the lane-major copy the RMS chain
// reads with 16-byte loads: element k at (k % 16) * lanemajor_stride(K) + k / 16.
__device__ __forceinline__ void load_vec(const Cs& m, const __half* src, int K, bool transposed) {
    const int4* s4 = reinterpret_cast<const int4*>(src);
    int4* d4 = reinterpret_cast<int4*>(m.xs);
    const int TS = lanemajor_stride(K);
    for (int i = threadIdx.x; i < K / 8; i += kPC) {
        const int4 v = src ? __ldcg(s4 + i) : d4[i];
        if (src) d4[i] = v;
        if (transposed) {
            const __half* h = reinterpret_cast<const __half*>(&v);
#pragma unroll
            for (int j = 0; j < 8; ++j) m.xsT[(8 * (i & 1) + j) * TS + (i >> 1)] = h[j];
        }
    }
    cbar();
}

constexpr int kMaxR = 3;  // 16-byte chunks of a tagged vector a consumer thread has in flight

// Stages K tagged fp16 activations (K % 4 == 0) into xs (with `transposed`, also the
// lane-major copy xsT) once every word carries `tag`: each thread issues the loads of up to
// kMaxR of its 16-byte chunks at once, then re-polls the ones not yet written. False (after
// the block barrier, in every thread) when a poll gave up.
__device__ __forceinline__ bool load_tagged(const Cs& m, const PArgs& a, const uint32_t* src, int K, unsigned tag,
                                            bool transposed) {
    const int tid = threadIdx.x, n4 = K / 4, TS = lanemajor_stride(K);
    for (int base = 0; base < n4; base += kPC * kMaxR) {
        uint4 v[kMaxR];
        unsigned pend = 0;
#pragma unroll
        for (int r = 0; r < kMaxR; ++r) {
            const int i = base + tid + r * kPC;
            if (i < n4) {
                v[r] = ld_relaxed_v4(src + 4 * i);
                if (!tagged4(v[r], tag)) pend |= 1u << r;
            }
        }
        for (uint32_t it = 0; pend; ++it) {
            if (!poll_go_on(a, it)) {
                *m.fail = 1;
                break;
            }
#pragma unroll
            for (int r = 0; r < kMaxR; ++r) {
                if (pend & (1u << r)) {
                    v[r] = ld_relaxed_v4(src + 4 * (base + tid + r * kPC));
                    if (tagged4(v[r], tag)) pend &= ~(1u << r);
                }
            }
        }
#pragma unroll
        for (int r = 0; r < kMaxR; ++r) {
            const int i = base + tid + r * kPC;
            if (i < n4) {
                *reinterpret_cast<uint2*>(m.xs + 4 * i) =
                    make_uint2((v[r].x & 0xFFFFu) | (v[r].y << 16), (v[r].z & 0xFFFFu) | (v[r].w << 16));
                if (transposed) {
                    const uint32_t w[4] = {v[r].x, v[r].y, v[r].z, v[r].w};
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const int k = 4 * i + j;
                        m.xsT[(k & 15) * TS + (k >> 4)] = word_h(w[j]);
                    }
                }
            }
        }
    }
    cbar();
    return *m.fail == 0;
}

// RMSNorm sum of squares (rms_sumsq_warp's order, K % 16 == 0) from the lane-major copy:
// lane l < 16 walks its 16-element tiles in order with one 16-byte load per 8 tiles.
__device__ __forceinline__ float rms_sumsq_lanemajor(const __half* xsT, int K) {
    const int lane = threadIdx.x & 31, l16 = lane & 15, T = K / 16, TS = lanemajor_stride(K);
    const int4* p = reinterpret_cast<const int4*>(xsT + l16 * TS);
    float acc = 0.0f;
    for (int c = 0; c < T / 8; ++c) {
        const int4 v = p[c];
        const __half* h = reinterpret_cast<const __half*>(&v);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float f = h2f(h[j]);
            acc = fmaf(f, f, acc);
        }
    }
    for (int t = (T / 8) * 8; t < T; ++t) {
        const float f = h2f(xsT[l16 * TS + t]);
        acc = fmaf(f, f, acc);
    }
    const float a4 = __shfl_sync(0xffffffffu, acc, (lane & 3) + 4);
    const float a8 = __shfl_sync(0xffffffffu, acc, (lane & 3) + 8);
    const float a12 = __shfl_sync(0xffffffffu, acc, (lane & 3) + 12);
    const float a0 = __shfl_sync(0xffffffffu, acc, lane & 3);
    const float t4 = __fadd_rn(__fadd_rn(__fadd_rn(a0, a4), a8), a12);
    const float t0 = __shfl_sync(0xffffffffu, t4, 0), t1 = __shfl_sync(0xffffffffu, t4, 1);
    const float t2 = __shfl_sync(0xffffffffu, t4, 2), t3 = __shfl_sync(0xffffffffu, t4, 3);
    return __fadd_rn(__fadd_rn(t0, t1), __fadd_rn(t2, t3));
}

// xs holds K fp16 activations (K % 8 == 0; K % 16 == 0 with a norm); optional RMSNorm with
// weights `normw` (the load_vec call must have passed transposed = true), then the
// activation quantisation (gemv.cuh prologues, same arithmetic) into act / *as. nw0 holds
// normw's 16-byte chunk `threadIdx.x`, loaded early by the caller (see norm_chunk).
__device__ __forceinline__ void prologue(const Cs& m, int K, const __half* normw, float eps, int4 nw0) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int nch = K / 8;
    int4* x4 = reinterpret_cast<int4*>(m.xs);
    float mx = 0.0f;
    if (normw) {
        if (warp == 0) {
            const float ss = rms_sumsq_lanemajor(m.xsT, K);
            if (lane == 0) m.red[32] = ss;
        }
        cbar();
        const float rms = __fsqrt_rn(__fadd_rn(__fdiv_rn(m.red[32], (float)K), eps));
        const float inv_rms = __fdiv_rn(1.0f, rms);
        const __half inv16 = __float2half_rn(inv_rms);
        const int4* w4 = reinterpret_cast<const int4*>(normw);
        for (int i = tid; i < nch; i += kPC) {
            int4 v = x4[i];
            const int4 w = i == tid ? nw0 : __ldg(w4 + i);
            __half* h = reinterpret_cast<__half*>(&v);
            const __half* hw = reinterpret_cast<const __half*>(&w);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                h[j] = __hmul(__hmul(h[j], inv16), hw[j]);
                mx = fmaxf(mx, fabsf(h2f(h[j])));
            }
            x4[i] = v;
        }
    } else {
        for (int i = tid; i < nch; i += kPC) {
            int4 v = x4[i];
            const __half* h = reinterpret_cast<const __half*>(&v);
#pragma unroll
            for (int j = 0; j < 8; ++j) mx = fmaxf(mx, fabsf(h2f(h[j])));
        }
    }
    mx = warp_max(mx);
    if (lane == 0) m.red[warp] = mx;
    cbar();
    // every warp folds the per-warp maxima itself (max is exact in any order)
    const float mxa = warp_max(lane < kPCW ? m.red[lane] : 0.0f);
    float scale = __fdiv_rn(mxa, 127.0f);
    if (scale < 1e-10f) scale = 1e-10f;
    const float inv = __fdiv_rn(1.0f, scale);
    int2* a2 = reinterpret_cast<int2*>(m.act);
    for (int i = tid; i < nch; i += kPC) {
        int4 v = x4[i];
        const __half* h = reinterpret_cast<const __half*>(&v);
        int2 q;
        int8_t* qb = reinterpret_cast<int8_t*>(&q);
#pragma unroll
        for (int j = 0; j < 8; ++j) qb[j] = quant_act(h2f(h[j]), inv, true);
        a2[i] = q;
    }
    if (tid == 0) *m.as = scale;
    cbar();
}

// The norm weights' 16-byte chunk of this thread, issued well before the prologue needs it so
// its global-memory latency overlaps the preceding phase.
__device__ __forceinline__ int4 norm_chunk(const __half* normw, int K) {
    return (normw && (int)threadIdx.x < K / 8) ? __ldg(reinterpret_cast<const int4*>(normw) + threadIdx.x)
                                               : make_int4(0, 0, 0, 0);
}

__device__ __forceinline__ unsigned long long argmax_key(float v, int i) {
    if (v != v) return 0ull;
    unsigned u = __float_as_uint(v);
    u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((unsigned long long)u << 32) | (0xFFFFFFFFu - (unsigned)i);
}

// One projection of the block's rows: grouped INT8 GEMV (exact int32 group sums, fp32 FMA
// chain over the groups in order, times the activation scale -> fp16) + epilogue.
// Outputs go to `out` as tagged words (`tag_out`; the residual read polls for `tag_res`),
// the lm head's logits to `lm_out` as plain fp16.
// CPG: 16-byte chunks per quantisation group (G / 16), a compile-time constant so the dot
// loop is unrolled for exactly the group's chunks.
template <int CPG>
__device__ __forceinline__ bool gemv_job(const PArgs& a, int j, int epi, const Cs& m, uint8_t* ring, uint64_t* full,
                                         uint64_t* empty, unsigned& kslot, uint32_t* out, __half* lm_out,
                                         unsigned tag_out, unsigned tag_res, unsigned long long& best) {
    const int tid = threadIdx.x;
    const JobW jw = job_w(a, j);
    int r0, r1;
    rows_of(jw.N, blockIdx.x, gridDim.x, r0, r1);
    // group sums / scales of row r at [r * gst, r * gst + ng): gst keeps rows 16-byte aligned
    // and puts consecutive rows in different banks for the 16-byte loads of the chain
    constexpr int G = CPG * 16;
    const int K = jw.K, ng = K / G, spr = rows_per_slot(a.slot_w, K), gst = ((ng + 3) & ~3) + 4;
    // thread -> (row, group): the group is fixed for the whole job (so its activation chunks
    // stay in registers) and a round covers rpr rows
    const int rpr = kPC / ng, g = tid % ng, r_first = tid / ng;
    const bool tactive = r_first < rpr;
    int4 ar[CPG];
#pragma unroll
    for (int c = 0; c < CPG; ++c)
        ar[c] = tactive ? *reinterpret_cast<const int4*>(m.act + g * G + c * 16) : make_int4(0, 0, 0, 0);
    const float as = *m.as;
    const int NS = a.nslots, sb = a.slot_w + a.slot_s;
    for (int r = r0; r < r1; r += spr, ++kslot) {
        const int s = (int)(kslot % NS);
        const unsigned par = (kslot / NS) & 1;
        const int rows = min(spr, r1 - r);
        // the residual row of this thread's output, read before the slot wait (written by this
        // block's previous projection into the same rows, or by the embedding)
        __half res = __float2half_rn(0.0f);
        if (epi == kEpiResid && tid < rows) {
            uint32_t w;
            if (!poll_word(a, out + r + tid, tag_res, w)) *m.fail = 1;
            res = word_h(w);
        }
        if (tid == 0) *m.flag = wait_abortable(&full[s], par, &a.sync->abort, 32, a.spin_limit) ? 1 : 0;
        cbar();
        if (!*m.flag) {
            if (tid == 0) set_abort(a, kDevTmaTimeout);
            return false;
        }
        if (*m.fail) return false;
        mbar_wait_bounded(&full[s], par);  // completed already: makes the copy visible to this thread
        const uint8_t* wsl = ring + (size_t)s * sb;
        const uint16_t* ssl = reinterpret_cast<const uint16_t*>(wsl + a.slot_w);
        // exact int32 sum of each (row, group): CPG 16-byte chunks, 4 dp4a each
        if (tactive) {
            for (int rr = r_first; rr < rows; rr += rpr) {
                const int4* wp = reinterpret_cast<const int4*>(wsl + (size_t)rr * K + g * G);
                int acc = 0;
#pragma unroll
                for (int c = 0; c < CPG; ++c) {
                    const int4 wv = wp[c];
                    acc = dp4a_ss(ar[c].x, wv.x, acc);
                    acc = dp4a_ss(ar[c].y, wv.y, acc);
                    acc = dp4a_ss(ar[c].z, wv.z, acc);
                    acc = dp4a_ss(ar[c].w, wv.w, acc);
                }
                m.gsm[rr * gst + g] = acc;
                m.gsf[rr * gst + g] = h2f_bits(ssl[rr * ng + g]);
            }
        }
        cbar();
        if (tid < rows) {
            const int4* gp = reinterpret_cast<const int4*>(m.gsm + tid * gst);
            const float4* fp = reinterpret_cast<const float4*>(m.gsf + tid * gst);
            float run = 0.0f;
            // group sums are below 2^22 in magnitude (G <= 128): exact integer -> float
            for (int c = 0; c < ng / 4; ++c) {
                const int4 gv = gp[c];
                const float4 fv = fp[c];
                run = fmaf(i2f_small(gv.x), fv.x, run);
                run = fmaf(i2f_small(gv.y), fv.y, run);
                run = fmaf(i2f_small(gv.z), fv.z, run);
                run = fmaf(i2f_small(gv.w), fv.w, run);
            }
            for (int g = ng & ~3; g < ng; ++g) run = fmaf(i2f_small(m.gsm[tid * gst + g]), m.gsf[tid * gst + g], run);
            const __half v = f2h(__fmul_rn(run, as));
            const int n = r + tid;
            if (epi == kEpiStore) {
                st_tagged(out + n, v, tag_out);
            } else if (epi == kEpiResid) {
                st_tagged(out + n, __hadd(res, v), tag_out);
            } else if (epi == kEpiLm) {
                lm_out[n] = v;
                const unsigned long long key = argmax_key(h2f(v), n);
                best = key > best ? key : best;
            } else {
                m.ob[tid] = v;
            }
        }
        cbar();
        if (tid == 0) mbar_arrive(&empty[s]);
        if (epi == kEpiGlu && tid < rows / 2)
            st_tagged(out + (r >> 1) + tid, __hmul(ref_silu(m.ob[2 * tid]), m.ob[2 * tid + 1]), tag_out);
    }
    return true;
}

template <int D>
__device__ __forceinline__ AttnCoreArgs attn_args(const PArgs& a, const PLayer& ly, int h, int cache_len,
                                                  int total_len, const float* qs, const __half* kr,
                                                  const __half* hv) {
    const int kvh = h / (a.Hq / a.Hkv);
    const int nqg = (D + 127) / 128;
    AttnCoreArgs c;
    c.qs = qs;
    c.Kc = ly.kc + (size_t)kvh * D;
    c.Vc = ly.vc + (size_t)kvh * D;
    c.ks = ly.ks + (size_t)kvh * nqg;
    c.vs = ly.vs + (size_t)kvh * nqg;
    c.Kn = kr;
    c.Vn = hv;
    c.kv_row = (long long)a.Hkv * D;
    c.sc_row = (long long)a.Hkv * nqg;
    c.kn_row = 0;
    c.cache_len = cache_len;
    c.new_len = 1;
    c.qgs = 128;
    c.aq = total_len;
    c.kv_end = min((long long)cache_len + 1, (long long)total_len + 1);
    c.causal = 1;
    c.scale = a.attn_scale;
    c.prestaged = 1;
    c.pages = a.pages;
    c.page_shift = a.page_shift;
    return c;
}

// attention work area: [core staging | qs float[D] | hq hk hv qr kr fp16[D] | qn kn fp16[D],
// ct st fp16[D/2]]
template <int D>
struct AttnSmem {
    float* qs;
    __half *hq, *hk, *hv, *qr, *kr, *qn, *kn, *crow, *srow;
    __device__ explicit AttnSmem(uint8_t* w) {
        qs = reinterpret_cast<float*>(w + attn_core_smem<D, kACH>());
        hq = reinterpret_cast<__half*>(qs + D);
        hk = hq + D;
        hv = hk + D;
        qr = hv + D;
        kr = qr + D;
        qn = kr + D;
        kn = qn + D;
        crow = kn + D;
        srow = crow + D / 2;
    }
};

// Attention blocks stage what their head needs for layer l before the layer's QKV
// projection — the cached K/V rows, the q/k norm weights and the RoPE rows of this position
// — since none of it depends on the step, the copies overlap the projection.
template <int D>
__device__ __forceinline__ void attention_prefetch(const PArgs& a, int l, int h, uint8_t* awork, int cache_len,
                                                   int total_len) {
    const PLayer& ly = a.layers[l];
    const AttnSmem<D> sm(awork);
    const int t = threadIdx.x;
    constexpr int C16 = D * 2 / 16;  // 16-byte chunks of one fp16 head vector
    if (t < C16) {
        if (ly.q_norm) cp_async16(sm.qn + t * 8, ly.q_norm + t * 8);
        if (ly.k_norm) cp_async16(sm.kn + t * 8, ly.k_norm + t * 8);
    } else if (ly.ct && t < C16 + C16 / 2) {
        const int c = t - C16;
        cp_async16(sm.crow + c * 8, ly.ct + (size_t)total_len * (D / 2) + c * 8);
        cp_async16(sm.srow + c * 8, ly.st + (size_t)total_len * (D / 2) + c * 8);
    }
    const AttnCoreArgs c = attn_args<D>(a, ly, h, cache_len, total_len, nullptr, nullptr, nullptr);
    attn_stage_chunk<D, kPC, kACH>(c, awork, 0);  // commits the group (the copies above included)
}

// Attention of head h in layer l: waits for the head's q and its kv head's k / v rows
// (tagged `tq`), writes its output rows tagged `ta`. False when a poll gave up.
template <int D>
__device__ __forceinline__ bool attention_head(const PArgs& a, const Cs& m, int l, int h, uint8_t* work, int cache_len,
                                               int total_len, unsigned tq, unsigned ta) {
    const int tid = threadIdx.x, warp = tid >> 5;
    const int grp = a.Hq / a.Hkv, kvh = h / grp;
    const int nqg = (D + 127) / 128;
    const AttnSmem<D> sm(work);
    float* qs = sm.qs;
    __half *hq = sm.hq, *hk = sm.hk, *hv = sm.hv, *qr = sm.qr, *kr = sm.kr;
    const PLayer& ly = a.layers[l];
    // every layer pointer is read here, next to the q/k/v loads: the block barriers below are
    // memory clobbers, so a read placed after one would add an L2 round trip to the phase
    const AttnCoreArgs c = attn_args<D>(a, ly, h, cache_len, total_len, qs, kr, hv);
    const bool rope = ly.ct != nullptr, qnorm = ly.q_norm != nullptr, knorm = ly.k_norm != nullptr;
    static_assert(D <= kPC, "one thread per dim");
    if (tid < D) {
        // the three words are requested together; only the ones not yet written are re-polled
        const uint32_t* pq = a.qkv + (size_t)h * D + tid;
        const uint32_t* pk = a.qkv + (size_t)(a.Hq + kvh) * D + tid;
        const uint32_t* pv = a.qkv + (size_t)(a.Hq + a.Hkv + kvh) * D + tid;
        uint32_t wq = ld_relaxed_gpu(pq), wk = ld_relaxed_gpu(pk), wv = ld_relaxed_gpu(pv);
        for (uint32_t it = 0; ((wq >> 16) != tq) | ((wk >> 16) != tq) | ((wv >> 16) != tq); ++it) {
            if (!poll_go_on(a, it)) {
                *m.fail = 1;
                break;
            }
            if ((wq >> 16) != tq) wq = ld_relaxed_gpu(pq);
            if ((wk >> 16) != tq) wk = ld_relaxed_gpu(pk);
            if ((wv >> 16) != tq) wv = ld_relaxed_gpu(pv);
        }
        hq[tid] = word_h(wq);
        hk[tid] = word_h(wk);
        hv[tid] = word_h(wv);
    }
    cp_async_wait<0>();  // the prefetched norm weights / RoPE rows / K/V of this thread
    cbar();
    if (*m.fail) return false;
    const __half* crow = rope ? sm.crow : nullptr;
    if (warp < 2) {  // warp 0: q, warp 1: k (one inlined copy of the routine)
        const bool isq = warp == 0;
        head_norm_rope_rows(isq ? hq : hk, D, isq ? (qnorm ? sm.qn : nullptr) : (knorm ? sm.kn : nullptr), a.eps,
                            crow, sm.srow, isq ? qr : kr);
    }
    cbar();
    for (int d = tid; d < D; d += kPC) qs[d] = h2f(qr[d]);
    cbar();
    const __half o = attn_exact_core<D, kPC, kACH>(c, work, SyncConsumers{});
    if (tid < D) st_tagged(a.attn + (size_t)h * D + tid, o, ta);
    // the first q head of each group appends the step's K/V to the cache at slot cache_len
    // (c.Kc / c.Vc / c.ks / c.vs point at this kv head's row 0). Only the next token reads
    // that row (this token's attention takes the new key and value from shared memory), so
    // the append runs after the output is published, off the critical path.
    if (h % grp == 0 && warp >= 2 && warp < 2 + 2 * nqg) {
        const int which = (warp - 2) / nqg, g = (warp - 2) % nqg;
        const int cnt = min(128, D - g * 128);
        const __half* src = (which ? hv : kr) + g * 128;
        const long long row = c.pages ? kv_page_row(c.pages, c.page_shift, cache_len) : cache_len;
        int8_t* dst = const_cast<int8_t*>(which ? c.Vc : c.Kc) + (size_t)row * c.kv_row + g * 128;
        float* sdst = const_cast<float*>(which ? c.vs : c.ks) + (size_t)row * c.sc_row + g;
        kv_quant_group_warp(src, cnt, dst, sdst);
    }
    return true;
}

// embedding row of `tok` (compute_embedding_node semantics, as embed_kernel) into xs; the
// block also stores its slice of the hidden state (tagged version 0)
__device__ __forceinline__ void embed_row(const PArgs& a, uint32_t tok, __half* xs) {
    const unsigned tag = vtag(a, 0);
    const int H = a.H;
    const int k0 = (int)(((long long)H * blockIdx.x) / gridDim.x), k1 = (int)(((long long)H * (blockIdx.x + 1)) / gridDim.x);
    for (int k = threadIdx.x; k < H; k += kPC) {
        __half v;
        if (a.emb_prec == 1) {
            v = reinterpret_cast<const __half*>(a.emb)[(size_t)tok * H + k];
        } else {
            int q;
            if (a.emb_prec == 0) {
                q = reinterpret_cast<const int8_t*>(a.emb)[(size_t)tok * H + k];
            } else {
                const uint8_t byte = reinterpret_cast<const uint8_t*>(a.emb)[((size_t)tok * H + k) >> 1];
                q = (k & 1) ? (byte >> 4) : (byte & 0x0F);
                q = (q & 8) ? q - 16 : q;
            }
            v = f2h(__fmul_rn((float)q, h2f(a.emb_s[(size_t)tok * (H / a.emb_G) + k / a.emb_G])));
        }
        xs[k] = v;
        if (k >= k0 && k < k1) st_tagged(a.hidden + k, v, tag);
    }
    cbar();
}

template <int D, int CPG>
__global__ void __launch_bounds__(kPT, 1) decode_persistent_kernel(PArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ float s_red[64];
    __shared__ float s_as;
    __shared__ int s_flag, s_fail;
    __shared__ unsigned long long s_best[16];
    const int NS = a.nslots, sb = a.slot_w + a.slot_s;
    uint8_t* ring = smem;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)NS * sb);
    uint64_t* empty = full + NS;
    uint8_t* work = smem + (size_t)NS * sb + a128(16 * NS);
    const int tid = threadIdx.x;
    if (tid == 0) {
        s_fail = 0;
        s_flag = ld_volatile_u32(&a.sync->abort) ? 0 : 1;
        for (int s = 0; s < NS; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        fence_mbar_init();
    }
    __syncthreads();
    if (!s_flag) return;  // an earlier block of this run failed
    if (tid >= kPC) {
        if (tid == kPC) producer(a, ring, full, empty);
        return;
    }
    Cs m;
    m.act = reinterpret_cast<int8_t*>(work);
    m.xs = reinterpret_cast<__half*>(work + a128(a.kmax));
    m.gsm = reinterpret_cast<int*>(work + a128(a.kmax) + a128(2 * a.kmax));
    m.gsf = reinterpret_cast<float*>(m.gsm + a.gsm_ints);
    m.ob = reinterpret_cast<__half*>(m.gsf + a.gsm_ints);
    m.xsT = reinterpret_cast<__half*>(reinterpret_cast<uint8_t*>(m.ob) + a128(a.max_rows * 2));
    m.red = s_red;
    m.as = &s_as;
    m.flag = &s_flag;
    m.fail = &s_fail;
    m.best = s_best;

    const int cache_len = __ldcg(a.state), total_len = __ldcg(a.state + 1);
    const uint32_t tok = __ldcg(a.tok_in);
    uint8_t* awork = work + a.attn_off;
    const bool attn_block = (int)blockIdx.x < a.Hq;
    unsigned kslot = 0;
    unsigned long long best = 0ull;
    embed_row(a, tok, m.xs);
    // One loop over the projection jobs (j = 4 l + {QKV, O, gate-up, down}, then the lm head)
    // with the phase-specific values selected at run time: the input / prologue / GEMV code
    // exists once in the kernel instead of once per phase, which keeps the instruction
    // footprint of the hot loop small.
    // Versions of the tagged words: the hidden state entering layer l is 5 l (the embedding,
    // or the previous layer's down projection), then QKV 5 l + 1, attention + 2, O + 3,
    // gate-up + 4, down + 5.
    for (int j = 0; j <= 4 * a.L; ++j) {
        const int l = j >> 2, p = j & 3;
        const bool lm = j == 4 * a.L;
        // attention blocks stage the layer's cached K/V rows, norm weights and RoPE rows
        // before its QKV phase (right after the previous layer's down projection): fixed for
        // this token, so the copies overlap the waits and the projection
        if (p == 0 && !lm && attn_block) attention_prefetch<D>(a, l, blockIdx.x, awork, cache_len, total_len);
        const __half* norm = nullptr;
        if (lm) norm = a.out_norm;
        else if (p == 0) norm = a.layers[l].in_norm;
        else if (p == 2) norm = a.layers[l].post_norm;
        const int4 nw = norm_chunk(norm, a.H);
        const uint32_t* src = p == 1 ? a.attn : (p == 3 ? a.gated : a.hidden);
        const int K = p == 1 ? a.Hq * D : (p == 3 ? a.F : a.H);
        const bool hid = p == 0 || p == 2;  // the hidden state (lane-major copy for the RMS chain)
        const int vin = 5 * l + (p == 0 ? 0 : p == 1 ? 2 : p == 2 ? 3 : 4);
        if (j > 0) {
            if (!load_tagged(m, a, src, K, vtag(a, vin), hid)) return;
        } else {
            load_vec(m, nullptr, a.H, true);  // xs holds the embedding row
        }
        prologue(m, K, norm, a.eps, nw);
        const int epi = lm ? kEpiLm : (p == 0 ? kEpiStore : p == 2 ? kEpiGlu : kEpiResid);
        uint32_t* out = lm ? nullptr : (p == 0 ? a.qkv : p == 2 ? a.gated : a.hidden);
        const unsigned t_out = vtag(a, 5 * l + (p == 0 ? 1 : p == 1 ? 3 : p == 2 ? 4 : 5));
        const unsigned t_res = vtag(a, 5 * l + (p == 1 ? 0 : 3));  // O / down: the residual's version
        if (!gemv_job<CPG>(a, j, epi, m, ring, full, empty, kslot, out, a.logits, t_out, t_res, best)) return;
        if (p == 0 && !lm && attn_block &&
            !attention_head<D>(a, m, l, blockIdx.x, awork, cache_len, total_len, t_out, vtag(a, 5 * l + 2)))
            return;
    }
    // block first-max, then the last block to finish picks the token
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long k2 = __shfl_xor_sync(0xffffffffu, best, o);
        best = k2 > best ? k2 : best;
    }
    if ((tid & 31) == 0) m.best[tid >> 5] = best;
    cbar();
    if (tid == 0) {
        unsigned long long b = m.best[0];
        for (int w = 1; w < kPCW; ++w) b = m.best[w] > b ? m.best[w] : b;
        if (b) atomicMax(&a.sync->key, b);
        __threadfence();
        const unsigned prev = atomicAdd(&a.sync->done, 1u);
        if (prev == gridDim.x - 1) {
            __threadfence();
            const unsigned long long key = atomicAdd(&a.sync->key, 0ull);
            const uint32_t next = key == 0ull ? 0u : 0xFFFFFFFFu - (unsigned)(key & 0xFFFFFFFFull);
            const int step = __ldcg(a.state + 2);
            a.tok_in[0] = next;
            if (a.ring) a.ring[step] = next;
            a.state[0] = cache_len + 1;
            a.state[1] = total_len + 1;
            a.state[2] = step + 1;
            a.sync->key = 0ull;
            a.sync->done = 0u;
            __threadfence();
        }
    }
}

template <int D>
int attn_work_bytes() {
    return attn_core_smem<D, kACH>() + D * 4 + 5 * D * 2 + 3 * D * 2;
}

}  // namespace

PPlan persistent_plan(PArgs& a, int num_sms, size_t smem_optin) {
    PPlan p;
    auto no = [&](const char* why) {
        p.ok = false;
        p.why = why;
        return p;
    };
    if (a.D != 64 && a.D != 128) return no("head_dim must be 64 or 128");
    // every block must own rows of the QKV and gate-up projections (the tagged hand-over
    // relies on it to order buffer reuse), so small models run on fewer blocks
    const int grid = std::min(num_sms, std::min(a.QKVN >> 3, a.F >> 2));
    if (a.Hq > grid || a.Hkv < 1 || a.Hq % a.Hkv) return no("head layout");
    if (ptag_span(a.L) >= 65535u) return no("too many layers for the 16-bit version tags");
    if (a.G < 16 || a.G % 16 || 32 % (a.G / 16)) return no("group size");
    const int Ks[3] = {a.H, a.Hq * a.D, a.F};
    int kmin = Ks[0], kmax = Ks[0];
    for (int K : Ks) {
        if (K % a.G || K % 16) return no("K not a multiple of the group size");
        kmin = K < kmin ? K : kmin;
        kmax = K > kmax ? K : kmax;
    }
    const int Ns[5] = {a.QKVN, a.H, 2 * a.F, a.H, a.V};
    for (int N : Ns) {
        if (N % 8) return no("rows not a multiple of 8");
        if ((long long)(N >> 3) * (num_sms + 1) >= (1LL << 31)) return no("too many rows for 32-bit row ranges");
    }
    a.kmax = kmax;
    // A slot holds 48 rows at K = 1024, so a block's share of every projection of a Qwen3-0.6B
    // layer (QKV 24-32 rows, gate-up 40-48 rows, O / down 8 rows) is one slot: no block trails
    // the others by a second slot before a grid barrier, and a phase waits on one ring slot.
    // Measured on B200 (decode tok/s): 24 KB slots 973, 32 KB 1008, 48 KB 1035 (two slots fit
    // beside the work area). CACTUS_B200_PSLOT overrides the size in bytes.
    int slot_min = 49152;
    if (const char* e = std::getenv("CACTUS_B200_PSLOT")) slot_min = std::max(8192, std::atoi(e));
    a.slot_w = a128(kmax * 8 > slot_min ? kmax * 8 : slot_min);
    a.slot_s = a128(a.slot_w / a.G * 2);
    a.max_rows = a.slot_w / kmin;
    if (a.max_rows > kPC) return no("hidden sizes too small for the slot size");
    a.gsm_ints = (a.slot_w / a.G + 8 * a.max_rows + 32 + 3) / 4 * 4;
    if (a.G > 16 * kMaxCpg) return no("group size above 128");
    if (kmax / a.G > kPC) return no("more groups per row than consumer threads");
    if (a.G & (a.G - 1)) return no("group size must be a power of two");
    if (a.H % 16) return no("hidden size must be a multiple of 16");
    const int gemv_work = a128(kmax) + a128(2 * kmax) + 2 * a.gsm_ints * 4 + a128(a.max_rows * 2) +
                          a128(16 * lanemajor_stride(a.H) * 2);
    const int attn_work = a.D == 64 ? attn_work_bytes<64>() : attn_work_bytes<128>();
    a.attn_off = a128(gemv_work);
    a.work_bytes = a.attn_off + a128(attn_work);
    const long long budget = (long long)smem_optin - kStaticSmem;
    const int sb = a.slot_w + a.slot_s;
    int NS = 0;
    while ((long long)(NS + 1) * sb + a128(16 * (NS + 1)) + a.work_bytes <= budget && NS < 16) ++NS;
    if (NS < 2) return no("shared memory too small for two weight slots");
    a.nslots = NS;
    p.smem = (size_t)NS * sb + a128(16 * NS) + a.work_bytes;
    p.grid = grid;
    p.threads = kPT;
    p.ok = true;
    return p;
}

cudaError_t launch_persistent_decode(const PArgs& a, const PPlan& p, cudaStream_t st) {
    // one instantiation per (head dim, chunks per group); persistent_plan admits G = 16 .. 128
    using Kfn = void (*)(PArgs);
    static const Kfn table[2][4] = {
        {decode_persistent_kernel<64, 1>, decode_persistent_kernel<64, 2>, decode_persistent_kernel<64, 4>,
         decode_persistent_kernel<64, 8>},
        {decode_persistent_kernel<128, 1>, decode_persistent_kernel<128, 2>, decode_persistent_kernel<128, 4>,
         decode_persistent_kernel<128, 8>}};
    const int gi = a.G == 16 ? 0 : a.G == 32 ? 1 : a.G == 64 ? 2 : 3;
    Kfn k = table[a.D == 64 ? 0 : 1][gi];
    static size_t attr_set[2][4] = {};  // largest dynamic shared memory enabled per variant
    size_t& done = attr_set[a.D == 64 ? 0 : 1][gi];
    if (p.smem > done) {
        cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)p.smem);
        if (e != cudaSuccess) return e;
        done = p.smem;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.grid);
    cfg.blockDim = dim3(p.threads);
    cfg.dynamicSmemBytes = p.smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, k, a);
}

}  // namespace eng
}  // namespace cb
