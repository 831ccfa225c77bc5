// Persistent decode step: one cooperative launch runs a whole batch-1 decode token —
// embedding, every transformer layer (Qwen/Llama block: RMSNorm -> fused QKV -> per-head
// q/k norm + RoPE -> KV append -> attention -> O + residual -> RMSNorm -> gate/up + SiLU-GLU
// -> down + residual), the final norm, the lm head and the greedy argmax — with the same
// arithmetic as the multi-kernel path (gemv.cuh, attention_core.cuh, head_ops.cuh), so the
// tokens are bit-identical to it and to the reference order.
//
// Why: at batch 1 each projection is a few MB, so a kernel per op is bound by launch and
// dependency latency, not by HBM. Here one block per SM stays resident for the token:
//  * warp 15 of every block is a producer that streams the block's share of every weight
//    matrix of the token (a fixed row range per matrix, 8-row units) through a ring of
//    shared-memory slots with 1-D TMA bulk copies (no multicast), full/empty mbarriers per
//    slot. Weights do not depend on activations, so the stream runs ahead of the layer
//    dependency chain by the ring's depth and HBM stays busy across phase boundaries;
//  * warps 0-14 consume: per phase they rebuild the quantised activations in shared memory
//    (every block redundantly, which is cheaper than another grid barrier), reduce their
//    rows and write outputs; grid-wide barriers (one counter, bounded spins, release/acquire)
//    separate phases: QKV | attention | O | gate-up | down, five per layer.
//  * blocks 0..Hq-1 run one attention head each (the reference-order core).
//  * the lm head keeps a per-block first-max key; the last block to finish combines them,
//    writes the next token, advances the device state and re-arms the sync words.
// Every wait is bounded; a timeout sets the abort word and the device error, every block
// leaves at its next wait, and producers first wait for their copies in flight.
#include "../attention_core.cuh"
#include "../common.cuh"
#include "../gemv.cuh"
#include "decode_persistent.h"
#include "head_ops.cuh"

namespace cb {
namespace eng {

namespace {

constexpr int kPT = 512;       // threads per block
constexpr int kPCW = 15;       // consumer warps
constexpr int kPC = kPCW * 32; // consumer threads
constexpr int kACH = 256;      // attention keys per staged chunk
constexpr int kStaticSmem = 1024;

enum : int { kEpiStore = 0, kEpiResid = 1, kEpiGlu = 2, kEpiLm = 3 };

__device__ __forceinline__ void cbar() { asm volatile("bar.sync 1, 480;" ::: "memory"); }
struct SyncConsumers {
    __device__ __forceinline__ void operator()() const { cbar(); }
};

__host__ __device__ inline int a128(int v) { return (v + 127) / 128 * 128; }

// rows of an [N, K] matrix owned by block c of P: 8-row units split evenly
__host__ __device__ inline void rows_of(int N, int c, int P, int& r0, int& r1) {
    const long long U = N >> 3;
    r0 = (int)((U * c) / P) * 8;
    r1 = (int)((U * (c + 1)) / P) * 8;
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
__device__ __forceinline__ bool wait_abortable(uint64_t* bar, unsigned par, const unsigned* abort, unsigned ns) {
    for (uint32_t i = 0; i < (1u << 22); ++i) {
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

// ------------------------------------------------------------------ producer (one thread)
__device__ void producer(const PArgs& a, uint8_t* ring, uint64_t* full, uint64_t* empty) {
    const int NS = a.nslots, sb = a.slot_w + a.slot_s;
    unsigned k = 0;
    bool ok = true;
    const int J = 4 * a.L + 1;
    for (int j = 0; j < J && ok; ++j) {
        const JobW jw = job_w(a, j);
        int r0, r1;
        rows_of(jw.N, blockIdx.x, gridDim.x, r0, r1);
        const int spr = rows_per_slot(a.slot_w, jw.K), ng = jw.K / a.G;
        for (int r = r0; r < r1; r += spr) {
            const int s = (int)(k % NS);
            if (k >= (unsigned)NS && !wait_abortable(&empty[s], ((k / NS) - 1) & 1, &a.sync->abort, 256)) {
                ok = false;
                break;
            }
            const int rows = min(spr, r1 - r);
            const unsigned wb = (unsigned)(rows * jw.K), sbytes = (unsigned)(rows * ng * 2);
            uint8_t* dst = ring + (size_t)s * sb;
            mbar_arrive_expect_tx(&full[s], wb + sbytes);
            tma_load_1d(dst, jw.w + (size_t)r * jw.K, wb, &full[s]);
            tma_load_1d(dst + a.slot_w, jw.s + (size_t)r * ng, sbytes, &full[s]);
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
    int* gsm;
    float* gsf;
    __half* ob;
    float* red;   // [64]
    float* as;    // activation scale of the current job
    int* flag;
    unsigned long long* best;  // [16]
};

constexpr int kMaxPerThread = 8;  // activation elements per consumer thread (K <= 3840)
constexpr int kMaxPass = 8;       // 512-element passes of one GEMV row (K <= 4096)

// Stages K fp16 activations written by other blocks (L2 loads) into xs; when `src` is null
// the caller has filled xs already. The optional RMSNorm weights of the following prologue
// are fetched into registers first, so their latency overlaps the staging.
__device__ __forceinline__ void load_vec(__half* xs, const __half* src, int K, const __half* norm,
                                         __half (&nw)[kMaxPerThread]) {
    if (norm) {
#pragma unroll
        for (int j = 0; j < kMaxPerThread; ++j) {
            const int k = threadIdx.x + j * kPC;
            if (k < K) nw[j] = norm[k];
        }
    }
    if (src) {
        const int4* s4 = reinterpret_cast<const int4*>(src);
        int4* d4 = reinterpret_cast<int4*>(xs);
        for (int i = threadIdx.x; i < K / 8; i += kPC) d4[i] = __ldcg(s4 + i);
    }
    cbar();
}

// xs holds K fp16 activations; optional RMSNorm with weights `nw` (registers, from
// load_vec), then the activation quantisation (gemv.cuh prologues, same arithmetic) into
// act / *as.
__device__ void prologue(const Cs& m, int K, bool norm, const __half (&nw)[kMaxPerThread], float eps) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int vec_end = (K / 8) * 8;
    float mx = 0.0f;
    if (norm) {
        if (warp == 0) {
            const float ss = rms_sumsq_warp(m.xs, K);
            if (lane == 0) m.red[32] = ss;
        }
        cbar();
        const float rms = __fsqrt_rn(__fadd_rn(__fdiv_rn(m.red[32], (float)K), eps));
        const float inv_rms = __fdiv_rn(1.0f, rms);
        const __half inv16 = __float2half_rn(inv_rms);
#pragma unroll
        for (int j = 0; j < kMaxPerThread; ++j) {
            const int k = tid + j * kPC;
            if (k < K) {
                __half v = m.xs[k];
                v = (k < vec_end) ? __hmul(__hmul(v, inv16), nw[j])
                                  : __float2half_rn(__fmul_rn(__fmul_rn(h2f(v), inv_rms), h2f(nw[j])));
                m.xs[k] = v;
                mx = fmaxf(mx, fabsf(h2f(v)));
            }
        }
    } else {
        for (int k = tid; k < K; k += kPC) mx = fmaxf(mx, fabsf(h2f(m.xs[k])));
    }
    mx = warp_max(mx);
    if (lane == 0) m.red[warp] = mx;
    cbar();
    // every warp folds the per-warp maxima itself (max is exact in any order)
    const float mxa = warp_max(lane < kPCW ? m.red[lane] : 0.0f);
    float scale = __fdiv_rn(mxa, 127.0f);
    if (scale < 1e-10f) scale = 1e-10f;
    const float inv = __fdiv_rn(1.0f, scale);
    for (int k = tid; k < K; k += kPC) m.act[k] = quant_act(h2f(m.xs[k]), inv, k < vec_end);
    if (tid == 0) *m.as = scale;
    cbar();
}

__device__ __forceinline__ unsigned long long argmax_key(float v, int i) {
    if (v != v) return 0ull;
    unsigned u = __float_as_uint(v);
    u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((unsigned long long)u << 32) | (0xFFFFFFFFu - (unsigned)i);
}

// One projection of the block's rows: grouped INT8 GEMV (exact int32 group sums, fp32 FMA
// chain over the groups in order, times the activation scale -> fp16) + epilogue.
__device__ bool gemv_job(const PArgs& a, int j, int epi, const Cs& m, uint8_t* ring, uint64_t* full,
                         uint64_t* empty, unsigned& kslot, __half* out, unsigned long long& best) {
    const int tid = threadIdx.x;
    const JobW jw = job_w(a, j);
    int r0, r1;
    rows_of(jw.N, blockIdx.x, gridDim.x, r0, r1);
    const int K = jw.K, ng = K / a.G, spr = rows_per_slot(a.slot_w, K), cpg = a.G / 16, gst = ng + 1;
    const int cpg_log2 = __ffs(cpg) - 1, chunks = K / 16, npass = (chunks + 31) / 32;
    const int lane = tid & 31, warp = tid >> 5;
    int4 areg[kMaxPass];  // this lane's activation chunks, one per pass
#pragma unroll
    for (int p = 0; p < kMaxPass; ++p) {
        const int c = p * 32 + lane;
        areg[p] = (p < npass && c < chunks) ? *reinterpret_cast<const int4*>(m.act + c * 16) : make_int4(0, 0, 0, 0);
    }
    const float as = *m.as;
    const int NS = a.nslots, sb = a.slot_w + a.slot_s;
    for (int r = r0; r < r1; r += spr, ++kslot) {
        const int s = (int)(kslot % NS);
        const unsigned par = (kslot / NS) & 1;
        const int rows = min(spr, r1 - r);
        if (tid == 0) *m.flag = wait_abortable(&full[s], par, &a.sync->abort, 32) ? 1 : 0;
        cbar();
        if (!*m.flag) {
            if (tid == 0) set_abort(a, kDevTmaTimeout);
            return false;
        }
        mbar_wait_bounded(&full[s], par);  // completed already: makes the copy visible to this thread
        const uint8_t* wsl = ring + (size_t)s * sb;
        const uint16_t* ssl = reinterpret_cast<const uint16_t*>(wsl + a.slot_w);
        // warp per row, lane per 16-byte chunk (chunk lane + 32p of pass p); the activation
        // chunks live in registers for the whole job; lanes of a group fold by xor shuffles
        for (int rr = warp; rr < rows; rr += kPCW) {
            const uint8_t* wrow = wsl + (size_t)rr * K;
            int part[kMaxPass];
#pragma unroll
            for (int p = 0; p < kMaxPass; ++p) {
                part[p] = 0;
                if (p < npass && (p * 32 + lane) < chunks) {
                    const int4 wv = *reinterpret_cast<const int4*>(wrow + (p * 32 + lane) * 16);
                    int acc = dp4a_ss(areg[p].x, wv.x, 0);
                    acc = dp4a_ss(areg[p].y, wv.y, acc);
                    acc = dp4a_ss(areg[p].z, wv.z, acc);
                    part[p] = dp4a_ss(areg[p].w, wv.w, acc);
                }
            }
#pragma unroll
            for (int p = 0; p < kMaxPass; ++p) {
                if (p < npass) {
                    int acc = part[p];
                    for (int o = 1; o < cpg; o <<= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
                    const int c = p * 32 + lane;
                    if (c < chunks && (lane & (cpg - 1)) == 0) {
                        const int g = c >> cpg_log2;
                        m.gsm[rr * gst + g] = acc;
                        m.gsf[rr * gst + g] = h2f_bits(ssl[rr * ng + g]);
                    }
                }
            }
        }
        cbar();
        if (tid < rows) {
            const int* gp = m.gsm + tid * gst;
            const float* fp = m.gsf + tid * gst;
            float run = 0.0f;
#pragma unroll 8
            for (int g = 0; g < ng; ++g) run = fmaf((float)gp[g], fp[g], run);
            const __half v = f2h(__fmul_rn(run, as));
            const int n = r + tid;
            if (epi == kEpiStore) {
                out[n] = v;
            } else if (epi == kEpiResid) {
                out[n] = __hadd(__ldcg(out + n), v);
            } else if (epi == kEpiLm) {
                out[n] = v;
                const unsigned long long key = argmax_key(h2f(v), n);
                best = key > best ? key : best;
            } else {
                m.ob[tid] = v;
            }
        }
        cbar();
        if (tid == 0) mbar_arrive(&empty[s]);
        if (epi == kEpiGlu && tid < rows / 2)
            out[(r >> 1) + tid] = __hmul(ref_silu(m.ob[2 * tid]), m.ob[2 * tid + 1]);
    }
    return true;
}

// grid-wide barrier over the consumer warps of all blocks
__device__ bool grid_sync(const PArgs& a, unsigned& nbar, int* flag) {
    cbar();
    ++nbar;
    if (threadIdx.x == 0) {
        bool ok = !ld_volatile_u32(&a.sync->abort);
        if (ok) {
            // release: the block's writes (ordered before by the consumer barrier) become
            // visible before the arrival; relaxed polling, one acquire fence at the end
            red_release_gpu_add(&a.sync->bar, 1u);
            const unsigned target = nbar * gridDim.x;
            uint32_t i = 0;
            while (ld_relaxed_gpu(&a.sync->bar) < target) {
                if (++i > (1u << 22) || ((i & 63) == 0 && ld_volatile_u32(&a.sync->abort))) {
                    ok = false;
                    break;
                }
            }
            fence_acq_rel_gpu();
        }
        if (!ok) set_abort(a, kDevFlagTimeout);
        *flag = ok ? 1 : 0;
    }
    cbar();
    return *flag != 0;
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

template <int D>
__device__ void attention_head(const PArgs& a, int l, int h, uint8_t* work, int cache_len, int total_len) {
    const int tid = threadIdx.x, warp = tid >> 5;
    const int grp = a.Hq / a.Hkv, kvh = h / grp;
    const int nqg = (D + 127) / 128;
    const AttnSmem<D> sm(work);
    float* qs = sm.qs;
    __half *hq = sm.hq, *hk = sm.hk, *hv = sm.hv, *qr = sm.qr, *kr = sm.kr;
    const PLayer& ly = a.layers[l];
    for (int d = tid; d < D; d += kPC) {
        hq[d] = __ldcg(a.qkv + (size_t)h * D + d);
        hk[d] = __ldcg(a.qkv + (size_t)(a.Hq + kvh) * D + d);
        hv[d] = __ldcg(a.qkv + (size_t)(a.Hq + a.Hkv + kvh) * D + d);
    }
    cp_async_wait<0>();  // the prefetched norm weights / RoPE rows / K/V of this thread
    cbar();
    const __half* crow = ly.ct ? sm.crow : nullptr;
    if (warp == 0) head_norm_rope_rows(hq, D, ly.q_norm ? sm.qn : nullptr, a.eps, crow, sm.srow, qr);
    else if (warp == 1) head_norm_rope_rows(hk, D, ly.k_norm ? sm.kn : nullptr, a.eps, crow, sm.srow, kr);
    cbar();
    for (int d = tid; d < D; d += kPC) qs[d] = h2f(qr[d]);
    // the first q head of each group appends the step's K/V to the cache at slot cache_len
    if (h % grp == 0 && warp >= 2 && warp < 2 + 2 * nqg) {
        const int which = (warp - 2) / nqg, g = (warp - 2) % nqg;
        const int cnt = min(128, D - g * 128);
        const __half* src = (which ? hv : kr) + g * 128;
        int8_t* dst = (which ? ly.vc : ly.kc) + ((size_t)cache_len * a.Hkv + kvh) * D + g * 128;
        float* sdst = (which ? ly.vs : ly.ks) + ((size_t)cache_len * a.Hkv + kvh) * nqg + g;
        kv_quant_group_warp(src, cnt, dst, sdst);
    }
    cbar();
    const AttnCoreArgs c = attn_args<D>(a, ly, h, cache_len, total_len, qs, kr, hv);
    const __half o = attn_exact_core<D, kPC, kACH>(c, work, SyncConsumers{});
    if (tid < D) a.attn[(size_t)h * D + tid] = o;
}

// embedding row of `tok` (compute_embedding_node semantics, as embed_kernel) into xs; the
// block also stores its slice of the hidden state
__device__ void embed_row(const PArgs& a, uint32_t tok, __half* xs) {
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
        if (k >= k0 && k < k1) a.hidden[k] = v;
    }
    cbar();
}

template <int D>
__global__ void __launch_bounds__(kPT, 1) decode_persistent_kernel(PArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ float s_red[64];
    __shared__ float s_as;
    __shared__ int s_flag;
    __shared__ unsigned long long s_best[16];
    const int NS = a.nslots, sb = a.slot_w + a.slot_s;
    uint8_t* ring = smem;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)NS * sb);
    uint64_t* empty = full + NS;
    uint8_t* work = smem + (size_t)NS * sb + a128(16 * NS);
    const int tid = threadIdx.x;
    if (tid == 0) {
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
    m.red = s_red;
    m.as = &s_as;
    m.flag = &s_flag;
    m.best = s_best;

    const int cache_len = __ldcg(a.state), total_len = __ldcg(a.state + 1);
    const uint32_t tok = __ldcg(a.tok_in);
    uint8_t* awork = work + a.attn_off;
    const bool attn_block = (int)blockIdx.x < a.Hq;
    unsigned kslot = 0, nbar = 0;
    unsigned long long best = 0ull;
    __half nw[kMaxPerThread];
    embed_row(a, tok, m.xs);
    for (int l = 0; l < a.L; ++l) {
        const PLayer& ly = a.layers[l];
        if (attn_block) attention_prefetch<D>(a, l, blockIdx.x, awork, cache_len, total_len);
        load_vec(m.xs, l > 0 ? a.hidden : nullptr, a.H, ly.in_norm, nw);
        prologue(m, a.H, true, nw, a.eps);
        if (!gemv_job(a, 4 * l, kEpiStore, m, ring, full, empty, kslot, a.qkv, best)) return;
        if (!grid_sync(a, nbar, m.flag)) return;
        if (attn_block) attention_head<D>(a, l, blockIdx.x, awork, cache_len, total_len);
        if (!grid_sync(a, nbar, m.flag)) return;
        load_vec(m.xs, a.attn, a.Hq * D, nullptr, nw);
        prologue(m, a.Hq * D, false, nw, a.eps);
        if (!gemv_job(a, 4 * l + 1, kEpiResid, m, ring, full, empty, kslot, a.hidden, best)) return;
        if (!grid_sync(a, nbar, m.flag)) return;
        load_vec(m.xs, a.hidden, a.H, ly.post_norm, nw);
        prologue(m, a.H, true, nw, a.eps);
        if (!gemv_job(a, 4 * l + 2, kEpiGlu, m, ring, full, empty, kslot, a.gated, best)) return;
        if (!grid_sync(a, nbar, m.flag)) return;
        load_vec(m.xs, a.gated, a.F, nullptr, nw);
        prologue(m, a.F, false, nw, a.eps);
        if (!gemv_job(a, 4 * l + 3, kEpiResid, m, ring, full, empty, kslot, a.hidden, best)) return;
        if (!grid_sync(a, nbar, m.flag)) return;
    }
    load_vec(m.xs, a.hidden, a.H, a.out_norm, nw);
    prologue(m, a.H, true, nw, a.eps);
    if (!gemv_job(a, 4 * a.L, kEpiLm, m, ring, full, empty, kslot, a.logits, best)) return;
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
            a.sync->bar = 0u;
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
    if (a.Hq > num_sms || a.Hkv < 1 || a.Hq % a.Hkv) return no("head layout");
    if (a.G < 16 || a.G % 16 || 32 % (a.G / 16)) return no("group size");
    const int Ks[3] = {a.H, a.Hq * a.D, a.F};
    int kmin = Ks[0], kmax = Ks[0];
    for (int K : Ks) {
        if (K % a.G || K % 16) return no("K not a multiple of the group size");
        kmin = K < kmin ? K : kmin;
        kmax = K > kmax ? K : kmax;
    }
    const int Ns[5] = {a.QKVN, a.H, 2 * a.F, a.H, a.V};
    for (int N : Ns)
        if (N % 8) return no("rows not a multiple of 8");
    a.kmax = kmax;
    a.slot_w = a128(kmax * 8 > 24576 ? kmax * 8 : 24576);
    a.slot_s = a128(a.slot_w / a.G * 2);
    a.max_rows = a.slot_w / kmin;
    if (a.max_rows > kPC) return no("hidden sizes too small for the slot size");
    a.gsm_ints = a.slot_w / a.G + a.max_rows + 32;
    if (a.H > kMaxPerThread * kPC) return no("hidden size above the per-thread RMSNorm limit");
    if (kmax > kMaxPass * 512) return no("projection width above 4096");
    if (a.G & (a.G - 1)) return no("group size must be a power of two");
    const int gemv_work = a128(kmax) + a128(2 * kmax) + 2 * a.gsm_ints * 4 + a.max_rows * 2 + 16;
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
    p.grid = num_sms;
    p.threads = kPT;
    p.ok = true;
    return p;
}

cudaError_t launch_persistent_decode(const PArgs& a, const PPlan& p, cudaStream_t st) {
    void (*k)(PArgs) = a.D == 64 ? decode_persistent_kernel<64> : decode_persistent_kernel<128>;
    static size_t attr_set[2] = {0, 0};  // largest dynamic shared memory enabled per variant
    size_t& done = attr_set[a.D == 64 ? 0 : 1];
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
