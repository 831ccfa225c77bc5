// Device kernels that only the engine uses: fused per-head q/k RMSNorm + RoPE (+ split of
// the fused QKV projection), KV-cache append, decode-state bookkeeping, embedding lookup,
// Gemma's norm + clipped residual, and the per-sequence argmax that feeds the next step.
#include "../common.cuh"
#include "../gemv.cuh"
#include "engine_kernels.h"
#include "head_ops.cuh"

namespace cb {
namespace eng {

// ------------------------------------------------------------------ q/k norm + RoPE
// One warp per (row, head) of the fused projection row [q heads | k heads | v heads].
// q/k heads: optional per-head RMSNorm (QwenModel::build_attention, model_qwen.cpp:63-70:
// rms_norm over [seq*heads, head_dim]) then RoPE at position pos_base + (row % S)
// (cactus_rope_f16, kernel_attention.cpp:614-676); v heads are copied.
__global__ void __launch_bounds__(128) qkv_post_kernel(QkvPostArgs a) {
    pdl_launch_dependents();
    pdl_wait();
    extern __shared__ __align__(16) uint8_t smem_raw[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __half* xs = reinterpret_cast<__half*>(smem_raw) + warp * a.D;
    const int heads = a.Hq + 2 * a.Hkv;
    const long long item = (long long)blockIdx.x * 4 + warp;
    if (item >= (long long)a.rows * heads) return;
    const int row = (int)(item / heads), hi = (int)(item % heads);
    const int D = a.D;
    const __half* src = a.qkv + (size_t)row * a.qkv_stride + (size_t)hi * D;
    if (hi >= a.Hq + a.Hkv) {  // value head: copy
        __half* dst = a.v_out + ((size_t)row * a.Hkv + (hi - a.Hq - a.Hkv)) * D;
        for (int d = lane; d < D; d += 32) dst[d] = src[d];
        return;
    }
    const bool is_q = hi < a.Hq;
    for (int d = lane; d < D; d += 32) xs[d] = src[d];
    __syncwarp();
    const long long pos = (a.dstate ? (long long)a.dstate[1] : a.pos_base) + (row % a.S);
    __half* dst = is_q ? a.q_out + ((size_t)row * a.Hq + hi) * D : a.k_out + ((size_t)row * a.Hkv + (hi - a.Hq)) * D;
    head_norm_rope_warp(xs, D, is_q ? a.q_norm : a.k_norm, a.eps, a.ct, a.st, pos, dst);
}

// ------------------------------------------------------------------ KV append
// Quantises tokens [src_tok0, src_tok0 + ntok) of every sequence (fp16 [B, S, Hkv, D]) with
// the KV rule (kernel_quants.cpp:223-264) into cache slots [dst0, dst0 + ntok) of each
// sequence's cache ([cap, Hkv, D] int8 + [cap, Hkv, ng] fp32). dst0 comes from the device
// state (cache_len) when `dstate` is set. One warp per (b, token, head, group).
__global__ void kv_append_kernel(KvAppendArgs a) {
    pdl_launch_dependents();
    pdl_wait();
    const long long wid = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    const int ng = (a.D + a.G - 1) / a.G;
    const long long total = (long long)a.B * a.ntok * a.Hkv * ng;
    if (wid >= total) return;
    const int g = (int)(wid % ng);
    long long r = wid / ng;
    const int h = (int)(r % a.Hkv);
    r /= a.Hkv;
    const int t = (int)(r % a.ntok);
    const int b = (int)(r / a.ntok);
    const long long dst0 = a.dstate ? (long long)a.dstate[0] : a.dst0;
    const int g0 = g * a.G, cnt = min(a.G, a.D - g0);
    for (int which = 0; which < 2; ++which) {
        const __half* src = (which ? a.v_new : a.k_new) +
                            (((size_t)b * a.S + a.src_tok0 + t) * a.Hkv + h) * a.D + g0;
        // contiguous: sequence b's rows at its stride; paged: the physical row of its table
        const long long row = a.pg.table ? kv_page_row(a.pg.table + (size_t)b * a.pg.pps, a.pg.shift, dst0 + t)
                                         : dst0 + t;
        const size_t kb = a.pg.table ? 0 : (size_t)b * a.cache_bstride;
        const size_t sb = a.pg.table ? 0 : (size_t)b * a.scale_bstride;
        int8_t* dst = (which ? a.v_cache : a.k_cache) + kb + ((size_t)row * a.Hkv + h) * a.D + g0;
        float* sdst = (which ? a.v_scales : a.k_scales) + sb + ((size_t)row * a.Hkv + h) * ng + g;
        kv_quant_group_warp(src, cnt, dst, sdst);
    }
}

// paged compaction: phase 0 gathers the source rows (keys, values, scales) into tmp, phase 1
// scatters them to the destination rows; one thread per 4-byte word
__global__ void kv_move_paged_kernel(KvMoveArgs a, int phase) {
    pdl_launch_dependents();
    pdl_wait();
    const long long rb = (long long)a.Hkv * a.D / 4, rs = (long long)a.Hkv * a.ng;  // words per row
    const long long per = 2 * rb + 2 * rs;
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= a.n * per) return;
    const long long r = i / per, w = i % per;
    const int* tb = a.pg.table + (size_t)a.b * a.pg.pps;
    const long long row = kv_page_row(tb, a.pg.shift, (phase == 0 ? a.src0 : a.dst0) + r);
    uint32_t* slot;
    if (w < rb) slot = reinterpret_cast<uint32_t*>(a.k_cache) + row * rb + w;
    else if (w < 2 * rb) slot = reinterpret_cast<uint32_t*>(a.v_cache) + row * rb + (w - rb);
    else if (w < 2 * rb + rs) slot = reinterpret_cast<uint32_t*>(a.k_scales) + row * rs + (w - 2 * rb);
    else slot = reinterpret_cast<uint32_t*>(a.v_scales) + row * rs + (w - 2 * rb - rs);
    uint32_t* t = reinterpret_cast<uint32_t*>(a.tmp) + i;
    if (phase == 0) *t = *slot;
    else *slot = *t;
}

// byte copy used for the sliding-window compaction (through a temporary, so overlap is safe)
__global__ void copy_bytes_kernel(uint8_t* __restrict__ dst, const uint8_t* __restrict__ src, long long n) {
    pdl_launch_dependents();
    pdl_wait();
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) dst[i] = src[i];
}

// state[0] = current_seq_len, state[1] = total_seq_len, state[2] = decode step (no sliding)
__global__ void state_advance_kernel(int* state, int ntok) {
    pdl_launch_dependents();
    pdl_wait();
    if (threadIdx.x == 0 && blockIdx.x == 0) {
        state[0] += ntok;
        state[1] += ntok;
        state[2] += 1;
    }
}

// ------------------------------------------------------------------ embedding (+ Gemma scale)
// compute_embedding_node (graph_ops_tensor.cpp:226-331); INT4 tables stay packed and are
// dequantised per element to the same value as the reference's unpack-then-INT8 path.
__global__ void embed_kernel(EmbedArgs a) {
    pdl_launch_dependents();
    pdl_wait();
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)a.n * a.hidden) return;
    const int t = (int)(i / a.hidden), k = (int)(i % a.hidden);
    const size_t row = a.ids[t];
    __half v;
    if (a.prec == 1) {
        v = reinterpret_cast<const __half*>(a.table)[row * a.hidden + k];
    } else {
        int q;
        if (a.prec == 0) {
            q = reinterpret_cast<const int8_t*>(a.table)[row * a.hidden + k];
        } else {
            const uint8_t byte = reinterpret_cast<const uint8_t*>(a.table)[(row * a.hidden + k) >> 1];
            q = (k & 1) ? (byte >> 4) : (byte & 0x0F);
            q = (q & 8) ? q - 16 : q;
        }
        v = f2h(__fmul_rn((float)q, h2f(a.scales[row * (a.hidden / a.G) + k / a.G])));
    }
    if (a.has_scale) v = __hmul(v, a.scale16);
    a.out[i] = v;
}

// ------------------------------------------------------------------ Gemma: hidden = add_clipped(hidden, rms_norm(o))
// GemmaModel::build_transformer_block (model_gemma.cpp:134-146); one CTA per row.
__global__ void norm_add_clipped_kernel(__half* __restrict__ hidden, const __half* __restrict__ o,
                                        const __half* __restrict__ w, int dims, float eps) {
    pdl_launch_dependents();
    pdl_wait();
    extern __shared__ __align__(16) uint8_t sm[];
    __half* xs = reinterpret_cast<__half*>(sm);
    __shared__ float ssum;
    const size_t r = blockIdx.x;
    for (int k = threadIdx.x; k < dims; k += blockDim.x) xs[k] = o[r * dims + k];
    __syncthreads();
    if (threadIdx.x < 32) {
        const float ss = rms_sumsq_warp(xs, dims);
        if (threadIdx.x == 0) ssum = ss;
    }
    __syncthreads();
    const float rms = __fsqrt_rn(__fadd_rn(__fdiv_rn(ssum, (float)dims), eps));
    const float inv = __fdiv_rn(1.0f, rms);
    const __half inv16 = __float2half_rn(inv);
    const int vec_end = dims >= 8 ? (dims / 8) * 8 : 0;
    for (int k = threadIdx.x; k < dims; k += blockDim.x) {
        const __half v = xs[k];
        const __half y = (k < vec_end) ? __hmul(__hmul(v, inv16), w[k])
                                       : __float2half_rn(__fmul_rn(__fmul_rn(h2f(v), inv), h2f(w[k])));
        float s = __fadd_rn(h2f(hidden[r * dims + k]), h2f(y));
        s = fminf(fmaxf(s, -65500.0f), 65500.0f);
        hidden[r * dims + k] = f2h(s);
    }
}

// ------------------------------------------------------------------ per-sequence argmax
// First maximum wins (kernel_nn.cpp:451-467). Writes the next input token of sequence b and
// appends it to the output ring at position state[2] (the decode step).
__global__ void argmax_rows_kernel(const __half* __restrict__ logits, int V, uint32_t* __restrict__ next_tok,
                                   uint32_t* __restrict__ ring, int ring_stride, const int* __restrict__ state) {
    pdl_launch_dependents();
    pdl_wait();
    __shared__ unsigned long long red[32];
    const int b = blockIdx.x;
    const __half* lg = logits + (size_t)b * V;
    // (value, ~index) keys: the maximum key is the first maximum whatever the scan order
    auto key = [](__half h, int i) -> unsigned long long {
        const float v = h2f(h);
        if (v != v) return 0ull;
        unsigned u = __float_as_uint(v);
        u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
        return ((unsigned long long)u << 32) | (0xFFFFFFFFu - (unsigned)i);
    };
    unsigned long long best = 0ull;
    int i0 = 0;
    if ((reinterpret_cast<uintptr_t>(lg) & 15) == 0) {
        // 16-byte loads of 8 logits, four in flight per thread (a vocabulary row is up to 512 KB)
        const int n8 = V / 8;
        const int4* l8 = reinterpret_cast<const int4*>(lg);
#pragma unroll 4
        for (int c = threadIdx.x; c < n8; c += blockDim.x) {
            const int4 q = __ldg(l8 + c);
            const __half* h = reinterpret_cast<const __half*>(&q);
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const unsigned long long k = key(h[e], 8 * c + e);
                best = k > best ? k : best;
            }
        }
        i0 = n8 * 8;
    }
    for (int i = i0 + threadIdx.x; i < V; i += blockDim.x) {
        const unsigned long long k = key(lg[i], i);
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
        if (threadIdx.x == 0) {
            const uint32_t tok = best == 0ull ? 0u : 0xFFFFFFFFu - (unsigned)(best & 0xFFFFFFFFull);
            next_tok[b] = tok;
            if (ring) ring[(size_t)b * ring_stride + (state ? state[2] : 0)] = tok;
        }
    }
}

// ------------------------------------------------------------------ launchers
static inline unsigned nb(long long n, int t) { return (unsigned)((n + t - 1) / t); }

void launch_qkv_post(const QkvPostArgs& a, cudaStream_t st) {
    const long long items = (long long)a.rows * (a.Hq + 2 * a.Hkv);
    launch_k(qkv_post_kernel, dim3(nb(items, 4)), dim3(128), 4 * a.D * 2, st, a);
}
void launch_kv_append(const KvAppendArgs& a, cudaStream_t st) {
    const int ng = (a.D + a.G - 1) / a.G;
    const long long warps = (long long)a.B * a.ntok * a.Hkv * ng;
    if (warps > 0) launch_k(kv_append_kernel, dim3(nb(warps * 32, 256)), dim3(256), 0, st, a);
}
void launch_kv_move_paged(const KvMoveArgs& a, cudaStream_t st) {
    const long long words = a.n * (2LL * a.Hkv * a.D / 4 + 2LL * a.Hkv * a.ng);
    if (words <= 0) return;
    launch_k(kv_move_paged_kernel, dim3(nb(words, 256)), dim3(256), 0, st, a, 0);
    launch_k(kv_move_paged_kernel, dim3(nb(words, 256)), dim3(256), 0, st, a, 1);
}
void launch_copy_bytes(void* dst, const void* src, long long n, cudaStream_t st) {
    if (n > 0)
        launch_k(copy_bytes_kernel, dim3(nb(n, 256)), dim3(256), 0, st, static_cast<uint8_t*>(dst), static_cast<const uint8_t*>(src), n);
}
void launch_state_advance(int* state, int ntok, cudaStream_t st) { launch_k(state_advance_kernel, dim3(1), dim3(32), 0, st, state, ntok); }
void launch_embed(const EmbedArgs& a, cudaStream_t st) {
    launch_k(embed_kernel, dim3(nb((long long)a.n * a.hidden, 256)), dim3(256), 0, st, a);
}
void launch_norm_add_clipped(__half* hidden, const __half* o, const __half* w, int rows, int dims, float eps,
                             cudaStream_t st) {
    launch_k(norm_add_clipped_kernel, dim3(rows), dim3(256), dims * 2, st, hidden, o, w, dims, eps);
}
void launch_argmax_rows(const __half* logits, int rows, int V, uint32_t* next_tok, uint32_t* ring, int ring_stride,
                        const int* state, cudaStream_t st) {
    launch_k(argmax_rows_kernel, dim3(rows), dim3(1024), 0, st, logits, V, next_tok, ring, ring_stride, state);
}

}  // namespace eng
}  // namespace cb
