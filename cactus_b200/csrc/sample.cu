// Device sampling: cactus_sample_f16's non-greedy branch (kernel_nn.cpp:469-651) and the
// normalised entropy that Model::decode reports (engine_model.cpp:255-290).
//
// One CTA of 1024 threads per row. Steps, each as in the reference:
//   1. filtered = logits, times fp16(1/temperature) when temperature > 0 (fp16 multiply);
//   2. repetition penalty 1.1 for every id in the history (in history order);
//   3. top-k: the k-th largest value is found by a two-level histogram over the fp16
//      ordering keys; values below it become -inf (ties with it are kept);
//   4. top-p: the surviving candidates are ordered by value (descending, lower index first
//      on ties), probabilities exp(x - max) normalised in that order, and the tail after the
//      cumulative probability passes top_p is removed (up to 1024 survivors sorted in
//      shared memory, more walked as runs of equal values: top_p_all_candidates);
//   5. probabilities exp(x - max) of the survivors summed in index order, the uniform
//      sample (drawn on the host with the reference's mt19937) picks the first index whose
//      cumulative probability reaches it (one warp walks all V entries in index order when
//      more than 1024 survive: draw_all_candidates).
#include "common.cuh"
#include "ops.h"

namespace cb {

constexpr int kSampleThreads = 1024;
constexpr int kMaxCand = 1024;

__device__ __forceinline__ unsigned h_key(__half h) {  // monotone key of an fp16 value
    const unsigned short u = __half_as_ushort(h);
    return (u & 0x8000u) ? (unsigned)(~u & 0xFFFFu) : (unsigned)(u | 0x8000u);
}
__device__ __forceinline__ __half key_h(unsigned k) {
    const unsigned short u = (k & 0x8000u) ? (unsigned short)(k & 0x7FFFu) : (unsigned short)(~k & 0xFFFFu);
    return __ushort_as_half(u);
}

struct SampleArgs {
    const __half* logits;
    int V;
    float temperature, top_p;
    int top_k;
    float uniform;                // sample in [0, 1)
    const uint32_t* history;      // repetition-penalty history
    int n_history;
    __half* work;                 // [V] scratch (filtered logits)
    uint32_t* out;
};

// Top-p over more candidates than fit in shared memory (kernel_nn.cpp:537-586 with any
// number of survivors). The reference sorts the survivors by value and sums exp(v - max) in
// that order; equal values give equal terms, so the sorted order is walked as runs of equal
// fp16 values (descending), each run's term added once per member in one thread, which is
// the same serial fp32 sum. Runs are found with a 256-bin histogram of the keys' high byte
// and, per non-empty high bin, a 256-bin histogram of the low byte (one pass over V each).
// The cut lands inside one run (value v*, r members kept): values below v* are removed, and
// of the members equal to v* the first r in index order stay (ties ordered by index, as in
// the fast path).
__device__ __noinline__ void top_p_all_candidates(const SampleArgs& a, unsigned* hist1, int t) {
    __shared__ unsigned hist2[256];
    __shared__ float s_mx, s_sum, s_cum;
    __shared__ int s_pos, s_have_mx, s_done, s_cut_key, s_keep, s_base;
    __shared__ int s_wsum[kSampleThreads / 32];
    const __half neg_inf = __ushort_as_half(0xFC00u);
    for (int i = t; i < 256; i += kSampleThreads) hist1[i] = 0;
    if (t == 0) { s_sum = 0.0f; s_cum = 0.0f; s_pos = 0; s_have_mx = 0; s_done = 0; s_cut_key = -1; s_keep = 0; }
    __syncthreads();
    for (int i = t; i < a.V; i += kSampleThreads) {
        const __half v = a.work[i];
        if (!__heq(v, neg_inf)) atomicAdd(&hist1[h_key(v) >> 8], 1u);
    }
    __syncthreads();
    for (int phase = 0; phase < 2; ++phase) {  // 0: the sum, 1: the cumulative cut
        for (int hb = 255; hb >= 0; --hb) {
            if (hist1[hb] == 0u || s_done) continue;  // uniform: shared values after a barrier
            for (int i = t; i < 256; i += kSampleThreads) hist2[i] = 0;
            __syncthreads();
            for (int i = t; i < a.V; i += kSampleThreads) {
                const __half v = a.work[i];
                const unsigned k = h_key(v);
                if (!__heq(v, neg_inf) && (k >> 8) == (unsigned)hb) atomicAdd(&hist2[k & 0xFFu], 1u);
            }
            __syncthreads();
            if (t == 0) {
                for (int lb = 255; lb >= 0 && !s_done; --lb) {
                    const unsigned c = hist2[lb];
                    if (!c) continue;
                    const unsigned key = ((unsigned)hb << 8) | (unsigned)lb;
                    const float v = h2f(key_h(key));
                    if (!s_have_mx) { s_mx = v; s_have_mx = 1; }
                    const float p = expf_cr(__fsub_rn(v, s_mx));
                    if (phase == 0) {
                        float sum = s_sum;
                        for (unsigned j = 0; j < c; ++j) sum = __fadd_rn(sum, p);
                        s_sum = sum;
                    } else {
                        const float q = __fdiv_rn(p, s_sum);
                        float cum = s_cum;
                        int pos = s_pos;
                        for (unsigned j = 0; j < c; ++j, ++pos) {
                            cum = __fadd_rn(cum, q);
                            if (cum > a.top_p && pos > 0) {
                                s_cut_key = (int)key;
                                s_keep = (int)j;
                                s_done = 1;
                                break;
                            }
                        }
                        s_cum = cum;
                        s_pos = pos;
                    }
                }
            }
            __syncthreads();
        }
    }
    if (s_cut_key < 0) return;  // no cut: every survivor stays
    const unsigned cut_key = (unsigned)s_cut_key;
    const int keep = s_keep;
    if (t == 0) s_base = 0;
    __syncthreads();
    const int lane = t & 31, w = t >> 5;
    for (int base = 0; base < a.V; base += kSampleThreads) {
        const int i = base + t;
        bool tie = false;
        if (i < a.V) {
            const __half v = a.work[i];
            if (!__heq(v, neg_inf)) {
                const unsigned k = h_key(v);
                if (k < cut_key) a.work[i] = neg_inf;
                tie = (k == cut_key);
            }
        }
        const unsigned bal = __ballot_sync(0xffffffffu, tie);
        if (lane == 0) s_wsum[w] = __popc(bal);
        __syncthreads();
        int before = s_base;
        for (int x = 0; x < w; ++x) before += s_wsum[x];
        before += __popc(bal & ((1u << lane) - 1u));
        if (tie && before >= keep) a.work[i] = neg_inf;
        __syncthreads();
        if (t == 0) {
            int tot = 0;
            for (int x = 0; x < kSampleThreads / 32; ++x) tot += s_wsum[x];
            s_base += tot;
        }
        __syncthreads();
    }
}

// The final draw over more survivors than fit in shared memory (kernel_nn.cpp:603-650): one
// warp walks the vocabulary in index order, 32 entries at a time; every lane computes its
// entry's exp(x - max) (0 for removed entries) and all lanes add the 32 terms in index order,
// so the fp32 sum and the cumulative scan are the reference's serial ones.
__device__ __noinline__ void draw_all_candidates(const SampleArgs& a, float maxv, int lane) {
    const __half neg_inf = __ushort_as_half(0xFC00u);
    const float mx = h2f(__float2half_rn(maxv));
    float sum = 0.0f;
    for (int base = 0; base < a.V; base += 32) {
        const int i = base + lane;
        float p = 0.0f;
        if (i < a.V) {
            const __half v = a.work[i];
            if (!__heq(v, neg_inf)) p = expf_cr(__fsub_rn(h2f(v), mx));
        }
        for (int j = 0; j < 32; ++j) sum = __fadd_rn(sum, __shfl_sync(0xffffffffu, p, j));
    }
    uint32_t result = 0;
    if (sum != 0.0f && a.uniform > 0.0f) {
        float cum = 0.0f;
        int found = -1, last = -1;
        for (int base = 0; base < a.V && found < 0; base += 32) {
            const int i = base + lane;
            float q = 0.0f;
            if (i < a.V) {
                const __half v = a.work[i];
                if (!__heq(v, neg_inf)) q = __fdiv_rn(expf_cr(__fsub_rn(h2f(v), mx)), sum);
            }
            for (int j = 0; j < 32; ++j) {
                const float qj = __shfl_sync(0xffffffffu, q, j);
                cum = __fadd_rn(cum, qj);
                if (qj > 0.0f) last = base + j;
                if (cum >= a.uniform) { found = base + j; break; }
            }
        }
        result = (uint32_t)(found >= 0 ? found : (last >= 0 ? last : 0));
    }
    if (lane == 0) a.out[0] = result;
}

__global__ void __launch_bounds__(kSampleThreads) sample_kernel(SampleArgs a) {
    pdl_launch_dependents();
    pdl_wait();
    __shared__ unsigned hist[256];
    __shared__ unsigned sel_hi, sel_lo, need;
    __shared__ float cval[kMaxCand];
    __shared__ int cidx[kMaxCand];
    __shared__ int ncand;
    __shared__ float red[32];
    const int t = threadIdx.x;
    const __half neg_inf = __ushort_as_half(0xFC00u);
    // 1. temperature
    const __half inv_t = __float2half_rn(a.temperature > 0.0f ? __fdiv_rn(1.0f, a.temperature) : 1.0f);
    for (int i = t; i < a.V; i += kSampleThreads)
        a.work[i] = a.temperature > 0.0f ? __hmul(a.logits[i], inv_t) : a.logits[i];
    __syncthreads();
    // 2. repetition penalty, sequential in history order
    if (t == 0 && a.n_history > 0) {
        const float pinv = __fdiv_rn(1.0f, 1.1f);
        const __half pinv16 = __float2half_rn(pinv), pen16 = __float2half_rn(1.1f);
        for (int j = 0; j < a.n_history; ++j) {
            const uint32_t id = a.history[j];
            if ((int)id >= a.V) continue;
            const __half f = a.work[id];
            a.work[id] = __float2half_rn(__fmul_rn(h2f(f), h2f(__hgt(f, __float2half_rn(0.0f)) ? pinv16 : pen16)));
        }
    }
    __syncthreads();
    // 3. top-k threshold by histogram select
    if (a.top_k > 0 && a.top_k < a.V) {
        for (int lvl = 0; lvl < 2; ++lvl) {
            for (int i = t; i < 256; i += kSampleThreads) hist[i] = 0;
            if (t == 0 && lvl == 0) need = (unsigned)a.top_k;
            __syncthreads();
            for (int i = t; i < a.V; i += kSampleThreads) {
                const unsigned k = h_key(a.work[i]);
                if (lvl == 0) atomicAdd(&hist[k >> 8], 1u);
                else if ((k >> 8) == sel_hi) atomicAdd(&hist[k & 0xFF], 1u);
            }
            __syncthreads();
            if (t == 0) {
                unsigned cum = 0, r = need;
                int bin = 255;
                for (; bin >= 0; --bin) {
                    if (cum + hist[bin] >= r) break;
                    cum += hist[bin];
                }
                if (bin < 0) bin = 0;
                if (lvl == 0) { sel_hi = (unsigned)bin; need = r - cum; }
                else sel_lo = (unsigned)bin;
            }
            __syncthreads();
        }
        const __half kth = key_h((sel_hi << 8) | sel_lo);
        for (int i = t; i < a.V; i += kSampleThreads)
            if (__hlt(a.work[i], kth)) a.work[i] = neg_inf;
        __syncthreads();
    }
    // 4. top-p over the surviving candidates
    if (a.top_p > 0.0f && a.top_p < 1.0f) {
        if (t == 0) ncand = 0;
        __syncthreads();
        for (int i = t; i < a.V; i += kSampleThreads) {
            if (!__heq(a.work[i], neg_inf)) {
                const int p = atomicAdd(&ncand, 1);
                if (p < kMaxCand) { cval[p] = h2f(a.work[i]); cidx[p] = i; }
            }
        }
        __syncthreads();
        if (ncand <= kMaxCand) {
            if (t == 0) {
                const int n = ncand;
                // insertion sort by (value desc, index asc): n is at most top_k plus ties
                for (int i = 1; i < n; ++i) {
                    const float v = cval[i];
                    const int id = cidx[i];
                    int j = i - 1;
                    while (j >= 0 && (cval[j] < v || (cval[j] == v && cidx[j] > id))) {
                        cval[j + 1] = cval[j];
                        cidx[j + 1] = cidx[j];
                        --j;
                    }
                    cval[j + 1] = v;
                    cidx[j + 1] = id;
                }
                if (n > 0) {
                    const __half mx = __float2half_rn(cval[0]);
                    float sum = 0.0f;
                    for (int i = 0; i < n; ++i) sum = __fadd_rn(sum, expf_cr(__fsub_rn(cval[i], h2f(mx))));
                    float cum = 0.0f;
                    bool cut = false;
                    for (int i = 0; i < n; ++i) {
                        cum = __fadd_rn(cum, __fdiv_rn(expf_cr(__fsub_rn(cval[i], h2f(mx))), sum));
                        if (cum > a.top_p && i > 0) cut = true;
                        if (cut) a.work[cidx[i]] = neg_inf;
                    }
                }
            }
        } else {
            top_p_all_candidates(a, hist, t);
        }
        __syncthreads();
    }
    // 5. sample: max, then in-order probabilities (only survivors are non-zero)
    float mx = -INFINITY;
    for (int i = t; i < a.V; i += kSampleThreads) mx = fmaxf(mx, h2f(a.work[i]));
    mx = warp_max(mx);
    if ((t & 31) == 0) red[t >> 5] = mx;
    __syncthreads();
    if (t == 0) {
        float m = red[0];
        for (int w = 1; w < kSampleThreads / 32; ++w) m = fmaxf(m, red[w]);
        red[0] = m;
        ncand = 0;
    }
    __syncthreads();
    const float maxv = red[0];
    for (int i = t; i < a.V; i += kSampleThreads) {
        if (!__heq(a.work[i], neg_inf)) {
            const int p = atomicAdd(&ncand, 1);
            if (p < kMaxCand) { cidx[p] = i; }
        }
    }
    __syncthreads();
    if (maxv == -INFINITY) {
        if (t == 0) a.out[0] = 0;
    } else if (ncand > kMaxCand) {
        if (t < 32) draw_all_candidates(a, maxv, t);
    } else if (t == 0) {
        uint32_t result = 0;
        const int n = ncand;
        for (int i = 1; i < n; ++i) {  // index order
            const int id = cidx[i];
            int j = i - 1;
            while (j >= 0 && cidx[j] > id) { cidx[j + 1] = cidx[j]; --j; }
            cidx[j + 1] = id;
        }
        const __half mx16 = __float2half_rn(maxv);
        float sum = 0.0f;
        for (int i = 0; i < n; ++i) {
            cval[i] = expf_cr(__fsub_rn(h2f(a.work[cidx[i]]), h2f(mx16)));
            sum = __fadd_rn(sum, cval[i]);
        }
        if (sum == 0.0f || a.uniform <= 0.0f) {
            result = 0;  // a zero sample stops the reference's in-order scan at index 0
        } else {
            float cum = 0.0f;
            int found = -1;
            for (int i = 0; i < n; ++i) {
                cum = __fadd_rn(cum, __fdiv_rn(cval[i], sum));
                if (cum >= a.uniform) { found = cidx[i]; break; }
            }
            if (found < 0)
                for (int i = n - 1; i >= 0; --i)
                    if (__fdiv_rn(cval[i], sum) > 0.0f) { found = cidx[i]; break; }
            result = found < 0 ? 0u : (uint32_t)found;
        }
        a.out[0] = result;
    }
}

// normalised entropy of softmax(logits) in double precision (engine_model.cpp:255-290)
__global__ void __launch_bounds__(1024) entropy_kernel(const __half* __restrict__ logits, int V, float* out) {
    pdl_launch_dependents();
    pdl_wait();
    __shared__ double red[32];
    __shared__ float fmx;
    const int t = threadIdx.x;
    float mx = -INFINITY;
    for (int i = t; i < V; i += 1024) mx = fmaxf(mx, h2f(logits[i]));
    mx = warp_max(mx);
    if ((t & 31) == 0) red[t >> 5] = mx;
    __syncthreads();
    if (t == 0) {
        double m = red[0];
        for (int w = 1; w < 32; ++w) m = fmax(m, red[w]);
        fmx = (float)m;
    }
    __syncthreads();
    double s = 0.0;
    for (int i = t; i < V; i += 1024) s += exp((double)__fsub_rn(h2f(logits[i]), fmx));
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    __syncthreads();
    if ((t & 31) == 0) red[t >> 5] = s;
    __syncthreads();
    __shared__ double lse;
    if (t == 0) {
        double tot = 0;
        for (int w = 0; w < 32; ++w) tot += red[w];
        lse = (double)fmx + log(tot);
    }
    __syncthreads();
    double e = 0.0;
    for (int i = t; i < V; i += 1024) {
        const double lp = (double)h2f(logits[i]) - lse;
        const double p = exp(lp);
        if (p > 1e-10) e -= p * lp;
    }
    for (int o = 16; o > 0; o >>= 1) e += __shfl_xor_sync(0xffffffffu, e, o);
    __syncthreads();
    if ((t & 31) == 0) red[t >> 5] = e;
    __syncthreads();
    if (t == 0) {
        double tot = 0;
        for (int w = 0; w < 32; ++w) tot += red[w];
        out[0] = (float)(tot / log((double)V));
    }
}

int launch_sample(const __half* logits, int V, float temperature, float top_p, int top_k, float uniform,
                  const uint32_t* history, int n_history, __half* work, uint32_t* out, cudaStream_t st) {
    SampleArgs a;
    a.logits = logits;
    a.V = V;
    a.temperature = temperature;
    a.top_p = top_p;
    a.top_k = top_k;
    a.uniform = uniform;
    a.history = history;
    a.n_history = n_history;
    a.work = work;
    a.out = out;
    launch_k(sample_kernel, dim3(1), dim3(kSampleThreads), 0, st, a);
    return 0;
}

int launch_entropy(const __half* logits, int V, float* out, cudaStream_t st) {
    launch_k(entropy_kernel, dim3(1), dim3(1024), 0, st, logits, V, out);
    return 0;
}

}  // namespace cb
