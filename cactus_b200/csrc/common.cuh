// Shared device helpers for the sm_100a kernels of cactus_b200.
//
// Arithmetic conventions (they reproduce the reference's rounding points):
//  * the library is compiled with --fmad=false, so a*b+c is never contracted
//    implicitly; every fused multiply-add is an explicit fmaf()/__hfma() placed
//    where the reference's NEON code fuses (vfmaq_f32 / vfmaq_f16 / contracted
//    `acc += a * b`);
//  * __hadd/__hmul/__hfma are the correctly rounded binary16 ops that NEON's
//    vaddq_f16/vmulq_f16/vfmaq_f16 perform.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

#include "kv_paging.h"

namespace cb {

constexpr int kNumSMs = 148;

__host__ __device__ __forceinline__ long long kv_page_row(const int* seq_table, int shift, long long c) {
    return ((long long)seq_table[c >> shift] << shift) + (c & ((1LL << shift) - 1));
}

// Device-side error word: kernels that give up a bounded wait record a code here and
// return; the host reads it with cactus_cuda_device_error().
enum DevError : unsigned {
    kDevOk = 0,
    kDevTmaTimeout = 1,
    kDevFlagTimeout = 2,
};
#ifdef __CUDACC_RDC__
extern __device__ unsigned g_dev_error;

__device__ __forceinline__ void report_dev_error(unsigned code) { atomicCAS(&g_dev_error, 0u, code); }
#endif
// Address of g_dev_error for kernels compiled as whole-program code (no extern device
// symbols there): they take it as a kernel argument.
unsigned* dev_error_ptr();

// ---------------------------------------------------------------- fp16 helpers
__device__ __forceinline__ float h2f(__half h) { return __half2float(h); }
// Exact int -> fp32 for |x| < 2^22 without the conversion pipe: 1.5 * 2^23 + x holds x in the
// low mantissa bits, so one integer add and one float subtract give (float)x exactly.
__device__ __forceinline__ float i2f_small(int x) { return __fsub_rn(__int_as_float(0x4B400000 + x), 12582912.0f); }
__device__ __forceinline__ __half f2h(float f) { return __float2half_rn(f); }
__device__ __forceinline__ float h2f_bits(uint16_t b) { return __half2float(__ushort_as_half(b)); }
__device__ __forceinline__ uint16_t f2h_bits(float f) { return __half_as_ushort(__float2half_rn(f)); }

// vcvtq_s32_f32: truncation toward zero with saturation (cvt.rzi saturates, NaN -> 0)
__device__ __forceinline__ int cvt_trunc_sat(float x) { return __float2int_rz(x); }
// vcvtnq_s32_f32: round half to even with saturation
__device__ __forceinline__ int cvt_rne_sat(float x) { return __float2int_rn(x); }
__device__ __forceinline__ int sat8(int v) { return v > 127 ? 127 : (v < -128 ? -128 : v); }

// Reference fast_exp (kernel_utils.h:108-141): clamp to +-87, split z = x*log2(e) into
// integer and fractional parts, degree-4 polynomial in (frac * ln2), scale by 2^int.
__device__ __forceinline__ float ref_fast_exp(float x) {
    x = fmaxf(x, -87.0f);
    x = fminf(x, 87.0f);
    float z = __fmul_rn(x, 1.4426950408889634f);
    int zi = cvt_trunc_sat(z);
    float zf = __fsub_rn(z, (float)zi);
    if (zf < 0.0f) { zi -= 1; zf = __fadd_rn(zf, 1.0f); }
    float t = __fmul_rn(zf, 0.6931471805599453f);
    float p = 0.009618129842071803f;
    p = fmaf(p, t, 0.05550410866482158f);
    p = fmaf(p, t, 0.2402265069591007f);
    p = fmaf(p, t, 0.6931471805599453f);
    p = fmaf(p, t, 1.0f);
    float sc = __uint_as_float((unsigned)(zi + 127) << 23);
    return __fmul_rn(p, sc);
}

// Reference fast_tanh (kernel_utils.h:143-163): x(27+x^2)/(27+9x^2), saturated beyond 4.5.
__device__ __forceinline__ float ref_fast_tanh(float x) {
    float x2 = __fmul_rn(x, x);
    float num = __fadd_rn(27.0f, x2);
    float den = fmaf(9.0f, x2, 27.0f);
    float r = __fmul_rn(x, __fdiv_rn(num, den));
    if (x > 4.5f) r = 1.0f;
    if (x < -4.5f) r = -1.0f;
    return r;
}

// exp / tanh rounded once from the double-precision result: correctly rounded except in
// vanishingly rare double-rounding cases, so the CPU restatement (which computes the same
// expression) matches bit for bit. The reference calls libm expf / tanhf, whose results
// are correctly rounded for all but rare arguments.
__device__ __forceinline__ float expf_cr(float x) { return (float)exp((double)x); }
__device__ __forceinline__ float tanhf_cr(float x) { return (float)tanh((double)x); }

// SiLU of one fp16 value as the vector path of cactus_silu_f16 (kernel_nn.cpp:22-35).
__device__ __forceinline__ __half ref_silu(__half h) {
    float x = h2f(h);
    float e = ref_fast_exp(-x);
    float sg = __fdiv_rn(1.0f, __fadd_rn(1.0f, e));
    return f2h(__fmul_rn(x, sg));
}
// GELU-tanh of one fp16 value as the vector path of cactus_gelu_f16 (kernel_nn.cpp:60-80).
__device__ __forceinline__ __half ref_gelu(__half h) {
    float x = h2f(h);
    float x3 = __fmul_rn(__fmul_rn(x, x), x);
    float inner = fmaf(0.044715f, x3, x);
    inner = __fmul_rn(0.7978845608028654f, inner);
    float t = ref_fast_tanh(inner);
    return f2h(__fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, t)));
}

// Quadratic 2^x approximation of the no-cache attention (kernel_attention.cpp:174-195).
__device__ __forceinline__ float attn_quad_exp(float s, float block_max) {
    float x = __fmul_rn(__fsub_rn(s, block_max), 1.442695f);
    int xi = cvt_trunc_sat(x);
    float xf = __fsub_rn(x, (float)xi);
    float y = fmaf(xf, 0.6931472f, 1.0f);
    y = fmaf(__fmul_rn(xf, xf), 0.2402265f, y);
    float sc = __uint_as_float((unsigned)(xi + 127) << 23);
    return __fmul_rn(y, sc);
}

// ---------------------------------------------------------------- integer dot products
__device__ __forceinline__ int dp4a_ss(int a, int b, int c) {
    int d;
    asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
// signed a x unsigned b
__device__ __forceinline__ int dp4a_su(int a, unsigned b, int c) {
    int d;
    asm("dp4a.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// ---------------------------------------------------------------- warp / block reductions
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ int warp_sum_i(int v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// ---------------------------------------------------------------- mbarrier + TMA bulk copy
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, unsigned bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, unsigned parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait: gives up after ~2^24 polls (each try_wait itself suspends for a while),
// i.e. seconds, far beyond any copy's latency; the caller turns `false` into an error.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, unsigned parity) {
    for (uint32_t i = 0; i < (1u << 24); ++i)
        if (mbar_try_wait(bar, parity)) return true;
    return false;
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// gpu-scope acquire load / relaxed volatile load of a flag word
__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ unsigned ld_relaxed_gpu(const unsigned* p) {
    unsigned v;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void red_release_gpu_add(unsigned* p, unsigned v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }
__device__ __forceinline__ unsigned ld_volatile_u32(const unsigned* p) {
    return *reinterpret_cast<const volatile unsigned*>(p);
}
// 1-D bulk async copy global -> shared (no multicast), completion on `bar`.
__device__ __forceinline__ void tma_load_1d(void* smem_dst, const void* gmem_src, unsigned bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(smem_dst)),
        "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}
// L2 policy for data read once per pass (streamed weights): evict it first so that small
// reused data (activations, norms, RoPE rows, the KV cache, the kernel's own instructions)
// stays resident in L2.
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
// 1-D bulk async copy global -> shared with an L2 cache-policy hint (no multicast).
__device__ __forceinline__ void tma_load_1d_hint(void* smem_dst, const void* gmem_src, unsigned bytes, uint64_t* bar,
                                                 uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            smem_u32(smem_dst)),
        "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}
// 2-D tiled TMA load (no multicast) at (x = innermost byte coordinate, y = row), with an L2
// cache-policy hint; `map` is a __grid_constant__ kernel parameter
__device__ __forceinline__ void tma_load_2d_tile(void* dst, const void* map, int x, int y, uint64_t* bar,
                                                 uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}
// orders this thread's generic-proxy shared-memory accesses before later async-proxy ones
// (a bulk copy into a buffer that was just read with ordinary loads)
__device__ __forceinline__ void fence_proxy_async_shared() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void prefetch_l2_bulk(const void* gmem_src, unsigned bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(gmem_src), "r"(bytes) : "memory");
}

// ---------------------------------------------------------------- programmatic dependent launch
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" :::); }

// Host side: kernels launched through launch_k() get the programmatic-stream-serialization
// attribute while pdl_scope is active on the calling thread (the engine enables it for its
// decode/prefill sequences; standalone C-ABI calls run without it, where griddepcontrol.wait
// is a no-op). Every kernel calls pdl_launch_dependents()/pdl_wait() before touching data
// produced by earlier launches.
bool& pdl_flag();
struct pdl_scope {
    bool prev;
    explicit pdl_scope(bool on) : prev(pdl_flag()) { pdl_flag() = on; }
    ~pdl_scope() { pdl_flag() = prev; }
};
template <typename... KArgs, typename... Args>
inline cudaError_t launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                            Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_flag() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// cp.async copies global -> shared (4 bytes through L1, 16 bytes bypassing it) and their groups
__device__ __forceinline__ void cp_async4(void* smem, const void* gmem) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(smem)), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem)), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// 16-byte global load that bypasses L1 allocation (read-only stream)
__device__ __forceinline__ int4 ldg_nc_v4(const void* p) {
    int4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.s32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

}  // namespace cb
