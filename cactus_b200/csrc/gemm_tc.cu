// Grouped INT8 GEMM for M >= 64 rows on the 5th-generation tensor cores (tcgen05, TMEM).
//
// Result bits are those of qgemm_kernel / qgemv_kernel (and of cactus_matmul_int8,
// kernel_gemm.cpp:128-327): C[m,n] = fp16(chain_g(fma(float(gsum[m,n,g]), Bs[n,g], acc)) * As[m]).
// The reference needs the exact int32 sum of every quantisation group before it enters the
// fp32 chain, so each group gets its own TMEM accumulator: a tcgen05.mma.kind::i8 of K = 32
// writes (G = 32) or accumulates (G = 64, 128) the group's int32 sums for a 128 x BN tile into
// its own BN TMEM columns; the epilogue warps read the groups back in order (tcgen05.ld) and
// continue the fp32 chains in registers — one thread per row.
//
// Per CTA: a 128-row x BN-column output tile, 128 threads (4 warps). K advances in chunks of
// 128 bytes (4 mma k-steps); chunks are staged with cp.async in the canonical K-major,
// no-swizzle UMMA layout (8-row x 16-byte core matrices) in a 3-stage ring; the TMEM holds two
// chunks of group accumulators, so the MMAs of chunk c overlap the epilogue fold of chunk c-1.
// One thread issues the MMAs; completion is signalled with tcgen05.commit to an mbarrier.
// Every wait is bounded (device error on timeout) and TMEM is freed on every path.
// This file is compiled as whole-program device code (build.py WHOLE_PROGRAM): as relocatable
// code the same MMAs read their shared-memory operands displaced and the products are wrong.
#include "attention_core.cuh"
#include "common.cuh"
#include "ops.h"

namespace cb {

namespace {
constexpr int kTM = 128, kTBN = 16, kTThreads = 128;
constexpr int kKC = 128;                      // K bytes per chunk (4 x K32 mma steps)
constexpr int kStages = 3;
constexpr int kStageA = kTM * kKC;            // 16 KB
constexpr int kStageB = kTBN * kKC;           // 2 KB
constexpr int kStageS = kTBN * 4 * 2;         // scales of up to 4 groups x BN columns (fp16)
constexpr int kStage = ((kStageA + kStageB + kStageS) + 1023) / 1024 * 1024;
constexpr int kTmemCols = 128;                // 2 chunks x up to 4 groups x 16 columns

struct TcArgs {
    const int8_t* aq;
    const float* as;
    const int8_t* w;
    const __half* ws;
    __half* out;
    const __half* resid;
    unsigned* err;  // the library's device error word
    int M, K, N, G;
};

__device__ __forceinline__ void cp_async16_z(void* smem, const void* gmem, unsigned src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem)), "l"(gmem), "r"(src_bytes)
                 : "memory");
}

// canonical K-major no-swizzle layout: 8-row x 16-byte core matrices, K-columns 128 B apart,
// 8-row groups (kKC / 16) * 128 B apart
__device__ __forceinline__ int umma_off(int row, int kc) { return (row >> 3) * (kKC / 16) * 128 + kc * 128 + (row & 7) * 16; }

__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr) {
    const uint64_t lbo = 128 >> 4, sbo = ((kKC / 16) * 128) >> 4;
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | (lbo << 16) | (sbo << 32) | (1ull << 46);  // version 1, no swizzle
}

// kind::i8, D = S32, A = B = S8, both K-major, N = kTBN, M = kTM
constexpr uint32_t kIdesc = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kTBN >> 3) << 17) | ((uint32_t)(kTM >> 4) << 24);

__device__ __forceinline__ void tc_mma(uint32_t dtmem, uint64_t da, uint64_t db, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n"
        :
        : "r"(dtmem), "l"(da), "l"(db), "r"(kIdesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0));
}
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// The load and its wait form one asm statement: the destination registers are written
// asynchronously, and a separate wait statement would let the compiler schedule their first
// use ahead of it (it only orders memory, not these registers).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, int (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr)
        : "memory");
}

template <int EPI>
__global__ void __launch_bounds__(kTThreads, 1) qgemm_tc_kernel(TcArgs a) {
    pdl_launch_dependents();
    pdl_wait();
    // The declared alignment of dynamic shared memory is not honoured when static shared
    // variables precede it; the stages are aligned to 1024 bytes by hand (1 KB of slack is
    // launched) so that operand addresses do not depend on the static layout.
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* const smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    __shared__ uint64_t mma_done[2];
    __shared__ uint32_t tmem_base_s;
    __shared__ int s_ok;
    const int tid = threadIdx.x, warp = tid >> 5;
    const int m0 = blockIdx.y * kTM, n0 = blockIdx.x * kTBN;
    const int G = a.G, ng = a.K / G, gpc = kKC / G, nchunks = a.K / kKC;

    if (warp == 0) {  // TMEM for two chunks of group accumulators
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base_s)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (tid == 0) {
        s_ok = 1;
        mbar_init(&mma_done[0], 1);
        mbar_init(&mma_done[1], 1);
        fence_mbar_init();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base_s;

    auto load = [&](int c) {
        uint8_t* st = smem + (c % kStages) * kStage;
        uint8_t* sA = st;
        uint8_t* sB = st + kStageA;
        __half* sS = reinterpret_cast<__half*>(st + kStageA + kStageB);
        const int k0 = c * kKC;
        for (int i = tid; i < kTM * (kKC / 16); i += kTThreads) {
            const int r = i >> 3, kc = i & 7, m = m0 + r;
            cp_async16_z(sA + umma_off(r, kc), a.aq + (size_t)min(m, a.M - 1) * a.K + k0 + kc * 16, m < a.M ? 16u : 0u);
        }
        {
            const int r = tid >> 3, kc = tid & 7;  // kTBN * 8 == kTThreads
            cp_async16(sB + umma_off(r, kc), a.w + (size_t)(n0 + r) * a.K + k0 + kc * 16);
        }
        if (tid < kTBN * gpc) {
            const int r = tid / gpc, g = tid % gpc;
            sS[r * 4 + g] = a.ws[(size_t)(n0 + r) * ng + c * gpc + g];
        }
        cp_async_commit();
    };

    float acc[kTBN];
#pragma unroll
    for (int j = 0; j < kTBN; ++j) acc[j] = 0.0f;
    const int row_local = warp * 32 + (tid & 31);                 // TMEM lane = tile row
    const uint32_t lane_addr = tmem + ((uint32_t)(warp * 32) << 16);

    // fold chunk c's group accumulators (in group order) into the per-row fp32 chains
    auto fold = [&](int c) -> bool {
        bool ok = true;
        if (tid == 0) *const_cast<volatile int*>(&s_ok) = mbar_wait_bounded(&mma_done[c & 1], (c >> 1) & 1) ? 1 : 0;
        __syncthreads();
        if (!s_ok) return false;
        mbar_wait_bounded(&mma_done[c & 1], (c >> 1) & 1);  // completed: orders this thread after the MMAs
        tc_fence_after();
        const __half* sS = reinterpret_cast<const __half*>(smem + (c % kStages) * kStage + kStageA + kStageB);
        for (int g = 0; g < gpc; ++g) {
            int v[16];
            tmem_ld16(lane_addr + (uint32_t)(((c & 1) * 4 + g) * kTBN), v);
#pragma unroll
            for (int j = 0; j < kTBN; ++j) acc[j] = fmaf((float)v[j], __half2float(sS[j * 4 + g]), acc[j]);
        }
        tc_fence_before();
        return ok;
    };

    bool ok = true;
    load(0);
    if (nchunks > 1) load(1);
    for (int c = 0; c < nchunks && ok; ++c) {
        if (c + 1 < nchunks) cp_async_wait<1>();
        else cp_async_wait<0>();
        fence_proxy_async();  // this thread's cp.async data -> visible to the tensor core
        __syncthreads();
        tc_fence_after();
        if (tid == 0) {
            const uint32_t base = smem_u32(smem + (c % kStages) * kStage);
            for (int s = 0; s < kKC / 32; ++s) {
                const int g = (s * 32) / G;
                const uint32_t dt = tmem + (uint32_t)(((c & 1) * 4 + g) * kTBN);
                tc_mma(dt, umma_desc(base + 2 * s * 128), umma_desc(base + kStageA + 2 * s * 128),
                       (s * 32) % G != 0 ? 1u : 0u);
            }
            tc_commit(&mma_done[c & 1]);
        }
        if (c >= 1) ok = fold(c - 1);
        if (ok && c + 2 < nchunks) {
            __syncthreads();  // every thread has read chunk c-1's scales
            load(c + 2);      // into the stage of chunk c-1, whose MMAs have completed
        }
    }
    if (ok) ok = fold(nchunks - 1);
    cp_async_wait<0>();
    if (!ok && tid == 0) atomicCAS(a.err, 0u, (unsigned)kDevTmaTimeout);
    tc_fence_before();
    __syncthreads();
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
    if (!ok) return;

    const int m = m0 + row_local;
    if (m >= a.M) return;
    const float asm_ = a.as[m];
#pragma unroll
    for (int j = 0; j < kTBN; j += 2) {
        const int n = n0 + j;
        const __half v0 = f2h(__fmul_rn(acc[j], asm_)), v1 = f2h(__fmul_rn(acc[j + 1], asm_));
        if constexpr (EPI == kEpiStore) {
            a.out[(size_t)m * a.N + n] = v0;
            a.out[(size_t)m * a.N + n + 1] = v1;
        } else if constexpr (EPI == kEpiResidual) {
            a.out[(size_t)m * a.N + n] = __hadd(a.resid[(size_t)m * a.N + n], v0);
            a.out[(size_t)m * a.N + n + 1] = __hadd(a.resid[(size_t)m * a.N + n + 1], v1);
        } else {
            const __half act = (EPI == kEpiGluSilu) ? ref_silu(v0) : ref_gelu(v0);
            a.out[(size_t)m * (a.N / 2) + n / 2] = __hmul(act, v1);
        }
    }
}

template <int EPI>
int launch_tc(const TcArgs& t, cudaStream_t st) {
    const size_t sm = (size_t)kStages * kStage + 1024;
    static bool attr = false;
    if (!attr) {
        if (cudaFuncSetAttribute(qgemm_tc_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm) !=
            cudaSuccess)
            return -1;
        attr = true;
    }
    const dim3 grid((unsigned)(t.N / kTBN), (unsigned)((t.M + kTM - 1) / kTM));
    launch_k(qgemm_tc_kernel<EPI>, grid, dim3(kTThreads), sm, st, t);
    return 0;
}
}  // namespace

bool gemm_tc_ok(int M, int K, int N, int G, int int4) {
    return !int4 && M >= 64 && N % kTBN == 0 && K % kKC == 0 && (G == 32 || G == 64 || G == 128) && K % G == 0;
}

int launch_gemm_tc(const int8_t* aq, const float* as, const int8_t* w, const __half* ws, __half* out,
                   const __half* resid, int M, int K, int N, int G, int epi, cudaStream_t st) {
    unsigned* err = dev_error_ptr();
    if (!err) return -1;
    TcArgs t = {aq, as, w, ws, out, resid, err, M, K, N, G};
    switch (epi) {
        case kEpiStore: return launch_tc<kEpiStore>(t, st);
        case kEpiResidual: return launch_tc<kEpiResidual>(t, st);
        case kEpiGluSilu: return launch_tc<kEpiGluSilu>(t, st);
        case kEpiGluGelu: return launch_tc<kEpiGluGelu>(t, st);
    }
    return -1;
}

}  // namespace cb
