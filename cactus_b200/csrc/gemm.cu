// Grouped INT8 / INT4 GEMM for M >= 16 rows (prefill) on the tensor cores, exact.
//
// Same result bits as cactus_matmul_int8 / cactus_matmul_int4 (kernel_gemm.cpp:128-529) and
// as qgemv_kernel: every output is
//   C[m,n] = fp16( chain_g( fma(float(gsum[m,n,g]), float(Bs[n,g]), acc) ) * As[m] )
// with the group sums exact in int32 and the fp32 chain over the groups in ascending g. A
// group of G = 32·s values is s mma.sync m16n8k32 (s8·s8 -> s32) steps accumulated in int32
// (|sum| <= 128·128·G < 2^24, so float(sum) is exact too); after each group the int32
// fragment is folded into the fp32 accumulators in group order.
//
// Tiles: a CTA (4 warps) owns 64 rows x 32 columns; warp w owns rows 16w..16w+15 as four
// n8 fragments. K advances in chunks of GPC groups (GPC = 4 or 2) staged with cp.async into a
// two-stage ring: the int8 activation rows, the weight rows (INT4 stays packed and is
// expanded to int8 when the B fragment is built: low nibble = even k) and the chunk's fp16
// group scales. Epilogues: store, residual add (fp16), SiLU / GELU gate x up on interleaved
// gate/up columns.
#include <cstdlib>
#include <string>

#include "attention_core.cuh"
#include "common.cuh"
#include "ops.h"

namespace cb {

namespace {
constexpr int kBM = 64, kBN = 32, kThreads = 128;

struct GemmArgs {
    const int8_t* aq;
    const float* as;
    const void* w;
    const __half* ws;
    __half* out;
    const __half* resid;
    int M, K, N, G, gpc;
};

__device__ __forceinline__ void cp_async16_zfill(void* smem, const void* gmem, unsigned src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem)), "l"(gmem), "r"(src_bytes)
                 : "memory");
}
__device__ __forceinline__ void cp_async8(void* smem, const void* gmem) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_u32(smem)), "l"(gmem) : "memory");
}

__device__ __forceinline__ void mma_s8(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                       uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// two packed bytes (k, k+1 | k+2, k+3 in low/high nibbles) -> four sign-extended int8
__device__ __forceinline__ uint32_t expand_nibbles(uint32_t x16) {
    const uint32_t v = (x16 & 0x000Fu) | ((x16 & 0x00F0u) << 4) | ((x16 & 0x0F00u) << 8) | ((x16 & 0xF000u) << 12);
    return __vsub4(v ^ 0x08080808u, 0x08080808u);
}

__device__ __forceinline__ uint32_t lds32(const uint8_t* p) { return *reinterpret_cast<const uint32_t*>(p); }

template <int EPI, int INT4>
__global__ void __launch_bounds__(kThreads) qgemm_kernel(GemmArgs a) {
    pdl_launch_dependents();
    pdl_wait();
    extern __shared__ __align__(128) uint8_t smem[];
    const int G = a.G, GPC = a.gpc, KC = GPC * G;
    const int AS = KC + 16;
    const int BW = INT4 ? KC / 2 : KC, BSd = BW + 16;
    const int stageA = kBM * AS, stageB = kBN * BSd, stageS = kBN * GPC * 2;
    const int stage = (stageA + stageB + stageS + 127) / 128 * 128;
    const int m0 = blockIdx.y * kBM, n0 = blockIdx.x * kBN;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, gid = lane >> 2, tig = lane & 3;
    const int ng = a.K / G, nchunks = ng / GPC;
    const size_t wrow = INT4 ? (size_t)a.K / 2 : (size_t)a.K;

    auto load = [&](int c, int s) {
        uint8_t* sA = smem + s * stage;
        uint8_t* sB = sA + stageA;
        uint8_t* sS = sB + stageB;
        const int k0 = c * KC;
        const int ap = KC / 16;
        for (int i = tid; i < kBM * ap; i += kThreads) {
            const int r = i / ap, p = i - r * ap, m = m0 + r;
            const int8_t* src = a.aq + (size_t)min(m, a.M - 1) * a.K + k0 + p * 16;
            cp_async16_zfill(sA + r * AS + p * 16, src, m < a.M ? 16u : 0u);
        }
        const int bp = BW / 16;
        for (int i = tid; i < kBN * bp; i += kThreads) {
            const int r = i / bp, p = i - r * bp;
            const uint8_t* src = static_cast<const uint8_t*>(a.w) + (size_t)(n0 + r) * wrow + (INT4 ? k0 / 2 : k0) + p * 16;
            cp_async16(sB + r * BSd + p * 16, src);
        }
        if (tid < kBN) {
            const __half* src = a.ws + (size_t)(n0 + tid) * ng + c * GPC;
            if (GPC == 4) cp_async8(sS + tid * 8, src);
            else cp_async4(sS + tid * 4, src);
        }
        cp_async_commit();
    };

    float acc[4][4];
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[j][e] = 0.0f;

    load(0, 0);
    for (int c = 0; c < nchunks; ++c) {
        if (c + 1 < nchunks) {
            load(c + 1, (c + 1) & 1);
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();
        const uint8_t* sA = smem + (c & 1) * stage;
        const uint8_t* sB = sA + stageA;
        const __half* sS = reinterpret_cast<const __half*>(sB + stageB);
        const uint8_t* pa = sA + (warp * 16 + gid) * AS + tig * 4;
        for (int gi = 0; gi < GPC; ++gi) {
            int ci[4][4];
#pragma unroll
            for (int j = 0; j < 4; ++j)
#pragma unroll
                for (int e = 0; e < 4; ++e) ci[j][e] = 0;
            for (int st = 0; st < G / 32; ++st) {
                const int kk = gi * G + st * 32;
                const uint32_t a0 = lds32(pa + kk), a1 = lds32(pa + 8 * AS + kk);
                const uint32_t a2 = lds32(pa + kk + 16), a3 = lds32(pa + 8 * AS + kk + 16);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const uint8_t* pb = sB + (8 * j + gid) * BSd;
                    uint32_t b0, b1;
                    if (INT4) {
                        b0 = expand_nibbles(*reinterpret_cast<const uint16_t*>(pb + kk / 2 + tig * 2));
                        b1 = expand_nibbles(*reinterpret_cast<const uint16_t*>(pb + kk / 2 + 8 + tig * 2));
                    } else {
                        b0 = lds32(pb + kk + tig * 4);
                        b1 = lds32(pb + kk + 16 + tig * 4);
                    }
                    mma_s8(ci[j], a0, a1, a2, a3, b0, b1);
                }
            }
            // the group's exact sums continue each output's fp32 chain
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int nc = 8 * j + 2 * tig;
                const float s0 = __half2float(sS[nc * GPC + gi]), s1 = __half2float(sS[(nc + 1) * GPC + gi]);
                acc[j][0] = fmaf((float)ci[j][0], s0, acc[j][0]);
                acc[j][1] = fmaf((float)ci[j][1], s1, acc[j][1]);
                acc[j][2] = fmaf((float)ci[j][2], s0, acc[j][2]);
                acc[j][3] = fmaf((float)ci[j][3], s1, acc[j][3]);
            }
        }
        __syncthreads();
    }

    // epilogue: C fragment element e of n8 tile j is row gid + 8*(e>>1), column 8j + 2*tig + (e&1)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int m = m0 + warp * 16 + gid + 8 * h;
        if (m >= a.M) continue;
        const float asm_ = a.as[m];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int n = n0 + 8 * j + 2 * tig;
            const __half v0 = f2h(__fmul_rn(acc[j][2 * h], asm_));
            const __half v1 = f2h(__fmul_rn(acc[j][2 * h + 1], asm_));
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
}

int gemm_gpc(int K, int G) {
    if (G < 32 || G % 32 || K % G) return 0;
    const int ng = K / G;
    return ng % 4 == 0 ? 4 : (ng % 2 == 0 ? 2 : 0);
}

size_t gemm_smem(int G, int gpc, int int4) {
    const int KC = gpc * G, AS = KC + 16, BW = int4 ? KC / 2 : KC;
    const int stage = (kBM * AS + kBN * (BW + 16) + kBN * gpc * 2 + 127) / 128 * 128;
    return (size_t)2 * stage;
}

template <int EPI, int INT4>
int launch_one(const GemmArgs& g, cudaStream_t st) {
    const size_t sm = gemm_smem(g.G, g.gpc, INT4);
    static size_t attr = 0;
    if (sm > 48 * 1024 && sm > attr) {
        if (cudaFuncSetAttribute(qgemm_kernel<EPI, INT4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm) !=
            cudaSuccess)
            return -1;
        attr = sm;
    }
    const dim3 grid((unsigned)(g.N / kBN), (unsigned)((g.M + kBM - 1) / kBM));
    launch_k(qgemm_kernel<EPI, INT4>, grid, dim3(kThreads), sm, st, g);
    return 0;
}
}  // namespace

// The tcgen05 GEMM (gemm_tc.cu: TMA-fed tcgen05.mma, TMEM group accumulators) takes the INT8 /
// INT4 shapes it supports that fill at least one wave of its tiles; CACTUS_B200_GEMM=mma keeps
// this file's mma.sync kernel for every shape, CACTUS_B200_GEMM=tc gives the tcgen05 kernel
// every shape it supports (read once per process).
int gemm_tc_mode() {
    static const int mode = [] {
        const char* e = std::getenv("CACTUS_B200_GEMM");
        if (e && std::string(e) == "mma") return 0;
        if (e && std::string(e) == "tc") return 2;
        return 1;
    }();
    return mode;
}

const char* gemm_check(int M, int K, int N, int G, int int4) {
    if (M < 1 || K < 1 || N < 1) return "empty matrix";
    if (N % kBN) return "N must be a multiple of 32";
    if (!gemm_gpc(K, G)) return "K / G must be even and G a multiple of 32";
    (void)int4;
    return nullptr;
}

bool gemm_tc_ok(int M, int K, int N, int G, int int4, bool any_size);
int launch_gemm_tc(const int8_t* aq, const float* as, const void* w, const __half* ws, __half* out,
                   const __half* resid, int M, int K, int N, int G, int int4, int epi, cudaStream_t st);

int launch_gemm(const int8_t* aq, const float* as, const void* w, const __half* ws, __half* out, const __half* resid,
                int M, int K, int N, int G, int int4, int epi, cudaStream_t st) {
    if (gemm_check(M, K, N, G, int4)) return -1;
    const int mode = gemm_tc_mode();
    if (mode != 0 && gemm_tc_ok(M, K, N, G, int4, mode == 2)) {
        const int rc = launch_gemm_tc(aq, as, w, ws, out, resid, M, K, N, G, int4, epi, st);
        if (rc != -2) return rc;  // -2: operands not addressable by a tensor map; mma.sync below
    }
    GemmArgs g = {aq, as, w, ws, out, resid, M, K, N, G, gemm_gpc(K, G)};
    switch (epi * 2 + (int4 ? 1 : 0)) {
        case kEpiStore * 2: return launch_one<kEpiStore, 0>(g, st);
        case kEpiStore * 2 + 1: return launch_one<kEpiStore, 1>(g, st);
        case kEpiResidual * 2: return launch_one<kEpiResidual, 0>(g, st);
        case kEpiResidual * 2 + 1: return launch_one<kEpiResidual, 1>(g, st);
        case kEpiGluSilu * 2: return launch_one<kEpiGluSilu, 0>(g, st);
        case kEpiGluSilu * 2 + 1: return launch_one<kEpiGluSilu, 1>(g, st);
        case kEpiGluGelu * 2: return launch_one<kEpiGluGelu, 0>(g, st);
        case kEpiGluGelu * 2 + 1: return launch_one<kEpiGluGelu, 1>(g, st);
    }
    return -1;
}

}  // namespace cb
