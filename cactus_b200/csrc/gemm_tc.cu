// Grouped INT8 / INT4 GEMM for prefill and batched rows on the 5th-generation tensor cores:
// TMA-fed tcgen05.mma.kind::i8 with TMEM accumulators, warp-specialised.
//
// Result bits are those of qgemm_kernel / qgemv_kernel and of cactus_matmul_int8 / _int4
// (kernel_gemm.cpp:128-529): C[m,n] = fp16(chain_g(fma(float(gsum[m,n,g]), Bs[n,g], acc)) * As[m]).
// The reference needs the exact int32 sum of every quantisation group before it enters the
// fp32 chain, so every group gets its own TMEM accumulator: the MMAs of group g (one K = 32
// step for G = 32, two for 64, four for 128, accumulating) write a 128 x 128 int32 tile into
// one of four TMEM buffers, and the epilogue warps read the groups back in order and continue
// the fp32 chains in registers while the tensor core fills the next buffers.
//
// CTA = 128 activation rows x 128 weight rows, 19 warps:
//   warp 0  producer: 2-D TMA tile loads (cp.async.bulk.tensor, 128-byte swizzle, no
//           multicast) of the A and B K-chunks (128 bytes of K) into a 4-stage ring;
//   warp 1  allocates TMEM (512 columns) and one thread issues the MMAs; tcgen05.commit
//           signals TMEM buffers full and ring stages free;
//   warp 18 loads the chunks' fp16 group scales (several chunks per batch of loads) into a
//           scale ring as fp32;
//   warps 2-17 epilogue: warp w reads TMEM lanes 32 * (w % 4) (its tile rows) and columns
//           32 * ((w - 2) / 4) of each group buffer (tcgen05.ld), continues 32 fp32 chains
//           per thread, then scales by As and writes fp16 (store / residual / GLU).
// INT4 weights ([N, K/2] nibbles, low = even k): the producer loads the packed chunk with a
// 2-D TMA tile and, one chunk behind its loads, unpacks it into the swizzled int8 layout
// before the MMAs (sign-extended nibbles; the group sums are exact).
// Every wait is bounded; a timeout raises the device error and every role leaves in order
// (TMEM freed by its allocator after all warps meet).
// This file is compiled as whole-program device code (build.py WHOLE_PROGRAM).
#include <cuda.h>

#include <cstring>
#include <mutex>

#include "common.cuh"
#include "ops.h"

namespace cb {

namespace {
constexpr int kBM = 128, kBN = 128, kKC = 128;  // tile rows (A), tile columns (B rows), K bytes per chunk
// ring depth: INT8 stages are 32 KB, INT4 stages 40 KB (with the packed chunk)
template <int I4>
constexpr int stages() { return I4 ? 4 : 6; }
constexpr int kTileA = kBM * kKC, kTileB = kBN * kKC;  // 16 KB each
constexpr int kPackB = kBN * kKC / 2;                  // INT4: the packed chunk, 8 KB
// a stage: A tile | B tile (int8, swizzled) | INT4 only: the packed B chunk
template <int I4>
constexpr int stage_bytes() { return I4 ? kTileA + kTileB + 8192 : kTileA + kTileB; }  // 40 / 32 KB
constexpr int kSStages = 8;                             // scale ring (one slot per chunk)
constexpr int kSSlot = 4 * kBN * 4;                     // up to 4 groups x 128 columns, fp32
constexpr int kTBufs = 4;                               // TMEM group buffers of 128 columns
constexpr int kTmemCols = kTBufs * kBN;                 // 512
// 18 warps: sixteen epilogue warps, four per TMEM lane quarter, each owning 32 columns. The
// epilogue is latency-bound (dependent TMEM reads and fp32 chains), so it takes as many warps
// as the register file holds: each SM sub-partition's 16K registers hold five warps at the
// 96 registers a thread the 32-column epilogue needs.
constexpr int kWarps = 19, kThreads = kWarps * 32;  // + producer, MMA issuer, scale loader
constexpr int kEpiWarps = 16;
constexpr int kCPT = kBN / 4;      // columns per epilogue thread
constexpr uint32_t kSpin = 1u << 24;

struct TcArgs {
    const float* as;
    const uint8_t* w4;      // INT4: packed weights [N, K/2]; INT8: null (tensor map B)
    const __half* ws;
    __half* out;
    const __half* resid;
    unsigned* err;  // the library's device error word
    int M, K, N, G;
};

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// smem matrix descriptor, K-major with 128-byte swizzle: 8-row x 128-byte atoms, 1024 bytes
// between 8-row groups (SBO), version 1, layout type 2 (SWIZZLE_128B). Stage bases are
// 1024-byte aligned; a K step of 32 bytes inside the atom advances the start address.
__device__ __forceinline__ uint64_t desc_sw128(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// kind::i8: D = S32, A = B = S8, both K-major; N = kBN, M = kBM
constexpr uint32_t kIdesc =
    (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kBN >> 3) << 17) | ((uint32_t)(kBM >> 4) << 24);

__device__ __forceinline__ void tc_mma(uint32_t dtmem, uint64_t da, uint64_t db, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}\n"
        :
        : "r"(dtmem), "l"(da), "l"(db), "r"(kIdesc), "r"(accumulate));
}
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// 2-D tiled TMA load of box {kKC bytes, 128 rows} at (x = k byte offset, y = row), no multicast
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar,
                                            uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}
__device__ __forceinline__ uint64_t l2_policy_evict_last() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// 64 TMEM columns of the warp's 32 lanes set to the integer 0x4B400000 (the store is
// asynchronous: tmem_wait_st before the columns are handed to the tensor core)
__device__ __forceinline__ void tmem_st64_bias(uint32_t taddr) {
    const int b = 0x4B400000;
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x64.b32 [%0], {%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,"
        "%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,"
        "%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1};" ::"r"(taddr),
        "r"(b)
        : "memory");
}
__device__ __forceinline__ void tmem_st32_bias(uint32_t taddr) {
    const int b = 0x4B400000;
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,"
        "%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1};" ::"r"(taddr),
        "r"(b)
        : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Two lanes of the fp32 group chain: run = fma(float(gsum), scale, run) for a pair of columns,
// with one f32x2 subtract and one f32x2 fused multiply-add (each lane rounded as the scalar
// instruction). The TMEM accumulators start at the integer 0x4B400000, so an accumulated
// group sum x (|x| < 2^22) reads back as the float 12582912 + x exactly and one subtraction
// of 12582912 gives float(x) exactly.
__device__ __forceinline__ void chain2(unsigned long long& run, int v0, int v1, unsigned long long s2,
                                       unsigned long long bias2) {
    asm("{\n\t.reg .b64 f;\n\t"
        "mov.b64 f, {%1, %2};\n\t"
        "sub.rn.f32x2 f, f, %4;\n\t"
        "fma.rn.f32x2 %0, f, %3, %0;\n\t}"
        : "+l"(run)
        : "r"(v0), "r"(v1), "l"(s2), "l"(bias2));
}

// one warp: 32 consecutive TMEM columns of its 32 lanes; load and wait in one statement (a
// separate wait would let the compiler schedule uses of the registers ahead of it)
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, int (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
          "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
          "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
        : "r"(taddr)
        : "memory");
}

__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, unsigned parity, volatile int* abort) {
    for (uint32_t i = 0; i < kSpin; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 255) == 255 && *abort) return false;
    }
    *abort = 1;
    return false;
}

// INT4: nibbles of the packed chunk (row-major [128][64] bytes, low nibble = even k) become
// sign-extended int8 in the swizzled K-major B tile. One 16-byte output chunk (16 k) comes
// from 8 packed bytes; lane l converts chunks l, l + 32, ... of the 1024.
__device__ __forceinline__ void unpack_chunk_int4(const uint8_t* packed, uint8_t* btile, int lane) {
#pragma unroll 4
    for (int i = 0; i < 32; ++i) {
        const int idx = lane + 32 * i, r = idx >> 3, j = idx & 7;
        const uint2 p = *reinterpret_cast<const uint2*>(packed + r * 64 + j * 8);
        uint4 o;
        const unsigned lo0 = __vsub4((p.x & 0x0F0F0F0Fu) ^ 0x08080808u, 0x08080808u);
        const unsigned hi0 = __vsub4(((p.x >> 4) & 0x0F0F0F0Fu) ^ 0x08080808u, 0x08080808u);
        const unsigned lo1 = __vsub4((p.y & 0x0F0F0F0Fu) ^ 0x08080808u, 0x08080808u);
        const unsigned hi1 = __vsub4(((p.y >> 4) & 0x0F0F0F0Fu) ^ 0x08080808u, 0x08080808u);
        o.x = __byte_perm(lo0, hi0, 0x5140);
        o.y = __byte_perm(lo0, hi0, 0x7362);
        o.z = __byte_perm(lo1, hi1, 0x5140);
        o.w = __byte_perm(lo1, hi1, 0x7362);
        *reinterpret_cast<uint4*>(btile + r * 128 + ((j ^ (r & 7)) << 4)) = o;
    }
}

template <int EPI, int I4>
__global__ void __launch_bounds__(kThreads, 1)
    qgemm_tc_kernel(const __grid_constant__ CUtensorMap mapA, const __grid_constant__ CUtensorMap mapB, TcArgs a) {
    pdl_launch_dependents();
    // Stage bases must be 1024-byte aligned for the swizzle atoms; the declared alignment of
    // dynamic shared memory is not relied on (1 KB of slack is launched).
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* const smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    constexpr int kStage = stage_bytes<I4>();
    constexpr int kStages = stages<I4>();
    float* const sscale = reinterpret_cast<float*>(smem + kStages * kStage);
    __shared__ uint64_t full[kStages], empty[kStages], cfull[kStages], sfull[kSStages], sempty[kSStages],
        tfull[kTBufs], tempty[kTBufs], drain;
    __shared__ uint32_t tmem_base_s;
    __shared__ int s_abort;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = blockIdx.y * kBM, n0 = blockIdx.x * kBN;
    const int G = a.G, nchunks = a.K / kKC, gpc = kKC / G, spg = G / 32, ngroups = a.K / G;

    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base_s)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (threadIdx.x == 0) {
        s_abort = 0;
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
            mbar_init(&cfull[s], 1);
        }
        for (int s = 0; s < kSStages; ++s) {
            mbar_init(&sfull[s], 32);
            mbar_init(&sempty[s], kEpiWarps);
        }
        for (int b = 0; b < kTBufs; ++b) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], kEpiWarps);
        }
        mbar_init(&drain, 1);
        fence_mbar_init();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base_s;
    volatile int* const abort = &s_abort;
    pdl_wait();  // A (and the residual) come from the previous kernel

    if (warp == 0) {
        // ---------------------------------------------------------------- producer
        const uint64_t pol_a = l2_policy_evict_last(), pol_b = l2_policy_evict_first();
        int issued = 0;
        // INT4: the chunk loaded one iteration earlier is unpacked after the next one is issued
        auto convert = [&](int c) -> bool {
            const int s = c % kStages;
            if (!wait_or_abort(&full[s], (c / kStages) & 1, abort)) return false;
            uint8_t* st = smem + s * kStage;
            unpack_chunk_int4(st + kTileA + kTileB, st + kTileA, lane);
            fence_proxy_async_smem();  // generic-proxy stores -> visible to the tensor core
            __syncwarp();
            if (lane == 0) mbar_arrive(&cfull[s]);
            return true;
        };
        for (int c = 0; c < nchunks; ++c) {
            const int s = c % kStages;
            if (c >= kStages && !wait_or_abort(&empty[s], ((c / kStages) - 1) & 1, abort)) break;
            if (lane == 0) {
                uint8_t* st = smem + s * kStage;
                if (I4) {
                    mbar_arrive_expect_tx(&full[s], (unsigned)(kTileA + kPackB));
                    tma_load_2d(st, &mapA, c * kKC, m0, &full[s], pol_a);
                    tma_load_2d(st + kTileA + kTileB, &mapB, c * (kKC / 2), n0, &full[s], pol_b);
                } else {
                    mbar_arrive_expect_tx(&full[s], (unsigned)kStage);
                    tma_load_2d(st, &mapA, c * kKC, m0, &full[s], pol_a);
                    tma_load_2d(st + kTileA, &mapB, c * kKC, n0, &full[s], pol_b);
                }
            }
            ++issued;
            if (I4 && c >= 1 && !convert(c - 1)) break;
        }
        if (I4 && !*abort && issued == nchunks) convert(nchunks - 1);
        // no copy may land after the block leaves: wait (bounded) for the last ones issued
        if (*abort && lane == 0)
            for (int c = issued > kStages ? issued - kStages : 0; c < issued; ++c)
                mbar_wait_bounded(&full[c % kStages], (c / kStages) & 1);
    } else if (warp == 1) {
        // ---------------------------------------------------------------- MMA issuer
        if (lane == 0) {
            for (int c = 0; c < nchunks; ++c) {
                const int s = c % kStages;
                if (!wait_or_abort(I4 ? &cfull[s] : &full[s], (c / kStages) & 1, abort)) break;
                tc_fence_after();
                const uint32_t base = smem_u32(smem + s * kStage);
                bool ok = true;
                for (int ks = 0; ks < kKC / 32 && ok; ++ks) {
                    const int kg = c * (kKC / 32) + ks, grp = kg / spg, b = grp % kTBufs;
                    const bool first = (kg % spg) == 0, last = (kg % spg) == spg - 1;
                    if (first) {  // the epilogue has re-armed this buffer with the bias
                        ok = wait_or_abort(&tempty[b], (grp / kTBufs) & 1, abort);
                        if (!ok) break;
                        tc_fence_after();
                    }
                    tc_mma(tmem + (uint32_t)(b * kBN), desc_sw128(base + ks * 32), desc_sw128(base + kTileA + ks * 32),
                           1u);
                    if (last) tc_commit(&tfull[b]);
                }
                tc_commit(&empty[s]);
                if (!ok) break;
            }
            // every MMA issued has completed before TMEM is released
            tc_commit(&drain);
            mbar_wait_bounded(&drain, 0);
        }
        __syncwarp();
    } else if (warp == kWarps - 1) {
        // ---------------------------------------------------------------- group scales
        // fp16 scales of the tile's rows (lane + 32 i) for kSB chunks at a time: all loads in
        // flight together (4 / 2 / 1 consecutive scales per row and chunk for G = 32 / 64 / 128,
        // one aligned 8 / 4 / 2-byte load; rows are ngroups * 2 bytes apart, a multiple of 8
        // since K % 128 == 0, and the launcher checks the base), then converted to fp32 into
        // the scale ring as [group][column]
        constexpr int kSB = kSStages / 2;
        bool ok = true;
        for (int c0 = 0; c0 < nchunks && ok; c0 += kSB) {
            uint2 sreg[kSB][4];
#pragma unroll
            for (int j = 0; j < kSB; ++j) {
                if (c0 + j < nchunks) {
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const __half* src = a.ws + (size_t)(n0 + lane + 32 * i) * ngroups + (c0 + j) * gpc;
                        if (gpc == 4) sreg[j][i] = __ldg(reinterpret_cast<const uint2*>(src));
                        else if (gpc == 2) sreg[j][i].x = __ldg(reinterpret_cast<const unsigned*>(src));
                        else sreg[j][i].x = __ldg(reinterpret_cast<const unsigned short*>(src));
                    }
                }
            }
#pragma unroll
            for (int j = 0; j < kSB; ++j) {
                const int c = c0 + j, ss = c % kSStages;
                if (c >= nchunks) break;
                if (c >= kSStages && !wait_or_abort(&sempty[ss], ((c / kSStages) - 1) & 1, abort)) {
                    ok = false;
                    break;
                }
                float* sl = sscale + ss * (kSSlot / 4);
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const __half2 lo = *reinterpret_cast<const __half2*>(&sreg[j][i].x);
                    const __half2 hi = *reinterpret_cast<const __half2*>(&sreg[j][i].y);
                    float* d = sl + lane + 32 * i;
                    d[0] = __low2float(lo);
                    if (gpc > 1) d[kBN] = __high2float(lo);
                    if (gpc > 2) {
                        d[2 * kBN] = __low2float(hi);
                        d[3 * kBN] = __high2float(hi);
                    }
                }
                mbar_arrive(&sfull[ss]);
            }
        }
    } else {
        // ---------------------------------------------------------------- epilogue
        const int q = warp & 3, h = (warp - 2) >> 2;  // TMEM lane quarter (warp id % 4), column block
        const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(h * kCPT);
        // arm every group buffer with the bias (completion 0 of tempty)
        for (int b = 0; b < kTBufs; ++b)
            for (int c32 = 0; c32 < kCPT / 32; ++c32) tmem_st32_bias(taddr + (uint32_t)(b * kBN + c32 * 32));
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0)
            for (int b = 0; b < kTBufs; ++b) mbar_arrive(&tempty[b]);
        const float bias = 12582912.0f;
        const unsigned long long bias2 =
            ((unsigned long long)__float_as_uint(bias) << 32) | (unsigned long long)__float_as_uint(bias);
        unsigned long long run[kCPT / 2];
#pragma unroll
        for (int j = 0; j < kCPT / 2; ++j) run[j] = 0ull;  // two fp32 zeros
        bool ok = true;
#pragma unroll 1
        for (int grp = 0; grp < ngroups && ok; ++grp) {
            const int b = grp % kTBufs, c = grp / gpc, gi = grp % gpc, ss = c % kSStages;
            if (gi == 0) ok = wait_or_abort(&sfull[ss], (c / kSStages) & 1, abort);
            if (ok) ok = wait_or_abort(&tfull[b], (grp / kTBufs) & 1, abort);
            if (!ok) break;
            tc_fence_after();
            const ulonglong2* sc = reinterpret_cast<const ulonglong2*>(sscale + ss * (kSSlot / 4) + gi * kBN + h * kCPT);
#pragma unroll
            for (int half = 0; half < kCPT / 32; ++half) {
                int v[32];
                tmem_ld32(taddr + (uint32_t)(b * kBN + half * 32), v);
                if (half == 0 && grp > 0) {  // the previous group's buffer: bias stored, hand it back
                    tmem_wait_st();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&tempty[(grp - 1) % kTBufs]);
                }
#pragma unroll
                for (int j4 = 0; j4 < 8; ++j4) {
                    const ulonglong2 sv = sc[half * 8 + j4];
                    chain2(run[half * 16 + 2 * j4], v[4 * j4], v[4 * j4 + 1], sv.x, bias2);
                    chain2(run[half * 16 + 2 * j4 + 1], v[4 * j4 + 2], v[4 * j4 + 3], sv.y, bias2);
                }
            }
            // re-arm this buffer for group grp + kTBufs; the store completes while the next group
            // is read, and the buffer is handed back after that (the previous group's below)
            if (grp + kTBufs < ngroups) {
#pragma unroll
                for (int c32 = 0; c32 < kCPT / 32; ++c32) tmem_st32_bias(taddr + (uint32_t)(b * kBN + c32 * 32));
            }
            if (gi == gpc - 1) {
                __syncwarp();
                if (lane == 0) mbar_arrive(&sempty[ss]);
            }
        }
        const int m = m0 + q * 32 + lane;
        // column j of this thread's kCPT: lane (j & 1) of the pair run[j >> 1]
        auto col = [&](int j) -> float {
            return __uint_as_float((j & 1) ? (unsigned)(run[j >> 1] >> 32) : (unsigned)(run[j >> 1] & 0xFFFFFFFFull));
        };
        if (ok && !*abort && m < a.M) {
            const float asm_ = a.as[m];
            const int nb = n0 + h * kCPT;
            if constexpr (EPI == kEpiGluSilu || EPI == kEpiGluGelu) {
                int4* o4 = reinterpret_cast<int4*>(a.out + (size_t)m * (a.N / 2) + nb / 2);
#pragma unroll
                for (int j8 = 0; j8 < kCPT / 16; ++j8) {
                    int4 ov;
                    __half* oh = reinterpret_cast<__half*>(&ov);
#pragma unroll
                    for (int t = 0; t < 8; ++t) {
                        const int j = j8 * 16 + 2 * t;
                        const __half g0 = f2h(__fmul_rn(col(j), asm_)), u1 = f2h(__fmul_rn(col(j + 1), asm_));
                        const __half act = (EPI == kEpiGluSilu) ? ref_silu(g0) : ref_gelu(g0);
                        oh[t] = __hmul(act, u1);
                    }
                    o4[j8] = ov;
                }
            } else {
                int4* o4 = reinterpret_cast<int4*>(a.out + (size_t)m * a.N + nb);
                const int4* r4 = reinterpret_cast<const int4*>(a.resid + (size_t)m * a.N + nb);
#pragma unroll
                for (int j8 = 0; j8 < kCPT / 8; ++j8) {
                    int4 ov;
                    __half* oh = reinterpret_cast<__half*>(&ov);
                    if constexpr (EPI == kEpiResidual) {
                        const int4 rv = r4[j8];
                        const __half* rh = reinterpret_cast<const __half*>(&rv);
#pragma unroll
                        for (int t = 0; t < 8; ++t) oh[t] = __hadd(rh[t], f2h(__fmul_rn(col(j8 * 8 + t), asm_)));
                    } else {
#pragma unroll
                        for (int t = 0; t < 8; ++t) oh[t] = f2h(__fmul_rn(col(j8 * 8 + t), asm_));
                    }
                    o4[j8] = ov;
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (threadIdx.x == 0 && *abort) atomicCAS(a.err, 0u, (unsigned)kDevTmaTimeout);
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
    }
}

// ---------------------------------------------------------------- host side
using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// cuTensorMapEncodeTiled through the runtime's driver entry points (the library does not link libcuda)
EncodeTiled encode_fn() {
    static EncodeTiled fn = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess) {
            cudaGetLastError();
            return static_cast<EncodeTiled>(nullptr);
        }
        return reinterpret_cast<EncodeTiled>(p);
    }();
    return fn;
}

// [rows, kbytes] bytes row-major, box {box_inner bytes, 128 rows}; rows past the end read as
// zeros. The base must be 16-byte aligned and kbytes a multiple of 16.
bool make_map(CUtensorMap* m, const void* base, int rows, int kbytes, int box_inner, bool swizzle) {
    const EncodeTiled fn = encode_fn();
    if (!fn || (reinterpret_cast<uintptr_t>(base) & 15u) || (kbytes % 16)) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)kbytes, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)kbytes};
    const cuuint32_t box[2] = {(cuuint32_t)box_inner, 128u};
    const cuuint32_t estr[2] = {1u, 1u};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int I4>
constexpr size_t smem_bytes() { return (size_t)stages<I4>() * stage_bytes<I4>() + (size_t)kSStages * kSSlot + 1024; }

template <int EPI, int I4>
int launch_tc(const CUtensorMap& ma, const CUtensorMap& mb, const TcArgs& t, cudaStream_t st) {
    static bool attr = false;
    if (!attr) {
        if (cudaFuncSetAttribute(qgemm_tc_kernel<EPI, I4>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)smem_bytes<I4>()) != cudaSuccess)
            return -1;
        attr = true;
    }
    const dim3 grid((unsigned)(t.N / kBN), (unsigned)((t.M + kBM - 1) / kBM));
    return launch_k(qgemm_tc_kernel<EPI, I4>, grid, dim3(kThreads), smem_bytes<I4>(), st, ma, mb, t) == cudaSuccess
               ? 0
               : -1;
}

template <int I4>
int launch_epi(const CUtensorMap& ma, const CUtensorMap& mb, const TcArgs& t, int epi, cudaStream_t st) {
    switch (epi) {
        case kEpiStore: return launch_tc<kEpiStore, I4>(ma, mb, t, st);
        case kEpiResidual: return launch_tc<kEpiResidual, I4>(ma, mb, t, st);
        case kEpiGluSilu: return launch_tc<kEpiGluSilu, I4>(ma, mb, t, st);
        case kEpiGluGelu: return launch_tc<kEpiGluGelu, I4>(ma, mb, t, st);
    }
    return -1;
}
}  // namespace

// Shapes the kernel takes, and only when they fill the GPU with at least one wave of 128 x 128
// tiles: below that the mma.sync GEMM, with four times as many (smaller) tiles, is faster
// (measured on B200: M = 256, K = 1024, N = 3072 runs 27 us here against 21 us there).
bool gemm_tc_ok(int M, int K, int N, int G, int int4, bool any_size) {
    (void)int4;
    const long long tiles = (long long)((M + kBM - 1) / kBM) * (N / kBN);
    return M >= 1 && N % kBN == 0 && K % kKC == 0 && (G == 32 || G == 64 || G == 128) && K % G == 0 &&
           (any_size || tiles >= kNumSMs) && encode_fn() != nullptr;
}

int launch_gemm_tc(const int8_t* aq, const float* as, const void* w, const __half* ws, __half* out,
                   const __half* resid, int M, int K, int N, int G, int int4, int epi, cudaStream_t st) {
    unsigned* err = dev_error_ptr();
    if (!err) return -1;
    CUtensorMap ma, mb;
    if (reinterpret_cast<uintptr_t>(ws) & (uintptr_t)(kKC / G * 2 - 1)) return -2;  // scale loads need alignment
    if (!make_map(&ma, aq, M, K, kKC, true)) return -2;  // not TMA-able: the caller falls back
    if (!(int4 ? make_map(&mb, w, N, K / 2, kKC / 2, false) : make_map(&mb, w, N, K, kKC, true))) return -2;
    TcArgs t = {as, nullptr, ws, out, resid, err, M, K, N, G};
    return int4 ? launch_epi<1>(ma, mb, t, epi, st) : launch_epi<0>(ma, mb, t, epi, st);
}

}  // namespace cb
