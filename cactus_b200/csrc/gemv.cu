// Host side of the grouped INT8/INT4 GEMV: shape checks, tile/stage selection and the
// launch (optionally with programmatic dependent launch). The kernel is in gemv.cuh.
#include <cuda.h>

#include <cstdlib>
#include <map>
#include <mutex>
#include <string>
#include <tuple>

#include "gemv.cuh"
#include "gemv_lanes.cuh"
#include "ops.h"

namespace cb {

namespace {

using KernelFn = void (*)(GemvArgs);
using KernelLanesFn = void (*)(const CUtensorMap, GemvArgs, int, int, int);

// GEMV kernel choice, read once per process. By default (1) the lane-per-row kernel
// (gemv_lanes.cuh) takes the wide shapes it supports and the TMA tile kernel (gemv.cuh) the
// rest (lanes_by_default); CACTUS_B200_GEMV=lanes (3) gives every supported shape to the lane kernel,
// CACTUS_B200_GEMV=tile (0) every shape to the tile kernel, CACTUS_B200_GEMV=rows (2) selects
// the row-streaming kernel where its group-size condition holds.
int gemv_mode() {
    static const int mode = [] {
        const char* e = std::getenv("CACTUS_B200_GEMV");
        if (e && std::string(e) == "rows") return 2;
        if (e && std::string(e) == "tile") return 0;
        if (e && std::string(e) == "lanes") return 3;
        return 1;
    }();
    return mode;
}
// The lane kernel gives each 32-row block to one warp, so narrow outputs leave most SMs idle;
// measured on B200 (M = 1 and 4, INT8 and INT4), it wins from 16384 rows at G = 32 and from
// 6144 rows at G = 128 (where the tile kernel's chain step costs more), and loses below.
bool lanes_by_default(int N, int G) {
    const int nrb = (N + 31) / 32;
    return nrb >= 512 || (G >= 128 && nrb >= 192);
}
bool gemv_rows_enabled() { return gemv_mode() == 2; }

template <int WF, int MT, int RPW, int PRO, int EPI>
KernelFn fn() {
    return &qgemv_kernel<WF, MT, RPW, PRO, EPI>;
}

// (pro, epi) combinations used by the op API and the models
constexpr int kCombos[][2] = {
    {kProPreq, kEpiStore},         {kProQuant, kEpiStore},          {kProQuant, kEpiResidual},
    {kProRmsNormQuant, kEpiStore}, {kProRmsNormQuant, kEpiGluSilu}, {kProRmsNormQuant, kEpiGluGelu},
};
constexpr int kNumCombos = sizeof(kCombos) / sizeof(kCombos[0]);

int combo_index(int pro, int epi) {
    for (int i = 0; i < kNumCombos; ++i)
        if (kCombos[i][0] == pro && kCombos[i][1] == epi) return i;
    return -1;
}

template <int WF, int MT, int RPW>
KernelFn pick_combo(int ci) {
    switch (ci) {
        case 0: return fn<WF, MT, RPW, kProPreq, kEpiStore>();
        case 1: return fn<WF, MT, RPW, kProQuant, kEpiStore>();
        case 2: return fn<WF, MT, RPW, kProQuant, kEpiResidual>();
        case 3: return fn<WF, MT, RPW, kProRmsNormQuant, kEpiStore>();
        case 4: return fn<WF, MT, RPW, kProRmsNormQuant, kEpiGluSilu>();
        case 5: return fn<WF, MT, RPW, kProRmsNormQuant, kEpiGluGelu>();
    }
    return nullptr;
}
template <int WF, int MT>
KernelFn pick_rpw(int rpw, int ci) {
    return rpw == 4 ? pick_combo<WF, MT, 4>(ci) : rpw == 2 ? pick_combo<WF, MT, 2>(ci) : pick_combo<WF, MT, 1>(ci);
}
template <int WF>
KernelFn pick_mt(int mt, int rpw, int ci) {
    switch (mt) {
        case 1: return pick_rpw<WF, 1>(rpw, ci);
        case 2: return pick_rpw<WF, 2>(rpw, ci);
        case 4: return pick_rpw<WF, 4>(rpw, ci);
        default: return pick_rpw<WF, 8>(rpw, ci);
    }
}

template <int WF, int MT>
KernelFn pick_rows_combo(int ci) {
    switch (ci) {
        case 0: return &qgemv_rows_kernel<WF, MT, kProPreq, kEpiStore>;
        case 1: return &qgemv_rows_kernel<WF, MT, kProQuant, kEpiStore>;
        case 2: return &qgemv_rows_kernel<WF, MT, kProQuant, kEpiResidual>;
        case 3: return &qgemv_rows_kernel<WF, MT, kProRmsNormQuant, kEpiStore>;
        case 4: return &qgemv_rows_kernel<WF, MT, kProRmsNormQuant, kEpiGluSilu>;
        case 5: return &qgemv_rows_kernel<WF, MT, kProRmsNormQuant, kEpiGluGelu>;
    }
    return nullptr;
}
template <int WF>
KernelFn pick_rows(int mt, int ci) {
    switch (mt) {
        case 1: return pick_rows_combo<WF, 1>(ci);
        case 2: return pick_rows_combo<WF, 2>(ci);
        case 4: return pick_rows_combo<WF, 4>(ci);
        default: return pick_rows_combo<WF, 8>(ci);
    }
}

template <int WF, int MT, int GT>
KernelLanesFn pick_lanes_combo(int ci) {
    switch (ci) {
        case 0: return &qgemv_lanes_kernel<WF, MT, GT, kProPreq, kEpiStore>;
        case 1: return &qgemv_lanes_kernel<WF, MT, GT, kProQuant, kEpiStore>;
        case 2: return &qgemv_lanes_kernel<WF, MT, GT, kProQuant, kEpiResidual>;
        case 3: return &qgemv_lanes_kernel<WF, MT, GT, kProRmsNormQuant, kEpiStore>;
        case 4: return &qgemv_lanes_kernel<WF, MT, GT, kProRmsNormQuant, kEpiGluSilu>;
        case 5: return &qgemv_lanes_kernel<WF, MT, GT, kProRmsNormQuant, kEpiGluGelu>;
    }
    return nullptr;
}
template <int WF, int GT>
KernelLanesFn pick_lanes_mt(int mt, int ci) {
    switch (mt) {
        case 1: return pick_lanes_combo<WF, 1, GT>(ci);
        case 2: return pick_lanes_combo<WF, 2, GT>(ci);
        default: return pick_lanes_combo<WF, 4, GT>(ci);
    }
}
// group sizes 32 and 128 (the others take the tile kernel)
template <int WF>
KernelLanesFn pick_lanes(int mt, int G, int ci) {
    return G == 32 ? pick_lanes_mt<WF, 32>(mt, ci) : G == 128 ? pick_lanes_mt<WF, 128>(mt, ci) : nullptr;
}

std::mutex g_attr_mu;
bool g_lanes_attr[2][5][2][kNumCombos] = {};
bool g_attr_set[2][9][5][kNumCombos] = {};
// row-streaming variants: shared-memory attribute set, resident blocks per SM (0: unknown)
bool g_rows_attr[2][9][kNumCombos] = {};
int g_rows_per_sm[2][9][kNumCombos] = {};

}  // namespace

constexpr int kSmemLimit = 227 * 1024;

int gemv_rows_per_launch(int int4, int pro, int K, int G) {
    for (int mt = 8; mt >= 1; mt >>= 1)
        if (gemv_layout(int4, mt, 1, 2, pro, K, G).total <= kSmemLimit) return mt;
    return 0;
}

static int mt_of(int M) { return M <= 1 ? 1 : M <= 2 ? 2 : M <= 4 ? 4 : 8; }

const char* gemv_check(const GemvCall& c) {
    if (c.M < 1 || c.M > 8) return "gemv: M must be in [1, 8]";
    if (c.N < 1 || c.K < 1 || c.G < 1) return "gemv: empty shape";
    if (c.K % c.G) return "gemv: K must be a multiple of group_size";
    if (!c.int4 && (c.G % 16 || c.G > 512)) return "gemv: INT8 group_size must be a multiple of 16 and <= 512";
    if (c.int4 && (c.G % 32 || c.G > 1024)) return "gemv: INT4 group_size must be a multiple of 32 and <= 1024";
    if ((reinterpret_cast<uintptr_t>(c.w) & 15) || (reinterpret_cast<uintptr_t>(c.ws) & 15))
        return "gemv: weights and scales must be 16-byte aligned";
    if ((c.epi == kEpiGluSilu || c.epi == kEpiGluGelu) && (c.N & 1)) return "gemv: GLU epilogue needs even N";
    if (combo_index(c.pro, c.epi) < 0) return "gemv: unsupported prologue/epilogue combination";
    const GemvLayout L = gemv_layout(c.int4, mt_of(c.M), 1, 2, c.pro, c.K, c.G);
    if (L.total > kSmemLimit) return "gemv: K too large for the shared-memory tile";
    return nullptr;
}

// Raises the dynamic shared-memory limit of every GEMV variant once, outside any stream
// capture (cudaFuncSetAttribute is not a stream operation).
void gemv_prepare() {
    std::lock_guard<std::mutex> lk(g_attr_mu);
    for (int wf = 0; wf < 2; ++wf)
        for (int mt : {1, 2, 4, 8})
            for (int rpw : {1, 2, 4})
                for (int ci = 0; ci < kNumCombos; ++ci) {
                    bool& done = g_attr_set[wf][mt][rpw][ci];
                    if (done) continue;
                    KernelFn f = wf ? pick_mt<1>(mt, rpw, ci) : pick_mt<0>(mt, rpw, ci);
                    if (f && cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024) ==
                                 cudaSuccess)
                        done = true;
                }
    for (int wf = 0; wf < 2; ++wf)
        for (int mt : {1, 2, 4})
            for (int gi = 0; gi < 2; ++gi)
            for (int ci = 0; ci < kNumCombos; ++ci) {
                bool& done = g_lanes_attr[wf][mt][gi][ci];
                if (done) continue;
                const int G = gi ? 128 : 32;
                KernelLanesFn f = wf ? pick_lanes<1>(mt, G, ci) : pick_lanes<0>(mt, G, ci);
                if (f && cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit) == cudaSuccess)
                    done = true;
            }
    for (int wf = 0; wf < 2; ++wf)
        for (int mt : {1, 2, 4, 8})
            for (int ci = 0; ci < kNumCombos; ++ci) {
                bool& done = g_rows_attr[wf][mt][ci];
                if (done) continue;
                KernelFn f = wf ? pick_rows<1>(mt, ci) : pick_rows<0>(mt, ci);
                if (f && cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024) == cudaSuccess)
                    done = true;
            }
}

// Row-streaming launch (gemv.cuh: qgemv_rows_kernel); -2 when the shape does not qualify.
static int launch_gemv_rows(const GemvCall& c, int mt, int ci, const GemvArgs& a, cudaStream_t st) {
    if (!gemv_rows_ok(c.int4, c.G)) return -2;
    const GemvRowsLayout L = gemv_rows_layout(c.int4, mt, c.pro, c.epi, c.K, c.G);
    if (L.total > kSmemLimit) return -2;
    KernelFn f = c.int4 ? pick_rows<1>(mt, ci) : pick_rows<0>(mt, ci);
    if (!f) return -2;
    int per_sm = 1;
    {
        std::lock_guard<std::mutex> lk(g_attr_mu);
        if (!g_rows_attr[c.int4][mt][ci]) {
            if (cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024) != cudaSuccess)
                return -1;
            g_rows_attr[c.int4][mt][ci] = true;
        }
        int& cached = g_rows_per_sm[c.int4][mt][ci];
        if (cached == 0) {
            int nb = 0;
            if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, f, kGemvThreads, 48 * 1024) != cudaSuccess)
                nb = 1;
            cached = nb < 1 ? 1 : nb;
        }
        per_sm = cached;
    }
    // resident blocks also limited by this shape's shared memory
    const int by_smem = (228 * 1024) / (L.total + 1024);
    if (by_smem < per_sm) per_sm = by_smem < 1 ? 1 : by_smem;
    const int nrg = (c.N + L.RW - 1) / L.RW;
    int grid = (nrg + kGemvWarps - 1) / kGemvWarps;
    if (grid < kNumSMs) grid = nrg < kNumSMs ? nrg : kNumSMs;  // spread small outputs over the SMs
    if (grid > per_sm * kNumSMs) grid = per_sm * kNumSMs;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kGemvThreads);
    cfg.dynamicSmemBytes = L.total;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = (c.pdl || pdl_flag()) ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, f, a) == cudaSuccess ? 0 : -1;
}

// Tensor map of a weight matrix for the lane-per-row GEMV: [rows, rowbytes] bytes, box of 128
// bytes x 32 rows, 128-byte swizzle (cuTensorMapEncodeTiled through the runtime's driver entry
// points; the library does not link libcuda). Encoded maps are cached per (base, rows, bytes).
static bool lanes_map(CUtensorMap* m, const void* base, int rows, int rowbytes) {
    using Encode = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
    static Encode fn = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess) {
            cudaGetLastError();
            return static_cast<Encode>(nullptr);
        }
        return reinterpret_cast<Encode>(p);
    }();
    if (!fn || (reinterpret_cast<uintptr_t>(base) & 15u) || (rowbytes % 16)) return false;
    static std::mutex mu;
    static std::map<std::tuple<const void*, int, int>, CUtensorMap> cache;
    std::lock_guard<std::mutex> lk(mu);
    const auto key = std::make_tuple(base, rows, rowbytes);
    auto it = cache.find(key);
    if (it != cache.end()) {
        *m = it->second;
        return true;
    }
    const cuuint64_t dims[2] = {(cuuint64_t)rowbytes, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)rowbytes};
    const cuuint32_t box[2] = {128u, 32u};
    const cuuint32_t estr[2] = {1u, 1u};
    if (fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return false;
    if (cache.size() > 4096) cache.clear();
    cache[key] = *m;
    return true;
}

// Lane-per-row launch (gemv_lanes.cuh); -2 when the shape does not qualify. One block per SM
// (its rings take most of the shared memory), warps with row blocks only, and as many ring
// slots per warp as fit (2 to 16).
static int launch_gemv_lanes(const GemvCall& c, int mt, int ci, const GemvArgs& a, cudaStream_t st) {
    if (mt > 4 || c.K % (c.int4 ? 256 : 128) || !(c.G == 32 || c.G == 128)) return -2;
    CUtensorMap wmap;
    if (!lanes_map(&wmap, c.w, c.N, c.int4 ? c.K / 2 : c.K)) return -2;
    const GemvLanesLayout L = gemv_lanes_layout(c.int4, mt, c.K, c.G);
    const int nrb = (c.N + 31) / 32;
    const int grid = nrb < kNumSMs ? nrb : kNumSMs;
    int wpc = (nrb + grid - 1) / grid;
    if (wpc > kLanesWarps) wpc = kLanesWarps;
    // two chunks per slot where K allows: each row's 256 bytes come in one burst. Measured on
    // the lm-head shape (INT8, G = 32), the ring's shared memory held fixed: 33.4 us with 8 warps
    // and two chunks per slot against 41.0 us with one chunk, 43.4 / 48.3 us with 4 warps and
    // four / two chunks, and 30.5 us with 12 warps and two chunks (more row-owning warps beat
    // deeper slots)
    const int nch = c.K / (c.int4 ? 256 : 128);
    const int nb = nch % 2 ? 1 : 2;
    int S = (kSmemLimit - L.fixed) / (wpc * nb * L.slot);
    if (S > kLaneMaxSlots) S = kLaneMaxSlots;
    if (S < 2) return -2;
    const size_t smem = (size_t)L.fixed + (size_t)wpc * S * nb * L.slot;
    KernelLanesFn f = c.int4 ? pick_lanes<1>(mt, c.G, ci) : pick_lanes<0>(mt, c.G, ci);
    if (!f) return -2;
    {
        std::lock_guard<std::mutex> lk(g_attr_mu);
        bool& done = g_lanes_attr[c.int4][mt][c.G == 128][ci];
        if (!done) {
            if (cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit) != cudaSuccess)
                return -1;
            done = true;
        }
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kLanesThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = (c.pdl || pdl_flag()) ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, f, wmap, a, S, wpc, nb) == cudaSuccess ? 0 : -1;
}

int launch_gemv(const GemvCall& c, cudaStream_t st) {
    const int mt = mt_of(c.M);
    // rows per tile: 8 for narrow outputs (>= 128 tiles at N = 1024), 16 for mid-size, 32 for
    // very wide ones (the vocabulary projection); fewer when two stages would not fit
    int rpw = c.N >= 32 * 2 * kNumSMs ? 4 : (c.N >= 16 * kNumSMs ? 2 : 1);
    while (rpw > 1 && gemv_layout(c.int4, mt, rpw, 2, c.pro, c.K, c.G).total > kSmemLimit) rpw >>= 1;
    const int R = 8 * rpw;
    const int ntiles = (c.N + R - 1) / R;
    int S = 4;
    GemvLayout L = gemv_layout(c.int4, mt, rpw, S, c.pro, c.K, c.G);
    while (S > 2 && L.total > 112 * 1024) {
        --S;
        L = gemv_layout(c.int4, mt, rpw, S, c.pro, c.K, c.G);
    }
    if (L.total > kSmemLimit) return -1;
    const int per_sm = L.total <= 112 * 1024 ? 2 : 1;
    const int grid = ntiles < per_sm * kNumSMs ? ntiles : per_sm * kNumSMs;
    const int ci = combo_index(c.pro, c.epi);
    KernelFn f = c.int4 ? pick_mt<1>(mt, rpw, ci) : pick_mt<0>(mt, rpw, ci);
    if (!f) return -1;
    {
        std::lock_guard<std::mutex> lk(g_attr_mu);
        bool& done = g_attr_set[c.int4][mt][rpw][ci];
        if (!done) {
            if (cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024) != cudaSuccess)
                return -1;
            done = true;
        }
    }
    GemvArgs a;
    a.x = c.x;
    a.norm_w = c.norm_w;
    a.eps = c.eps;
    a.aq = c.aq;
    a.as = c.as;
    a.w = c.w;
    a.ws = c.ws;
    a.out = c.out;
    a.resid = c.resid;
    a.aq_out = c.aq_out;
    a.as_out = c.as_out;
    a.M = c.M;
    a.K = c.K;
    a.N = c.N;
    a.G = c.G;
    a.S = S;
    if (gemv_rows_enabled()) {
        const int r = launch_gemv_rows(c, mt, ci, a, st);
        if (r != -2) return r;
    }
    if (gemv_mode() == 3 || (gemv_mode() == 1 && lanes_by_default(c.N, c.G))) {
        const int r = launch_gemv_lanes(c, mt, ci, a, st);
        if (r != -2) return r;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kGemvThreads);
    cfg.dynamicSmemBytes = L.total;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = (c.pdl || pdl_flag()) ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, f, a) == cudaSuccess ? 0 : -1;
}

}  // namespace cb
