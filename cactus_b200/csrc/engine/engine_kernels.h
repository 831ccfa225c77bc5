// Engine-only kernel launchers (engine_kernels.cu).
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../kv_paging.h"

namespace cb {
namespace eng {

struct QkvPostArgs {
    const __half* qkv;  // [rows, qkv_stride]: q heads, k heads, v heads
    long long qkv_stride;
    __half* q_out;  // [rows, Hq, D]
    __half* k_out;  // [rows, Hkv, D]
    __half* v_out;  // [rows, Hkv, D]
    const __half* q_norm;  // [D] or null
    const __half* k_norm;  // [D] or null
    float eps;
    const __half* ct;  // rope tables or null
    const __half* st;
    long long pos_base;  // position of row 0 when dstate is null
    const int* dstate;   // {cache_len, total_len, step}: position base = total_len
    int rows, S, Hq, Hkv, D;
};
void launch_qkv_post(const QkvPostArgs& a, cudaStream_t st);

struct KvAppendArgs {
    const __half* k_new;  // [B, S, Hkv, D]
    const __half* v_new;
    int8_t* k_cache;  // [B][cap, Hkv, D]
    int8_t* v_cache;
    float* k_scales;  // [B][cap, Hkv, ng]
    float* v_scales;
    long long cache_bstride, scale_bstride;
    int B, S, Hkv, D, G;
    int src_tok0, ntok;
    long long dst0;
    const int* dstate;  // dst0 = cache_len when set
    KvPaging pg;        // paged cache: caches / scales are the pools, rows through the table
};
// Sliding-window compaction of a paged cache: logical rows [src0, src0 + n) of sequence b
// move to [dst0, dst0 + n) (through `tmp`, so the ranges may overlap); keys, values and scales.
struct KvMoveArgs {
    int8_t* k_cache;
    int8_t* v_cache;
    float* k_scales;
    float* v_scales;
    uint8_t* tmp;  // n * row bytes * 2 + n * scale bytes * 2
    KvPaging pg;
    int b, Hkv, D, ng;
    long long src0, dst0, n;
};
void launch_kv_move_paged(const KvMoveArgs& a, cudaStream_t st);
void launch_kv_append(const KvAppendArgs& a, cudaStream_t st);
void launch_copy_bytes(void* dst, const void* src, long long n, cudaStream_t st);
void launch_state_advance(int* state, int ntok, cudaStream_t st);

struct EmbedArgs {
    const void* table;
    const __half* scales;
    int prec;  // 0 int8, 1 fp16, 3 int4
    int G, hidden;
    const uint32_t* ids;
    int n;
    __half* out;
    int has_scale;
    __half scale16;
};
void launch_embed(const EmbedArgs& a, cudaStream_t st);
void launch_norm_add_clipped(__half* hidden, const __half* o, const __half* w, int rows, int dims, float eps,
                             cudaStream_t st);
void launch_argmax_rows(const __half* logits, int rows, int V, uint32_t* next_tok, uint32_t* ring, int ring_stride,
                        const int* state, cudaStream_t st);

}  // namespace eng
}  // namespace cb
