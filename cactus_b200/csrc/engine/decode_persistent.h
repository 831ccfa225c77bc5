// Persistent single-launch decode step for batch-1 greedy decoding (see decode_persistent.cu).
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <string>

namespace cb {
namespace eng {

struct PLayer {
    const int8_t *wqkv, *wo, *wgu, *wd;   // [N, K] int8, rows 16-byte aligned
    const __half *sqkv, *so, *sgu, *sd;   // [N, K/G] fp16 group scales
    const __half *in_norm, *post_norm, *q_norm, *k_norm;  // q/k norm may be null
    int8_t *kc, *vc;                      // sequence 0 of this layer's cache [cap, Hkv, D]
    float *ks, *vs;                       // [cap, Hkv, ceil(D/128)]
    const __half *ct, *st;                // RoPE tables [positions, D/2] (null: no RoPE)
};

// Device-resident synchronisation words. Zero before the first launch of a run; the last
// block of every launch zeroes done/key again. `abort` stays set after a failure.
struct PSync {
    unsigned done, abort, pad0, pad1;
    unsigned long long key;
};

// Activations that cross blocks travel as tagged words: the fp16 bits in the low half and the
// writer's 16-bit version tag in the high half. A reader polls the words it needs until they
// carry the version it expects, so the data is its own ready flag and no grid barrier is
// needed. Version v of a launch (v = 0 for the embedding, 5 l + 1 .. 5 l + 5 for layer l's
// QKV, attention, O, gate-up and down outputs) has tag 1 + (tag_base + v) % 65535: never 0
// (the buffers start zeroed), and the host advances tag_base by ptag_span(L) per launch.
__host__ __device__ inline unsigned ptag_span(int L) { return 5u * (unsigned)L + 1u; }

struct PArgs {
    const PLayer* layers;
    int L, H, F, Hq, Hkv, D, V, G, QKVN;
    const int8_t* lm_w;
    const __half* lm_s;
    const __half* out_norm;
    const void* emb;        // embedding table: int8 / fp16 / packed int4 (emb_prec 0 / 1 / 3)
    const __half* emb_s;
    int emb_prec, emb_G;
    float eps, attn_scale;
    uint32_t *hidden, *qkv, *attn, *gated;  // tagged words: [H], [QKVN], [Hq*D], [F]
    __half* logits;                         // [V]
    unsigned tag_base;                      // this launch's tag offset (see ptag_span)
    uint32_t* tok_in;       // input token of the step; the next token is written back here
    uint32_t* ring;         // optional: ring[state[2]] = next token
    int* state;             // [cache_len, total_len, step], advanced by the kernel
    PSync* sync;
    const int* pages;       // paged KV cache: the sequence's page table (null: contiguous)
    int page_shift;
    unsigned spin_limit;    // polls before a wait gives up (2^22; CACTUS_B200_SPIN_LIMIT lowers it in tests)
    // filled by persistent_plan
    int slot_w, slot_s, nslots, kmax, gsm_ints, max_rows, work_bytes, attn_off;
};

struct PPlan {
    bool ok = false;
    std::string why;
    int grid = 0, threads = 0;
    size_t smem = 0;
};

// Checks the model shape against the kernel's requirements and sizes the weight ring for
// `smem_optin` bytes of shared memory per block (fills a.slot_* / work fields).
PPlan persistent_plan(PArgs& a, int num_sms, size_t smem_optin);
cudaError_t launch_persistent_decode(const PArgs& a, const PPlan& p, cudaStream_t st);

}  // namespace eng
}  // namespace cb
