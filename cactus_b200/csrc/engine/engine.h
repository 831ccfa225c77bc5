// Device-resident engine state (see engine.cu).
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <stdexcept>
#include <string>
#include <vector>

#include "decode_persistent.h"
#include "../kv_paging.h"
#include "weights_io.h"

namespace cb {
namespace eng {

enum ModelType : int { kQwen = 0, kGemma = 1, kSmol = 2, kOther = 99 };

// Subset of cactus::engine::Config (engine.h:43-116) used by the hot path; defaults are the
// reference's (Qwen3-0.6B).
struct Config {
    uint32_t vocab_size = 151936, bos_token_id = 151643, eos_token_id = 151645;
    uint32_t num_layers = 28, hidden_dim = 1024, ffn_intermediate_dim = 3072;
    uint32_t attention_heads = 16, attention_kv_heads = 8, attention_head_dim = 128;
    float layer_norm_eps = 1e-6f, rope_theta = 1000000.0f;
    bool tie_word_embeddings = true;
    int model_type = kQwen;
    float default_temperature = 0.6f, default_top_p = 0.95f;
    size_t default_top_k = 20;
    bool load(const std::string& path, std::string& err);
};

struct Mat {  // weight matrix [N, K] resident in HBM
    int prec = kFp16;  // kInt8 / kInt4 / kFp16
    int N = 0, K = 0, G = 0, ng = 0;
    void* data = nullptr;
    __half* scales = nullptr;  // [N, ng]
};

struct LayerW {
    Mat qkv, o, gateup, down;  // qkv rows = [q | k | v]; gateup rows interleaved (gate_i, up_i)
    __half *in_norm = nullptr, *post_attn_norm = nullptr, *q_norm = nullptr, *k_norm = nullptr;
    __half *pre_ffn_norm = nullptr, *post_ffn_norm = nullptr;
};

class Engine {
public:
    Engine() = default;
    ~Engine();
    void init(const std::string& folder, size_t context_size, size_t max_batch, int device);
    void reset();
    // causal-correct masking inside a prefill chunk after the window has slid (off: the
    // reference's behaviour, whose mask uses the total position and so lets a chunk's queries
    // see its later keys once total > cache index; kernel_attention.cpp:331-346)
    void set_causal_fix(bool on) { causal_fix_ = on; }
    void set_window(size_t w, size_t s) {
        if (cfg_.model_type == kGemma) return;  // Gemma keeps its cache unbounded
        if (w > cap_) throw std::runtime_error("window exceeds the KV cache capacity");
        window_ = w;
        sink_ = s;
    }
    void info(uint32_t* o) const {
        o[0] = (uint32_t)V_; o[1] = (uint32_t)L_; o[2] = (uint32_t)H_; o[3] = (uint32_t)Hq_;
        o[4] = (uint32_t)Hkv_; o[5] = (uint32_t)D_; o[6] = (uint32_t)F_; o[7] = (uint32_t)cfg_.model_type;
    }
    int device() const { return device_; }
    size_t cache_len() const { return cache_len_; }
    size_t total_len() const { return total_len_; }
    const Config& config() const { return cfg_; }
    size_t weight_bytes() const { return weight_bytes_; }

    void prefill(const uint32_t* tokens, size_t n, size_t chunk);
    uint32_t decode(const uint32_t* tokens, size_t n, float temperature, float top_p, size_t top_k, float* entropy);
    uint32_t decode_argmax(const uint32_t* tokens, size_t n, float* entropy);
    void generate(const uint32_t* prompts, int B, size_t P, size_t max_new, uint32_t* out);
    void last_logits(uint16_t* host, size_t vocab);
    void read_kv(size_t layer, int8_t* k, int8_t* v, float* ks, float* vs);
    cudaStream_t stream() const { return stream_; }
    // timing of the last generate(): device time of the prefill and decode phases (CUDA
    // events on the engine stream), kernels launched, graph replays and nodes per replay
    void stats(double* out8) const {
        out8[0] = last_prefill_ms_; out8[1] = last_decode_ms_; out8[2] = (double)last_launches_;
        out8[3] = (double)last_graph_replays_; out8[4] = (double)graph_nodes_; out8[5] = (double)weight_bytes_;
        out8[6] = (double)cap_; out8[7] = (double)window_;
    }

    bool use_graph_ = true;
    bool use_pdl_ = true;
    bool use_persistent_ = true;
    int last_path_ = 0;  // 0 host loop, 1 CUDA graph, 2 persistent step
    const std::string& persistent_reason() const { return pplan_.why; }

private:
    Mat upload_mat(const std::vector<const HostTensor*>& parts, bool interleave_rows);
    __half* upload_vec(const HostTensor& t, size_t expect);
    bool is_global(int layer) const;
    void push_state(int step);
    void gemv(const Mat& w, int pro, int epi, const __half* x, const __half* norm, __half* out, const __half* resid,
              int M);
    void forward(int B, int S, bool graph_mode);
    void update_kv(int l, int B, int S, const __half* kl, const __half* vl, int8_t* kcl, int8_t* vcl, float* ksl,
                   float* vsl, bool graph_mode, bool sliding, bool cache_empty);
    void advance(int S);
    void embed(const uint32_t* d_ids, int n, __half* out);
    void lm_head(const __half* last_rows, int B);
    void check_tokens(const uint32_t* t, size_t n) const;
    void run_forward_tokens(const uint32_t* tokens, int B, int S);
    void gather_last(int B, int S);
    void decode_step_device(int B, uint32_t* ring, int ring_stride, bool graph_mode);
    void setup_persistent();

    Config cfg_;
    int device_ = 0;
    cudaStream_t stream_ = nullptr;
    std::vector<void*> owned_;
    size_t weight_bytes_ = 0;
    int V_ = 0, L_ = 0, H_ = 0, F_ = 0, Hq_ = 0, Hkv_ = 0, D_ = 0, QKVN_ = 0;
    int max_batch_ = 1, max_rows_ = 256;
    Mat embed_, lm_;
    __half* out_norm_ = nullptr;
    std::vector<LayerW> layers_;
    float attention_scale_ = 1.0f;
    size_t window_ = 512, sink_ = 4, cap_ = 512;
    long long cache_bstride_ = 0, scale_bstride_ = 0;
    int seq0_ = 0;  // cache slot of sequence 0 of the current forward (per-sequence prefill)
    bool causal_fix_ = false;
    // paged KV cache (CACTUS_B200_KV_PAGE = tokens per page, a power of two; 0 = contiguous):
    // each layer's cache is a pool of pages, sequences own pages through a block table that
    // every cache access (attention, append, window compaction) goes through
    int page_shift_ = 0, pps_ = 0;
    int* dtable_ = nullptr;         // device [max_batch, pps]
    int* htable_ = nullptr;         // pinned host mirror
    std::vector<int> free_pages_;
    std::vector<int> seq_pages_;    // pages held by each sequence slot
    KvPaging paging(int seq) const {
        KvPaging p;
        if (page_shift_) {
            p.table = dtable_ + (size_t)seq * pps_;
            p.shift = page_shift_;
            p.pps = pps_;
        }
        return p;
    }
    void release_pages();
    void ensure_pages(int seq0, int B, size_t rows);
    int8_t *kc_ = nullptr, *vc_ = nullptr;
    float *ks_ = nullptr, *vs_ = nullptr;
    uint8_t* tmp_kv_ = nullptr;
    size_t cache_len_ = 0, total_len_ = 0;
    int* dstate_ = nullptr;
    int* h_state_ = nullptr;  // pinned ring of 64 state slots
    int h_state_slot_ = 0;
    __half *hidden_ = nullptr, *qkv_ = nullptr, *q_ = nullptr, *kall_ = nullptr, *vall_ = nullptr;
    __half *attn_ = nullptr, *tmp_o_ = nullptr, *gated_ = nullptr, *last_ = nullptr, *xnorm_ = nullptr;
    __half* logits_ = nullptr;
    __half* gm_xn_ = nullptr;  // prefill GEMM staging: normalised rows, int8 rows, row scales
    int8_t* gm_aq_ = nullptr;
    float* gm_as_ = nullptr;
    uint32_t *ids_ = nullptr, *tok_in_ = nullptr, *ring_ = nullptr, *hist_dev_ = nullptr;
    __half* sample_work_ = nullptr;
    float* f32_scratch_ = nullptr;
    size_t ring_cap_ = 0;
    std::vector<const __half*> ct_, st_;
    // exact key-split attention inside decode graphs (long caches): scratch sized for the
    // capacity; split_graph_ selects it while a decode graph is captured
    float* split_scr_ = nullptr;
    size_t split_scr_bytes_ = 0;
    bool split_graph_ = false, graph_split_ = false;
    cudaGraphExec_t graph_exec_ = nullptr;
    size_t graph_nodes_ = 0;
    cudaEvent_t ev_[3] = {nullptr, nullptr, nullptr};
    double last_prefill_ms_ = 0, last_decode_ms_ = 0;
    long long launches_ = 0, last_launches_ = 0, last_graph_replays_ = 0;
    int graph_batch_ = 0, graph_ring_stride_ = 0;
    uint32_t* graph_ring_ = nullptr;
    // persistent decode step
    PArgs pargs_ = {};
    PPlan pplan_;
    PLayer* d_players_ = nullptr;
    PSync* psync_ = nullptr;
    uint32_t* ptagged_ = nullptr;  // the persistent step's tagged activation words (zeroed)
    size_t ptagged_words_ = 0;
    unsigned ptag_base_ = 0;       // advanced by ptag_span(L) per persistent launch
};

}  // namespace eng
}  // namespace cb
