// C entry points over the reference's own sources (cactus/kernel, cactus/graph,
// cactus/engine, cactus/models), compiled on this x86-64 host against oracle/neon_shim.
// TEST INFRASTRUCTURE ONLY: the library built from this file (oracle/_ref/libcactus_ref.so)
// is loaded by tests/ and bench.py's reference leg as the checker, never by the product.
//
// Kernels are forwarded as they are. For the engine, ref_model_decode_greedy is
// Model::decode (cactus/engine/engine_model.cpp:221-297) with the graph-level greedy sample
// sample(logits, 0, 0, 0) (kernel_nn.cpp:451-467) in place of the per-model default top_k,
// and it can hand back the fp16 logits of the step; every other step is the reference's.
#include <cstdint>
#include <cstring>
#include <exception>
#include <memory>
#include <random>
#include <string>
#include <vector>

#include "engine/engine.h"
#include "kernel/kernel_utils.h"
#include "graph/graph.h"
#include "kernel/kernel.h"
#include "models/model.h"

using namespace cactus::engine;

namespace {

thread_local std::string g_err;

struct RefModel {
    virtual ~RefModel() = default;
    virtual Model& model() = 0;
    virtual uint32_t decode_greedy(const std::vector<uint32_t>& tokens, uint16_t* logits_out, size_t vocab) = 0;
    virtual void forward_hidden(const std::vector<uint32_t>& tokens, uint16_t* out, bool update_cache) = 0;
    virtual size_t cache_copy(size_t layer, int8_t* k, int8_t* v, float* ks, float* vs) = 0;
};

template <class M>
struct GreedyModel final : M, RefModel {
    explicit GreedyModel(const Config& c) : M(c) {}
    Model& model() override { return *this; }
    uint32_t decode_greedy(const std::vector<uint32_t>& tokens, uint16_t* logits_out, size_t vocab) override {
        const size_t final_hidden = this->forward(tokens, true);
        auto* gb = static_cast<CactusGraph*>(this->graph_handle_);
        size_t last = gb->index(final_hidden, tokens.size() - 1, 0);
        const size_t hidden_dim = gb->get_output_buffer(last).shape[0];
        last = gb->reshape(last, {1, hidden_dim});
        const size_t logits = gb->matmul(last, this->output_weight_node_id_, true, ComputeBackend::CPU);
        const size_t tok = gb->sample(logits, 0.0f, 0.0f, 0);
        gb->execute();
        if (logits_out) {
            const auto& buf = gb->get_output_buffer(logits);
            if (buf.precision != Precision::FP16 || buf.shape.back() != vocab)
                throw std::runtime_error("unexpected logits buffer");
            std::memcpy(logits_out, gb->get_output(logits), vocab * 2);
        }
        this->post_execute_updates(gb, tokens.size());
        this->update_kv_cache(gb, tokens.size());
        return *static_cast<uint32_t*>(gb->get_output(tok));
    }
    // one graph execution of forward(tokens, use_cache = true): the final normed hidden
    // states [S, hidden] (the prefill step of Model::prefill when update_cache is set)
    void forward_hidden(const std::vector<uint32_t>& tokens, uint16_t* out, bool update_cache) override {
        const size_t final_hidden = this->forward(tokens, true);
        auto* gb = static_cast<CactusGraph*>(this->graph_handle_);
        gb->execute();
        const auto& buf = gb->get_output_buffer(final_hidden);
        std::memcpy(out, gb->get_output(final_hidden), buf.total_size * 2);
        if (update_cache) {
            this->post_execute_updates(gb, tokens.size());
            this->update_kv_cache(gb, tokens.size());
        }
    }
    // the INT8 cache of one layer as the attention reads it ([len, kv_heads, dim] + scales)
    size_t cache_copy(size_t layer, int8_t* k, int8_t* v, float* ks, float* vs) override {
        auto& kv = this->kv_cache_;
        const size_t n = kv.current_seq_len;
        const size_t heads = this->config_.attention_kv_heads, dim = this->config_.attention_head_dim;
        const size_t groups = (dim + KV_QUANT_GROUP_SIZE - 1) / KV_QUANT_GROUP_SIZE;
        if (k) std::memcpy(k, kv.get_keys_int8(layer), n * heads * dim);
        if (v) std::memcpy(v, kv.get_values_int8(layer), n * heads * dim);
        if (ks) std::memcpy(ks, kv.get_key_scales(layer), n * heads * groups * 4);
        if (vs) std::memcpy(vs, kv.get_value_scales(layer), n * heads * groups * 4);
        return n;
    }
};

template <class F>
int guarded(F&& f) {
    try {
        f();
        return 0;
    } catch (const std::exception& e) {
        g_err = e.what();
    } catch (...) {
        g_err = "unknown exception";
    }
    return -1;
}

}  // namespace

extern "C" {

const char* ref_last_error() { return g_err.c_str(); }

// ---- engine ----
void* ref_model_create(const char* folder, size_t context_size) {
    RefModel* out = nullptr;
    guarded([&] {
        Config cfg;
        const std::string dir(folder);
        if (!cfg.from_json(dir + "/config.txt")) throw std::runtime_error("cannot read config.txt");
        std::unique_ptr<RefModel> m;
        switch (cfg.model_type) {
            case Config::ModelType::QWEN: m = std::make_unique<GreedyModel<QwenModel>>(cfg); break;
            case Config::ModelType::GEMMA: m = std::make_unique<GreedyModel<GemmaModel>>(cfg); break;
            case Config::ModelType::SMOL: m = std::make_unique<GreedyModel<SmolModel>>(cfg); break;
            default: throw std::runtime_error("model type not on the hot path");
        }
        if (!m->model().init(dir, context_size, "", false)) throw std::runtime_error("Model::init failed");
        out = m.release();
    });
    return out;
}
void ref_model_destroy(void* h) { delete static_cast<RefModel*>(h); }
int ref_model_prefill(void* h, const uint32_t* tokens, size_t n, size_t chunk) {
    return guarded([&] { static_cast<RefModel*>(h)->model().prefill(std::vector<uint32_t>(tokens, tokens + n), chunk); });
}
int ref_model_decode_greedy(void* h, const uint32_t* tokens, size_t n, uint32_t* out, uint16_t* logits, size_t vocab) {
    return guarded([&] { *out = static_cast<RefModel*>(h)->decode_greedy(std::vector<uint32_t>(tokens, tokens + n), logits, vocab); });
}
int ref_model_decode(void* h, const uint32_t* tokens, size_t n, float temperature, float top_p, size_t top_k,
                     uint32_t* out) {
    return guarded([&] {
        *out = static_cast<RefModel*>(h)->model().decode(std::vector<uint32_t>(tokens, tokens + n), temperature, top_p, top_k);
    });
}
int ref_model_forward_hidden(void* h, const uint32_t* tokens, size_t n, uint16_t* out, int update_cache) {
    return guarded([&] {
        static_cast<RefModel*>(h)->forward_hidden(std::vector<uint32_t>(tokens, tokens + n), out, update_cache != 0);
    });
}
size_t ref_model_cache(void* h, size_t layer, int8_t* k, int8_t* v, float* ks, float* vs) {
    size_t n = 0;
    guarded([&] { n = static_cast<RefModel*>(h)->cache_copy(layer, k, v, ks, vs); });
    return n;
}
int ref_model_reset(void* h) { return guarded([&] { static_cast<RefModel*>(h)->model().reset_cache(); }); }
int ref_model_set_window(void* h, size_t window, size_t sink) {
    return guarded([&] { static_cast<RefModel*>(h)->model().set_cache_window(window, sink); });
}

// ---- kernels (cactus/kernel/kernel.h), fp16 passed as raw 16-bit storage ----
#define HP(p) reinterpret_cast<const __fp16*>(p)
#define HW(p) reinterpret_cast<__fp16*>(p)
void ref_matmul_int8(const int8_t* A, const float* As, const int8_t* B, const uint16_t* Bs, uint16_t* C, size_t M,
                     size_t K, size_t N, size_t G) {
    cactus_matmul_int8(A, As, B, HP(Bs), HW(C), M, K, N, G);
}
void ref_matmul_int4(const int8_t* A, const float* As, const uint8_t* B, const uint16_t* Bs, uint16_t* C, size_t M,
                     size_t K, size_t N, size_t G) {
    cactus_matmul_int4(A, As, B, HP(Bs), HW(C), M, K, N, G);
}
void ref_matmul_f16(const uint16_t* a, const uint16_t* bt, uint16_t* c, size_t M, size_t K, size_t N) {
    cactus_matmul_f16(HP(a), HP(bt), HW(c), M, K, N);
}
void ref_fp16_to_int8(const uint16_t* src, int8_t* dst, size_t count, float scale) {
    cactus_fp16_to_int8(HP(src), dst, count, scale);
}
float ref_fp16_max_abs(const uint16_t* src, size_t count) { return cactus_fp16_max_abs(HP(src), count); }
void ref_rms_norm(const uint16_t* x, const uint16_t* w, uint16_t* y, size_t rows, size_t dims, float eps) {
    cactus_rms_norm_f16(HP(x), HP(w), HW(y), rows, dims, eps);
}
void ref_conv1d_causal_depthwise(const uint16_t* x, const uint16_t* w, uint16_t* y, size_t N, size_t L, size_t C,
                                 size_t K, size_t dil) {
    cactus_conv1d_causal_depthwise_f16(HP(x), HP(w), HW(y), N, L, C, K, dil);
}
void ref_conv1d_k3(const uint16_t* x, const uint16_t* w, uint16_t* y, size_t N, size_t L, size_t Cin, size_t Cout,
                   size_t stride) {
    cactus_conv1d_f16_k3(HP(x), HP(w), HW(y), N, L, Cin, Cout, stride);
}
// The reference's layernorm is a graph node (compute_layernorm_node): one-node graph, fp16 in / out.
int ref_layernorm(const uint16_t* x, const uint16_t* w, const uint16_t* b, uint16_t* y, size_t rows, size_t F,
                  float eps) {
    try {
        CactusGraph g;
        const size_t xi = g.input({rows, F}, Precision::FP16);
        const size_t wi = g.input({F}, Precision::FP16);
        const size_t bi = g.input({F}, Precision::FP16);
        const size_t o = g.layernorm(xi, wi, bi, eps);
        g.set_input(xi, x, Precision::FP16);
        g.set_input(wi, w, Precision::FP16);
        g.set_input(bi, b, Precision::FP16);
        g.execute();
        const auto& buf = g.get_output_buffer(o);
        if (buf.precision != Precision::FP16 || buf.total_size != rows * F) {
            g_err = "layernorm: unexpected output buffer";
            return -1;
        }
        std::memcpy(y, g.get_output(o), rows * F * 2);
        return 0;
    } catch (const std::exception& e) {
        g_err = e.what();
        return -1;
    }
}
void ref_rope(const uint16_t* x, uint16_t* y, size_t B, size_t S, size_t H, size_t D, size_t start, float theta) {
    cactus_rope_f16(HP(x), HW(y), B, S, H, D, start, theta);
}
void ref_softmax(const uint16_t* x, uint16_t* y, size_t B, size_t S, size_t V) { cactus_softmax_f16(HP(x), HW(y), B, S, V); }
void ref_silu(const uint16_t* x, uint16_t* y, size_t n) { cactus_silu_f16(HP(x), HW(y), n); }
void ref_gelu(const uint16_t* x, uint16_t* y, size_t n) { cactus_gelu_f16(HP(x), HW(y), n); }
void ref_add(const uint16_t* a, const uint16_t* b, uint16_t* y, size_t n) { cactus_add_f16(HP(a), HP(b), HW(y), n); }
void ref_add_clipped(const uint16_t* a, const uint16_t* b, uint16_t* y, size_t n) {
    cactus_add_f16_clipped(HP(a), HP(b), HW(y), n);
}
void ref_multiply(const uint16_t* a, const uint16_t* b, uint16_t* y, size_t n) { cactus_multiply_f16(HP(a), HP(b), HW(y), n); }
void ref_attention_f16(const uint16_t* q, const uint16_t* k, const uint16_t* v, uint16_t* o, size_t B, size_t S,
                       size_t Skv, size_t Hq, size_t Hkv, size_t D, float scale, size_t pos_offset, size_t window,
                       int causal) {
    cactus_attention_f16(HP(q), HP(k), HP(v), HW(o), B, S, Skv, Hq, Hkv, D, scale, nullptr, pos_offset, window, causal != 0);
}
void ref_attention_hybrid(const uint16_t* q, const int8_t* kc, const int8_t* vc, const float* ks, const float* vs,
                          const uint16_t* kn, const uint16_t* vn, uint16_t* o, size_t B, size_t S, size_t cache_len,
                          size_t new_len, size_t Hq, size_t Hkv, size_t D, float scale, size_t pos_offset, int causal) {
    cactus_attention_hybrid_int8_fp16(HP(q), kc, vc, ks, vs, HP(kn), HP(vn), HW(o), B, S, cache_len, new_len, Hq, Hkv,
                                      D, scale, pos_offset, causal != 0);
}
void ref_quantize_kv(const uint16_t* src, int8_t* dst, float* scales, size_t S, size_t H, size_t D) {
    cactus_quantize_kv_fp16_to_int8(HP(src), dst, scales, S, H, D);
}
void ref_unpack_int4(const uint8_t* packed, int8_t* out, size_t count) { cactus_unpack_int4_to_int8(packed, out, count); }
void ref_sample_f16(const uint16_t* logits, uint32_t* out, size_t V, float temperature, float top_p, size_t top_k,
                    size_t seed) {
    cactus_sample_f16(HP(logits), out, V, temperature, top_p, top_k, seed);
}

// workers of the reference's thread pool (min(hardware threads, 16), kernel_utils.h:265-311):
// parallel_for splits element-wise work into that many chunks at most, and SiLU / GELU use
// libm on each chunk's tail (fewer than 8 elements), so those positions depend on it
size_t ref_pool_workers() { return CactusThreading::get_thread_pool().num_workers(); }

// the uniform sample cactus_sample_f16 draws for a non-zero seed (kernel_nn.cpp:627-630)
float ref_mt19937_uniform(size_t seed) {
    std::mt19937 gen(static_cast<uint32_t>(seed));
    std::uniform_real_distribution<float> dist(0.0f, 1.0f);
    return dist(gen);
}

}  // extern "C"
