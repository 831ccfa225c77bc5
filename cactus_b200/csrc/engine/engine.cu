// Device-resident engine: config, weight upload, INT8 KV cache, chunked prefill, decode
// (optionally as one CUDA-graph replay per token) and the C ABI of
// include/cactus_b200_engine.h.
//
// Model graphs follow the reference model builders:
//   Qwen3  QwenModel  (cactus/models/model_qwen.cpp:51-172)
//   Gemma3 GemmaModel (cactus/models/model_gemma.cpp:57-176)
//   Llama  SmolModel  (cactus/models/model_smol.cpp:43-143)
// with the per-node arithmetic of the kernels they call; fusions keep every rounding point:
//   rms_norm -> matmul                  = one GEMV with an RMSNorm+quantise prologue
//   matmul -> add(hidden, .)            = one GEMV with a residual epilogue
//   gate/up matmuls -> act -> multiply  = one GEMV over row-interleaved gate/up weights
//   q/k rms_norm -> rope (-> kv quant)  = qkv_post (+ kv_append)
#include <chrono>
#include <cmath>
#include <cstdlib>
#include <random>
#include <cstring>
#include <fstream>
#include <memory>
#include <mutex>
#include <sstream>
#include <string>
#include <vector>

#include "../../../include/cactus_b200_engine.h"
#include "../gemv.cuh"
#include "../ops.h"
#include "engine.h"
#include "engine_kernels.h"
#include "weights_io.h"

namespace cb {
namespace eng {

static void ck(cudaError_t e, const char* what) {
    if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

// ------------------------------------------------------------------ config.txt (engine_model.cpp:403-539)
bool Config::load(const std::string& path, std::string& err) {
    std::ifstream f(path);
    if (!f) {
        err = "Failed to open config file: " + path;
        return false;
    }
    std::string line;
    while (std::getline(f, line)) {
        if (line.empty() || line[0] == '#') continue;
        const size_t eq = line.find('=');
        if (eq == std::string::npos) continue;
        std::string key = line.substr(0, eq), value = line.substr(eq + 1);
        auto trim = [](std::string& s) {
            s.erase(0, s.find_first_not_of(" \t\r"));
            s.erase(s.find_last_not_of(" \t\r") + 1);
        };
        trim(key);
        trim(value);
        try {
            if (key == "vocab_size") vocab_size = (uint32_t)std::stoul(value);
            else if (key == "bos_token_id") bos_token_id = (uint32_t)std::stoul(value);
            else if (key == "eos_token_id") eos_token_id = (uint32_t)std::stoul(value);
            else if (key == "num_layers") num_layers = (uint32_t)std::stoul(value);
            else if (key == "hidden_dim") hidden_dim = (uint32_t)std::stoul(value);
            else if (key == "ffn_intermediate_dim") ffn_intermediate_dim = (uint32_t)std::stoul(value);
            else if (key == "attention_heads") attention_heads = (uint32_t)std::stoul(value);
            else if (key == "attention_kv_heads") attention_kv_heads = (uint32_t)std::stoul(value);
            else if (key == "attention_head_dim") attention_head_dim = (uint32_t)std::stoul(value);
            else if (key == "layer_norm_eps") layer_norm_eps = std::stof(value);
            else if (key == "rope_theta") rope_theta = std::stof(value);
            else if (key == "tie_word_embeddings") tie_word_embeddings = (value == "true" || value == "1");
            else if (key == "model_type") {
                if (value == "gemma" || value == "GEMMA") model_type = kGemma;
                else if (value == "smol" || value == "SMOL" || value == "Smol") model_type = kSmol;
                else if (value == "qwen" || value == "QWEN" || value == "qwen3") model_type = kQwen;
                else model_type = kOther;
            }
        } catch (const std::exception&) {
            err = "bad value for " + key + " in " + path;
            return false;
        }
    }
    if (model_type == kGemma) {
        default_temperature = 1.0f;
        default_top_p = 0.95f;
        default_top_k = 64;
    } else if (model_type == kSmol) {
        default_temperature = 0.2f;
        default_top_p = 0.95f;
        default_top_k = 20;
    } else {
        default_temperature = 0.6f;
        default_top_p = 0.95f;
        default_top_k = 20;
    }
    return true;
}

// ------------------------------------------------------------------ weight upload
static void* dmalloc(size_t bytes, std::vector<void*>& owned) {
    void* p = nullptr;
    ck(cudaMalloc(&p, bytes ? bytes : 16), "cudaMalloc");
    owned.push_back(p);
    return p;
}

Mat Engine::upload_mat(const std::vector<const HostTensor*>& parts, bool interleave_rows) {
    const HostTensor& p0 = *parts[0];
    if (p0.shape.size() != 2) throw std::runtime_error("weight matrix must be 2-D");
    Mat m;
    m.prec = p0.prec;
    m.K = (int)p0.shape[1];
    m.G = (int)p0.group_size;
    m.ng = (int)p0.num_groups;
    size_t N = 0;
    for (auto* p : parts) {
        if (p->prec != p0.prec || p->shape.size() != 2 || p->shape[1] != p0.shape[1] || p->group_size != p0.group_size)
            throw std::runtime_error("fused projections need equal precision, K and group size");
        N += p->shape[0];
    }
    m.N = (int)N;
    if (m.prec == kInt8 || m.prec == kInt4) {
        if (m.G <= 0 || m.ng * m.G != m.K) throw std::runtime_error("quantized weight without group scales");
    } else if (m.prec != kFp16) {
        throw std::runtime_error("unsupported weight precision");
    }
    const size_t row_bytes = m.prec == kInt8 ? (size_t)m.K : m.prec == kInt4 ? (size_t)m.K / 2 : (size_t)m.K * 2;
    std::vector<uint8_t> data(N * row_bytes);
    std::vector<uint16_t> scales(m.prec == kFp16 ? 0 : N * (size_t)m.ng);
    if (!interleave_rows) {
        size_t r0 = 0;
        for (auto* p : parts) {
            const size_t n = p->shape[0];
            if (p->data.size() != n * row_bytes) throw std::runtime_error("weight data size mismatch");
            std::memcpy(data.data() + r0 * row_bytes, p->data.data(), n * row_bytes);
            if (!scales.empty()) std::memcpy(scales.data() + r0 * m.ng, p->scales.data(), n * m.ng * 2);
            r0 += n;
        }
    } else {  // rows 2i / 2i+1 = part0 row i / part1 row i (gate / up)
        const HostTensor& a = *parts[0];
        const HostTensor& b = *parts[1];
        if (a.shape[0] != b.shape[0]) throw std::runtime_error("gate/up row counts differ");
        const size_t n = a.shape[0];
        for (size_t i = 0; i < n; ++i) {
            std::memcpy(data.data() + (2 * i) * row_bytes, a.data.data() + i * row_bytes, row_bytes);
            std::memcpy(data.data() + (2 * i + 1) * row_bytes, b.data.data() + i * row_bytes, row_bytes);
            if (!scales.empty()) {
                std::memcpy(scales.data() + (2 * i) * m.ng, a.scales.data() + i * m.ng, m.ng * 2);
                std::memcpy(scales.data() + (2 * i + 1) * m.ng, b.scales.data() + i * m.ng, m.ng * 2);
            }
        }
    }
    m.data = dmalloc(data.size(), owned_);
    ck(cudaMemcpy(m.data, data.data(), data.size(), cudaMemcpyHostToDevice), "upload weights");
    weight_bytes_ += data.size();
    if (!scales.empty()) {
        m.scales = static_cast<__half*>(dmalloc(scales.size() * 2, owned_));
        ck(cudaMemcpy(m.scales, scales.data(), scales.size() * 2, cudaMemcpyHostToDevice), "upload scales");
        weight_bytes_ += scales.size() * 2;
    }
    return m;
}

__half* Engine::upload_vec(const HostTensor& t, size_t expect) {
    if (t.prec != kFp16) throw std::runtime_error("norm weights must be FP16");
    if (t.data.size() != expect * 2) throw std::runtime_error("norm weight size mismatch");
    __half* p = static_cast<__half*>(dmalloc(expect * 2, owned_));
    ck(cudaMemcpy(p, t.data.data(), expect * 2, cudaMemcpyHostToDevice), "upload norm");
    return p;
}

Engine::~Engine() {
    for (auto& e : ev_)
        if (e) cudaEventDestroy(e);
    if (graph_exec_) cudaGraphExecDestroy(graph_exec_);
    if (stream_) cudaStreamDestroy(stream_);
    for (void* p : owned_) cudaFree(p);
    if (h_state_) cudaFreeHost(h_state_);
    if (htable_) cudaFreeHost(htable_);
}

void Engine::init(const std::string& folder, size_t context_size, size_t max_batch, int device) {
    device_ = device;
    ck(cudaSetDevice(device), "cudaSetDevice");
    std::string err;
    if (!cfg_.load(folder + "/config.txt", err)) throw std::runtime_error(err);
    if (cfg_.model_type == kOther) throw std::runtime_error("model_type not supported by the B200 engine");
    ck(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking), "stream");
    ck(cudaMallocHost(&h_state_, 64 * 4 * sizeof(int)), "pinned state");
    gemv_prepare();
    attention_prepare();
    V_ = (int)cfg_.vocab_size;
    L_ = (int)cfg_.num_layers;
    H_ = (int)cfg_.hidden_dim;
    F_ = (int)cfg_.ffn_intermediate_dim;
    Hq_ = (int)cfg_.attention_heads;
    Hkv_ = (int)cfg_.attention_kv_heads;
    D_ = (int)cfg_.attention_head_dim;
    QKVN_ = (Hq_ + 2 * Hkv_) * D_;
    max_batch_ = (int)(max_batch ? max_batch : 1);
    max_rows_ = std::max(256, max_batch_);
    if (D_ % 32 || D_ > 256) throw std::runtime_error("head_dim must be a multiple of 32 and <= 256");

    // weights
    HostTensor emb = read_weights_file(folder + "/token_embeddings.weights");
    if (emb.shape.size() != 2 || emb.shape[1] != (size_t)H_)
        throw std::runtime_error("Memory-mapped embeddings must be 2D [vocab_size, embedding_dim]");
    embed_ = upload_mat({&emb}, false);
    if (cfg_.tie_word_embeddings) {
        lm_ = embed_;
    } else {
        HostTensor ow = read_weights_file(folder + "/output_weight.weights");
        lm_ = upload_mat({&ow}, false);
    }
    if (lm_.N != V_) V_ = lm_.N;
    out_norm_ = upload_vec(read_weights_file(folder + "/output_norm.weights"), H_);
    layers_.resize(L_);
    for (int i = 0; i < L_; ++i) {
        const std::string p = folder + "/layer_" + std::to_string(i) + "_";
        LayerW& lw = layers_[i];
        {
            HostTensor q = read_weights_file(p + "attn_q.weights");
            HostTensor k = read_weights_file(p + "attn_k.weights");
            HostTensor v = read_weights_file(p + "attn_v.weights");
            lw.qkv = upload_mat({&q, &k, &v}, false);
        }
        {
            HostTensor o = read_weights_file(p + "attn_output.weights");
            lw.o = upload_mat({&o}, false);
        }
        {
            HostTensor g = read_weights_file(p + "ffn_gate.weights");
            HostTensor u = read_weights_file(p + "ffn_up.weights");
            lw.gateup = upload_mat({&g, &u}, true);
        }
        {
            HostTensor d = read_weights_file(p + "ffn_down.weights");
            lw.down = upload_mat({&d}, false);
        }
        lw.in_norm = upload_vec(read_weights_file(p + "input_norm.weights"), H_);
        lw.post_attn_norm = upload_vec(read_weights_file(p + "post_attn_norm.weights"), H_);
        if (cfg_.model_type != kSmol) {
            lw.q_norm = upload_vec(read_weights_file(p + "attn_q_norm.weights"), D_);
            lw.k_norm = upload_vec(read_weights_file(p + "attn_k_norm.weights"), D_);
        }
        if (cfg_.model_type == kGemma) {
            lw.pre_ffn_norm = upload_vec(read_weights_file(p + "pre_ffn_norm.weights"), H_);
            lw.post_ffn_norm = upload_vec(read_weights_file(p + "post_ffn_norm.weights"), H_);
        }
        if (lw.qkv.N != QKVN_ || lw.o.N != H_ || lw.gateup.N != 2 * F_ || lw.down.N != H_)
            throw std::runtime_error("layer weight shapes do not match config.txt");
        if (lw.qkv.prec == kFp16 || lw.o.prec == kFp16 || lw.gateup.prec == kFp16 || lw.down.prec == kFp16)
            throw std::runtime_error("FP16 layer projections are not supported by the B200 engine");
    }
    if (lm_.prec == kFp16 && lm_.K != H_) throw std::runtime_error("lm_head shape mismatch");

    // attention scale (engine_model.cpp:125-129) and per-layer window / rope theta
    attention_scale_ = cfg_.model_type == kGemma ? 1.0f / std::sqrt(256.0f) : 1.0f / std::sqrt((float)D_);
    // KV window (engine_model.cpp:136-146), Gemma disables it in post_init (model_gemma.cpp:17-19)
    window_ = std::min(context_size, (size_t)512);
    sink_ = 4;
    if (const char* w = std::getenv("CACTUS_KV_WINDOW_SIZE")) window_ = std::strtoul(w, nullptr, 10);
    if (const char* s = std::getenv("CACTUS_KV_SINK_SIZE")) sink_ = std::strtoul(s, nullptr, 10);
    if (const char* f = std::getenv("CACTUS_B200_CAUSAL_FIX")) causal_fix_ = std::strtoul(f, nullptr, 10) != 0;
    if (cfg_.model_type == kGemma) window_ = 0, sink_ = 0;
    cap_ = std::max<size_t>(context_size, 1);
    if (const char* c = std::getenv("CACTUS_B200_KV_CAPACITY")) cap_ = std::max(cap_, (size_t)std::strtoul(c, nullptr, 10));
    if (window_ > cap_) cap_ = window_;

    const int ng = (D_ + 127) / 128;
    size_t cap_rows = cap_;
    if (const char* pg = std::getenv("CACTUS_B200_KV_PAGE")) {
        const long pt = std::strtol(pg, nullptr, 10);
        if (pt > 0) {
            if (pt < 16 || (pt & (pt - 1))) throw std::runtime_error("CACTUS_B200_KV_PAGE must be a power of two >= 16");
            while ((1L << page_shift_) < pt) ++page_shift_;
            pps_ = (int)((cap_ + pt - 1) / pt);
            cap_rows = (size_t)pps_ * pt;  // a sequence slot's share of the pool, in rows
        }
    }
    cache_bstride_ = (long long)cap_rows * Hkv_ * D_;
    scale_bstride_ = (long long)cap_rows * Hkv_ * ng;
    const size_t cache_elems = (size_t)L_ * max_batch_ * cache_bstride_;
    const size_t scale_elems = (size_t)L_ * max_batch_ * scale_bstride_;
    kc_ = static_cast<int8_t*>(dmalloc(cache_elems, owned_));
    vc_ = static_cast<int8_t*>(dmalloc(cache_elems, owned_));
    ks_ = static_cast<float*>(dmalloc(scale_elems * 4, owned_));
    vs_ = static_cast<float*>(dmalloc(scale_elems * 4, owned_));
    tmp_kv_ = static_cast<uint8_t*>(dmalloc((size_t)cache_bstride_ * 4 + 256, owned_));
    if (page_shift_) {
        dtable_ = static_cast<int*>(dmalloc((size_t)max_batch_ * pps_ * 4, owned_));
        ck(cudaMallocHost(&htable_, (size_t)max_batch_ * pps_ * 4), "page table");
        for (int i = 0; i < max_batch_ * pps_; ++i) htable_[i] = -1;
        release_pages();
    }

    const size_t R = (size_t)max_rows_;
    hidden_ = static_cast<__half*>(dmalloc(R * H_ * 2, owned_));
    qkv_ = static_cast<__half*>(dmalloc(R * QKVN_ * 2, owned_));
    q_ = static_cast<__half*>(dmalloc(R * Hq_ * D_ * 2, owned_));
    kall_ = static_cast<__half*>(dmalloc((size_t)L_ * R * Hkv_ * D_ * 2, owned_));
    vall_ = static_cast<__half*>(dmalloc((size_t)L_ * R * Hkv_ * D_ * 2, owned_));
    attn_ = static_cast<__half*>(dmalloc(R * Hq_ * D_ * 2, owned_));
    tmp_o_ = static_cast<__half*>(dmalloc(R * H_ * 2, owned_));
    gated_ = static_cast<__half*>(dmalloc(R * F_ * 2, owned_));
    last_ = static_cast<__half*>(dmalloc((size_t)max_batch_ * H_ * 2, owned_));
    xnorm_ = static_cast<__half*>(dmalloc((size_t)max_batch_ * H_ * 2, owned_));
    logits_ = static_cast<__half*>(dmalloc((size_t)max_batch_ * V_ * 2, owned_));
    ids_ = static_cast<uint32_t*>(dmalloc(R * 4, owned_));
    const size_t kmax = (size_t)std::max({H_, Hq_ * D_, F_});
    gm_xn_ = static_cast<__half*>(dmalloc(R * H_ * 2, owned_));
    gm_aq_ = static_cast<int8_t*>(dmalloc(R * kmax, owned_));
    gm_as_ = static_cast<float*>(dmalloc(R * 4, owned_));
    tok_in_ = static_cast<uint32_t*>(dmalloc((size_t)max_batch_ * 4, owned_));
    dstate_ = static_cast<int*>(dmalloc(4 * sizeof(int), owned_));
    hist_dev_ = static_cast<uint32_t*>(dmalloc(128 * 4, owned_));
    sample_work_ = static_cast<__half*>(dmalloc((size_t)V_ * 2, owned_));
    f32_scratch_ = static_cast<float*>(dmalloc(64, owned_));
    if ((long long)cap_ + 1 >= kSplitMinKeys && attention_split_prepare(D_, Hq_, Hkv_, (long long)cap_ + 1) == 0) {
        split_scr_bytes_ = attention_split_scratch_bytes((long long)max_batch_ * Hq_, (long long)cap_ + 1);
        split_scr_ = static_cast<float*>(dmalloc(split_scr_bytes_, owned_));
    }

    // RoPE tables per layer (Gemma: global every 6th layer theta 1e6, local 1e4; model_gemma.cpp:84-88)
    ct_.assign(L_, nullptr);
    st_.assign(L_, nullptr);
    if (cfg_.rope_theta > 0) {
        for (int i = 0; i < L_; ++i) {
            float theta = cfg_.rope_theta;
            if (cfg_.model_type == kGemma) theta = is_global(i) ? 1000000.0f : 10000.0f;
            if (!rope_tables(theta, D_, (long long)cap_ + 4096 + R, &ct_[i], &st_[i]))
                throw std::runtime_error("rope table allocation failed");
        }
    }
    setup_persistent();
    reset();
    ck(cudaStreamSynchronize(stream_), "init");
}

// Prepares the persistent decode step (decode_persistent.cu) when the model fits it: a
// Qwen/Llama-style block with grouped INT8 projections and lm head sharing one group size.
void Engine::setup_persistent() {
    pplan_ = PPlan();
    if (const char* m = std::getenv("CACTUS_B200_DECODE"))
        if (std::string(m) == "graph") use_persistent_ = false;
    auto no = [&](const char* why) { pplan_.ok = false; pplan_.why = why; };
    if (cfg_.model_type == kGemma) return no("Gemma blocks use the per-op path");
    const int G = lm_.G;
    if (lm_.prec != kInt8) return no("lm head is not grouped INT8");
    if (embed_.N < V_) return no("embedding table has fewer rows than the vocabulary");
    for (const LayerW& lw : layers_)
        for (const Mat* m : {&lw.qkv, &lw.o, &lw.gateup, &lw.down})
            if (m->prec != kInt8 || m->G != G) return no("projections are not grouped INT8 with one group size");
    std::vector<PLayer> pl(L_);
    const size_t lstride = (size_t)max_batch_;
    for (int l = 0; l < L_; ++l) {
        const LayerW& lw = layers_[l];
        PLayer& p = pl[l];
        p.wqkv = static_cast<const int8_t*>(lw.qkv.data);
        p.sqkv = lw.qkv.scales;
        p.wo = static_cast<const int8_t*>(lw.o.data);
        p.so = lw.o.scales;
        p.wgu = static_cast<const int8_t*>(lw.gateup.data);
        p.sgu = lw.gateup.scales;
        p.wd = static_cast<const int8_t*>(lw.down.data);
        p.sd = lw.down.scales;
        p.in_norm = lw.in_norm;
        p.post_norm = lw.post_attn_norm;
        p.q_norm = lw.q_norm;
        p.k_norm = lw.k_norm;
        p.kc = kc_ + (size_t)l * lstride * cache_bstride_;
        p.vc = vc_ + (size_t)l * lstride * cache_bstride_;
        p.ks = ks_ + (size_t)l * lstride * scale_bstride_;
        p.vs = vs_ + (size_t)l * lstride * scale_bstride_;
        p.ct = ct_[l];
        p.st = st_[l];
    }
    d_players_ = static_cast<PLayer*>(dmalloc(sizeof(PLayer) * L_, owned_));
    ck(cudaMemcpy(d_players_, pl.data(), sizeof(PLayer) * L_, cudaMemcpyHostToDevice), "persistent layers");
    psync_ = static_cast<PSync*>(dmalloc(sizeof(PSync), owned_));
    ptagged_words_ = (size_t)H_ + QKVN_ + (size_t)Hq_ * D_ + F_;
    ptagged_ = static_cast<uint32_t*>(dmalloc(ptagged_words_ * 4, owned_));
    ck(cudaMemset(ptagged_, 0, ptagged_words_ * 4), "persistent activations");
    PArgs& a = pargs_;
    a = PArgs{};
    a.layers = d_players_;
    a.L = L_, a.H = H_, a.F = F_, a.Hq = Hq_, a.Hkv = Hkv_, a.D = D_, a.V = V_, a.G = G, a.QKVN = QKVN_;
    a.lm_w = static_cast<const int8_t*>(lm_.data);
    a.lm_s = lm_.scales;
    a.out_norm = out_norm_;
    a.emb = embed_.data;
    a.emb_s = embed_.scales;
    a.emb_prec = embed_.prec;
    a.emb_G = embed_.G;
    a.eps = cfg_.layer_norm_eps;
    a.attn_scale = attention_scale_;
    a.hidden = ptagged_;
    a.qkv = a.hidden + H_;
    a.attn = a.qkv + QKVN_;
    a.gated = a.attn + (size_t)Hq_ * D_;
    a.logits = logits_;
    a.tok_in = tok_in_;
    a.state = dstate_;
    a.sync = psync_;
    a.pages = page_shift_ ? dtable_ : nullptr;  // sequence slot 0's table
    a.spin_limit = 1u << 22;
    if (const char* e = std::getenv("CACTUS_B200_SPIN_LIMIT")) a.spin_limit = (unsigned)std::max(1L, std::strtol(e, nullptr, 10));
    a.page_shift = page_shift_;
    int sms = 0, optin = 0;
    ck(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device_), "sm count");
    ck(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device_), "smem");
    pplan_ = persistent_plan(a, sms, (size_t)optin);
}

bool Engine::is_global(int layer) const { return cfg_.model_type == kGemma && ((layer + 1) % 6) == 0; }

// All pages back to the pool. Pages are handed out from the end of the pool first, so a
// sequence's logical pages do not sit in physical order (the table is always exercised).
void Engine::release_pages() {
    if (!page_shift_) return;
    free_pages_.resize((size_t)max_batch_ * pps_);
    for (size_t i = 0; i < free_pages_.size(); ++i) free_pages_[i] = (int)i;
    seq_pages_.assign(max_batch_, 0);
}

// Gives sequence slots [seq0, seq0 + B) pages for `rows` logical rows and uploads the table
// when it changed. The host mirror is only rewritten after the stream has drained, so a copy
// still queued never sees a later edit.
void Engine::ensure_pages(int seq0, int B, size_t rows) {
    if (!page_shift_) return;
    const int need = (int)((rows + ((size_t)1 << page_shift_) - 1) >> page_shift_);
    if (need > pps_) throw std::runtime_error("KV cache capacity exceeded");
    bool synced = false, changed = false;
    for (int b = seq0; b < seq0 + B; ++b) {
        while (seq_pages_[b] < need) {
            if (free_pages_.empty()) throw std::runtime_error("KV page pool exhausted");
            if (!synced) {
                ck(cudaStreamSynchronize(stream_), "page table");
                synced = true;
            }
            htable_[(size_t)b * pps_ + seq_pages_[b]++] = free_pages_.back();
            free_pages_.pop_back();
            changed = true;
        }
    }
    if (changed)
        ck(cudaMemcpyAsync(dtable_, htable_, (size_t)max_batch_ * pps_ * 4, cudaMemcpyHostToDevice, stream_),
           "page table");
}

void Engine::reset() {
    release_pages();
    seq0_ = 0;
    cache_len_ = 0;
    total_len_ = 0;
    push_state(0);
}

// Copies {cache_len, total_len, step} to the device state. Each copy reads its own slot of a
// 64-entry pinned ring, so a queued copy never sees a later update; the stream is
// synchronised whenever the ring wraps.
void Engine::push_state(int step) {
    if (h_state_slot_ == 64) {
        ck(cudaStreamSynchronize(stream_), "state ring");
        h_state_slot_ = 0;
    }
    int* h = h_state_ + 4 * h_state_slot_++;
    h[0] = (int)cache_len_;
    h[1] = (int)total_len_;
    h[2] = step;
    h[3] = 0;
    ck(cudaMemcpyAsync(dstate_, h, 4 * sizeof(int), cudaMemcpyHostToDevice, stream_), "state");
}

// ------------------------------------------------------------------ GEMV helper (chunks of 8 rows)
void Engine::gemv(const Mat& w, int pro, int epi, const __half* x, const __half* norm, __half* out,
                  const __half* resid, int M) {
    if (M >= kGemmMinRows && w.prec != kFp16 && gemm_check(M, w.K, w.N, w.G, w.prec == kInt4) == nullptr) {
        // prefill: normalise / quantise the rows once, then the tensor-core GEMM (same bits)
        const __half* xq = x;
        if (pro == kProRmsNormQuant) {
            launch_rms_norm(x, norm, gm_xn_, M, w.K, cfg_.layer_norm_eps, stream_);
            xq = gm_xn_;
            ++launches_;
        }
        launch_quantize_act(xq, gm_aq_, gm_as_, M, w.K, stream_);
        if (launch_gemm(gm_aq_, gm_as_, w.data, w.scales, out, resid, M, w.K, w.N, w.G, w.prec == kInt4 ? 1 : 0, epi,
                        stream_) != 0)
            throw std::runtime_error("gemm launch failed");
        ck(cudaGetLastError(), "gemm launch");
        launches_ += 2;
        return;
    }
    const int per = gemv_rows_per_launch(w.prec == kInt4 ? 1 : 0, pro, w.K, w.G);
    if (per == 0) throw std::runtime_error("gemv: K too large for the shared-memory tile");
    for (int m0 = 0; m0 < M; m0 += per) {
        GemvCall c = {};
        c.int4 = w.prec == kInt4 ? 1 : 0;
        c.pro = pro;
        c.epi = epi;
        c.x = x + (size_t)m0 * w.K;
        c.norm_w = norm;
        c.eps = cfg_.layer_norm_eps;
        c.w = w.data;
        c.ws = w.scales;
        const int outN = (epi == kEpiGluSilu || epi == kEpiGluGelu) ? w.N / 2 : w.N;
        c.out = out + (size_t)m0 * outN;
        c.resid = resid ? resid + (size_t)m0 * outN : nullptr;
        c.M = std::min(per, M - m0);
        c.K = w.K;
        c.N = w.N;
        c.G = w.G;
        c.pdl = use_pdl_;
        if (const char* why = gemv_check(c)) throw std::runtime_error(why);
        if (launch_gemv(c, stream_) != 0) ck(cudaGetLastError(), "gemv launch");
        ++launches_;
    }
}

// ------------------------------------------------------------------ forward
// Processes B sequences x S new tokens whose embeddings are already in hidden_ ([B*S, H]).
// `graph_mode` reads positions / cache lengths from the device state (decode graphs).
void Engine::forward(int B, int S, bool graph_mode) {
    const int rows = B * S;
    const bool cache_empty = cache_len_ == 0;
    const bool sliding = window_ > 0 && cache_len_ + S > window_;
    const int* ds = graph_mode ? dstate_ : nullptr;
    const int ng = (D_ + 127) / 128;
    const size_t kv_rows_stride = (size_t)max_rows_ * Hkv_ * D_;
    for (int l = 0; l < L_; ++l) {
        const LayerW& lw = layers_[l];
        __half* kl = kall_ + (size_t)l * kv_rows_stride;
        __half* vl = vall_ + (size_t)l * kv_rows_stride;
        // contiguous: sequence seq0_'s slot; paged: the layer's pool (rows through the table)
        const size_t slot = page_shift_ ? 0 : (size_t)seq0_;
        int8_t* kcl = kc_ + ((size_t)l * max_batch_ + slot) * cache_bstride_;
        int8_t* vcl = vc_ + ((size_t)l * max_batch_ + slot) * cache_bstride_;
        float* ksl = ks_ + ((size_t)l * max_batch_ + slot) * scale_bstride_;
        float* vsl = vs_ + ((size_t)l * max_batch_ + slot) * scale_bstride_;

        gemv(lw.qkv, kProRmsNormQuant, kEpiStore, hidden_, lw.in_norm, qkv_, nullptr, rows);
        QkvPostArgs qa = {};
        qa.qkv = qkv_;
        qa.qkv_stride = QKVN_;
        qa.q_out = q_;
        qa.k_out = kl;
        qa.v_out = vl;
        qa.q_norm = lw.q_norm;
        qa.k_norm = lw.k_norm;
        qa.eps = cfg_.layer_norm_eps;
        qa.ct = ct_[l];
        qa.st = st_[l];
        qa.pos_base = (long long)total_len_;
        qa.dstate = ds;
        qa.rows = rows;
        qa.S = S;
        qa.Hq = Hq_;
        qa.Hkv = Hkv_;
        qa.D = D_;
        launch_qkv_post(qa, stream_);
        ++launches_;

        if (cache_empty && !graph_mode) {
            // no-cache attention (QwenModel::build_attention -> gb->attention, model_qwen.cpp:100);
            // Gemma local layers pass window 512 on this path only (model_gemma.cpp:99-113)
            const long long win = (cfg_.model_type == kGemma && !is_global(l)) ? 512 : 0;
            launch_attention_f16(q_, kl, vl, attn_, B, S, S, Hq_, Hkv_, D_, attention_scale_, (long long)total_len_,
                                 win, 1, stream_);
        } else {
            // reference-order (bit-exact) hybrid attention (kernel_attention.cpp:257-482); in a
            // decode graph over a long cache the same arithmetic split over the keys
            if (graph_mode && split_graph_ && S == 1) {
                if (launch_attention_split_dev(q_, kcl, vcl, ksl, vsl, kl, vl, attn_, B, S, S, Hq_, Hkv_, D_,
                                               attention_scale_, 1, 128, cache_bstride_, scale_bstride_,
                                               (long long)cap_ + 1, ds, split_scr_, split_scr_bytes_, stream_,
                                               paging(seq0_)) != 0)
                    throw std::runtime_error("split attention launch failed");
                ++launches_;
            } else if (launch_attention_hybrid_exact(q_, kcl, vcl, ksl, vsl, kl, vl, attn_, B, S, (int)cache_len_, S, Hq_,
                                              Hkv_, D_, attention_scale_,
                                              causal_fix_ ? (long long)cache_len_ : (long long)total_len_, 1, 128,
                                              cache_bstride_, scale_bstride_, stream_, ds, paging(seq0_)) != 0)
                throw std::runtime_error("unsupported head_dim for the hybrid attention kernel");
        }
        ck(cudaGetLastError(), "attention launch");
        ++launches_;
        update_kv(l, B, S, kl, vl, kcl, vcl, ksl, vsl, graph_mode, sliding, cache_empty);

        if (cfg_.model_type == kGemma) {
            gemv(lw.o, kProQuant, kEpiStore, attn_, nullptr, tmp_o_, nullptr, rows);
            launch_norm_add_clipped(hidden_, tmp_o_, lw.post_attn_norm, rows, H_, cfg_.layer_norm_eps, stream_);
            ++launches_;
            gemv(lw.gateup, kProRmsNormQuant, kEpiGluGelu, hidden_, lw.pre_ffn_norm, gated_, nullptr, rows);
            gemv(lw.down, kProQuant, kEpiStore, gated_, nullptr, tmp_o_, nullptr, rows);
            launch_norm_add_clipped(hidden_, tmp_o_, lw.post_ffn_norm, rows, H_, cfg_.layer_norm_eps, stream_);
            ++launches_;
        } else {
            gemv(lw.o, kProQuant, kEpiResidual, attn_, nullptr, hidden_, hidden_, rows);
            gemv(lw.gateup, kProRmsNormQuant, kEpiGluSilu, hidden_, lw.post_attn_norm, gated_, nullptr, rows);
            gemv(lw.down, kProQuant, kEpiResidual, gated_, nullptr, hidden_, hidden_, rows);
        }
    }
    (void)ng;
}

// KVCache::update_from_graph (engine_cache.cpp:101-337) for one layer: quantise the new
// tokens' keys/values into the cache; with a sliding window keep `sink_` sink tokens plus
// the most recent tokens, as the reference does.
void Engine::update_kv(int l, int B, int S, const __half* kl, const __half* vl, int8_t* kcl, int8_t* vcl, float* ksl,
                       float* vsl, bool graph_mode, bool sliding, bool cache_empty) {
    KvAppendArgs a = {};
    a.k_new = kl;
    a.v_new = vl;
    a.k_cache = kcl;
    a.v_cache = vcl;
    a.k_scales = ksl;
    a.v_scales = vsl;
    a.cache_bstride = cache_bstride_;
    a.scale_bstride = scale_bstride_;
    a.B = B;
    a.S = S;
    a.Hkv = Hkv_;
    a.D = D_;
    a.G = 128;
    a.pg = paging(seq0_);
    if (graph_mode) {  // non-sliding append at cache_len (checked by the caller)
        a.src_tok0 = 0;
        a.ntok = S;
        a.dstate = dstate_;
        launch_kv_append(a, stream_);
        ++launches_;
        return;
    }
    if (!sliding) {
        a.src_tok0 = 0;
        a.ntok = S;
        a.dst0 = (long long)cache_len_;
        launch_kv_append(a, stream_);
        ++launches_;
        return;
    }
    launches_ += 2;
    const int ng = (D_ + 127) / 128;
    const size_t tok_bytes = (size_t)Hkv_ * D_, tok_scales = (size_t)Hkv_ * ng;
    if (cache_empty) {
        // first branch: the graph output holds the whole sequence (engine_cache.cpp:172-231)
        const size_t new_total = cache_len_ + S;
        const size_t skip = new_total - window_;
        a.src_tok0 = 0;
        a.ntok = (int)std::min(sink_, (size_t)S);
        a.dst0 = 0;
        launch_kv_append(a, stream_);
        a.src_tok0 = (int)(sink_ + skip);
        a.ntok = (int)(window_ - sink_);
        a.dst0 = (long long)sink_;
        launch_kv_append(a, stream_);
        return;
    }
    // incremental branch (engine_cache.cpp:267-329)
    const long long tts = (long long)window_ - (long long)sink_ - S;
    const size_t old = cache_len_;
    if (tts > 0 && old > sink_) {
        const long long shift_src = (long long)old - tts;
        if (shift_src > (long long)sink_ && page_shift_) {
            for (int b = 0; b < B; ++b) {
                KvMoveArgs mv = {};
                mv.k_cache = kcl;
                mv.v_cache = vcl;
                mv.k_scales = ksl;
                mv.v_scales = vsl;
                mv.tmp = tmp_kv_;
                mv.pg = paging(seq0_);
                mv.b = b;
                mv.Hkv = Hkv_;
                mv.D = D_;
                mv.ng = ng;
                mv.src0 = shift_src;
                mv.dst0 = (long long)sink_;
                mv.n = tts;
                launch_kv_move_paged(mv, stream_);
            }
        } else if (shift_src > (long long)sink_) {
            for (int b = 0; b < B; ++b) {
                for (int which = 0; which < 2; ++which) {
                    int8_t* c = (which ? vcl : kcl) + (size_t)b * cache_bstride_;
                    float* sc = (which ? vsl : ksl) + (size_t)b * scale_bstride_;
                    const long long nb = tts * (long long)tok_bytes, ns = tts * (long long)tok_scales * 4;
                    launch_copy_bytes(tmp_kv_, c + shift_src * tok_bytes, nb, stream_);
                    launch_copy_bytes(c + sink_ * tok_bytes, tmp_kv_, nb, stream_);
                    launch_copy_bytes(tmp_kv_, sc + shift_src * tok_scales, ns, stream_);
                    launch_copy_bytes(sc + sink_ * tok_scales, tmp_kv_, ns, stream_);
                }
            }
        }
    }
    a.src_tok0 = 0;
    a.ntok = S;
    a.dst0 = (long long)(window_ - S);
    launch_kv_append(a, stream_);
}

void Engine::advance(int S) {
    const size_t new_total = cache_len_ + S;
    cache_len_ = (window_ > 0 && new_total > window_) ? window_ : new_total;
    total_len_ += S;
}

void Engine::embed(const uint32_t* d_ids, int n, __half* out) {
    EmbedArgs e = {};
    e.table = embed_.data;
    e.scales = embed_.scales;
    e.prec = embed_.prec;
    e.G = embed_.G;
    e.hidden = H_;
    e.ids = d_ids;
    e.n = n;
    e.out = out;
    if (cfg_.model_type == kGemma) {  // hidden * sqrt(hidden_dim) (model_gemma.cpp:173-174)
        e.has_scale = 1;
        e.scale16 = __float2half_rn(std::sqrt((float)H_));
    }
    launch_embed(e, stream_);
    ++launches_;
}

// final norm + lm_head on rows `last_rows` ([B, H]) -> logits_ [B, V]
void Engine::lm_head(const __half* last_rows, int B) {
    if (lm_.prec == kFp16) {
        launch_rms_norm(last_rows, out_norm_, xnorm_, B, H_, cfg_.layer_norm_eps, stream_);
        launch_matmul_f16(xnorm_, static_cast<const __half*>(lm_.data), logits_, B, H_, V_, stream_);
        launches_ += 2;
    } else {
        gemv(lm_, kProRmsNormQuant, kEpiStore, last_rows, out_norm_, logits_, nullptr, B);
    }
}

void Engine::check_tokens(const uint32_t* t, size_t n) const {
    for (size_t i = 0; i < n; ++i)
        if (t[i] >= (uint32_t)embed_.N)
            throw std::runtime_error("Embedding index out of bounds: " + std::to_string(t[i]) +
                                     " >= " + std::to_string(embed_.N));
}

void Engine::run_forward_tokens(const uint32_t* tokens, int B, int S) {
    if (B * S > max_rows_) throw std::runtime_error("too many rows for the engine buffers");
    if (cache_len_ + S > cap_) throw std::runtime_error("KV cache capacity exceeded");
    check_tokens(tokens, (size_t)B * S);
    // rows this forward writes: the cache grows to cache_len + S, or to the window once it slides
    ensure_pages(seq0_, B, window_ > 0 ? std::min(cache_len_ + S, window_) : cache_len_ + S);
    ck(cudaMemcpyAsync(ids_, tokens, (size_t)B * S * 4, cudaMemcpyHostToDevice, stream_), "ids");
    embed(ids_, B * S, hidden_);
    forward(B, S, false);
    advance(S);
}

// Model::prefill (engine_model.cpp:170-219)
void Engine::prefill(const uint32_t* tokens, size_t n, size_t chunk) {
    if (n == 0) return;
    pdl_scope pdl(use_pdl_);
    if (chunk == 0) chunk = 256;
    chunk = std::min(chunk, (size_t)max_rows_);
    if (n <= chunk) {
        run_forward_tokens(tokens, 1, (int)n);
    } else {
        const size_t full = (n - 1) / chunk;
        for (size_t c = 0; c < full; ++c) run_forward_tokens(tokens + c * chunk, 1, (int)chunk);
        run_forward_tokens(tokens + full * chunk, 1, (int)(n - full * chunk));
    }
    push_state(0);
}

// rows b*S + S-1 of hidden_ -> last_
void Engine::gather_last(int B, int S) {
    if (S == 1) {
        ck(cudaMemcpyAsync(last_, hidden_, (size_t)B * H_ * 2, cudaMemcpyDeviceToDevice, stream_), "last");
    } else {
        ck(cudaMemcpy2DAsync(last_, (size_t)H_ * 2, hidden_ + (size_t)(S - 1) * H_, (size_t)S * H_ * 2,
                             (size_t)H_ * 2, B, cudaMemcpyDeviceToDevice, stream_),
           "last rows");
    }
}

// The reference keeps one process-wide repetition-penalty history of the last 128 sampled
// tokens (kernel_nn.cpp:498-513), appended only on the sampling path.
static std::mutex g_hist_mu;
static std::vector<uint32_t> g_history;

// Model::decode (engine_model.cpp:221-297): defaulting rule, forward, lm_head on the last
// row, optional normalised entropy, then greedy argmax or device sampling with a uniform
// sample from std::mt19937 seeded by the clock (graph_builder.cpp:408).
uint32_t Engine::decode(const uint32_t* tokens, size_t n, float temperature, float top_p, size_t top_k, float* entropy) {
    if (temperature < 0) temperature = cfg_.default_temperature;
    if (top_p < 0) top_p = cfg_.default_top_p;
    if (top_k == 0) top_k = cfg_.default_top_k;
    const bool greedy = temperature == 0.0f && top_p <= 0.0f && top_k == 0;
    if (greedy) return decode_argmax(tokens, n, entropy);
    pdl_scope pdl(use_pdl_);
    if (n == 0) throw std::runtime_error("Token sequence cannot be empty");
    run_forward_tokens(tokens, 1, (int)n);
    gather_last(1, (int)n);
    lm_head(last_, 1);
    if (entropy) launch_entropy(logits_, V_, f32_scratch_, stream_);
    std::vector<uint32_t> hist;
    {
        std::lock_guard<std::mutex> lk(g_hist_mu);
        hist = g_history;
    }
    if (!hist.empty())
        ck(cudaMemcpyAsync(hist_dev_, hist.data(), hist.size() * 4, cudaMemcpyHostToDevice, stream_), "history");
    std::mt19937 gen((uint32_t)std::chrono::high_resolution_clock::now().time_since_epoch().count());
    std::uniform_real_distribution<float> dist(0.0f, 1.0f);
    const float u = dist(gen);
    launch_sample(logits_, V_, temperature, top_p, (int)top_k, u, hist_dev_, (int)hist.size(), sample_work_,
                  tok_in_, stream_);
    launches_ += entropy ? 2 : 1;
    push_state(0);
    uint32_t tok = 0;
    float ent = 0.0f;
    ck(cudaMemcpyAsync(&tok, tok_in_, 4, cudaMemcpyDeviceToHost, stream_), "token");
    if (entropy) ck(cudaMemcpyAsync(&ent, f32_scratch_, 4, cudaMemcpyDeviceToHost, stream_), "entropy");
    ck(cudaStreamSynchronize(stream_), "decode");
    if (entropy) *entropy = ent;
    {
        std::lock_guard<std::mutex> lk(g_hist_mu);
        g_history.push_back(tok);
        if (g_history.size() > 128) g_history.erase(g_history.begin());
    }
    return tok;
}

uint32_t Engine::decode_argmax(const uint32_t* tokens, size_t n, float* entropy) {
    if (n == 0) throw std::runtime_error("Token sequence cannot be empty");
    pdl_scope pdl(use_pdl_);
    run_forward_tokens(tokens, 1, (int)n);
    gather_last(1, (int)n);
    lm_head(last_, 1);
    launch_argmax_rows(logits_, 1, V_, tok_in_, nullptr, 0, nullptr, stream_);
    if (entropy) launch_entropy(logits_, V_, f32_scratch_, stream_);
    launches_ += entropy ? 2 : 1;
    push_state(0);
    uint32_t tok = 0;
    float ent = 0.0f;
    ck(cudaMemcpyAsync(&tok, tok_in_, 4, cudaMemcpyDeviceToHost, stream_), "token");
    if (entropy) ck(cudaMemcpyAsync(&ent, f32_scratch_, 4, cudaMemcpyDeviceToHost, stream_), "entropy");
    ck(cudaStreamSynchronize(stream_), "decode");
    if (entropy) *entropy = ent;
    return tok;
}

// One decode step of B sequences whose input tokens are in tok_in_ (device); appends the
// argmax token to ring[b*ring_stride + step] and feeds it back into tok_in_.
void Engine::decode_step_device(int B, uint32_t* ring, int ring_stride, bool graph_mode) {
    embed(tok_in_, B, hidden_);
    forward(B, 1, graph_mode);
    lm_head(hidden_, B);
    launch_argmax_rows(logits_, B, V_, tok_in_, ring, ring_stride, dstate_, stream_);
    launch_state_advance(dstate_, 1, stream_);
    launches_ += 2;
}

void Engine::generate(const uint32_t* prompts, int B, size_t P, size_t max_new, uint32_t* out) {
    if (B < 1 || B > max_batch_) throw std::runtime_error("batch exceeds max_batch");
    if (P == 0) throw std::runtime_error("Cannot generate from empty prompt");
    if (max_new == 0) return;
    pdl_scope pdl(use_pdl_);
    reset();
    check_tokens(prompts, (size_t)B * P);
    if (P + max_new > cap_ + 1) throw std::runtime_error("prompt + max_new exceeds the KV cache capacity");
    if (!ev_[0])
        for (auto& e : ev_) ck(cudaEventCreate(&e), "event");
    const long long launches0 = launches_;
    long long replays = 0;
    ck(cudaEventRecord(ev_[0], stream_), "event");
    // prefill prompt[:-1] of every sequence as Model::prefill does it for one sequence
    // (engine_model.cpp:170-219): chunks of 256 tokens, each sequence into its own cache slot,
    // so every sequence sees the reference's chunking whatever the batch size
    if (P > 1) {
        const size_t pre = P - 1;
        const size_t chunk = std::min<size_t>(256, (size_t)max_rows_);
        const size_t full = pre > chunk ? (pre - 1) / chunk : 0;
        for (int b = 0; b < B; ++b) {
            cache_len_ = 0;
            total_len_ = 0;
            seq0_ = b;
            for (size_t c = 0; c <= full; ++c) {
                const size_t s0 = c * chunk;
                const size_t sl = (c == full) ? pre - s0 : chunk;
                run_forward_tokens(prompts + (size_t)b * P + s0, 1, (int)sl);
            }
        }
        seq0_ = 0;
    }
    // last prompt token of each sequence -> tok_in_
    std::vector<uint32_t> last(B);
    for (int b = 0; b < B; ++b) last[b] = prompts[(size_t)b * P + P - 1];
    ck(cudaMemcpyAsync(tok_in_, last.data(), (size_t)B * 4, cudaMemcpyHostToDevice, stream_), "tok_in");
    ck(cudaEventRecord(ev_[1], stream_), "event");
    // output ring
    const size_t ring_bytes = (size_t)B * max_new * 4;
    if (ring_bytes > ring_cap_) {
        if (ring_) cudaFree(ring_);
        ck(cudaMalloc(&ring_, ring_bytes), "ring");
        ring_cap_ = ring_bytes;
    }
    push_state(0);
    const bool no_slide = cache_len_ > 0 && (window_ == 0 || cache_len_ + max_new <= window_) &&
                          cache_len_ + max_new <= cap_;
    // pages for every row the decode steps write (the device-side decode paths append rows
    // without returning to the host)
    ensure_pages(0, B, window_ > 0 ? std::min(cache_len_ + max_new, window_) : std::min(cache_len_ + max_new, cap_));
    const bool can_graph = use_graph_ && no_slide;
    const bool can_persist = use_persistent_ && pplan_.ok && no_slide && B == 1;
    size_t step = 0;
    if (can_persist) {
        pargs_.ring = ring_;
        ck(cudaMemsetAsync(psync_, 0, sizeof(PSync), stream_), "persistent sync");
        for (; step < max_new; ++step) {
            pargs_.tag_base = ptag_base_;  // every launch writes new versions of the tagged words
            ptag_base_ = (ptag_base_ + ptag_span(L_)) % 65535u;
            ck(launch_persistent_decode(pargs_, pplan_, stream_), "persistent decode");
        }
        cache_len_ += max_new;
        total_len_ += max_new;
        launches_ += (long long)max_new;
        last_path_ = 2;
    } else if (!can_graph) {
        last_path_ = 0;
        for (; step < max_new; ++step) {
            // host-driven step: positions from the host mirror
            if (cache_len_ + 1 > cap_) throw std::runtime_error("KV cache capacity exceeded");
            embed(tok_in_, B, hidden_);
            forward(B, 1, false);
            lm_head(hidden_, B);
            launch_argmax_rows(logits_, B, V_, tok_in_, ring_, (int)max_new, dstate_, stream_);
            advance(1);
            launch_state_advance(dstate_, 1, stream_);  // keeps the device step counter in sync
            launches_ += 2;
        }
    } else {
        // long caches decode through the key-split attention (two kernels, exact); the choice is
        // part of the captured graph
        const bool want_split = split_scr_ && (long long)cache_len_ + 1 >= kSplitMinKeys &&
                                attention_split_scratch_bytes((long long)B * Hq_, (long long)cap_ + 1) <= split_scr_bytes_;
        if (!graph_exec_ || graph_batch_ != B || graph_ring_ != ring_ || graph_ring_stride_ != (int)max_new ||
            graph_split_ != want_split) {
            if (graph_exec_) {
                cudaGraphExecDestroy(graph_exec_);
                graph_exec_ = nullptr;
            }
            cudaGraph_t g = nullptr;
            split_graph_ = want_split;
            ck(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal), "capture");
            try {
                decode_step_device(B, ring_, (int)max_new, true);
            } catch (...) {
                split_graph_ = false;
                cudaStreamEndCapture(stream_, &g);
                if (g) cudaGraphDestroy(g);
                throw;
            }
            ck(cudaStreamEndCapture(stream_, &g), "end capture");
            split_graph_ = false;
            graph_split_ = want_split;
            ck(cudaGraphInstantiate(&graph_exec_, g, 0), "instantiate");
            ck(cudaGraphGetNodes(g, nullptr, &graph_nodes_), "graph nodes");
            cudaGraphDestroy(g);
            graph_batch_ = B;
            graph_ring_ = ring_;
            graph_ring_stride_ = (int)max_new;
        }
        last_path_ = 1;
        const long long before = launches_;
        for (; step < max_new; ++step) ck(cudaGraphLaunch(graph_exec_, stream_), "graph launch");
        replays = (long long)max_new;
        cache_len_ += max_new;
        total_len_ += max_new;
        launches_ = before + (long long)graph_nodes_ * replays;
    }
    ck(cudaEventRecord(ev_[2], stream_), "event");
    for (int b = 0; b < B; ++b)
        ck(cudaMemcpyAsync(out + (size_t)b * max_new, ring_ + (size_t)b * max_new, max_new * 4, cudaMemcpyDeviceToHost,
                           stream_),
           "tokens out");
    ck(cudaStreamSynchronize(stream_), "generate");
    if (last_path_ == 2) {
        PSync ps;
        ck(cudaMemcpy(&ps, psync_, sizeof(ps), cudaMemcpyDeviceToHost), "persistent sync");
        if (ps.abort) {
            // words of the abandoned launch must not pass for a later version
            ck(cudaMemset(ptagged_, 0, ptagged_words_ * 4), "persistent activations");
            throw std::runtime_error("persistent decode step gave up a bounded wait (device error recorded)");
        }
    }
    float a = 0, b = 0;
    ck(cudaEventElapsedTime(&a, ev_[0], ev_[1]), "elapsed");
    ck(cudaEventElapsedTime(&b, ev_[1], ev_[2]), "elapsed");
    last_prefill_ms_ = a;
    last_decode_ms_ = b;
    last_launches_ = launches_ - launches0;
    last_graph_replays_ = replays;
}

void Engine::last_logits(uint16_t* host, size_t vocab) {
    if (vocab > (size_t)V_) vocab = V_;
    ck(cudaMemcpyAsync(host, logits_, vocab * 2, cudaMemcpyDeviceToHost, stream_), "logits");
    ck(cudaStreamSynchronize(stream_), "logits");
}

void Engine::read_kv(size_t layer, int8_t* k, int8_t* v, float* ks, float* vs) {
    if (layer >= (size_t)L_) throw std::runtime_error("layer out of range");
    const int ng = (D_ + 127) / 128;
    const size_t nb = cache_len_ * Hkv_ * D_, ns = cache_len_ * Hkv_ * ng;
    const size_t lo = layer * max_batch_;
    if (page_shift_) {  // sequence 0's rows, page by page through the table
        const size_t P = (size_t)1 << page_shift_, rb = (size_t)Hkv_ * D_, rs = (size_t)Hkv_ * ng;
        for (size_t r0 = 0; r0 < cache_len_; r0 += P) {
            const size_t n = std::min(P, cache_len_ - r0), pr = (size_t)htable_[r0 >> page_shift_] << page_shift_;
            ck(cudaMemcpyAsync(k + r0 * rb, kc_ + lo * cache_bstride_ + pr * rb, n * rb, cudaMemcpyDeviceToHost, stream_), "kv");
            ck(cudaMemcpyAsync(v + r0 * rb, vc_ + lo * cache_bstride_ + pr * rb, n * rb, cudaMemcpyDeviceToHost, stream_), "kv");
            ck(cudaMemcpyAsync(ks + r0 * rs, ks_ + lo * scale_bstride_ + pr * rs, n * rs * 4, cudaMemcpyDeviceToHost,
                               stream_), "kv");
            ck(cudaMemcpyAsync(vs + r0 * rs, vs_ + lo * scale_bstride_ + pr * rs, n * rs * 4, cudaMemcpyDeviceToHost,
                               stream_), "kv");
        }
        ck(cudaStreamSynchronize(stream_), "read kv");
        return;
    }
    ck(cudaMemcpyAsync(k, kc_ + lo * cache_bstride_, nb, cudaMemcpyDeviceToHost, stream_), "kv");
    ck(cudaMemcpyAsync(v, vc_ + lo * cache_bstride_, nb, cudaMemcpyDeviceToHost, stream_), "kv");
    ck(cudaMemcpyAsync(ks, ks_ + lo * scale_bstride_, ns * 4, cudaMemcpyDeviceToHost, stream_), "kv");
    ck(cudaMemcpyAsync(vs, vs_ + lo * scale_bstride_, ns * 4, cudaMemcpyDeviceToHost, stream_), "kv");
    ck(cudaStreamSynchronize(stream_), "read kv");
}

}  // namespace eng
}  // namespace cb

// ==================================================================== C ABI
namespace {
thread_local std::string g_engine_error;
cb::eng::Engine* E(cactus_engine_t h) { return static_cast<cb::eng::Engine*>(h); }
template <class F>
int guarded(F&& f) {
    try {
        f();
        return CB_OK;
    } catch (const std::exception& e) {
        g_engine_error = e.what();
        return CB_ERR_ARG;
    }
}
}  // namespace

extern "C" {

CB_API const char* cactus_engine_last_error(void) { return g_engine_error.c_str(); }

CB_API cactus_engine_t cactus_engine_create(const char* model_folder, size_t context_size, size_t max_batch,
                                            int device) {
    if (!model_folder) {
        g_engine_error = "model_folder is NULL";
        return nullptr;
    }
    auto* e = new cb::eng::Engine();
    try {
        e->init(model_folder, context_size ? context_size : 512, max_batch, device);
        return e;
    } catch (const std::exception& ex) {
        g_engine_error = ex.what();
        delete e;
        return nullptr;
    }
}

CB_API void cactus_engine_destroy(cactus_engine_t engine) {
    if (engine) {
        cudaSetDevice(E(engine)->device());
        delete E(engine);
    }
}

CB_API int cactus_engine_reset(cactus_engine_t engine) {
    if (!engine) return CB_ERR_ARG;
    return guarded([&] { E(engine)->reset(); });
}

CB_API int cactus_engine_set_cache_window(cactus_engine_t engine, size_t window_size, size_t sink_size) {
    if (!engine) return CB_ERR_ARG;
    return guarded([&] { E(engine)->set_window(window_size, sink_size); });
}

CB_API int cactus_engine_set_causal_fix(cactus_engine_t engine, int on) {
    if (!engine) return CB_ERR_ARG;
    return guarded([&] { E(engine)->set_causal_fix(on != 0); });
}

CB_API int cactus_engine_info(cactus_engine_t engine, uint32_t* out8) {
    if (!engine || !out8) return CB_ERR_ARG;
    E(engine)->info(out8);
    return CB_OK;
}

CB_API int cactus_engine_prefill(cactus_engine_t engine, const uint32_t* tokens, size_t n, size_t chunk_size) {
    if (!engine || (!tokens && n)) return CB_ERR_ARG;
    return guarded([&] {
        cudaSetDevice(E(engine)->device());
        E(engine)->prefill(tokens, n, chunk_size);
    });
}

CB_API int cactus_engine_decode(cactus_engine_t engine, const uint32_t* tokens, size_t n, float temperature,
                                float top_p, size_t top_k, uint32_t* out_token, float* out_entropy) {
    if (!engine || !tokens || !out_token) return CB_ERR_ARG;
    return guarded([&] {
        cudaSetDevice(E(engine)->device());
        *out_token = E(engine)->decode(tokens, n, temperature, top_p, top_k, out_entropy);
    });
}

CB_API int cactus_engine_generate_greedy(cactus_engine_t engine, const uint32_t* prompt, size_t n, size_t max_new,
                                         uint32_t* out_tokens) {
    if (!engine || !prompt || (!out_tokens && max_new)) return CB_ERR_ARG;
    return guarded([&] {
        cudaSetDevice(E(engine)->device());
        E(engine)->generate(prompt, 1, n, max_new, out_tokens);
    });
}

CB_API int cactus_engine_generate_batch_greedy(cactus_engine_t engine, const uint32_t* prompts, size_t batch,
                                               size_t prompt_len, size_t max_new, uint32_t* out_tokens) {
    if (!engine || !prompts || (!out_tokens && max_new)) return CB_ERR_ARG;
    return guarded([&] {
        cudaSetDevice(E(engine)->device());
        E(engine)->generate(prompts, (int)batch, prompt_len, max_new, out_tokens);
    });
}

CB_API int cactus_engine_last_logits(cactus_engine_t engine, uint16_t* host_logits, size_t vocab) {
    if (!engine || !host_logits) return CB_ERR_ARG;
    return guarded([&] { E(engine)->last_logits(host_logits, vocab); });
}

CB_API int cactus_engine_stats(cactus_engine_t engine, double* out8) {
    if (!engine || !out8) return CB_ERR_ARG;
    E(engine)->stats(out8);
    return CB_OK;
}

CB_API int cactus_engine_decode_path(cactus_engine_t engine, int mode) {
    if (!engine) return -1;
    if (mode == -1) E(engine)->use_persistent_ = true;
    if (mode == 1) E(engine)->use_persistent_ = false;
    return E(engine)->last_path_;
}

CB_API int cactus_engine_kv_state(cactus_engine_t engine, size_t* out2) {
    if (!engine || !out2) return CB_ERR_ARG;
    out2[0] = E(engine)->cache_len();
    out2[1] = E(engine)->total_len();
    return CB_OK;
}

CB_API int cactus_engine_read_kv(cactus_engine_t engine, size_t layer, int8_t* keys, int8_t* values, float* k_scales,
                                 float* v_scales) {
    if (!engine || !keys || !values || !k_scales || !v_scales) return CB_ERR_ARG;
    return guarded([&] { E(engine)->read_kv(layer, keys, values, k_scales, v_scales); });
}

}  // extern "C"
