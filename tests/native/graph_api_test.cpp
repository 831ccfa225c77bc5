// CactusGraph API test program (built and run by tests/test_graph_gpu.py).
//
// Part 1 restates the known answers of the reference's graph tests (tests/test_graph.cpp:
// matrix multiplication :75-90, transpose :92-104, reshape :106-118, RMS norm :176-204,
// softmax :206-218, attention :220-240, embedding :778-816, embedding from file :818-864)
// through the B200 graph. Part 2 builds a quantized attention block from .weights files in
// <dir> and writes every node the Python side compares against the oracle to <dir>/*.bin.
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <string>
#include <vector>

#include "cactus/graph.h"

namespace {
// IEEE binary16 <-> binary32 on the host (round to nearest even)
uint16_t f2h(float f) {
    uint32_t x;
    std::memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t absx = x & 0x7FFFFFFFu;
    if (absx >= 0x7F800000u) return (uint16_t)(sign | (absx > 0x7F800000u ? 0x7E00u : 0x7C00u));
    if (absx >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u);  // rounds past 65504
    if (absx < 0x38800000u) {                                    // subnormal half
        const int shift = 113 - (int)(absx >> 23);
        if (shift > 24) return (uint16_t)sign;
        const uint32_t mant = (absx & 0x7FFFFFu) | 0x800000u;
        uint32_t h = mant >> (shift + 13);
        const uint32_t rem = mant & ((1u << (shift + 13)) - 1);
        const uint32_t half = 1u << (shift + 12);
        if (rem > half || (rem == half && (h & 1))) ++h;
        return (uint16_t)(sign | h);
    }
    uint32_t h = ((absx - 0x38000000u) >> 13);
    const uint32_t rem = absx & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1))) ++h;
    return (uint16_t)(sign | h);
}
float h2f(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t e = (h >> 10) & 0x1F, m = h & 0x3FF;
    uint32_t x;
    if (e == 0) {
        if (m == 0) {
            x = sign;
        } else {
            float f = std::ldexp((float)m, -24);
            std::memcpy(&x, &f, 4);
            x |= sign;
        }
    } else if (e == 31) {
        x = sign | 0x7F800000u | (m << 13);
    } else {
        x = sign | ((e + 112) << 23) | (m << 13);
    }
    float f;
    std::memcpy(&f, &x, 4);
    return f;
}
std::vector<uint16_t> H(const std::vector<float>& v) {
    std::vector<uint16_t> o;
    for (float f : v) o.push_back(f2h(f));
    return o;
}

int failures = 0;
void report(const char* name, bool ok) {
    std::printf("%s %s\n", ok ? "PASS" : "FAIL", name);
    if (!ok) ++failures;
}
bool close_h(const void* out, const std::vector<float>& exp, float tol) {
    const uint16_t* o = static_cast<const uint16_t*>(out);
    for (size_t i = 0; i < exp.size(); ++i)
        if (!(std::fabs(h2f(o[i]) - exp[i]) <= tol)) {
            std::printf("  index %zu: got %g expected %g\n", i, h2f(o[i]), exp[i]);
            return false;
        }
    return true;
}
template <class F>
bool throws(F f) {
    try {
        f();
    } catch (const std::exception&) {
        return true;
    }
    return false;
}
void dump(CactusGraph& g, size_t node, const std::string& path) {
    const BufferDesc& b = g.get_output_buffer(node);
    const void* p = g.get_output(node);
    std::ofstream f(path, std::ios::binary);
    f.write(static_cast<const char*>(p), (std::streamsize)b.byte_size);
}
std::vector<uint16_t> read_f16(const std::string& path, size_t n) {
    std::vector<uint16_t> v(n);
    std::ifstream f(path, std::ios::binary);
    f.read(reinterpret_cast<char*>(v.data()), (std::streamsize)(n * 2));
    if (!f) throw std::runtime_error("cannot read " + path);
    return v;
}

void known_answers(const std::string& dir) {
    {
        CactusGraph g;
        size_t a = g.input({2, 3}, Precision::FP16), b = g.input({3, 2}, Precision::FP16);
        size_t c = g.matmul(a, b, false);
        auto da = H({1, 2, 3, 4, 5, 6});
        g.set_input(a, da.data(), Precision::FP16);
        g.set_input(b, da.data(), Precision::FP16);
        g.execute();
        report("matmul_f16", close_h(g.get_output(c), {22, 28, 49, 64}, 0.0f));
    }
    {
        CactusGraph g;
        size_t a = g.input({2, 3}, Precision::FP16);
        size_t t = g.transpose(a);
        size_t r = g.reshape(a, {3, 2});
        auto da = H({1, 2, 3, 4, 5, 6});
        g.set_input(a, da.data(), Precision::FP16);
        g.execute();
        report("transpose", close_h(g.get_output(t), {1, 4, 2, 5, 3, 6}, 0.0f));
        report("reshape", close_h(g.get_output(r), {1, 2, 3, 4, 5, 6}, 0.0f) &&
                              g.get_output_buffer(r).shape == std::vector<size_t>({3, 2}));
    }
    {
        CactusGraph g;
        size_t a = g.input({1, 8}, Precision::FP16), w = g.input({8}, Precision::FP16);
        size_t n = g.rms_norm(a, w);
        std::vector<float> x = {1, 2, 3, 4, 5, 6, 7, 8};
        auto dx = H(x), dw = H({1, 1, 1, 1, 1, 1, 1, 1});
        g.set_input(a, dx.data(), Precision::FP16);
        g.set_input(w, dw.data(), Precision::FP16);
        g.execute();
        float ss = 0;
        for (float v : x) ss += v * v;
        const float inv = 1.0f / std::sqrt(ss / 8.0f + 1e-5f);
        std::vector<float> e;
        for (float v : x) e.push_back(v * inv);
        report("rms_norm", close_h(g.get_output(n), e, 0.01f));
    }
    {
        CactusGraph g;
        size_t a = g.input({2, 3}, Precision::FP16);
        size_t s = g.softmax(a, -1);
        auto d = H({1, 2, 3, 4, 5, 6});
        g.set_input(a, d.data(), Precision::FP16);
        g.execute();
        report("softmax", close_h(g.get_output(s), {0.09003f, 0.24473f, 0.66524f, 0.09003f, 0.24473f, 0.66524f}, 0.01f));
    }
    {
        CactusGraph g;
        size_t q = g.input({1, 2, 1, 4}, Precision::FP16), k = g.input({1, 2, 1, 4}, Precision::FP16),
               v = g.input({1, 2, 1, 4}, Precision::FP16);
        size_t o = g.attention(q, k, v, 0.5f);
        auto dq = H({1, 0, 0, 0, 0, 1, 0, 0}), dv = H({1, 2, 3, 4, 5, 6, 7, 8});
        g.set_input(q, dq.data(), Precision::FP16);
        g.set_input(k, dq.data(), Precision::FP16);
        g.set_input(v, dv.data(), Precision::FP16);
        g.execute();
        // head_dim 4 < 8: the reference accumulates V only over head_dim rounded down to a
        // multiple of 8 and writes zeros past it (kernel_attention.cpp:203-245), so every
        // output is 0
        report("attention_head_dim_4", close_h(g.get_output(o), std::vector<float>(8, 0.0f), 0.0f));
    }
    {
        CactusGraph g;
        size_t q = g.input({1, 2, 1, 8}, Precision::FP16), k = g.input({1, 2, 1, 8}, Precision::FP16),
               v = g.input({1, 2, 1, 8}, Precision::FP16);
        size_t o = g.attention(q, k, v, 0.5f);
        std::vector<float> qf(16, 0.0f), vf(16);
        qf[0] = 1;
        qf[9] = 1;
        for (int i = 0; i < 16; ++i) vf[i] = (float)(i + 1);
        auto dq = H(qf), dv = H(vf);
        g.set_input(q, dq.data(), Precision::FP16);
        g.set_input(k, dq.data(), Precision::FP16);
        g.set_input(v, dv.data(), Precision::FP16);
        g.execute();
        // causal: token 0 sees key 0 only; token 1 weighs keys 0/1 by softmax(0, 0.5)
        const float w1 = 1.0f / (1.0f + std::exp(-0.5f)), w0 = 1.0f - w1;
        std::vector<float> e(vf.begin(), vf.begin() + 8);
        for (int d = 0; d < 8; ++d) e.push_back(w0 * vf[d] + w1 * vf[8 + d]);
        report("attention_head_dim_8", close_h(g.get_output(o), e, 0.02f));
    }
    {
        CactusGraph g;
        size_t emb = g.input({4, 3}, Precision::INT8), idx = g.input({2, 2}, Precision::INT8);
        size_t e = g.embedding(emb, idx);
        std::vector<int8_t> table = {1, 5, 9, 2, 6, 10, 3, 7, 11, 4, 8, 12}, ids = {0, 2, 3, 1};
        g.set_input(emb, table.data(), Precision::INT8);
        g.set_input(idx, ids.data(), Precision::INT8);
        g.execute();
        report("embedding_int8", close_h(g.get_output(e), {1, 5, 9, 3, 7, 11, 4, 8, 12, 2, 6, 10}, 0.0f) &&
                                     g.get_output_buffer(e).shape == std::vector<size_t>({2, 2, 3}));
    }
    {
        CactusGraph g;
        size_t idx = g.input({3}, Precision::INT8);
        size_t e = g.embedding(dir + "/emb_f16.weights", idx);
        std::vector<int8_t> ids = {2, 0, 3};
        g.set_input(idx, ids.data(), Precision::INT8);
        g.execute();
        report("embedding_from_file", close_h(g.get_output(e), {3, 7, 11, 1, 5, 9, 4, 8, 12}, 0.01f));
        std::vector<int8_t> bad = {2, 9, 3};
        g.set_input(idx, bad.data(), Precision::INT8);
        report("embedding_out_of_range_throws", throws([&] { g.execute(); }));
    }
    {
        CactusGraph g;
        size_t a = g.input({2, 3}, Precision::FP16), b = g.input({4, 3}, Precision::FP16);
        report("matmul_shape_mismatch_throws", throws([&] { g.matmul(a, b, false); }));
        report("index_out_of_bounds_throws", throws([&] { g.index(a, 2, 0); }));
        report("quantize_requires_fp16", throws([&] { g.quantize_activations(g.input({2, 2}, Precision::INT8)); }));
        size_t w = g.mmap_weights(dir + "/wq.weights");
        report("mmap_weights_cached", g.mmap_weights(dir + "/wq.weights") == w);
        size_t x = g.input({2, 128}, Precision::FP16);
        report("grouped_int8_requires_pretransposed", throws([&] {
                   g.matmul(x, w, false);
                   g.execute();
               }));
    }
}

// quantized attention block: the composition the Python side restates with the oracle
void block(const std::string& dir) {
    const size_t M = 3, K = 128, Hq = 2, Hkv = 1, D = 64, V = 500;
    CactusGraph g;
    size_t x = g.input({M, K}, Precision::FP16);
    size_t nw = g.mmap_weights(dir + "/attn_norm.weights");
    size_t wq = g.mmap_weights(dir + "/wq.weights"), wk = g.mmap_weights(dir + "/wk.weights"),
           wv = g.mmap_weights(dir + "/wv.weights"), wo = g.mmap_weights(dir + "/wo.weights"),
           wlm = g.mmap_weights(dir + "/lm.weights");
    size_t xn = g.rms_norm(x, nw, 1e-6f);
    size_t q = g.rope(g.reshape(g.matmul(xn, wq, true), {1, M, Hq, D}), 1000000.0f, 0);
    size_t xq = g.quantize_activations(xn);
    size_t k = g.rope(g.reshape(g.matmul(xq, wk, true), {1, M, Hkv, D}), 1000000.0f, 0);
    size_t v = g.reshape(g.matmul(xq, wv, true), {1, M, Hkv, D});
    size_t att = g.attention(q, k, v, 0.125f);
    size_t o = g.matmul(g.reshape(att, {M, Hq * D}), wo, true);
    size_t h = g.add(o, x);
    size_t act = g.multiply(g.silu(h), g.gelu(h));
    size_t logits = g.matmul(g.scalar_multiply(g.add_clipped(act, h), 0.5f), wlm, true);
    size_t last = g.index(logits, M - 1, 0);
    size_t probs = g.softmax(logits);
    size_t tok = g.sample(logits, 0.0f, 0.0f, 0);
    auto xd = read_f16(dir + "/x.bin", M * K);
    g.set_input(x, xd.data(), Precision::FP16);
    g.execute(dir + "/profile.txt");
    dump(g, xn, dir + "/out_xn.bin");
    dump(g, q, dir + "/out_q.bin");
    dump(g, k, dir + "/out_k.bin");
    dump(g, v, dir + "/out_v.bin");
    dump(g, att, dir + "/out_att.bin");
    dump(g, h, dir + "/out_h.bin");
    dump(g, logits, dir + "/out_logits.bin");
    dump(g, last, dir + "/out_last.bin");
    dump(g, probs, dir + "/out_probs.bin");
    dump(g, tok, dir + "/out_tok.bin");
    report("block_shapes", g.get_output_buffer(logits).shape == std::vector<size_t>({M, V}) &&
                               g.get_output_buffer(last).shape == std::vector<size_t>({V}));
    // a second execute with the same inputs reproduces the logits bit for bit
    std::vector<uint8_t> first(static_cast<uint8_t*>(g.get_output(logits)),
                               static_cast<uint8_t*>(g.get_output(logits)) + M * V * 2);
    g.execute();
    report("block_repeatable", std::memcmp(first.data(), g.get_output(logits), first.size()) == 0);
    // soft_reset keeps the cached weights
    g.soft_reset();
    report("soft_reset_keeps_weights", g.get_node_count() == 6 && g.mmap_weights(dir + "/wq.weights") == wq);
}
// LFM2 / Whisper / encoder ops: causal depthwise conv, conv1d k=3 (stride 2), layernorm; the
// inputs come from the Python side, the outputs are compared there with the oracle
void families(const std::string& dir) {
    CactusGraph g;
    const size_t N = 1, L = 20, C = 16, K = 4, Cin = 8, Lk = 12, Cout = 6, R = 3, F = 40;
    auto in = [&](const std::vector<size_t>& shape, const std::string& name) {
        size_t n = 1;
        for (size_t d : shape) n *= d;
        const size_t id = g.input(shape, Precision::FP16);
        const std::vector<uint16_t> v = read_f16(dir + "/" + name, n);
        g.set_input(id, v.data(), Precision::FP16);
        return id;
    };
    const size_t xd = in({N, L, C}, "x_dw.bin"), wd = in({C, 1, K}, "w_dw.bin");
    const size_t xk = in({N, Cin, Lk}, "x_k3.bin"), wk = in({Cout, Cin, 3}, "w_k3.bin");
    const size_t xl = in({R, F}, "x_ln.bin"), wl = in({F}, "w_ln.bin"), bl = in({F}, "b_ln.bin");
    const size_t dw = g.conv1d_causal(xd, wd, K, 2);
    const size_t k3 = g.conv1d_k3(xk, wk, 2);
    const size_t ln = g.layernorm(xl, wl, bl, 1e-5f);
    g.execute();
    report("families_shapes", g.get_output_buffer(dw).shape == std::vector<size_t>({N, L, C}) &&
                                  g.get_output_buffer(k3).shape == std::vector<size_t>({N, Cout, (Lk - 1) / 2 + 1}) &&
                                  g.get_output_buffer(ln).shape == std::vector<size_t>({R, F}));
    dump(g, dw, dir + "/out_dw.bin");
    dump(g, k3, dir + "/out_k3.bin");
    dump(g, ln, dir + "/out_ln.bin");
}
}  // namespace

int main(int argc, char** argv) {
    if (argc < 2) {
        std::fprintf(stderr, "usage: %s <dir>\n", argv[0]);
        return 2;
    }
    try {
        known_answers(argv[1]);
        block(argv[1]);
        families(argv[1]);
    } catch (const std::exception& e) {
        std::printf("FAIL exception: %s\n", e.what());
        return 1;
    }
    std::printf("%d failures\n", failures);
    return failures ? 1 : 0;
}
