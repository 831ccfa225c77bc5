// The reference's text-completion FFI (include/cactus_ffi.h) on top of the B200 engine.
// Control flow, JSON fields, defaults and error behaviour follow cactus/ffi/cactus_init.cpp
// (cactus_init / destroy / reset / stop), cactus/ffi/cactus_complete.cpp (cactus_complete,
// cactus_tokenize) and cactus/ffi/cactus_utils.h (option parsing, response JSON).
#include <atomic>
#include <chrono>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <iomanip>
#include <memory>
#include <sstream>
#include <string>
#include <unistd.h>
#include <vector>

#include "../../../include/cactus_ffi.h"
#include "engine.h"

namespace {

std::string g_last_error;

struct Handle {
    std::unique_ptr<cb::eng::Engine> engine;
    std::atomic<bool> should_stop{false};
    std::vector<uint32_t> processed_tokens;
    std::string model_name;
};

struct Message {
    std::string role, content;
};

// id tokenizer: whitespace / comma separated decimal ids
std::vector<uint32_t> encode(const std::string& text) {
    std::vector<uint32_t> out;
    std::string cur;
    auto flush = [&] {
        if (cur.empty()) return;
        size_t pos = 0;
        const unsigned long v = std::stoul(cur, &pos);
        if (pos != cur.size()) throw std::runtime_error("id tokenizer: '" + cur + "' is not a token id");
        out.push_back((uint32_t)v);
        cur.clear();
    };
    for (char c : text) {
        if (c == ' ' || c == ',' || c == '\n' || c == '\t' || c == '\r') flush();
        else cur.push_back(c);
    }
    flush();
    return out;
}
std::string decode_ids(const std::vector<uint32_t>& ids) {
    std::string s;
    for (size_t i = 0; i < ids.size(); ++i) {
        if (i) s += ' ';
        s += std::to_string(ids[i]);
    }
    return s;
}

std::string escape_json(const std::string& s) {
    std::ostringstream o;
    for (char c : s) {
        switch (c) {
            case '"': o << "\\\""; break;
            case '\\': o << "\\\\"; break;
            case '\n': o << "\\n"; break;
            case '\r': o << "\\r"; break;
            case '\t': o << "\\t"; break;
            default: o << c;
        }
    }
    return o.str();
}

double ram_usage_mb() {
    long pages = 0, resident = 0;
    FILE* f = std::fopen("/proc/self/statm", "r");
    if (f) {
        if (std::fscanf(f, "%ld %ld", &pages, &resident) != 2) resident = 0;
        std::fclose(f);
    }
    return (double)resident * (double)sysconf(_SC_PAGESIZE) / (1024.0 * 1024.0);
}

void error_json(const std::string& msg, char* buf, size_t size) {
    std::ostringstream j;
    j << "{\"success\":false,\"error\":\"" << escape_json(msg) << "\",\"cloud_handoff\":false,\"response\":null,"
      << "\"function_calls\":[],\"confidence\":0.0,\"time_to_first_token_ms\":0.0,\"total_time_ms\":0.0,"
      << "\"prefill_tps\":0.0,\"decode_tps\":0.0,\"ram_usage_mb\":" << std::fixed << std::setprecision(2)
      << ram_usage_mb() << ",\"prefill_tokens\":0,\"decode_tokens\":0,\"total_tokens\":0}";
    const std::string s = j.str();
    if (buf && s.size() < size) std::strcpy(buf, s.c_str());
}

// parse_messages_json (cactus_utils.h:155-238), without images
std::vector<Message> parse_messages(const std::string& json) {
    std::vector<Message> msgs;
    size_t pos = json.find('[');
    if (pos == std::string::npos) throw std::runtime_error("Invalid JSON: expected array");
    pos = json.find('{', pos);
    while (pos != std::string::npos) {
        Message m;
        size_t end = pos + 1;
        int depth = 1;
        while (end < json.size() && depth > 0) {
            if (json[end] == '{') depth++;
            else if (json[end] == '}') depth--;
            end++;
        }
        const size_t rp = json.find("\"role\"", pos);
        if (rp == std::string::npos || rp >= end) break;
        const size_t rs = json.find('"', rp + 6) + 1;
        const size_t re = json.find('"', rs);
        m.role = json.substr(rs, re - rs);
        const size_t cp = json.find("\"content\"", re);
        if (cp != std::string::npos && cp < end) {
            const size_t cs = json.find('"', cp + 9) + 1;
            size_t ce = cs;
            while (ce < json.size()) {
                ce = json.find('"', ce);
                if (ce == std::string::npos) break;
                if (json[ce - 1] != '\\') break;
                ce++;
            }
            m.content = json.substr(cs, ce - cs);
            size_t e = 0;
            while ((e = m.content.find("\\n", e)) != std::string::npos) m.content.replace(e, 2, "\n"), e += 1;
            e = 0;
            while ((e = m.content.find("\\\"", e)) != std::string::npos) m.content.replace(e, 2, "\""), e += 1;
        }
        msgs.push_back(m);
        pos = json.find('{', end);
    }
    return msgs;
}

struct Options {
    float temperature = 0.0f, top_p = 0.0f, confidence_threshold = 0.7f;
    size_t top_k = 0, max_tokens = 100;
    std::vector<std::string> stop_sequences;
    bool include_stop_sequences = false;
};

// parse_options_json (cactus_utils.h:296-…)
Options parse_options(const std::string& json) {
    Options o;
    if (json.empty()) return o;
    auto num = [&](const char* key, auto setter) {
        size_t p = json.find(key);
        if (p != std::string::npos) setter(json.substr(json.find(':', p) + 1));
    };
    num("\"temperature\"", [&](const std::string& v) { o.temperature = std::stof(v); });
    num("\"top_p\"", [&](const std::string& v) { o.top_p = std::stof(v); });
    num("\"top_k\"", [&](const std::string& v) { o.top_k = std::stoul(v); });
    num("\"max_tokens\"", [&](const std::string& v) { o.max_tokens = std::stoul(v); });
    num("\"confidence_threshold\"", [&](const std::string& v) { o.confidence_threshold = std::stof(v); });
    size_t p = json.find("\"include_stop_sequences\"");
    if (p != std::string::npos) {
        p = json.find(':', p) + 1;
        while (p < json.size() && std::isspace((unsigned char)json[p])) p++;
        o.include_stop_sequences = json.compare(p, 4, "true") == 0;
    }
    p = json.find("\"stop_sequences\"");
    if (p != std::string::npos) {
        const size_t a = json.find('[', p), b = json.find(']', a);
        size_t q = a;
        while (a != std::string::npos && b != std::string::npos) {
            q = json.find('"', q + 1);
            if (q == std::string::npos || q >= b) break;
            const size_t e = json.find('"', q + 1);
            o.stop_sequences.push_back(json.substr(q + 1, e - q - 1));
            q = e;
        }
    }
    return o;
}

bool ends_with_any(const std::vector<uint32_t>& gen, const std::vector<std::vector<uint32_t>>& stops) {
    for (const auto& s : stops) {
        if (s.empty() || gen.size() < s.size()) continue;
        if (std::equal(s.rbegin(), s.rend(), gen.rbegin())) return true;
    }
    return false;
}

}  // namespace

extern "C" {

CACTUS_FFI_EXPORT const char* cactus_get_last_error(void) { return g_last_error.c_str(); }

CACTUS_FFI_EXPORT cactus_model_t cactus_init(const char* model_path, const char* corpus_dir) {
    (void)corpus_dir;  // RAG corpus indexing is outside this backend
    const std::string path = model_path ? model_path : "unknown";
    try {
        auto* h = new Handle();
        const size_t slash = path.find_last_of("/\\");
        h->model_name = slash == std::string::npos ? path : path.substr(slash + 1);
        h->engine = std::make_unique<cb::eng::Engine>();
        int device = 0;
        if (const char* d = std::getenv("CACTUS_B200_DEVICE")) device = std::atoi(d);
        try {
            h->engine->init(path, 512, 1, device);  // DEFAULT_CONTEXT_SIZE (cactus_init.cpp:350)
        } catch (const std::exception& e) {
            g_last_error = "Failed to initialize model - check weight files at: " + path + " (" + e.what() + ")";
            delete h;
            return nullptr;
        }
        return h;
    } catch (const std::exception& e) {
        g_last_error = "Exception during init: " + std::string(e.what());
        return nullptr;
    }
}

CACTUS_FFI_EXPORT void cactus_destroy(cactus_model_t model) { delete static_cast<Handle*>(model); }

CACTUS_FFI_EXPORT void cactus_reset(cactus_model_t model) {
    if (!model) return;
    auto* h = static_cast<Handle*>(model);
    h->engine->reset();
    h->processed_tokens.clear();
}

CACTUS_FFI_EXPORT void cactus_stop(cactus_model_t model) {
    if (model) static_cast<Handle*>(model)->should_stop = true;
}

CACTUS_FFI_EXPORT int cactus_tokenize(cactus_model_t model, const char* text, uint32_t* token_buffer,
                                      size_t token_buffer_len, size_t* out_token_len) {
    if (!model || !text || !out_token_len) return -1;
    try {
        const std::vector<uint32_t> t = encode(text);
        *out_token_len = t.size();
        if (!token_buffer || token_buffer_len == 0) return 0;
        if (token_buffer_len < t.size()) return -2;
        std::memcpy(token_buffer, t.data(), t.size() * 4);
        return 0;
    } catch (...) {
        return -1;
    }
}

CACTUS_FFI_EXPORT int cactus_complete(cactus_model_t model, const char* messages_json, char* response_buffer,
                                      size_t buffer_size, const char* options_json, const char* tools_json,
                                      cactus_token_callback callback, void* user_data) {
    (void)tools_json;
    if (!model) {
        error_json(g_last_error.empty() ? "Model not initialized. Check model path and files." : g_last_error,
                   response_buffer, buffer_size);
        return -1;
    }
    if (!messages_json || !response_buffer || buffer_size == 0) {
        error_json("Invalid parameters", response_buffer, buffer_size);
        return -1;
    }
    auto* h = static_cast<Handle*>(model);
    try {
        using clock = std::chrono::high_resolution_clock;
        const auto t_start = clock::now();
        h->should_stop = false;
        const std::vector<Message> messages = parse_messages(messages_json);
        if (messages.empty()) {
            error_json("No messages provided", response_buffer, buffer_size);
            return -1;
        }
        const Options opt = parse_options(options_json ? options_json : "");
        std::string prompt;  // id tokenizer "chat template": the messages' ids in order
        for (const auto& m : messages) prompt += m.content + " ";
        const std::vector<uint32_t> current = encode(prompt);
        std::vector<uint32_t> todo;
        const bool is_prefix = current.size() >= h->processed_tokens.size() &&
                               std::equal(h->processed_tokens.begin(), h->processed_tokens.end(), current.begin());
        if (h->processed_tokens.empty() || !is_prefix) {
            h->engine->reset();
            todo = current;
        } else {
            todo.assign(current.begin() + h->processed_tokens.size(), current.end());
        }
        const size_t prompt_tokens = todo.size();
        std::vector<std::vector<uint32_t>> stops = {{h->engine->config().eos_token_id}};
        for (const auto& s : opt.stop_sequences) stops.push_back(encode(s));

        std::vector<uint32_t> generated;
        float first_entropy = 0.0f;
        uint32_t next = 0;
        cb::eng::Engine& eng = *h->engine;
        if (todo.empty()) {
            if (h->processed_tokens.empty()) {
                error_json("Cannot generate from empty prompt", response_buffer, buffer_size);
                return -1;
            }
            const uint32_t last = h->processed_tokens.back();
            next = eng.decode(&last, 1, opt.temperature, opt.top_p, opt.top_k, &first_entropy);
        } else if (todo.size() > 1) {
            eng.prefill(todo.data(), todo.size() - 1, 256);
            next = eng.decode(&todo.back(), 1, opt.temperature, opt.top_p, opt.top_k, &first_entropy);
        } else {
            next = eng.decode(todo.data(), 1, opt.temperature, opt.top_p, opt.top_k, &first_entropy);
        }
        h->processed_tokens = current;
        const double ttft = std::chrono::duration_cast<std::chrono::microseconds>(clock::now() - t_start).count() / 1e3;
        float confidence = 1.0f - first_entropy;
        if (confidence < opt.confidence_threshold) {  // cloud handoff (cactus_complete.cpp:216-238)
            const double prefill_tps = ttft > 0 ? prompt_tokens * 1000.0 / ttft : 0.0;
            std::ostringstream j;
            j << "{\"success\":false,\"error\":null,\"cloud_handoff\":true,\"response\":null,\"function_calls\":[],"
              << "\"confidence\":" << std::fixed << std::setprecision(4) << confidence
              << ",\"time_to_first_token_ms\":" << std::setprecision(2) << ttft << ",\"total_time_ms\":" << ttft
              << ",\"prefill_tps\":" << prefill_tps << ",\"decode_tps\":0.0,\"ram_usage_mb\":" << ram_usage_mb()
              << ",\"prefill_tokens\":" << prompt_tokens << ",\"decode_tokens\":0,\"total_tokens\":" << prompt_tokens
              << "}";
            const std::string r = j.str();
            if (r.size() >= buffer_size) {
                error_json("Response buffer too small", response_buffer, buffer_size);
                return -1;
            }
            std::strcpy(response_buffer, r.c_str());
            return (int)r.size();
        }
        generated.push_back(next);
        h->processed_tokens.push_back(next);
        std::vector<float> window = {first_entropy};
        float window_sum = first_entropy, total_entropy = first_entropy;
        size_t n_entropy = 1;
        bool handoff = false;
        auto trim = [&] {
            if (opt.include_stop_sequences) return;
            for (const auto& s : stops) {
                if (s.empty() || generated.size() < s.size()) continue;
                if (std::equal(s.rbegin(), s.rend(), generated.rbegin())) {
                    generated.resize(generated.size() - s.size());
                    break;
                }
            }
        };
        if (!ends_with_any(generated, stops)) {
            if (callback) callback(std::to_string(next).c_str(), next, user_data);
            for (size_t i = 1; i < opt.max_tokens; ++i) {
                if (h->should_stop) break;
                float ent = 0.0f;
                next = eng.decode(&next, 1, opt.temperature, opt.top_p, opt.top_k, &ent);
                generated.push_back(next);
                h->processed_tokens.push_back(next);
                total_entropy += ent;
                n_entropy++;
                window.push_back(ent);
                window_sum += ent;
                if (window.size() > 10) {
                    window_sum -= window.front();
                    window.erase(window.begin());
                }
                if (1.0f - window_sum / window.size() < opt.confidence_threshold) {
                    handoff = true;
                    break;
                }
                if (ends_with_any(generated, stops)) {
                    trim();
                    break;
                }
                if (callback) callback(std::to_string(next).c_str(), next, user_data);
            }
        } else {
            trim();
        }
        confidence = 1.0f - total_entropy / (float)n_entropy;
        const double total_ms = std::chrono::duration_cast<std::chrono::microseconds>(clock::now() - t_start).count() / 1e3;
        const size_t completion = generated.size();
        const double decode_ms = total_ms - ttft;
        const double prefill_tps = ttft > 0 ? prompt_tokens * 1000.0 / ttft : 0.0;
        const double decode_tps = (completion > 1 && decode_ms > 0) ? (completion - 1) * 1000.0 / decode_ms : 0.0;
        std::ostringstream j;
        j << "{\"success\":" << (handoff ? "false" : "true") << ",\"error\":null,\"cloud_handoff\":"
          << (handoff ? "true" : "false") << ",\"response\":\"" << escape_json(decode_ids(generated))
          << "\",\"function_calls\":[],\"confidence\":" << std::fixed << std::setprecision(4) << confidence
          << ",\"time_to_first_token_ms\":" << std::setprecision(2) << ttft << ",\"total_time_ms\":" << total_ms
          << ",\"prefill_tps\":" << prefill_tps << ",\"decode_tps\":" << decode_tps
          << ",\"ram_usage_mb\":" << ram_usage_mb() << ",\"prefill_tokens\":" << prompt_tokens
          << ",\"decode_tokens\":" << completion << ",\"total_tokens\":" << (prompt_tokens + completion) << "}";
        const std::string r = j.str();
        if (r.size() >= buffer_size) {
            error_json("Response buffer too small", response_buffer, buffer_size);
            return -1;
        }
        std::strcpy(response_buffer, r.c_str());
        return (int)r.size();
    } catch (const std::exception& e) {
        error_json(e.what(), response_buffer, buffer_size);
        return -1;
    } catch (...) {
        error_json("Unknown error during completion", response_buffer, buffer_size);
        return -1;
    }
}

}  // extern "C"
