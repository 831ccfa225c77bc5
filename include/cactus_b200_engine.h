/*
 * cactus_b200_engine.h — C ABI of the device-resident engine (model + KV cache).
 *
 * These entry points are the C image of the reference's C++ engine API
 * (cactus/engine/engine.h:473-579): create_model + Model::init, Model::prefill,
 * Model::decode, reset_cache and set_cache_window. The engine keeps weights, KV cache
 * and the decode state in HBM; token ids cross the boundary as HOST arrays.
 * Calls on one handle must not overlap (as in the reference); different handles
 * may live on different devices.
 */
#ifndef CACTUS_B200_ENGINE_H
#define CACTUS_B200_ENGINE_H

#include <stddef.h>
#include <stdint.h>

#include "cactus_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef void* cactus_engine_t;

/* create_model (engine_model.cpp:545-582) + Model::init (engine_model.cpp:73-164):
 * reads <model_folder>/config.txt and the .weights files, uploads them to `device`,
 * allocates the INT8 KV cache for `context_size` tokens per sequence and `max_batch`
 * sequences. The KV window defaults to min(context_size, 512) with 4 sink tokens
 * (CACTUS_KV_WINDOW_SIZE / CACTUS_KV_SINK_SIZE override it; Gemma uses no window).
 * Returns NULL on failure (message in cactus_engine_last_error()). */
CB_API cactus_engine_t cactus_engine_create(const char* model_folder, size_t context_size, size_t max_batch,
                                            int device);
CB_API void cactus_engine_destroy(cactus_engine_t engine);
CB_API const char* cactus_engine_last_error(void);

/* Model::reset_cache (engine.h:525) */
CB_API int cactus_engine_reset(cactus_engine_t engine);
/* Model::set_cache_window (engine.h:531); window 0 disables sliding */
CB_API int cactus_engine_set_cache_window(cactus_engine_t engine, size_t window_size, size_t sink_size);
/* Causal-correct masking of prefill chunks after the KV window has slid (on != 0). No
 * reference counterpart: off (the default) is the reference's behaviour, where the mask of
 * cactus_attention_hybrid_int8_fp16 uses the total position (kernel_attention.cpp:331-346 with
 * engine_cache.cpp:111-120), so once total > cache index a chunk's queries also see the
 * chunk's later keys; on masks by the cache index. Decode steps are the same in both modes.
 * Also set by CACTUS_B200_CAUSAL_FIX=1 at creation. */
CB_API int cactus_engine_set_causal_fix(cactus_engine_t engine, int on);
/* model dimensions: out[0..7] = vocab, layers, hidden, heads, kv_heads, head_dim, ffn, model_type */
CB_API int cactus_engine_info(cactus_engine_t engine, uint32_t* out8);

/* Model::prefill (engine_model.cpp:170-219): processes `tokens` in chunks of
 * `chunk_size` (256 in the reference) and appends them to the KV cache. */
CB_API int cactus_engine_prefill(cactus_engine_t engine, const uint32_t* tokens, size_t n, size_t chunk_size);

/* Model::decode (engine_model.cpp:221-297): forward of `tokens` (usually one), then the
 * logits of the last row are sampled. Greedy (first-max argmax, kernel_nn.cpp:451-467)
 * when temperature == 0, top_p <= 0 and top_k == 0 after Model::decode's defaulting rule
 * (negative temperature / top_p and top_k == 0 take the model defaults); other settings
 * sample on the device (top-k, top-p, temperature). `out_entropy` may be NULL. */
CB_API int cactus_engine_decode(cactus_engine_t engine, const uint32_t* tokens, size_t n, float temperature,
                                float top_p, size_t top_k, uint32_t* out_token, float* out_entropy);

/* Graph-level greedy generation (CactusGraph::sample(logits, 0, 0, 0), kernel_nn.cpp:451-467):
 * prefill(prompt[:-1]) then `max_new` decode steps, each step one CUDA-graph replay whose
 * argmax token feeds the next step on the device. out_tokens receives max_new ids. */
CB_API int cactus_engine_generate_greedy(cactus_engine_t engine, const uint32_t* prompt, size_t n, size_t max_new,
                                         uint32_t* out_tokens);

/* Batched greedy decode of `batch` independent sequences that share a prompt length:
 * prompts [batch, prompt_len] (host), out_tokens [batch, max_new] (host). The sequences
 * never interact; each has its own KV cache. */
CB_API int cactus_engine_generate_batch_greedy(cactus_engine_t engine, const uint32_t* prompts, size_t batch,
                                               size_t prompt_len, size_t max_new, uint32_t* out_tokens);

/* statistics of the last generate call: out[0] prefill ms, out[1] decode ms (CUDA events on
 * the engine stream), out[2] kernels launched, out[3] decode-graph replays, out[4] kernel
 * nodes per replay, out[5] weight bytes in HBM, out[6] KV capacity, out[7] KV window */
CB_API int cactus_engine_stats(cactus_engine_t engine, double* out8);

/* decode path of the last generate call: 0 host-driven launches, 1 CUDA-graph replay of
 * the per-op kernels, 2 persistent single-launch decode step (batch 1, non-Gemma models).
 * `mode` selects the path for later calls: -1 automatic (persistent where it applies),
 * 1 never use the persistent step. Returns the last path, or -1 for a null engine. */
CB_API int cactus_engine_decode_path(cactus_engine_t engine, int mode);

/* fp16 logits of the last decoded row of sequence 0 (for parity checks) */
CB_API int cactus_engine_last_logits(cactus_engine_t engine, uint16_t* host_logits, size_t vocab);
/* KV state of sequence 0: out[0] = current_seq_len, out[1] = total_seq_len (engine_cache.cpp:101-337) */
CB_API int cactus_engine_kv_state(cactus_engine_t engine, size_t* out2);
/* copy layer `layer`'s INT8 keys/values and fp32 scales of sequence 0 to host buffers
 * ([current_seq_len, kv_heads, head_dim] int8 and [current_seq_len, kv_heads, groups] fp32) */
CB_API int cactus_engine_read_kv(cactus_engine_t engine, size_t layer, int8_t* keys, int8_t* values, float* k_scales,
                                 float* v_scales);

#ifdef __cplusplus
}
#endif
#endif
