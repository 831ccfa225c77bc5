/*
 * cactus_ffi.h — the reference's text-completion C FFI (cactus/ffi/cactus_ffi.h:38-232),
 * implemented on the B200 engine. Signatures, ownership and error behaviour are the
 * reference's: the handle is owned by the library and freed by cactus_destroy, buffers are
 * the caller's, exceptions never cross the ABI (functions return -1 and write an error JSON
 * / set cactus_get_last_error()), one call at a time per handle, cactus_stop is atomic.
 *
 * Only the text path is provided (transcription, embeddings, RAG, index and telemetry
 * entry points of the reference are out of this backend's scope). Model folders written by
 * the converter without tokenizer files use an id tokenizer: message text is a
 * whitespace- or comma-separated list of decimal token ids, and generated tokens are
 * rendered as their ids.
 */
#ifndef CACTUS_FFI_H
#define CACTUS_FFI_H

#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

#if __GNUC__ >= 4
#define CACTUS_FFI_EXPORT __attribute__((visibility("default")))
#else
#define CACTUS_FFI_EXPORT
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef void* cactus_model_t;
typedef void (*cactus_token_callback)(const char* token, uint32_t token_id, void* user_data);

/* cactus_init.cpp:347-428: create + init with context 512; NULL on failure */
CACTUS_FFI_EXPORT cactus_model_t cactus_init(const char* model_path, const char* corpus_dir);
/* cactus_init.cpp:430-445 */
CACTUS_FFI_EXPORT void cactus_destroy(cactus_model_t model);
CACTUS_FFI_EXPORT void cactus_reset(cactus_model_t model);
CACTUS_FFI_EXPORT void cactus_stop(cactus_model_t model);

/* cactus_complete.cpp:14-374: returns the response JSON length, or -1 with an error JSON */
CACTUS_FFI_EXPORT int cactus_complete(cactus_model_t model, const char* messages_json, char* response_buffer,
                                      size_t buffer_size, const char* options_json, const char* tools_json,
                                      cactus_token_callback callback, void* user_data);

/* cactus_complete.cpp:376-400: 0 on success, -2 if token_buffer_len is too small, -1 on error */
CACTUS_FFI_EXPORT int cactus_tokenize(cactus_model_t model, const char* text, uint32_t* token_buffer,
                                      size_t token_buffer_len, size_t* out_token_len);

/* cactus_init.cpp:343-345 */
CACTUS_FFI_EXPORT const char* cactus_get_last_error(void);

#ifdef __cplusplus
}
#endif
#endif
