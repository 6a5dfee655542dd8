/* Bloom C ABI, revision 2 -- implemented by libbloom_ffi.so of bloom_b200.
 *
 * The declarations are the public contract of the reference's C ABI
 * (crates/ffi/bloom.h) and are kept identical so existing C/C++ consumers
 * link unchanged: function names, argument order, status codes, buffer
 * ownership rules and the JSON shapes (ModelInput such as
 * {"Text":{"prompt":"..."}}, GenerationParams such as
 * {"max_tokens":10,"temperature":0.7,"top_p":0.9,"seed":null}, ModelOutput
 * {"text":...}, stream chunks {"TextDelta":"..."} ... "End").
 */
#ifndef BLOOM_H
#define BLOOM_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct BloomPipeline BloomPipeline;
typedef struct BloomCancellationToken BloomCancellationToken;

#define BLOOM_ABI_VERSION 2u

typedef enum BloomStatus {
    BLOOM_STATUS_OK = 0,
    BLOOM_STATUS_INVALID_ARGUMENT = -1,
    BLOOM_STATUS_INVALID_UTF8 = -2,
    BLOOM_STATUS_INVALID_INPUT_JSON = -3,
    BLOOM_STATUS_INVALID_PARAMS_JSON = -4,
    BLOOM_STATUS_INFERENCE_ERROR = -5,
    BLOOM_STATUS_OUTPUT_ERROR = -6,
    BLOOM_STATUS_PANIC = -7,
    BLOOM_STATUS_CANCELLED = -8
} BloomStatus;

/* Borrowed bytes; the caller keeps ownership for the whole call. */
typedef struct BloomSlice {
    const uint8_t* data;
    size_t len;
} BloomSlice;

/* Bytes owned by the library; initialise to {NULL, 0}, release with bloom_buffer_free. */
typedef struct BloomOwnedBuffer {
    uint8_t* data;
    size_t len;
} BloomOwnedBuffer;

typedef void (*BloomStreamCallback)(void* user_data, const char* chunk_json);
typedef void (*BloomStreamCallbackV2)(void* user_data, const uint8_t* chunk_json, size_t chunk_json_len);

uint32_t bloom_abi_version(void);

BloomPipeline* bloom_pipeline_load_v2(BloomSlice model_path, BloomSlice engine_name, BloomSlice device_name,
                                      size_t context_size, char* error_buffer, size_t error_buffer_len);

int32_t bloom_pipeline_run_v2(BloomPipeline* pipeline, BloomSlice input_json, BloomSlice params_json,
                              BloomOwnedBuffer* output, char* error_buffer, size_t error_buffer_len);

BloomCancellationToken* bloom_cancellation_token_new(void);
int32_t bloom_cancellation_token_cancel(BloomCancellationToken* token);
void bloom_cancellation_token_free(BloomCancellationToken* token);

int32_t bloom_pipeline_run_stream_v2(BloomPipeline* pipeline, BloomSlice input_json, BloomSlice params_json,
                                     BloomStreamCallbackV2 callback, void* user_data,
                                     const BloomCancellationToken* cancellation, char* error_buffer,
                                     size_t error_buffer_len);

void bloom_buffer_free(BloomOwnedBuffer* buffer);

/* ABI revision 1 compatibility symbols. */
BloomPipeline* bloom_pipeline_load(const char* model_path, const char* engine_name, const char* device_name,
                                   size_t context_size, char* error_buffer, size_t error_buffer_len);
void bloom_pipeline_free(BloomPipeline* pipeline);
char* bloom_pipeline_run(BloomPipeline* pipeline, const char* input_json, const char* params_json,
                         char* error_buffer, size_t error_buffer_len);
int32_t bloom_pipeline_run_stream(BloomPipeline* pipeline, const char* input_json, const char* params_json,
                                  BloomStreamCallback callback, void* user_data, char* error_buffer,
                                  size_t error_buffer_len);
void bloom_string_free(char* s);

#ifdef __cplusplus
}
#endif

#endif /* BLOOM_H */
