/* Compiles bloom.h as C99 and checks the ABI surface a C consumer relies on:
 * the version, every status value, the layout of the two buffer structs,
 * zero initialisation, and that every exported function and callback type
 * has the declared signature (assigned to typed function pointers). */
#include <stddef.h>
#include <stdint.h>

#include "../bloom.h"

static void on_chunk(void* user, const char* chunk) { (void)user; (void)chunk; }
static void on_chunk_v2(void* user, const uint8_t* chunk, size_t len) { (void)user; (void)chunk; (void)len; }

int main(void) {
  int bad = 0;
  BloomSlice input = {0};
  BloomOwnedBuffer output = {0};
  BloomStatus status = BLOOM_STATUS_OK;
  bad |= !(input.data == NULL && input.len == 0 && output.data == NULL && output.len == 0);
  bad |= !(status == BLOOM_STATUS_OK && BLOOM_ABI_VERSION >= 2u);
  /* statuses 0 .. -8, in order */
  bad |= !(BLOOM_STATUS_INVALID_ARGUMENT == -1 && BLOOM_STATUS_INVALID_UTF8 == -2 &&
           BLOOM_STATUS_INVALID_INPUT_JSON == -3 && BLOOM_STATUS_INVALID_PARAMS_JSON == -4 &&
           BLOOM_STATUS_INFERENCE_ERROR == -5 && BLOOM_STATUS_OUTPUT_ERROR == -6 && BLOOM_STATUS_PANIC == -7 &&
           BLOOM_STATUS_CANCELLED == -8);
  /* {pointer, size_t} layouts, no padding surprises */
  bad |= !(offsetof(BloomSlice, data) == 0 && offsetof(BloomSlice, len) == sizeof(void*) &&
           sizeof(BloomSlice) == sizeof(void*) + sizeof(size_t));
  bad |= !(offsetof(BloomOwnedBuffer, data) == 0 && offsetof(BloomOwnedBuffer, len) == sizeof(void*) &&
           sizeof(BloomOwnedBuffer) == sizeof(void*) + sizeof(size_t));
  /* callback and function signatures */
  BloomStreamCallback cb = on_chunk;
  BloomStreamCallbackV2 cb2 = on_chunk_v2;
  uint32_t (*abi)(void) = bloom_abi_version;
  BloomPipeline* (*load2)(BloomSlice, BloomSlice, BloomSlice, size_t, char*, size_t) = bloom_pipeline_load_v2;
  int32_t (*run2)(BloomPipeline*, BloomSlice, BloomSlice, BloomOwnedBuffer*, char*, size_t) = bloom_pipeline_run_v2;
  int32_t (*stream2)(BloomPipeline*, BloomSlice, BloomSlice, BloomStreamCallbackV2, void*,
                     const BloomCancellationToken*, char*, size_t) = bloom_pipeline_run_stream_v2;
  BloomCancellationToken* (*tok_new)(void) = bloom_cancellation_token_new;
  int32_t (*tok_cancel)(BloomCancellationToken*) = bloom_cancellation_token_cancel;
  void (*tok_free)(BloomCancellationToken*) = bloom_cancellation_token_free;
  void (*buf_free)(BloomOwnedBuffer*) = bloom_buffer_free;
  BloomPipeline* (*load1)(const char*, const char*, const char*, size_t, char*, size_t) = bloom_pipeline_load;
  void (*pfree)(BloomPipeline*) = bloom_pipeline_free;
  char* (*run1)(BloomPipeline*, const char*, const char*, char*, size_t) = bloom_pipeline_run;
  int32_t (*stream1)(BloomPipeline*, const char*, const char*, BloomStreamCallback, void*, char*, size_t) =
      bloom_pipeline_run_stream;
  void (*sfree)(char*) = bloom_string_free;
  bad |= !(cb && cb2 && abi && load2 && run2 && stream2 && tok_new && tok_cancel && tok_free && buf_free && load1 &&
           pfree && run1 && stream1 && sfree);
  return bad;
}
