/* A C host of the Bloom ABI: loads a pipeline, runs one prompt, then streams
 * it, printing every chunk.
 *
 *   gcc demo.c -I.. -L../../../bloom_b200/ffi -lbloom_ffi -o demo
 *   PYTHONPATH=<repo> ./demo [model] [engine] [device]
 */
#include <stdio.h>
#include <string.h>

#include "../bloom.h"

static BloomSlice sl(const char* s) {
  BloomSlice r = {(const uint8_t*)s, strlen(s)};
  return r;
}

static void on_chunk(void* user, const uint8_t* json, size_t len) {
  int* n = (int*)user;
  ++*n;
  printf("chunk %d: %.*s\n", *n, (int)len, (const char*)json);
}

int main(int argc, char** argv) {
  const char* model = argc > 1 ? argv[1] : ".";
  const char* engine = argc > 2 ? argv[2] : "mock";
  const char* device = argc > 3 ? argv[3] : "cpu";
  char err[512];
  printf("abi %u\n", bloom_abi_version());
  BloomPipeline* p = bloom_pipeline_load_v2(sl(model), sl(engine), sl(device), 2048, err, sizeof err);
  if (!p) {
    fprintf(stderr, "load failed: %s\n", err);
    return 1;
  }
  const char* params = "{\"max_tokens\":16,\"temperature\":0.0,\"top_p\":1.0,\"seed\":7}";
  BloomOwnedBuffer out = {0};
  int32_t st = bloom_pipeline_run_v2(p, sl("{\"Text\":{\"prompt\":\"Hello from C\"}}"), sl(params), &out, err,
                                     sizeof err);
  if (st != BLOOM_STATUS_OK) {
    fprintf(stderr, "run failed (%d): %s\n", st, err);
    return 1;
  }
  printf("output: %.*s\n", (int)out.len, (const char*)out.data);
  bloom_buffer_free(&out);
  int chunks = 0;
  st = bloom_pipeline_run_stream_v2(p, sl("{\"Text\":{\"prompt\":\"stream me\"}}"), sl(params), on_chunk, &chunks,
                                    NULL, err, sizeof err);
  printf("stream status %d, %d chunks\n", st, chunks);
  bloom_pipeline_free(p);
  return st == BLOOM_STATUS_OK ? 0 : 1;
}
