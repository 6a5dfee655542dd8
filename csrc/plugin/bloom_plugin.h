/* Native engine plugin ABI.
 *
 * A plugin is a shared library exporting
 *     int bloom_plugin_init(CBloomEngine* out);
 * which fills the function table below and returns 0.  The table layout,
 * field order and JSON conventions are those of the reference's native plugin
 * ABI (crates/engine/src/plugin/mod.rs, `ffi::CBloomEngine`), so plugins built
 * for it load here unchanged.  Strings returned through out-pointers are owned
 * by the plugin and released with free_string; name() returns a static string.
 * Modality codes: 0 Text, 1 Audio, 2 Vision, 3 Embedding.  Device codes:
 * 0 Cpu, 1 Cuda, 2 Metal, 3 Npu.  Streaming callbacks return 0 to continue.
 */
#ifndef BLOOM_PLUGIN_H
#define BLOOM_PLUGIN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef int32_t (*CBloomStreamCallback)(void* user_data, const char* chunk_json);

typedef struct CBloomEngine {
  const char* (*name)(void);
  int32_t (*supported_modalities)(int32_t* out_modalities, size_t* out_len);
  int32_t (*supported_devices)(int32_t* out_devices, size_t* out_len);
  int32_t (*load_model)(const char* model_path, int32_t device_kind, void** out_model);
  void (*free_model)(void* model);
  int32_t (*model_metadata)(void* model, char** out_json);
  int32_t (*model_infer)(void* model, const char* input_json, char** out_json);
  int32_t (*model_infer_stream)(void* model, const char* input_json, CBloomStreamCallback callback,
                                void* user_data);
  void (*free_string)(char* s);
} CBloomEngine;

typedef int32_t (*BloomPluginInitFn)(CBloomEngine* out);

#ifdef __cplusplus
}
#endif

#endif /* BLOOM_PLUGIN_H */
