// libbloom_ffi: the C ABI of bloom.h (revision 2 plus the revision-1 symbols)
// over the Python engine, for C and C++ hosts.
//
// The library embeds CPython: a host that is not Python starts an
// interpreter on first use (Py_InitializeEx, then releases the GIL); a
// Python host that loaded the library through ctypes already has one.  Every
// entry point takes the GIL (PyGILState_Ensure) for its Python work and
// releases it around user callbacks, so a callback may cancel, or call into
// the library from another thread, without deadlock.
//
// Behaviour follows the reference ABI (crates/ffi/src/lib.rs): borrowed
// inputs are validated as UTF-8 before any parse (16 MiB JSON limit, 4 KiB
// identifiers), errors are written NUL-terminated and truncated into the
// caller's buffer, output buffers are malloc'd and released with
// bloom_buffer_free, cancellation is observed before and after every
// callback and reported as BLOOM_STATUS_CANCELLED, and no C++ exception
// crosses the boundary (BLOOM_STATUS_PANIC).
#define PY_SSIZE_T_CLEAN
#include <Python.h>

#include <atomic>
#include <cstdlib>
#include <cstring>
#include <exception>
#include <mutex>
#include <string>

#include "bloom.h"

#define BLOOM_EXPORT extern "C" __attribute__((visibility("default")))

struct BloomPipeline {
  PyObject* handle;  // bloom_b200.ffi.backend._Handle (strong reference)
};

struct BloomCancellationToken {
  std::atomic<bool> cancelled{false};
};

namespace {

constexpr size_t kMaxJsonBytes = 16u * 1024u * 1024u;
constexpr size_t kMaxIdentifierBytes = 4u * 1024u;

std::once_flag g_init_once;

void ensure_python() {
  std::call_once(g_init_once, [] {
    if (!Py_IsInitialized()) {
      Py_InitializeEx(0);
      PyEval_SaveThread();  // drop the GIL taken by initialisation
    }
  });
}

struct Gil {
  PyGILState_STATE s;
  Gil() : s(PyGILState_Ensure()) {}
  ~Gil() { PyGILState_Release(s); }
};

void write_error(const std::string& msg, char* buf, size_t len) {
  if (buf == nullptr || len == 0) return;
  const size_t n = msg.size() < len - 1 ? msg.size() : len - 1;
  std::memcpy(buf, msg.data(), n);
  buf[n] = '\0';
}

void clear_error(char* buf, size_t len) {
  if (buf != nullptr && len > 0) buf[0] = '\0';
}

// Strict UTF-8 check (RFC 3629: no overlongs, no surrogates, <= U+10FFFF).
bool valid_utf8(const uint8_t* s, size_t n) {
  size_t i = 0;
  while (i < n) {
    const uint8_t c = s[i];
    if (c < 0x80) {
      ++i;
      continue;
    }
    int extra;
    uint32_t cp;
    if ((c & 0xE0) == 0xC0) {
      extra = 1;
      cp = c & 0x1F;
    } else if ((c & 0xF0) == 0xE0) {
      extra = 2;
      cp = c & 0x0F;
    } else if ((c & 0xF8) == 0xF0) {
      extra = 3;
      cp = c & 0x07;
    } else {
      return false;
    }
    if (i + static_cast<size_t>(extra) >= n) return false;  // truncated sequence
    for (int k = 1; k <= extra; ++k) {
      const uint8_t d = s[i + k];
      if ((d & 0xC0) != 0x80) return false;
      cp = (cp << 6) | (d & 0x3F);
    }
    if ((extra == 1 && cp < 0x80) || (extra == 2 && cp < 0x800) || (extra == 3 && cp < 0x10000)) return false;
    if (cp > 0x10FFFF || (cp >= 0xD800 && cp <= 0xDFFF)) return false;
    i += extra + 1;
  }
  return true;
}

// Validates a borrowed slice; on success `out` holds the text.
int32_t slice_text(BloomSlice s, const char* what, size_t limit, std::string& out, std::string& err) {
  if (s.data == nullptr && s.len != 0) {
    err = std::string("NULL pointer passed for ") + what;
    return BLOOM_STATUS_INVALID_ARGUMENT;
  }
  if (s.len > limit) {
    err = std::string(what) + " exceeds " + std::to_string(limit) + " bytes";
    return BLOOM_STATUS_INVALID_ARGUMENT;
  }
  if (!valid_utf8(s.data, s.len)) {
    err = std::string(what) + " is not valid UTF-8";
    return BLOOM_STATUS_INVALID_UTF8;
  }
  out.assign(reinterpret_cast<const char*>(s.data), s.len);
  return BLOOM_STATUS_OK;
}

PyObject* backend() {
  static PyObject* mod = nullptr;  // owned for the process lifetime
  if (mod == nullptr) mod = PyImport_ImportModule("bloom_b200.ffi.backend");
  return mod;
}

// Maps the pending Python exception to a status code and message; clears it.
int32_t take_py_error(std::string& msg, int32_t fallback) {
  PyObject *type = nullptr, *value = nullptr, *tb = nullptr;
  PyErr_Fetch(&type, &value, &tb);
  PyErr_NormalizeException(&type, &value, &tb);
  int32_t st = fallback;
  msg = "unknown error";
  if (value != nullptr) {
    PyObject* s = PyObject_Str(value);
    if (s != nullptr) {
      const char* c = PyUnicode_AsUTF8(s);
      if (c != nullptr) msg = c;
      Py_DECREF(s);
    }
  }
  if (type != nullptr) {
    const char* name = reinterpret_cast<PyTypeObject*>(type)->tp_name;
    const std::string n = name ? name : "";
    auto ends = [&](const char* suf) {
      const size_t k = std::strlen(suf);
      return n.size() >= k && n.compare(n.size() - k, k, suf) == 0;
    };
    if (ends("InvalidArgument")) st = BLOOM_STATUS_INVALID_ARGUMENT;
    else if (ends("InvalidInputJson")) st = BLOOM_STATUS_INVALID_INPUT_JSON;
    else if (ends("InvalidParamsJson")) st = BLOOM_STATUS_INVALID_PARAMS_JSON;
    else if (ends("InferenceError")) st = BLOOM_STATUS_INFERENCE_ERROR;
  }
  Py_XDECREF(type);
  Py_XDECREF(value);
  Py_XDECREF(tb);
  PyErr_Clear();
  return st;
}

BloomPipeline* load_impl(const std::string& model, const std::string& engine, const std::string& device,
                         size_t ctx, char* ebuf, size_t elen) {
  if (ctx == 0) {
    write_error("context_size must be greater than zero", ebuf, elen);
    return nullptr;
  }
  ensure_python();
  Gil gil;
  PyObject* mod = backend();
  if (mod == nullptr) {
    std::string m;
    take_py_error(m, BLOOM_STATUS_INFERENCE_ERROR);
    write_error("cannot import bloom_b200.ffi.backend: " + m, ebuf, elen);
    return nullptr;
  }
  PyObject* h = PyObject_CallMethod(mod, "load", "sssn", model.c_str(), engine.c_str(), device.c_str(),
                                    static_cast<Py_ssize_t>(ctx));
  if (h == nullptr) {
    std::string m;
    take_py_error(m, BLOOM_STATUS_INFERENCE_ERROR);
    write_error(m, ebuf, elen);
    return nullptr;
  }
  auto* p = new BloomPipeline;
  p->handle = h;
  clear_error(ebuf, elen);
  return p;
}

int32_t run_impl(BloomPipeline* p, const std::string& input, const std::string& params, std::string& out,
                 std::string& err) {
  Gil gil;
  PyObject* r = PyObject_CallMethod(backend(), "run", "Oss", p->handle, input.c_str(), params.c_str());
  if (r == nullptr) return take_py_error(err, BLOOM_STATUS_INFERENCE_ERROR);
  const char* c = PyUnicode_AsUTF8(r);
  if (c == nullptr) {
    Py_DECREF(r);
    take_py_error(err, BLOOM_STATUS_OUTPUT_ERROR);
    err = "Failed to serialize ModelOutput: " + err;
    return BLOOM_STATUS_OUTPUT_ERROR;
  }
  out = c;
  Py_DECREF(r);
  return BLOOM_STATUS_OK;
}

// Streams chunks; `emit` is called without the GIL.  Returns a status.
template <typename Emit>
int32_t stream_impl(BloomPipeline* p, const std::string& input, const std::string& params,
                    const BloomCancellationToken* cancel, std::string& err, Emit&& emit) {
  auto cancelled = [&] { return cancel != nullptr && cancel->cancelled.load(std::memory_order_acquire); };
  if (cancelled()) {
    err = "stream cancelled";
    return BLOOM_STATUS_CANCELLED;
  }
  PyGILState_STATE st = PyGILState_Ensure();
  PyObject* it = PyObject_CallMethod(backend(), "stream", "Oss", p->handle, input.c_str(), params.c_str());
  if (it == nullptr) {
    const int32_t s = take_py_error(err, BLOOM_STATUS_INFERENCE_ERROR);
    PyGILState_Release(st);
    return s;
  }
  int32_t status = BLOOM_STATUS_OK;
  for (;;) {
    if (cancelled()) {
      err = "stream cancelled";
      status = BLOOM_STATUS_CANCELLED;
      break;
    }
    PyObject* item = PyIter_Next(it);
    if (item == nullptr) {
      if (PyErr_Occurred()) status = take_py_error(err, BLOOM_STATUS_INFERENCE_ERROR);
      break;
    }
    Py_ssize_t n = 0;
    const char* c = PyUnicode_AsUTF8AndSize(item, &n);
    if (c == nullptr) {
      Py_DECREF(item);
      take_py_error(err, BLOOM_STATUS_OUTPUT_ERROR);
      status = BLOOM_STATUS_OUTPUT_ERROR;
      break;
    }
    std::string chunk(c, static_cast<size_t>(n));
    Py_DECREF(item);
    PyGILState_Release(st);
    emit(chunk);
    st = PyGILState_Ensure();
    if (cancelled()) {
      err = "stream cancelled";
      status = BLOOM_STATUS_CANCELLED;
      break;
    }
  }
  PyObject* close = PyObject_GetAttrString(it, "close");  // stop the generator (frees engine state)
  if (close != nullptr) {
    PyObject* r = PyObject_CallNoArgs(close);
    Py_XDECREF(r);
    Py_DECREF(close);
  }
  PyErr_Clear();
  Py_DECREF(it);
  PyGILState_Release(st);
  return status;
}

}  // namespace

BLOOM_EXPORT uint32_t bloom_abi_version(void) { return BLOOM_ABI_VERSION; }

BLOOM_EXPORT BloomCancellationToken* bloom_cancellation_token_new(void) {
  try {
    return new BloomCancellationToken;
  } catch (...) {
    return nullptr;
  }
}

BLOOM_EXPORT int32_t bloom_cancellation_token_cancel(BloomCancellationToken* token) {
  if (token == nullptr) return BLOOM_STATUS_INVALID_ARGUMENT;
  token->cancelled.store(true, std::memory_order_release);
  return BLOOM_STATUS_OK;
}

BLOOM_EXPORT void bloom_cancellation_token_free(BloomCancellationToken* token) { delete token; }

BLOOM_EXPORT BloomPipeline* bloom_pipeline_load_v2(BloomSlice model_path, BloomSlice engine_name,
                                                   BloomSlice device_name, size_t context_size, char* error_buffer,
                                                   size_t error_buffer_len) {
  try {
    std::string model, engine, device, err;
    if (slice_text(model_path, "model_path", kMaxIdentifierBytes, model, err) != BLOOM_STATUS_OK ||
        slice_text(engine_name, "engine_name", kMaxIdentifierBytes, engine, err) != BLOOM_STATUS_OK ||
        slice_text(device_name, "device_name", kMaxIdentifierBytes, device, err) != BLOOM_STATUS_OK) {
      write_error(err, error_buffer, error_buffer_len);
      return nullptr;
    }
    return load_impl(model, engine, device, context_size, error_buffer, error_buffer_len);
  } catch (const std::exception& e) {
    write_error(std::string("internal error: ") + e.what(), error_buffer, error_buffer_len);
    return nullptr;
  } catch (...) {
    write_error("internal error", error_buffer, error_buffer_len);
    return nullptr;
  }
}

BLOOM_EXPORT BloomPipeline* bloom_pipeline_load(const char* model_path, const char* engine_name,
                                                const char* device_name, size_t context_size, char* error_buffer,
                                                size_t error_buffer_len) {
  if (model_path == nullptr || engine_name == nullptr || device_name == nullptr) {
    write_error("Null argument passed to bloom_pipeline_load", error_buffer, error_buffer_len);
    return nullptr;
  }
  auto sl = [](const char* s) {
    return BloomSlice{reinterpret_cast<const uint8_t*>(s), std::strlen(s)};
  };
  return bloom_pipeline_load_v2(sl(model_path), sl(engine_name), sl(device_name), context_size, error_buffer,
                                error_buffer_len);
}

BLOOM_EXPORT void bloom_pipeline_free(BloomPipeline* pipeline) {
  if (pipeline == nullptr) return;
  if (Py_IsInitialized()) {
    Gil gil;
    Py_XDECREF(pipeline->handle);
  }
  delete pipeline;
}

BLOOM_EXPORT int32_t bloom_pipeline_run_v2(BloomPipeline* pipeline, BloomSlice input_json, BloomSlice params_json,
                                           BloomOwnedBuffer* output, char* error_buffer, size_t error_buffer_len) {
  try {
    if (pipeline == nullptr || output == nullptr) {
      write_error("NULL argument passed to bloom_pipeline_run_v2", error_buffer, error_buffer_len);
      return BLOOM_STATUS_INVALID_ARGUMENT;
    }
    output->data = nullptr;
    output->len = 0;
    std::string input, params, err, out;
    int32_t st = slice_text(input_json, "input_json", kMaxJsonBytes, input, err);
    if (st == BLOOM_STATUS_OK) st = slice_text(params_json, "params_json", kMaxJsonBytes, params, err);
    if (st == BLOOM_STATUS_OK) st = run_impl(pipeline, input, params, out, err);
    if (st != BLOOM_STATUS_OK) {
      write_error(err, error_buffer, error_buffer_len);
      return st;
    }
    auto* p = static_cast<uint8_t*>(std::malloc(out.size() ? out.size() : 1));
    if (p == nullptr) {
      write_error("Failed to allocate the output buffer", error_buffer, error_buffer_len);
      return BLOOM_STATUS_OUTPUT_ERROR;
    }
    std::memcpy(p, out.data(), out.size());
    output->data = p;
    output->len = out.size();
    clear_error(error_buffer, error_buffer_len);
    return BLOOM_STATUS_OK;
  } catch (...) {
    write_error("internal error at the FFI boundary", error_buffer, error_buffer_len);
    return BLOOM_STATUS_PANIC;
  }
}

BLOOM_EXPORT char* bloom_pipeline_run(BloomPipeline* pipeline, const char* input_json, const char* params_json,
                                      char* error_buffer, size_t error_buffer_len) {
  if (pipeline == nullptr || input_json == nullptr || params_json == nullptr) {
    write_error("Null argument passed to bloom_pipeline_run", error_buffer, error_buffer_len);
    return nullptr;
  }
  BloomOwnedBuffer out{nullptr, 0};
  const int32_t st = bloom_pipeline_run_v2(
      pipeline, BloomSlice{reinterpret_cast<const uint8_t*>(input_json), std::strlen(input_json)},
      BloomSlice{reinterpret_cast<const uint8_t*>(params_json), std::strlen(params_json)}, &out, error_buffer,
      error_buffer_len);
  if (st != BLOOM_STATUS_OK) return nullptr;
  char* s = static_cast<char*>(std::malloc(out.len + 1));
  if (s != nullptr) {
    std::memcpy(s, out.data, out.len);
    s[out.len] = '\0';
  }
  bloom_buffer_free(&out);
  return s;
}

BLOOM_EXPORT int32_t bloom_pipeline_run_stream_v2(BloomPipeline* pipeline, BloomSlice input_json,
                                                  BloomSlice params_json, BloomStreamCallbackV2 callback,
                                                  void* user_data, const BloomCancellationToken* cancellation,
                                                  char* error_buffer, size_t error_buffer_len) {
  try {
    if (pipeline == nullptr || callback == nullptr) {
      write_error("Null argument passed to bloom_pipeline_run_stream_v2", error_buffer, error_buffer_len);
      return BLOOM_STATUS_INVALID_ARGUMENT;
    }
    std::string input, params, err;
    int32_t st = slice_text(input_json, "input_json", kMaxJsonBytes, input, err);
    if (st == BLOOM_STATUS_OK) st = slice_text(params_json, "params_json", kMaxJsonBytes, params, err);
    if (st == BLOOM_STATUS_OK)
      st = stream_impl(pipeline, input, params, cancellation, err, [&](const std::string& chunk) {
        callback(user_data, reinterpret_cast<const uint8_t*>(chunk.data()), chunk.size());
      });
    if (st != BLOOM_STATUS_OK) {
      write_error(err, error_buffer, error_buffer_len);
      return st;
    }
    clear_error(error_buffer, error_buffer_len);
    return BLOOM_STATUS_OK;
  } catch (...) {
    write_error("internal error at the FFI boundary", error_buffer, error_buffer_len);
    return BLOOM_STATUS_PANIC;
  }
}

BLOOM_EXPORT int32_t bloom_pipeline_run_stream(BloomPipeline* pipeline, const char* input_json,
                                               const char* params_json, BloomStreamCallback callback, void* user_data,
                                               char* error_buffer, size_t error_buffer_len) {
  if (pipeline == nullptr || input_json == nullptr || params_json == nullptr || callback == nullptr) {
    write_error("Null argument passed to bloom_pipeline_run_stream", error_buffer, error_buffer_len);
    return BLOOM_STATUS_INVALID_ARGUMENT;
  }
  try {
    std::string input(input_json), params(params_json), err;
    int32_t st = BLOOM_STATUS_OK;
    if (!valid_utf8(reinterpret_cast<const uint8_t*>(input.data()), input.size()) ||
        !valid_utf8(reinterpret_cast<const uint8_t*>(params.data()), params.size())) {
      err = "input is not valid UTF-8";
      st = BLOOM_STATUS_INVALID_UTF8;
    } else {
      st = stream_impl(pipeline, input, params, nullptr, err, [&](const std::string& chunk) {
        callback(user_data, chunk.c_str());  // NUL-terminated for revision-1 callbacks
      });
    }
    if (st != BLOOM_STATUS_OK) {
      write_error(err, error_buffer, error_buffer_len);
      return st;
    }
    clear_error(error_buffer, error_buffer_len);
    return BLOOM_STATUS_OK;
  } catch (...) {
    write_error("internal error at the FFI boundary", error_buffer, error_buffer_len);
    return BLOOM_STATUS_PANIC;
  }
}

BLOOM_EXPORT void bloom_buffer_free(BloomOwnedBuffer* buffer) {
  if (buffer == nullptr) return;
  std::free(buffer->data);
  buffer->data = nullptr;
  buffer->len = 0;
}

BLOOM_EXPORT void bloom_string_free(char* s) { std::free(s); }
