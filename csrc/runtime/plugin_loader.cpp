// Native engine plugins: dlopen a shared library, resolve bloom_plugin_init,
// and drive its CBloomEngine function table (csrc/plugin/bloom_plugin.h).
// Exposed to Python as bloom_b200._runtime.NativePlugin; the Python side
// (bloom_b200/engine/plugins.py) validates the manifest and adapts the
// plugin to the engine registry and InferencePipeline.
//
// Behaviour follows the reference loader (crates/engine/src/plugin/mod.rs:
// load_engine_plugin, FfiPluginEngine): only "native" entry points are
// loaded, a non-zero init code is an error, and plugin-owned strings are
// returned through free_string.
#include <dlfcn.h>
#include <pybind11/functional.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "../plugin/bloom_plugin.h"

namespace py = pybind11;

namespace bloom {
namespace rt {

class NativePlugin {
 public:
  explicit NativePlugin(const std::string& path) {
    handle_ = ::dlopen(path.c_str(), RTLD_NOW | RTLD_LOCAL);
    if (handle_ == nullptr) {
      const char* e = ::dlerror();
      throw std::runtime_error("failed to load plugin library " + path + ": " + (e ? e : "unknown error"));
    }
    auto init = reinterpret_cast<BloomPluginInitFn>(::dlsym(handle_, "bloom_plugin_init"));
    if (init == nullptr) {
      ::dlclose(handle_);
      handle_ = nullptr;
      throw std::runtime_error("plugin library does not export 'bloom_plugin_init'");
    }
    const int32_t rc = init(&eng_);
    if (rc != 0) {
      ::dlclose(handle_);
      handle_ = nullptr;
      throw std::runtime_error("bloom_plugin_init failed with error code " + std::to_string(rc));
    }
    if (eng_.name == nullptr || eng_.load_model == nullptr || eng_.model_infer == nullptr ||
        eng_.free_model == nullptr || eng_.free_string == nullptr)
      throw std::runtime_error("plugin function table is incomplete");
  }
  ~NativePlugin() {
    if (handle_ != nullptr) ::dlclose(handle_);
  }
  NativePlugin(const NativePlugin&) = delete;
  NativePlugin& operator=(const NativePlugin&) = delete;

  std::string name() const {
    const char* n = eng_.name();
    return n ? n : "";
  }
  std::vector<int32_t> codes(bool devices) const {
    int32_t buf[64];
    size_t n = 64;
    auto fn = devices ? eng_.supported_devices : eng_.supported_modalities;
    if (fn == nullptr || fn(buf, &n) != 0) return {};
    return std::vector<int32_t>(buf, buf + (n < 64 ? n : 64));
  }
  uintptr_t load_model(const std::string& path, int32_t device) {
    void* m = nullptr;
    const int32_t rc = eng_.load_model(path.c_str(), device, &m);
    if (rc != 0 || m == nullptr) throw std::runtime_error("plugin load_model failed with code " + std::to_string(rc));
    return reinterpret_cast<uintptr_t>(m);
  }
  void free_model(uintptr_t m) { eng_.free_model(reinterpret_cast<void*>(m)); }
  std::string take(char* s) {
    std::string r = s ? s : "";
    if (s) eng_.free_string(s);
    return r;
  }
  std::string metadata(uintptr_t m) {
    if (eng_.model_metadata == nullptr) return "{}";
    char* out = nullptr;
    const int32_t rc = eng_.model_metadata(reinterpret_cast<void*>(m), &out);
    if (rc != 0) throw std::runtime_error("plugin model_metadata failed with code " + std::to_string(rc));
    return take(out);
  }
  std::string infer(uintptr_t m, const std::string& input_json) {
    char* out = nullptr;
    int32_t rc;
    {
      py::gil_scoped_release nogil;
      rc = eng_.model_infer(reinterpret_cast<void*>(m), input_json.c_str(), &out);
    }
    if (rc != 0) {
      take(out);
      throw std::runtime_error("plugin model_infer failed with code " + std::to_string(rc));
    }
    return take(out);
  }
  // Streams chunks to `cb`; returning False from cb stops the stream.
  int32_t infer_stream(uintptr_t m, const std::string& input_json, const std::function<bool(std::string)>& cb) {
    if (eng_.model_infer_stream == nullptr) throw std::runtime_error("plugin does not stream");
    struct Ctx {
      const std::function<bool(std::string)>* cb;
      bool error = false;
      std::string what;
    } ctx{&cb};
    auto tramp = [](void* user, const char* chunk) -> int32_t {
      auto* c = static_cast<Ctx*>(user);
      py::gil_scoped_acquire gil;
      try {
        return (*c->cb)(chunk ? std::string(chunk) : std::string()) ? 0 : 1;
      } catch (const std::exception& e) {
        c->error = true;
        c->what = e.what();
        return 1;
      }
    };
    int32_t rc;
    {
      py::gil_scoped_release nogil;
      rc = eng_.model_infer_stream(reinterpret_cast<void*>(m), input_json.c_str(), tramp, &ctx);
    }
    if (ctx.error) throw std::runtime_error("stream callback raised: " + ctx.what);
    return rc;
  }

 private:
  void* handle_ = nullptr;
  CBloomEngine eng_{};
};

}  // namespace rt
}  // namespace bloom

void register_plugin(py::module_& m) {
  using bloom::rt::NativePlugin;
  py::class_<NativePlugin>(m, "NativePlugin")
      .def(py::init<const std::string&>())
      .def("name", &NativePlugin::name)
      .def("supported_modalities", [](const NativePlugin& p) { return p.codes(false); })
      .def("supported_devices", [](const NativePlugin& p) { return p.codes(true); })
      .def("load_model", &NativePlugin::load_model)
      .def("free_model", &NativePlugin::free_model)
      .def("metadata", &NativePlugin::metadata)
      .def("infer", &NativePlugin::infer)
      .def("infer_stream", &NativePlugin::infer_stream);
}
