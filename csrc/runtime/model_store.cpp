// Model package hashing for the acquisition control plane (import,
// integrity verification, inventory): SHA-256 (FIPS 180-4) of files, read
// with large sequential reads, one thread per file up to a limit, so a
// multi-shard safetensors package of tens of GB hashes at disk speed
// instead of one core's hashing speed.  A package digest is the SHA-256 of
// the sorted lines "<relative path>\t<size>\t<file sha256>\n".
// Reference behaviour: model_integrity.rs (re-hash of installed files against
// the recorded checksum), model_import.rs (checksummed import).
#include <pybind11/functional.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <functional>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

namespace py = pybind11;

namespace bloom {
namespace rt {
namespace {

// SHA-256 round constants and initial hash value (FIPS 180-4, section 4.2.2 / 5.3.3)
constexpr uint32_t kK[64] = {
    0x428a2f98, 0x71374491, 0xb5c0fbcf, 0xe9b5dba5, 0x3956c25b, 0x59f111f1, 0x923f82a4, 0xab1c5ed5,
    0xd807aa98, 0x12835b01, 0x243185be, 0x550c7dc3, 0x72be5d74, 0x80deb1fe, 0x9bdc06a7, 0xc19bf174,
    0xe49b69c1, 0xefbe4786, 0x0fc19dc6, 0x240ca1cc, 0x2de92c6f, 0x4a7484aa, 0x5cb0a9dc, 0x76f988da,
    0x983e5152, 0xa831c66d, 0xb00327c8, 0xbf597fc7, 0xc6e00bf3, 0xd5a79147, 0x06ca6351, 0x14292967,
    0x27b70a85, 0x2e1b2138, 0x4d2c6dfc, 0x53380d13, 0x650a7354, 0x766a0abb, 0x81c2c92e, 0x92722c85,
    0xa2bfe8a1, 0xa81a664b, 0xc24b8b70, 0xc76c51a3, 0xd192e819, 0xd6990624, 0xf40e3585, 0x106aa070,
    0x19a4c116, 0x1e376c08, 0x2748774c, 0x34b0bcb5, 0x391c0cb3, 0x4ed8aa4a, 0x5b9cca4f, 0x682e6ff3,
    0x748f82ee, 0x78a5636f, 0x84c87814, 0x8cc70208, 0x90befffa, 0xa4506ceb, 0xbef9a3f7, 0xc67178f2};

inline uint32_t rotr(uint32_t x, int n) { return (x >> n) | (x << (32 - n)); }

class Sha256 {
 public:
  Sha256() { reset(); }
  void reset() {
    h_[0] = 0x6a09e667;
    h_[1] = 0xbb67ae85;
    h_[2] = 0x3c6ef372;
    h_[3] = 0xa54ff53a;
    h_[4] = 0x510e527f;
    h_[5] = 0x9b05688c;
    h_[6] = 0x1f83d9ab;
    h_[7] = 0x5be0cd19;
    len_ = 0;
    fill_ = 0;
  }
  void update(const uint8_t* p, size_t n) {
    len_ += n;
    if (fill_) {
      const size_t take = std::min(n, size_t(64) - fill_);
      std::memcpy(buf_ + fill_, p, take);
      fill_ += take;
      p += take;
      n -= take;
      if (fill_ == 64) {
        block(buf_);
        fill_ = 0;
      }
    }
    while (n >= 64) {
      block(p);
      p += 64;
      n -= 64;
    }
    if (n) {
      std::memcpy(buf_, p, n);
      fill_ = n;
    }
  }
  std::string hex() {
    const uint64_t bits = len_ * 8;
    const uint8_t one = 0x80;
    update(&one, 1);
    const uint8_t zero = 0;
    while (fill_ != 56) update(&zero, 1);
    uint8_t lb[8];
    for (int i = 0; i < 8; ++i) lb[i] = static_cast<uint8_t>(bits >> (56 - 8 * i));
    update(lb, 8);
    static const char* d = "0123456789abcdef";
    std::string s(64, '0');
    for (int i = 0; i < 8; ++i)
      for (int b = 0; b < 4; ++b) {
        const uint8_t v = static_cast<uint8_t>(h_[i] >> (24 - 8 * b));
        s[i * 8 + b * 2] = d[v >> 4];
        s[i * 8 + b * 2 + 1] = d[v & 15];
      }
    return s;
  }

 private:
  void block(const uint8_t* p) {
    uint32_t w[64];
    for (int i = 0; i < 16; ++i)
      w[i] = (uint32_t(p[4 * i]) << 24) | (uint32_t(p[4 * i + 1]) << 16) | (uint32_t(p[4 * i + 2]) << 8) | p[4 * i + 3];
    for (int i = 16; i < 64; ++i) {
      const uint32_t s0 = rotr(w[i - 15], 7) ^ rotr(w[i - 15], 18) ^ (w[i - 15] >> 3);
      const uint32_t s1 = rotr(w[i - 2], 17) ^ rotr(w[i - 2], 19) ^ (w[i - 2] >> 10);
      w[i] = w[i - 16] + s0 + w[i - 7] + s1;
    }
    uint32_t a = h_[0], b = h_[1], c = h_[2], d = h_[3], e = h_[4], f = h_[5], g = h_[6], h = h_[7];
    for (int i = 0; i < 64; ++i) {
      const uint32_t S1 = rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25);
      const uint32_t ch = (e & f) ^ (~e & g);
      const uint32_t t1 = h + S1 + ch + kK[i] + w[i];
      const uint32_t S0 = rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22);
      const uint32_t mj = (a & b) ^ (a & c) ^ (b & c);
      const uint32_t t2 = S0 + mj;
      h = g;
      g = f;
      f = e;
      e = d + t1;
      d = c;
      c = b;
      b = a;
      a = t1 + t2;
    }
    h_[0] += a;
    h_[1] += b;
    h_[2] += c;
    h_[3] += d;
    h_[4] += e;
    h_[5] += f;
    h_[6] += g;
    h_[7] += h;
  }
  uint32_t h_[8];
  uint64_t len_;
  uint8_t buf_[64];
  size_t fill_;
};

struct FileDigest {
  std::string path;
  int64_t size = -1;
  std::string sha256;
  std::string error;
};

// Hash one file; `done` accumulates bytes read (progress), `cancel` stops early.
FileDigest hash_file(const std::string& path, std::atomic<int64_t>* done, const std::atomic<bool>* cancel) {
  FileDigest r;
  r.path = path;
  FILE* f = std::fopen(path.c_str(), "rb");
  if (!f) {
    r.error = "cannot open " + path;
    return r;
  }
  std::vector<uint8_t> buf(size_t(4) << 20);
  Sha256 h;
  int64_t total = 0;
  for (;;) {
    if (cancel && cancel->load()) {
      r.error = "cancelled";
      break;
    }
    const size_t n = std::fread(buf.data(), 1, buf.size(), f);
    if (n > 0) {
      h.update(buf.data(), n);
      total += static_cast<int64_t>(n);
      if (done) done->fetch_add(static_cast<int64_t>(n));
    }
    if (n < buf.size()) {
      if (std::ferror(f)) r.error = "read error in " + path;
      break;
    }
  }
  std::fclose(f);
  if (r.error.empty()) {
    r.size = total;
    r.sha256 = h.hex();
  }
  return r;
}

}  // namespace

std::string sha256_bytes(const std::string& data) {
  Sha256 h;
  h.update(reinterpret_cast<const uint8_t*>(data.data()), data.size());
  return h.hex();
}

// Hash files on up to `threads` threads; progress(bytes_done) is called from
// the calling thread roughly every 100 ms while the GIL is held; it may
// return False to cancel.
std::vector<FileDigest> hash_files(const std::vector<std::string>& paths, int threads,
                                   const std::function<bool(int64_t)>& progress) {
  std::vector<FileDigest> out(paths.size());
  std::atomic<size_t> next{0};
  std::atomic<int64_t> done{0};
  std::atomic<bool> cancel{false};
  std::atomic<int> running{0};
  const int nt = std::max(1, std::min<int>(threads, static_cast<int>(paths.size())));
  std::vector<std::thread> pool;
  running = nt;
  for (int t = 0; t < nt; ++t)
    pool.emplace_back([&] {
      for (size_t i; (i = next.fetch_add(1)) < paths.size();) out[i] = hash_file(paths[i], &done, &cancel);
      running.fetch_sub(1);
    });
  if (progress) {
    while (running.load() > 0) {
      std::this_thread::sleep_for(std::chrono::milliseconds(100));
      py::gil_scoped_acquire gil;
      if (!progress(done.load())) cancel = true;
    }
  }
  for (auto& th : pool) th.join();
  return out;
}

}  // namespace rt
}  // namespace bloom

void register_model_store(py::module_& m) {
  using namespace bloom::rt;
  m.def("sha256_bytes", [](const py::bytes& b) { return sha256_bytes(std::string(b)); });
  m.def(
      "hash_files",
      [](const std::vector<std::string>& paths, int threads, std::function<bool(int64_t)> progress) {
        std::vector<FileDigest> res;
        {
          py::gil_scoped_release nogil;
          res = hash_files(paths, threads, progress);
        }
        py::list out;
        for (const auto& r : res) {
          py::dict d;
          d["path"] = r.path;
          d["size"] = r.size;
          d["sha256"] = r.sha256;
          d["error"] = r.error;
          out.append(d);
        }
        return out;
      },
      py::arg("paths"), py::arg("threads") = 4, py::arg("progress") = std::function<bool(int64_t)>());
}

// ---------------------------------------------------------------- PNG scanline reconstruction
// Reverses the five PNG filter types (None, Sub, Up, Average, Paeth; PNG
// specification section 9) over the inflated IDAT stream of a non-interlaced
// 8-bit image: `raw` holds h rows of (1 filter byte + w * bpp bytes).
// The per-pixel dependency on the left neighbour makes this sequential per
// row, so it runs here rather than in Python.
namespace {
inline uint8_t paeth(int a, int b, int c) {
  const int p = a + b - c;
  const int pa = std::abs(p - a), pb = std::abs(p - b), pc = std::abs(p - c);
  if (pa <= pb && pa <= pc) return static_cast<uint8_t>(a);
  if (pb <= pc) return static_cast<uint8_t>(b);
  return static_cast<uint8_t>(c);
}
}  // namespace

py::bytes png_unfilter(const py::bytes& raw_b, int h, int w, int bpp) {
  const std::string raw(raw_b);
  const size_t stride = static_cast<size_t>(w) * bpp;
  if (h <= 0 || w <= 0 || bpp <= 0 || raw.size() < static_cast<size_t>(h) * (stride + 1))
    throw std::invalid_argument("png_unfilter: truncated image data");
  std::string out(static_cast<size_t>(h) * stride, '\0');
  uint8_t* o = reinterpret_cast<uint8_t*>(&out[0]);
  const uint8_t* r = reinterpret_cast<const uint8_t*>(raw.data());
  for (int y = 0; y < h; ++y) {
    const uint8_t ft = r[y * (stride + 1)];
    const uint8_t* src = r + y * (stride + 1) + 1;
    uint8_t* cur = o + y * stride;
    const uint8_t* prev = y > 0 ? o + (y - 1) * stride : nullptr;
    for (size_t x = 0; x < stride; ++x) {
      const int a = x >= static_cast<size_t>(bpp) ? cur[x - bpp] : 0;
      const int b = prev ? prev[x] : 0;
      const int c = (prev && x >= static_cast<size_t>(bpp)) ? prev[x - bpp] : 0;
      int v = src[x];
      switch (ft) {
        case 0: break;
        case 1: v += a; break;
        case 2: v += b; break;
        case 3: v += (a + b) >> 1; break;
        case 4: v += paeth(a, b, c); break;
        default: throw std::invalid_argument("png_unfilter: unknown filter type");
      }
      cur[x] = static_cast<uint8_t>(v);
    }
  }
  return py::bytes(out);
}

void register_image(py::module_& m) { m.def("png_unfilter", &png_unfilter); }
