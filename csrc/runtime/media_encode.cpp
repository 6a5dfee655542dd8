// Video / image output of the diffusion pipeline: animated GIF (GIF89a,
// LZW) and PNG frames, written from u8 RGB frames on the host.
//
// Reference behaviour: executor/wan/video_encoder.rs (encode_gif :43-83 with
// an LZW stream per frame and a per-frame delay, PNG / JPEG frame dumps
// :359-384).  Colour quantisation here is a fixed 6 x 7 x 6 RGB cube (252
// colours, ordered so that index = r6 * 42 + g7 * 6 + b6) with a 4 x 4
// Bayer ordered dither, so frames need no palette search and quantise in
// one pass.  PNG frames are zlib streams of stored (uncompressed) deflate
// blocks with the CRC-32 and Adler-32 checksums of the specifications
// (RFC 1950 / 1951, PNG section 5).
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <array>
#include <cstdint>
#include <fstream>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <vector>

namespace py = pybind11;

namespace {

constexpr int kR = 6, kG = 7, kB = 6;
constexpr int kBayer[4][4] = {{0, 8, 2, 10}, {12, 4, 14, 6}, {3, 11, 1, 9}, {15, 7, 13, 5}};

inline int level(int v, int levels, int y, int x) {
  // ordered dither: threshold offset in [-0.5, 0.5) of one quantisation step
  const float step = 255.f / (levels - 1);
  const float t = (kBayer[y & 3][x & 3] + 0.5f) / 16.f - 0.5f;
  int q = static_cast<int>(v / step + 0.5f + t);
  return q < 0 ? 0 : (q >= levels ? levels - 1 : q);
}

struct BitWriter {
  std::string& out;
  std::string block;
  uint32_t acc = 0;
  int nbits = 0;
  explicit BitWriter(std::string& o) : out(o) {}
  void put(int code, int width) {
    acc |= static_cast<uint32_t>(code) << nbits;
    nbits += width;
    while (nbits >= 8) {
      byte(static_cast<char>(acc & 0xff));
      acc >>= 8;
      nbits -= 8;
    }
  }
  void byte(char c) {
    block.push_back(c);
    if (block.size() == 255) flush_block();
  }
  void flush_block() {
    if (block.empty()) return;
    out.push_back(static_cast<char>(block.size()));
    out += block;
    block.clear();
  }
  void finish() {
    if (nbits > 0) byte(static_cast<char>(acc & 0xff));
    acc = 0;
    nbits = 0;
    flush_block();
    out.push_back('\0');  // block terminator
  }
};

// LZW image data of one frame of palette indices (GIF89a appendix F)
void lzw(const std::vector<uint8_t>& idx, std::string& out) {
  const int min_code = 8;
  out.push_back(static_cast<char>(min_code));
  BitWriter bw(out);
  const int clear = 1 << min_code, eoi = clear + 1;
  std::unordered_map<uint32_t, int> dict;
  dict.reserve(8192);
  int next = eoi + 1, width = min_code + 1;
  bw.put(clear, width);
  if (idx.empty()) {
    bw.put(eoi, width);
    bw.finish();
    return;
  }
  int prefix = idx[0];
  for (size_t i = 1; i < idx.size(); ++i) {
    const uint32_t key = (static_cast<uint32_t>(prefix) << 8) | idx[i];
    auto it = dict.find(key);
    if (it != dict.end()) {
      prefix = it->second;
      continue;
    }
    bw.put(prefix, width);
    if (next < 4096) {
      dict.emplace(key, next);
      if (next == (1 << width) && width < 12) ++width;
      ++next;
    } else {  // table full: restart
      bw.put(clear, width);
      dict.clear();
      next = eoi + 1;
      width = min_code + 1;
    }
    prefix = idx[i];
  }
  bw.put(prefix, width);
  bw.put(eoi, width);
  bw.finish();
}

void le16(std::string& o, int v) {
  o.push_back(static_cast<char>(v & 0xff));
  o.push_back(static_cast<char>((v >> 8) & 0xff));
}

std::string gif_bytes(const std::string& rgb, int frames, int h, int w, int delay_cs, int loops) {
  if (frames <= 0 || h <= 0 || w <= 0 || w > 65535 || h > 65535)
    throw std::invalid_argument("gif: bad dimensions");
  if (rgb.size() != static_cast<size_t>(frames) * h * w * 3) throw std::invalid_argument("gif: frames * h * w * 3 bytes");
  std::string o = "GIF89a";
  le16(o, w);
  le16(o, h);
  o.push_back(static_cast<char>(0xF7));  // global colour table, 8 bits, 256 entries
  o.push_back('\0');
  o.push_back('\0');
  for (int i = 0; i < 256; ++i) {
    int r = 0, g = 0, b = 0;
    if (i < kR * kG * kB) {
      r = (i / (kG * kB)) * 255 / (kR - 1);
      g = ((i / kB) % kG) * 255 / (kG - 1);
      b = (i % kB) * 255 / (kB - 1);
    }
    o.push_back(static_cast<char>(r));
    o.push_back(static_cast<char>(g));
    o.push_back(static_cast<char>(b));
  }
  // NETSCAPE2.0 application extension: loop count (0 = forever)
  o += std::string("\x21\xFF\x0BNETSCAPE2.0\x03\x01", 16);
  le16(o, loops);
  o.push_back('\0');
  const uint8_t* px = reinterpret_cast<const uint8_t*>(rgb.data());
  std::vector<uint8_t> idx(static_cast<size_t>(h) * w);
  for (int f = 0; f < frames; ++f) {
    o += std::string("\x21\xF9\x04\x04", 4);  // graphic control: dispose "do not dispose"
    le16(o, delay_cs);
    o.push_back('\0');
    o.push_back('\0');
    o.push_back(',');  // image descriptor
    le16(o, 0);
    le16(o, 0);
    le16(o, w);
    le16(o, h);
    o.push_back('\0');
    const uint8_t* fp = px + static_cast<size_t>(f) * h * w * 3;
    for (int y = 0; y < h; ++y)
      for (int x = 0; x < w; ++x) {
        const uint8_t* p = fp + (static_cast<size_t>(y) * w + x) * 3;
        idx[static_cast<size_t>(y) * w + x] =
            static_cast<uint8_t>(level(p[0], kR, y, x) * kG * kB + level(p[1], kG, y, x) * kB + level(p[2], kB, y, x));
      }
    lzw(idx, o);
  }
  o.push_back(';');
  return o;
}

// ---------------------------------------------------------------- PNG
uint32_t crc32(const uint8_t* d, size_t n, uint32_t c = 0xffffffffu) {
  static const std::array<uint32_t, 256> table = [] {
    std::array<uint32_t, 256> t{};
    for (uint32_t i = 0; i < 256; ++i) {
      uint32_t v = i;
      for (int k = 0; k < 8; ++k) v = (v & 1) ? 0xEDB88320u ^ (v >> 1) : v >> 1;
      t[i] = v;
    }
    return t;
  }();
  for (size_t i = 0; i < n; ++i) c = table[(c ^ d[i]) & 0xff] ^ (c >> 8);
  return c;
}

void be32(std::string& o, uint32_t v) {
  for (int s = 24; s >= 0; s -= 8) o.push_back(static_cast<char>((v >> s) & 0xff));
}

void chunk(std::string& o, const char* type, const std::string& data) {
  be32(o, static_cast<uint32_t>(data.size()));
  std::string td(type, 4);
  td += data;
  o += td;
  be32(o, crc32(reinterpret_cast<const uint8_t*>(td.data()), td.size()) ^ 0xffffffffu);
}

std::string png_bytes(const std::string& rgb, int h, int w) {
  if (h <= 0 || w <= 0 || rgb.size() != static_cast<size_t>(h) * w * 3) throw std::invalid_argument("png: h * w * 3 bytes");
  std::string raw;
  raw.reserve(static_cast<size_t>(h) * (w * 3 + 1));
  for (int y = 0; y < h; ++y) {
    raw.push_back('\0');  // filter type None
    raw.append(rgb, static_cast<size_t>(y) * w * 3, static_cast<size_t>(w) * 3);
  }
  std::string z = "\x78\x01";  // zlib header: deflate, 32 KiB window, no preset dictionary
  uint32_t a = 1, b = 0;
  for (unsigned char c : raw) {
    a = (a + c) % 65521;
    b = (b + a) % 65521;
  }
  for (size_t pos = 0; pos < raw.size() || pos == 0; pos += 65535) {
    const size_t n = std::min<size_t>(65535, raw.size() - pos);
    const bool last = pos + n >= raw.size();
    z.push_back(last ? '\x01' : '\x00');  // stored block
    z.push_back(static_cast<char>(n & 0xff));
    z.push_back(static_cast<char>(n >> 8));
    z.push_back(static_cast<char>(~n & 0xff));
    z.push_back(static_cast<char>((~n >> 8) & 0xff));
    z.append(raw, pos, n);
    if (last) break;
  }
  be32(z, (b << 16) | a);
  std::string o = "\x89PNG\r\n\x1a\n";
  std::string ihdr;
  be32(ihdr, static_cast<uint32_t>(w));
  be32(ihdr, static_cast<uint32_t>(h));
  ihdr += std::string("\x08\x02\x00\x00\x00", 5);  // 8-bit RGB, deflate, adaptive filter, no interlace
  chunk(o, "IHDR", ihdr);
  chunk(o, "IDAT", z);
  chunk(o, "IEND", "");
  return o;
}

}  // namespace

void register_media_encode(py::module_& m) {
  m.def(
      "encode_gif",
      [](const py::bytes& rgb, int frames, int h, int w, int delay_cs, int loops) {
        std::string s(rgb);
        std::string out;
        {
          py::gil_scoped_release nogil;
          out = gif_bytes(s, frames, h, w, delay_cs, loops);
        }
        return py::bytes(out);
      },
      "u8 RGB frames [frames, h, w, 3] -> animated GIF89a bytes (6x7x6 colour cube, ordered dither)",
      py::arg("rgb"), py::arg("frames"), py::arg("height"), py::arg("width"), py::arg("delay_cs") = 6,
      py::arg("loops") = 0);
  m.def(
      "encode_png",
      [](const py::bytes& rgb, int h, int w) { return py::bytes(png_bytes(std::string(rgb), h, w)); },
      "u8 RGB [h, w, 3] -> PNG bytes (stored deflate blocks)", py::arg("rgb"), py::arg("height"), py::arg("width"));
}
