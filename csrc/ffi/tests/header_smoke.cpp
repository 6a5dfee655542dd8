// Compiles bloom.h as C++17 (extern "C" linkage, no name clashes).
#include "../bloom.h"

#include <type_traits>

static_assert(std::is_same<decltype(&bloom_abi_version), uint32_t (*)()>::value, "abi version signature");
static_assert(sizeof(BloomSlice) == sizeof(void*) + sizeof(size_t), "BloomSlice layout");

int main() {
  BloomSlice s{nullptr, 0};
  BloomOwnedBuffer b{nullptr, 0};
  return (s.len == 0 && b.data == nullptr && BLOOM_ABI_VERSION == 2u) ? 0 : 1;
}
