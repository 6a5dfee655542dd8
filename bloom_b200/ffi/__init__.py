"""C ABI support: the Python side of libbloom_ffi (csrc/ffi/bloom_ffi.cpp) and
a ctypes client (`BloomClient`) for the same library."""
