/* Compiles bloom.h as C99 and checks the ABI constants and zero-initialised structs. */
#include "../bloom.h"

int main(void) {
  BloomSlice input = {0};
  BloomOwnedBuffer output = {0};
  BloomStatus status = BLOOM_STATUS_OK;
  return (input.len == 0 && output.len == 0 && status == BLOOM_STATUS_OK && BLOOM_ABI_VERSION >= 2u &&
          BLOOM_STATUS_CANCELLED == -8)
             ? 0
             : 1;
}
