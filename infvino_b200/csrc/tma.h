// Host-side TMA tensor-map encoding through the driver entry point (no link
// dependency on libcuda).
#pragma once

#include <cstdint>
#include <cuda.h>
#include <string>

namespace ivb {

// Encodes a tiled fp16 tensor map.  dims/box/elem_strides have `rank` entries,
// byte_strides has rank-1 entries (dimension 1..rank-1).  Returns false and fills
// `err` if the driver rejects the description.
bool encode_tiled_f16(CUtensorMap *map, int rank, const void *base, const uint64_t *dims,
                      const uint64_t *byte_strides, const uint32_t *box, const uint32_t *elem_strides,
                      CUtensorMapSwizzle swizzle, std::string *err);

CUtensorMapSwizzle swizzle_for_row_bytes(int row_bytes);

}  // namespace ivb
