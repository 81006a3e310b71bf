// Host helpers shared by the kernel translation units.
#pragma once

#include <cuda.h>
#include <stdint.h>

namespace algx {

// 2-D TMA descriptor over a row-major [outer][inner] tensor with the given
// row stride; box = box_outer rows x box_inner elements; optional 128-byte
// swizzle (box_inner * element size must then be <= 128).
int make_tmap_2d(CUtensorMap* map, const void* base, int32_t dtype, uint64_t inner, uint64_t outer,
                 uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer, bool swizzle128);

// Per-device error word (see DeviceError); nullptr if it cannot be created.
int* device_error_word();

}  // namespace algx
