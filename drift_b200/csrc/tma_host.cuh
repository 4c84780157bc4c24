// Host-side tensor maps for the TMA copies: the driver's cuTensorMapEncodeTiled,
// reached through the runtime's entry-point query (no link to libcuda).
#pragma once

#include <cuda.h>
#include <stdint.h>

namespace drift {

// Whether the driver offers tensor maps at all.
bool tensor_maps_available();

// Rows of 32-bit words: dims {row_words, rows}, row stride row_words * 4
// bytes, a box of {box_words, box_rows}, no swizzle, zero fill past the ends.
int encode_word_rows(CUtensorMap* map, const void* base, int64_t row_words, int64_t rows,
                     int box_words, int box_rows);

// F16 rows: dims {cols, rows}, a box of {64, box_rows} (128 bytes wide) in the
// 128-byte swizzle that UMMA's K-major canonical layout reads.
int encode_f16_sw128(CUtensorMap* map, const void* base, int64_t cols, int64_t rows, int box_rows);

}  // namespace drift
