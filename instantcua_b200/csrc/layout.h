// Device weight layout shared by the host packer (pack.cpp) and the kernels (gemv.cuh).
//
// A matrix [n_rows, K] is cut into 16-row tiles and 64-column units; a unit's bytes are the
// A-operand registers of four mma.sync.m16n8k16 of one warp, followed by its 32-column-group
// scales.  Units are stored slice-major: K is split into `slices` equal slices (one per warp of
// the GEMV that reads the matrix) and unit (tile, kk) of slice w = kk / ku sits at
// ((w * n_tiles + tile) * ku + kk % ku), ku = (K / 64) / slices, so a warp's share of a run of
// consecutive tiles is one contiguous byte range.
#pragma once
#include <cstdint>

namespace icua_layout {

constexpr int FMT_Q8 = 1, FMT_Q4A = 2, FMT_Q4S = 3;
// q4s: 32 lanes x 16 B nibbles + 8 rows x 2 groups x (2 x fp16) scales;
// q4a (reference affine q4, groups of 64): the same nibbles + 8 x (scale, bias) of rows g, g+8
constexpr int Q4_UNIT_BYTES = 576;
constexpr int Q8_UNIT_BYTES = 1088;  // 32 lanes x 32 B bytes + scales

#if defined(__CUDACC__)
#define ICUA_HD __host__ __device__
#else
#define ICUA_HD
#endif

ICUA_HD constexpr int unit_bytes(int fmt) { return fmt == FMT_Q8 ? Q8_UNIT_BYTES : Q4_UNIT_BYTES; }
// K slices (= GEMV warps): q4 decode projections 16, q8 matrices 8.
ICUA_HD constexpr int fmt_slices(int fmt) { return fmt == FMT_Q8 ? 8 : 16; }

ICUA_HD inline long long unit_offset(int fmt, int n_tiles, int upt, int tile, int kk) {
    const int ku = upt / fmt_slices(fmt);
    const int w = kk / ku, u = kk - w * ku;
    return (((long long)w * n_tiles + tile) * ku + u) * unit_bytes(fmt);
}

}  // namespace icua_layout
