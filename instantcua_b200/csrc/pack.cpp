// Host-side quantizers and the repack from the reference (file) layout to the device tile layout.
//
// Quantizers restate the reference Converter (Sources/Engine/Convert.swift:215-241 for q8) and the
// BASELINE symmetric q4 defined by analogy with it; results are bit-identical to the numpy
// restatement in oracle/qwen3vl_oracle.py (checked by tests/test_cpu_abi.py).  Compiled without
// fast-math so every fp32 operation rounds as IEEE-754 single precision.
#include <cmath>
#include <cstdint>
#include <cstring>
#include <thread>
#include <vector>

#include "../../include/icua.h"
#include "layout.h"

namespace icua_host {

// fp32 -> fp16 bits, round to nearest even (as numpy's astype(float16) and Swift's Float16(x)).
uint16_t f32_to_f16_bits(float f) {
    uint32_t x;
    std::memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t absx = x & 0x7FFFFFFFu;
    if (absx >= 0x7F800000u) return (uint16_t)(sign | (absx > 0x7F800000u ? 0x7E00u : 0x7C00u));
    if (absx >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u);  // rounds to inf
    if (absx < 0x38800000u) {                                     // subnormal or zero in fp16
        if (absx < 0x33000000u) return (uint16_t)sign;            // < 2^-25 rounds to 0
        const uint32_t e = absx >> 23;
        const uint32_t m = (absx & 0x7FFFFFu) | 0x800000u;
        // value = m * 2^(e-150); the fp16 subnormal unit is 2^-24, so q = m * 2^(e-126)
        const uint32_t sh = 126 - e;  // bits to drop (>= 14)
        uint32_t q = m >> sh;
        const uint32_t rem = m & ((1u << sh) - 1u);
        const uint32_t half = 1u << (sh - 1);
        if (rem > half || (rem == half && (q & 1u))) q += 1;
        return (uint16_t)(sign | q);
    }
    uint32_t r = absx - 0x38000000u;  // rebias exponent 127 -> 15
    const uint32_t mant_drop = r & 0x1FFFu;
    r >>= 13;
    if (mant_drop > 0x1000u || (mant_drop == 0x1000u && (r & 1u))) r += 1;
    return (uint16_t)(sign | r);
}

float f16_bits_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t e = (h >> 10) & 0x1Fu;
    const uint32_t m = h & 0x3FFu;
    uint32_t x;
    if (e == 0) {
        if (m == 0) {
            x = sign;
        } else {  // subnormal: m * 2^-24
            float v = (float)m * 5.9604644775390625e-08f;
            std::memcpy(&x, &v, 4);
            x |= sign;
        }
    } else if (e == 31) {
        x = sign | 0x7F800000u | (m << 13);
    } else {
        x = sign | ((e + 112) << 23) | (m << 13);
    }
    float f;
    std::memcpy(&f, &x, 4);
    return f;
}

template <typename F>
static void parallel_rows(int rows, F&& fn) {
    unsigned nt = std::thread::hardware_concurrency();
    if (nt == 0) nt = 1;
    if (nt > 32) nt = 32;
    if (rows < 256) nt = 1;
    std::vector<std::thread> th;
    for (unsigned t = 0; t < nt; ++t) {
        th.emplace_back([&, t] {
            const int a = (int)((long long)rows * t / nt), b = (int)((long long)rows * (t + 1) / nt);
            for (int r = a; r < b; ++r) fn(r);
        });
    }
    for (auto& x : th) x.join();
}

// Symmetric group-32 quantizer shared by q8 (qmax 127) and q4s (qmax 7).
static void quant_sym_g32(const float* w, int rows, int cols, int qmax, int8_t* q_out, uint16_t* scales) {
    const int groups = cols / 32;
    parallel_rows(rows, [&](int r) {
        for (int g = 0; g < groups; ++g) {
            const float* src = w + (long long)r * cols + g * 32;
            float amax = 0.f;
            for (int i = 0; i < 32; ++i) amax = std::fmax(amax, std::fabs(src[i]));
            uint16_t sh = f32_to_f16_bits(amax / (float)qmax);
            if (f16_bits_to_f32(sh) * (float)qmax < amax) sh = (uint16_t)(sh + 1);
            const float s = f16_bits_to_f32(sh);
            scales[(long long)r * groups + g] = sh;
            const float inv = s > 0.f ? 1.0f / s : 0.f;
            for (int i = 0; i < 32; ++i) {
                float v = std::round(src[i] * inv);  // ties away from zero, as Swift .rounded()
                if (v > (float)qmax) v = (float)qmax;
                if (v < -(float)qmax) v = -(float)qmax;
                q_out[(long long)r * cols + g * 32 + i] = (int8_t)v;
            }
        }
    });
}

// ---- repack to the device tile layout (layout.h) ----------------------------------------------
// Unit = 16 rows x 64 columns; per lane (g = lane / 4, t = lane % 4) and k16 step, the A fragment
// of mma.m16n8k16 holds rows g and g+8 at columns 2t, 2t+1, 2t+8, 2t+9.

static inline int src_row(const int* map, int r) { return map ? map[r] : r; }

void pack_q4s(int n_rows, int k, const uint8_t* packed, const uint16_t* scales, const int* row_map, uint8_t* out) {
    const int upt = k / 64, groups = k / 32;
    parallel_rows(n_rows / 16, [&](int tile) {
        for (int kk = 0; kk < upt; ++kk) {
            uint8_t* ub = out + icua_layout::unit_offset(icua_layout::FMT_Q4S, n_rows / 16, upt, tile, kk);
            for (int lane = 0; lane < 32; ++lane) {
                const int g = lane >> 2, t = lane & 3;
                const int ra = src_row(row_map, tile * 16 + g), rb = src_row(row_map, tile * 16 + g + 8);
                auto u = [&](int r, int kc) -> uint32_t {
                    const uint8_t b = packed[(long long)r * (k / 2) + (kc >> 1)];
                    return (kc & 1) ? (b >> 4) : (b & 0xF);
                };
                for (int step = 0; step < 4; ++step) {
                    const int k0 = kk * 64 + step * 16 + 2 * t;
                    const uint32_t w = u(ra, k0) | (u(rb, k0) << 4) | (u(ra, k0 + 8) << 8) | (u(rb, k0 + 8) << 12) |
                                       (u(ra, k0 + 1) << 16) | (u(rb, k0 + 1) << 20) | (u(ra, k0 + 9) << 24) |
                                       (u(rb, k0 + 9) << 28);
                    std::memcpy(ub + lane * 16 + step * 4, &w, 4);
                }
            }
            for (int g = 0; g < 8; ++g) {
                const int ra = src_row(row_map, tile * 16 + g), rb = src_row(row_map, tile * 16 + g + 8);
                for (int grp = 0; grp < 2; ++grp) {
                    const uint16_t sa = scales[(long long)ra * groups + kk * 2 + grp];
                    const uint16_t sb = scales[(long long)rb * groups + kk * 2 + grp];
                    std::memcpy(ub + 512 + g * 8 + grp * 4, &sa, 2);
                    std::memcpy(ub + 512 + g * 8 + grp * 4 + 2, &sb, 2);
                }
            }
        }
    });
}

// Reference affine q4 (Convert.swift:246-320): nibbles placed exactly as pack_q4s (codes 0..15,
// no offset); the unit's 64 bytes hold, per lane group g, the fp16 (scale, bias) of rows g and g+8
// for the unit's one 64-column group.  `sb` is the reference's half2 [rows][K / 64] array.
void pack_q4a(int n_rows, int k, const uint8_t* packed, const uint16_t* sb, const int* row_map, uint8_t* out) {
    const int upt = k / 64;
    parallel_rows(n_rows / 16, [&](int tile) {
        for (int kk = 0; kk < upt; ++kk) {
            uint8_t* ub = out + icua_layout::unit_offset(icua_layout::FMT_Q4A, n_rows / 16, upt, tile, kk);
            for (int lane = 0; lane < 32; ++lane) {
                const int g = lane >> 2, t = lane & 3;
                const int ra = src_row(row_map, tile * 16 + g), rb = src_row(row_map, tile * 16 + g + 8);
                auto u = [&](int r, int kc) -> uint32_t {
                    const uint8_t b = packed[(long long)r * (k / 2) + (kc >> 1)];
                    return (kc & 1) ? (b >> 4) : (b & 0xF);
                };
                for (int step = 0; step < 4; ++step) {
                    const int k0 = kk * 64 + step * 16 + 2 * t;
                    const uint32_t w = u(ra, k0) | (u(rb, k0) << 4) | (u(ra, k0 + 8) << 8) | (u(rb, k0 + 8) << 12) |
                                       (u(ra, k0 + 1) << 16) | (u(rb, k0 + 1) << 20) | (u(ra, k0 + 9) << 24) |
                                       (u(rb, k0 + 9) << 28);
                    std::memcpy(ub + lane * 16 + step * 4, &w, 4);
                }
            }
            for (int g = 0; g < 8; ++g) {
                const int ra = src_row(row_map, tile * 16 + g), rb = src_row(row_map, tile * 16 + g + 8);
                std::memcpy(ub + 512 + g * 8, sb + ((long long)ra * upt + kk) * 2, 4);      // scale, bias of row g
                std::memcpy(ub + 512 + g * 8 + 4, sb + ((long long)rb * upt + kk) * 2, 4);  // of row g + 8
            }
        }
    });
}

void pack_q8(int n_rows, int k, const int8_t* codes, const uint16_t* scales, const int* row_map, uint8_t* out) {
    const int upt = k / 64, groups = k / 32;
    parallel_rows(n_rows / 16, [&](int tile) {
        for (int kk = 0; kk < upt; ++kk) {
            uint8_t* ub = out + icua_layout::unit_offset(icua_layout::FMT_Q8, n_rows / 16, upt, tile, kk);
            for (int lane = 0; lane < 32; ++lane) {
                const int g = lane >> 2, t = lane & 3;
                const int ra = src_row(row_map, tile * 16 + g), rb = src_row(row_map, tile * 16 + g + 8);
                auto b = [&](int r, int kc) -> uint32_t {
                    return (uint32_t)(uint8_t)(codes[(long long)r * k + kc] + 128);
                };
                for (int step = 0; step < 4; ++step) {
                    const int k0 = kk * 64 + step * 16 + 2 * t;
                    const uint32_t w0 = b(ra, k0) | (b(rb, k0) << 8) | (b(ra, k0 + 1) << 16) | (b(rb, k0 + 1) << 24);
                    const uint32_t w1 =
                        b(ra, k0 + 8) | (b(rb, k0 + 8) << 8) | (b(ra, k0 + 9) << 16) | (b(rb, k0 + 9) << 24);
                    uint8_t* dst = ub + (step >> 1) * 512 + lane * 16 + (step & 1) * 8;
                    std::memcpy(dst, &w0, 4);
                    std::memcpy(dst + 4, &w1, 4);
                }
            }
            for (int g = 0; g < 8; ++g) {
                const int ra = src_row(row_map, tile * 16 + g), rb = src_row(row_map, tile * 16 + g + 8);
                for (int grp = 0; grp < 2; ++grp) {
                    const uint16_t sa = scales[(long long)ra * groups + kk * 2 + grp];
                    const uint16_t sb = scales[(long long)rb * groups + kk * 2 + grp];
                    std::memcpy(ub + 1024 + g * 8 + grp * 4, &sa, 2);
                    std::memcpy(ub + 1024 + g * 8 + grp * 4 + 2, &sb, 2);
                }
            }
        }
    });
}

}  // namespace icua_host

using namespace icua_host;

extern "C" {

icua_status icua_quantize_q8(const float* w, int32_t rows, int32_t cols, int8_t* codes, uint16_t* scales) {
    if (!w || !codes || !scales || rows <= 0 || cols <= 0 || cols % 32) return ICUA_ERR_INVALID;
    quant_sym_g32(w, rows, cols, 127, codes, scales);
    return ICUA_OK;
}

icua_status icua_quantize_q4s(const float* w, int32_t rows, int32_t cols, uint8_t* packed, uint16_t* scales) {
    if (!w || !packed || !scales || rows <= 0 || cols <= 0 || cols % 32) return ICUA_ERR_INVALID;
    std::vector<int8_t> q((size_t)rows * cols);
    quant_sym_g32(w, rows, cols, 7, q.data(), scales);
    parallel_rows(rows, [&](int r) {
        for (int c = 0; c < cols; c += 2) {
            const uint8_t lo = (uint8_t)(q[(size_t)r * cols + c] + 8);
            const uint8_t hi = (uint8_t)(q[(size_t)r * cols + c + 1] + 8);
            packed[(size_t)r * (cols / 2) + c / 2] = (uint8_t)(lo | (hi << 4));
        }
    });
    return ICUA_OK;
}

uint64_t icua_packed_bytes(int32_t fmt, int32_t n_rows, int32_t k) {
    if (n_rows <= 0 || k <= 0 || n_rows % 16 || k % 1024) return 0;
    const uint64_t units = (uint64_t)(n_rows / 16) * (uint64_t)(k / 64);
    if (fmt == ICUA_FMT_Q4S || fmt == ICUA_FMT_Q4) return units * 576;
    if (fmt == ICUA_FMT_Q8) return units * 1088;
    return 0;
}

icua_status icua_pack_matrix(int32_t fmt, int32_t n_rows, int32_t k, const void* codes, const uint16_t* scales,
                             void* packed_out) {
    if (!codes || !scales || !packed_out || icua_packed_bytes(fmt, n_rows, k) == 0) return ICUA_ERR_INVALID;
    if (fmt == ICUA_FMT_Q4S)
        pack_q4s(n_rows, k, (const uint8_t*)codes, scales, nullptr, (uint8_t*)packed_out);
    else if (fmt == ICUA_FMT_Q4)
        pack_q4a(n_rows, k, (const uint8_t*)codes, scales, nullptr, (uint8_t*)packed_out);
    else
        pack_q8(n_rows, k, (const int8_t*)codes, scales, nullptr, (uint8_t*)packed_out);
    return ICUA_OK;
}

}  // extern "C"
