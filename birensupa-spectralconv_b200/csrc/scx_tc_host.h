// Host-side helpers for the tensor-core operand tables: bf16 hi/lo splits of double
// precision twiddles, exact angle reduction, and writers for the K-major and MN-major
// 128-byte-swizzled shared-memory operand layouts (scx_tc.cuh documents both layouts).
#pragma once

#include <cmath>
#include <cstdint>
#include <cstring>
#include <vector>

namespace scx {
namespace host {

// Round-to-nearest-even fp32 -> bf16 bits (NaN stays NaN).
inline uint16_t bf16_bits(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return 0x7fc0;
    return static_cast<uint16_t>((u + 0x7fffu + ((u >> 16) & 1u)) >> 16);
}

inline float bf16_float(uint16_t b) {
    const uint32_t u = static_cast<uint32_t>(b) << 16;
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

// v ~= hi + lo, both bf16 (lo carries the rounding error of hi).
inline void bf16_split(double v, uint16_t& hi, uint16_t& lo) {
    hi = bf16_bits(static_cast<float>(v));
    lo = bf16_bits(static_cast<float>(v - static_cast<double>(bf16_float(hi))));
}

// 2*pi*((k*n) mod N)/N with the product reduced exactly in integers.
inline double ang(long long k, long long n, long long N) {
    return 2.0 * M_PI * static_cast<double>((k * n) % N) / static_cast<double>(N);
}

// Spectrum row held by corner slot s (s < m1: corner 1, else corner 2).
inline int slot_row(int s, int H, int m1) { return s < m1 ? s : H - m1 + (s - m1); }

inline int round_up(int v, int m) { return (v + m - 1) / m * m; }

// Byte offset of element (r, k) of a K-major SW128 bf16 operand with `rows` rows.
inline uint32_t kmajor_offset(int rows, int r, int k) {
    const int kb = k >> 6, kk = k & 63;
    return static_cast<uint32_t>(kb) * static_cast<uint32_t>(rows) * 128u + static_cast<uint32_t>(r >> 3) * 1024u +
           static_cast<uint32_t>(r & 7) * 128u + static_cast<uint32_t>(((kk >> 3) ^ (r & 7)) << 4) +
           static_cast<uint32_t>((kk & 7) << 1);
}

// A bf16 operand image (rows x kdim, K-major SW128), filled element by element.  The
// swizzle spans whole 128-byte rows, so K is padded to a multiple of 64 elements.
struct KMajor {
    int rows, kdim;
    std::vector<uint16_t> data;
    KMajor(int r, int k) : rows(r), kdim(k), data(static_cast<size_t>(r) * round_up(k, 64), 0) {}
    void set(int r, int k, uint16_t v) { data.at(kmajor_offset(rows, r, k) / 2) = v; }
    size_t bytes() const { return data.size() * 2; }
};

}  // namespace host
}  // namespace scx
