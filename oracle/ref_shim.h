// TEST INFRASTRUCTURE ONLY -- lets the reference's Metal decode source compile as C++20.
//
// oracle/build_ref.py takes the decode kernel text that the reference generates at run time
// (daig/omlx-exl3 src/omlx/exl3/kernels.py: HEADER :26-49 and _decode_source(K) :328-334) and
// compiles it, unchanged, against this header.  The header supplies the Metal names that code
// uses, with IEEE fp16 semantics: each fp16 add and fma is evaluated exactly in double and rounded
// once to nearest-even, which is what one fp16 instruction does.
#pragma once
#include <cmath>
#include <cstdint>
#include <cstring>

typedef uint32_t uint;
typedef uint16_t ushort;
typedef uint64_t ulong;

#define device
#define thread
#define constant

namespace refshim {
inline double h2d(uint16_t h)
{
    const int s = h >> 15, e = (h >> 10) & 0x1f, m = h & 0x3ff;
    double v;
    if (e == 0) v = std::ldexp((double)m, -24);
    else if (e == 31) v = m ? NAN : INFINITY;
    else v = std::ldexp((double)(m | 0x400), e - 25);
    return s ? -v : v;
}

inline uint16_t d2h(double x)
{
    uint16_t sign = 0;
    if (std::signbit(x)) { sign = 0x8000; x = -x; }
    if (std::isnan(x)) return sign | 0x7e00;
    if (x >= 65520.0) return sign | 0x7c00;
    if (x < std::ldexp(1.0, -14)) return sign | (uint16_t)std::nearbyint(x * std::ldexp(1.0, 24));
    int e;
    double f = std::frexp(x, &e);
    double r = std::nearbyint(std::ldexp(f, 11));
    if (r >= 2048.0) { r = 1024.0; e += 1; }
    const int be = e - 1 + 15;
    if (be >= 31) return sign | 0x7c00;
    return sign | (uint16_t)(be << 10) | (uint16_t)((int)r - 1024);
}
}  // namespace refshim

struct half {
    uint16_t bits = 0;
    half() = default;
    static half from_bits(uint16_t b) { half h; h.bits = b; return h; }
    explicit half(double v) : bits(refshim::d2h(v)) {}
    double to_double() const { return refshim::h2d(bits); }
};
inline half operator+(half a, half b) { return half(a.to_double() + b.to_double()); }
inline half fma(half a, half b, half c) { return half(a.to_double() * b.to_double() + c.to_double()); }

struct half2 { half x, y; };
struct half4 {
    half x, y, z, w;
    half4() = default;
    half4(half a, half b, half c, half d) : x(a), y(b), z(c), w(d) {}
};
struct uint2 { uint x, y; };
struct uint4 { uint x, y, z, w; };
struct uint3 { uint x, y, z; };

template <typename T, typename S>
inline T as_type(S s)
{
    static_assert(sizeof(T) == sizeof(S), "as_type size mismatch");
    T t;
    std::memcpy(&t, &s, sizeof(T));
    return t;
}

// Metal: bits [offset, offset + bits) of x, zero-extended.
inline uint extract_bits(uint x, uint offset, uint bits)
{
    const uint mask = bits >= 32 ? 0xffffffffu : ((1u << bits) - 1u);
    return (x >> offset) & mask;
}

// Metal: base with bits [offset, offset + bits) replaced by the low bits of insert.
inline uint insert_bits(uint base, uint insert, uint offset, uint bits)
{
    const uint mask = (bits >= 32 ? 0xffffffffu : ((1u << bits) - 1u)) << offset;
    return (base & ~mask) | ((insert << offset) & mask);
}
