// cuju-b200: scalar and vector primitives shared by every device module.
//
// Every float operation here keeps the operation order and the float/double split of Google
// Research Football (GRF 2.10.3), because each environment must produce the same bits as the
// reference CPU backend (cuju include/cuju/vector3.h, quaternion.h, math_utilities.h, x86.h).
// The whole library is compiled with --fmad=false -prec-div=true -prec-sqrt=true -ftz=false, so a
// `a * b + c` written here is two rounded operations, as GRF's x86-64 build computes it; a fused
// step is always an explicit `fma`.
#pragma once

#include <cstdint>
#include <cstring>
#include <cmath>

#if defined(__CUDACC__)
#define CB_HD __host__ __device__ __forceinline__
#define CB_HDNI __host__ __device__ __noinline__ inline
#define CB_FN __host__ __device__
#else
#define CB_HD inline
#define CB_HDNI inline
#define CB_FN
#endif

#if defined(__CUDA_ARCH__)
#define CB_DEVICE_PASS 1
#else
#define CB_DEVICE_PASS 0
#endif

#if defined(__FAST_MATH__)
#error "cuju-b200 needs IEEE-754 semantics; build without fast math"
#endif

namespace cb {

// ---------------------------------------------------------------------------------------------
// The per-thread crew byte (its layout and the crews themselves: crew.cuh). One bit of it marks
// that the environment the thread works on reached an iteration cap of GRF's arithmetic.
constexpr int kCrewSlots = 128;  // threads per block at most (the kernels launch 64)
constexpr uint8_t kCrewWidthBits = 0x07;
constexpr uint8_t kCrewDividedBit = 0x08;
constexpr uint8_t kCrewCapBit = 0x10;
#if CB_DEVICE_PASS
__device__ __forceinline__ uint8_t &crew_byte() {
    __shared__ uint8_t bytes[kCrewSlots];
    return bytes[threadIdx.x];
}
CB_HD int lane_id() { return (int)(threadIdx.x & 31); }
#else
inline uint8_t &crew_byte() {
    static thread_local uint8_t byte = 0;
    return byte;
}
CB_HD int lane_id() { return 0; }
#endif
CB_HD void crew_note_cap() { crew_byte() |= kCrewCapBit; }
CB_HD bool crew_cap_reached() { return (crew_byte() & kCrewCapBit) != 0; }
CB_HD void crew_clear_cap() { crew_byte() &= (uint8_t)~kCrewCapBit; }

// ---------------------------------------------------------------------------------------------
// Bit casts
CB_HD uint32_t f2u(float v) {
#if CB_DEVICE_PASS
    return __float_as_uint(v);
#else
    uint32_t b; memcpy(&b, &v, 4); return b;
#endif
}
CB_HD float u2f(uint32_t b) {
#if CB_DEVICE_PASS
    return __uint_as_float(b);
#else
    float v; memcpy(&v, &b, 4); return v;
#endif
}
CB_HD uint64_t d2u(double v) {
#if CB_DEVICE_PASS
    return (uint64_t)__double_as_longlong(v);
#else
    uint64_t b; memcpy(&b, &v, 8); return b;
#endif
}
CB_HD double u2d(uint64_t b) {
#if CB_DEVICE_PASS
    return __longlong_as_double((long long)b);
#else
    double v; memcpy(&v, &b, 8); return v;
#endif
}

// ---------------------------------------------------------------------------------------------
// x86-64 conversion semantics (GRF's build): cuju include/cuju/x86.h:13-33.
// cvttss2si to 32 bits: NaN and out-of-range give INT32_MIN ("integer indefinite").
CB_HD int32_t cvt_f_i32(float v) {
    if (!(v >= -2147483648.0f && v < 2147483648.0f)) return INT32_MIN;
    return (int32_t)v;
}
// float -> unsigned on x86-64 goes through a 64-bit signed conversion, low word kept.
CB_HD uint32_t cvt_f_u32(float v) {
    if (!(v >= -9223372036854775808.0f && v < 9223372036854775808.0f)) return 0u;
    return (uint32_t)(uint64_t)(int64_t)v;
}
CB_HD int32_t cvt_d_i32(double v) {
    if (!(v > -2147483649.0 && v < 2147483648.0)) return INT32_MIN;
    return (int32_t)v;
}

// ---------------------------------------------------------------------------------------------
// Scalars (cuju include/cuju/math_utilities.h)
constexpr float kPi = 3.1415926535897932384626433832795028841972f;
// The float just above the double 1e-6: `v < kAboveMicro` iff `(double)v < 1e-6`.
constexpr float kAboveMicro = 0x1.0c6f7cp-20f;

CB_HD float clampf_(float v, float lo, float hi) {
    if (lo > v) return lo;
    if (hi < v) return hi;
    return v;
}
CB_HD float nclamp(float v, float lo, float hi) {
    float c = clampf_(v, lo, hi);
    return (c - lo) / (hi - lo);
}
CB_HD int sign_side(float v) { return v >= 0 ? 1 : -1; }
// One period added or removed per iteration, so each keeps its rounding. With the span of 2*pi
// that every caller passes, the loops end for |v| below 2^27 (above it v - span rounds back to v)
// and take at most about 18.1 million iterations there; the cap of 2^25 per loop changes no
// result where they end, and stops them where they would not (an infinite or huge angle, which
// GRF leaves undefined) instead of holding the launch forever. Reaching the cap marks the
// environment (crew_note_cap), so its step ends in the unsupported-path status.
CB_HD float wrap_range(float lo, float hi, float v) {
    constexpr unsigned kCap = 1u << 25;
    float span = hi - lo;
    float r = v;
    for (unsigned i = 0; r < lo && i < kCap; i++) r += span;
    if (r < lo) crew_note_cap();
    for (unsigned i = 0; r > hi && i < kCap; i++) r -= span;
    if (r > hi) crew_note_cap();
    return r;
}
// A float written with printf("%f") and read back with atof, then narrowed to float: the exact
// binary value is rounded to a multiple of 1e-6 (ties to even) and the decimal N/1e6 is converted
// to the nearest double (one IEEE division, exact for |v| < 2^33) and then to float.
// cuju include/cuju/real_to_string.h:17 (RoundTripSixDecimals).
CB_HDNI float round_trip_six(float v) {
    const uint32_t b = f2u(v);
    const int e8 = (int)((b >> 23) & 0xffu);
    if (e8 == 0xff) return v;
    uint64_t man = b & 0x7fffffu;
    int e2 = -149;
    if (e8 != 0) {
        man |= 0x800000u;
        e2 = e8 - 150;
    }
    const uint64_t scaled = man * 1000000ull;  // below 2^44
    uint64_t n;
    if (e2 >= 0) {
        n = scaled << e2;
    } else if (-e2 >= 64) {
        n = 0;
    } else {
        const int sh = -e2;
        n = scaled >> sh;
        const uint64_t rem = scaled & ((1ull << sh) - 1), half = 1ull << (sh - 1);
        if (rem > half || (rem == half && (n & 1))) n++;
    }
    const float r = (float)((double)n / 1e6);
    return (b >> 31) ? -r : r;
}
CB_HD float fminf_(float a, float b) { return a < b ? a : b; }
CB_HD float fmaxf_(float a, float b) { return a > b ? a : b; }

// ---------------------------------------------------------------------------------------------
// Vec3: GRF's float 3-vector (cuju include/cuju/vector3.h:21-176).
struct Vec3 {
    float c[3];
    CB_HD constexpr Vec3() : c{0, 0, 0} {}
    CB_HD constexpr Vec3(float s) : c{s, s, s} {}
    CB_HD constexpr Vec3(float x, float y, float z) : c{x, y, z} {}
    CB_HD float &operator[](int i) { return c[i]; }
    CB_HD const float &operator[](int i) const { return c[i]; }
    CB_HD void set(float x, float y, float z) { c[0] = x; c[1] = y; c[2] = z; }
    CB_HD void mirror() { c[0] = -c[0]; c[1] = -c[1]; }
    CB_HD bool operator==(const Vec3 &o) const { return c[0] == o.c[0] && c[1] == o.c[1] && c[2] == o.c[2]; }
    CB_HD bool operator!=(const Vec3 &o) const { return !(*this == o); }
    CB_HD Vec3 operator*(float s) const { return Vec3(c[0] * s, c[1] * s, c[2] * s); }
    CB_HD Vec3 operator*(const Vec3 &o) const { return Vec3(c[0] * o.c[0], c[1] * o.c[1], c[2] * o.c[2]); }
    CB_HD Vec3 &operator*=(float s) { c[0] *= s; c[1] *= s; c[2] *= s; return *this; }
    CB_HD Vec3 &operator*=(const Vec3 &o) { c[0] *= o.c[0]; c[1] *= o.c[1]; c[2] *= o.c[2]; return *this; }
    CB_HD Vec3 operator/(float s) const { return Vec3(c[0] / s, c[1] / s, c[2] / s); }
    CB_HD Vec3 &operator/=(const Vec3 &o) { c[0] /= o.c[0]; c[1] /= o.c[1]; c[2] /= o.c[2]; return *this; }
    CB_HD Vec3 &operator+=(float s) { c[0] += s; c[1] += s; c[2] += s; return *this; }
    CB_HD Vec3 &operator+=(const Vec3 &o) { c[0] += o.c[0]; c[1] += o.c[1]; c[2] += o.c[2]; return *this; }
    CB_HD Vec3 &operator-=(const Vec3 &o) { c[0] -= o.c[0]; c[1] -= o.c[1]; c[2] -= o.c[2]; return *this; }
    CB_HD Vec3 operator+(const Vec3 &o) const { return Vec3(c[0] + o.c[0], c[1] + o.c[1], c[2] + o.c[2]); }
    CB_HD Vec3 operator+(float s) const { return Vec3(c[0] + s, c[1] + s, c[2] + s); }
    CB_HD Vec3 operator-(const Vec3 &o) const { return Vec3(c[0] - o.c[0], c[1] - o.c[1], c[2] - o.c[2]); }
    CB_HD Vec3 operator-() const { return Vec3(-c[0], -c[1], -c[2]); }
    CB_HD Vec3 operator-(float s) const { return Vec3(c[0] - s, c[1] - s, c[2] - s); }
    CB_HD Vec3 cross(const Vec3 &o) const {
        return Vec3(c[1] * o.c[2] - c[2] * o.c[1], c[2] * o.c[0] - c[0] * o.c[2],
                    c[0] * o.c[1] - c[1] * o.c[0]);
    }
    CB_HD float dot(const Vec3 &o) const { return c[0] * o.c[0] + c[1] * o.c[1] + c[2] * o.c[2]; }
    // GRF Vector3::Normalize(fallback).
    CB_HD void normalize(const Vec3 &fb) {
        if (fabsf(c[0]) < 0.000001f && fabsf(c[1]) < 0.000001f && fabsf(c[2]) < 0.000001f) {
            c[0] = fb.c[0]; c[1] = fb.c[1]; c[2] = fb.c[2];
        } else {
            float inv = 1.0f / sqrtf(dot(*this));
            c[0] *= inv; c[1] *= inv; c[2] *= inv;
        }
    }
    // A zero vector becomes NaN, as in GRF.
    CB_HD void normalize() {
        float inv = 1.0f / sqrtf(dot(*this));
        c[0] *= inv; c[1] *= inv; c[2] *= inv;
    }
    CB_HD Vec3 normalized(const Vec3 &fb) const { Vec3 t(*this); t.normalize(fb); return t; }
    CB_HD Vec3 normalized() const { Vec3 t(*this); t.normalize(); return t; }
    // The length is taken in double and rounded; below 1e-6 it is 0.
    CB_HD float length() const {
        double x = c[0], y = c[1], z = c[2];
        float l = (float)sqrt(x * x + y * y + z * z);
        if (l < kAboveMicro) l = 0;
        return l;
    }
    CB_HD float length_sq() const { return c[0] * c[0] + c[1] * c[1] + c[2] * c[2]; }
    CB_HD Vec3 flat() const { return Vec3(c[0], c[1], 0); }
    CB_HD Vec3 abs() const { return Vec3(fabsf(c[0]), fabsf(c[1]), fabsf(c[2])); }
    CB_HD Vec3 max_deviation(const Vec3 &dev, float maxDev) const {
        Vec3 r = *this;
        Vec3 d = dev - *this;
        float dl = d.length();
        if (dl > maxDev) r += d.normalized() * (dl - maxDev);
        return r;
    }
};

struct Radian;  // see state.cuh

}  // namespace cb
