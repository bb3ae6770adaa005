// OpenCL-C -> C++ shim used ONLY to compile the reference's kernel sources
// (kernels/llm_*.cl) as plain host C++ so they can serve as the CPU checker.
// This is test infrastructure: nothing in the product links it.
//
// Must be included AFTER every standard header: it redefines `kernel`,
// `global` and `__attribute__`, which would break libstdc++ otherwise.
#pragma once
#include <cmath>
#include <cstdint>
#include <cstring>
#include <cstddef>

namespace clshim {
// get_global_id() for the thread that is currently "being" a work item.
extern thread_local uint32_t tl_gid;
}

typedef uint32_t uint;

struct uint2 { uint x, y; };
struct uint4 {
    uint x, y, z, w;
    uint4() = default;
    // `(uint4)(0u, 0u, 0u, 0u)` in OpenCL parses as a cast of a comma
    // expression in C++, i.e. a broadcast of the last value.
    explicit uint4(uint v) : x(v), y(v), z(v), w(v) {}
    uint4& operator+=(const uint4& o) { x += o.x; y += o.y; z += o.z; w += o.w; return *this; }
};
struct float4 { float x, y, z, w; };

inline float dot(const float4& a, const float4& b) {
    // OpenCL dot(): evaluated left to right in fp32.
    float s = a.x * b.x;
    s += a.y * b.y;
    s += a.z * b.z;
    s += a.w * b.w;
    return s;
}
inline float as_float(uint u) { float f; std::memcpy(&f, &u, 4); return f; }
inline uint  as_uint(float f) { uint u; std::memcpy(&u, &f, 4); return u; }
inline size_t get_global_id(uint) { return clshim::tl_gid; }

// Float overloads so unqualified calls inside the kernel namespaces stay fp32.
inline float exp(float x)  { return std::exp(x); }
inline float exp2(float x) { return std::exp2(x); }
inline float log2(float x) { return std::log2(x); }
inline float sin(float x)  { return std::sin(x); }
inline float cos(float x)  { return std::cos(x); }
inline float sqrt(float x) { return std::sqrt(x); }
inline float rsqrt(float x) { return 1.0f / std::sqrt(x); }
inline float fmax(float a, float b) { return std::fmax(a, b); }
inline float fmin(float a, float b) { return std::fmin(a, b); }
inline float fabs(float a) { return std::fabs(a); }
inline bool  isfinite(float a) { return std::isfinite(a); }
inline float clamp(float v, float lo, float hi) { return std::fmin(std::fmax(v, lo), hi); }
inline uint  min(uint a, uint b) { return a < b ? a : b; }
inline uint  max(uint a, uint b) { return a > b ? a : b; }

#define kernel
#define global
#define __kernel
#define __global
#define constant const
#define __attribute__(x)
