/*
 * msl_host.h -- lets g++ compile the reference's Metal Shading Language
 * kernel sources as plain host C++ (test infrastructure only).
 *
 * The build recipe (oracle/Makefile, target `ref`) strips the MSL
 * `[[...]]` argument attributes with sed and includes this header in place
 * of <metal_stdlib>.  Address-space qualifiers become nothing, `half` becomes
 * the compiler's IEEE binary16 type, and the few Metal library calls the
 * kernels use are mapped onto <cmath>.  A kernel then becomes an ordinary
 * function whose thread-position arguments the driver (ref_driver.cpp)
 * passes explicitly, one call per Metal thread.
 *
 * simd_sum / threadgroup_barrier are only reached by the RMSNorm kernel when
 * it runs with more than one thread per threadgroup; the driver runs it with
 * one thread per row, where the reduction is the identity.
 */
#pragma once
#include <cmath>
#include <cstdint>

typedef _Float16 half;
typedef unsigned char uchar;
typedef unsigned short ushort;
typedef unsigned int uint;
struct uint3 {
  uint x, y, z;
};

#define device
#define constant
#define thread
#define threadgroup
#define kernel

namespace metal {
inline float max(float a, float b) { return a > b ? a : b; }
inline float min(float a, float b) { return a < b ? a : b; }
inline float simd_sum(float v) { return v; }
enum class mem_flags { mem_none, mem_threadgroup, mem_device };
inline void threadgroup_barrier(mem_flags) {}
using std::abs;
using std::ceil;
using std::cos;
using std::exp;
using std::floor;
using std::isinf;
using std::isnan;
using std::log;
using std::pow;
using std::sin;
using std::sqrt;
}  // namespace metal

/* MSL half literal suffix (e.g. 1.0h) */
inline half operator""h(long double v) { return (half)(float)v; }
