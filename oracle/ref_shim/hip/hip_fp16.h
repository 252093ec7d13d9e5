/* Host-only stand-in for hip_fp16.h (see hip_runtime.h in this folder).  The
 * __half2float here is only reachable from the reference's dead GPU kernels. */
#pragma once
#include <cstdint>
struct __half { uint16_t bits; };
static inline float __half2float(__half) { return 0.0f; }
