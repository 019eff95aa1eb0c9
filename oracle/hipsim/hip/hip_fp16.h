// Host stand-in for HIP's f16 types (test infrastructure only; see hip_runtime.h).
#pragma once

#include "hip_runtime.h"

struct __half2 {
    _Float16 x, y;
};
inline float2 __half22float2(__half2 h) { return float2{static_cast<float>(h.x), static_cast<float>(h.y)}; }
