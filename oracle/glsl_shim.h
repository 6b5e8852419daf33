// glsl_shim.h -- the few GLSL built-ins laguna-raw's compute shaders use,
// expressed in C++ so the shader bodies compile for the CPU unchanged.
//
// TEST INFRASTRUCTURE ONLY (oracle/_ref).  Included by oracle/build_ref.py in
// front of each reference shader; each shader becomes its own translation unit.
#pragma once
#include <cmath>
#include <cstdint>
#include <cstring>
#include <algorithm>

typedef unsigned int uint;

struct uvec3 {
    uint x, y, z;
};

// One invocation runs at a time per host thread.
static thread_local uvec3 gl_GlobalInvocationID;

static inline float uintBitsToFloat(uint u) {
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}
static inline float inversesqrt(float v) { return 1.0f / std::sqrt(v); }
static inline float exp(float v) { return std::exp(v); }
static inline float cos(float v) { return std::cos(v); }
static inline float sin(float v) { return std::sin(v); }
static inline float max(float a, float b) { return std::max(a, b); }
static inline uint max(uint a, uint b) { return std::max(a, b); }
