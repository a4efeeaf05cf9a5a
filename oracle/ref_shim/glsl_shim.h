// glsl_shim.h — the GLSL built-ins that VoxGen's BaseLM compute shaders use,
// as C++, so the shader bodies compile unchanged with g++ and run on the CPU.
//
// TEST INFRASTRUCTURE ONLY (the parity pin of the oracle): nothing in the
// product links this.
//
// Semantics follow the GLSL 4.60 specification: 32-bit uint/int/float,
// unpackHalf2x16 (low half in .x), packHalf2x16 (round to nearest even, the
// conversion the oracle and the CUDA path use), inversesqrt as 1/sqrt.
// Translation units that include this header must not include <cmath> or
// <math.h>: the unqualified exp/pow/cos/sin/tanh/round/max/min calls of a shader have to
// resolve to the float overloads below.
//
// Workgroup model: every invocation of a workgroup is a fiber on one host
// thread; barrier() switches to the next fiber, and `shared` variables are
// thread-local, so one workgroup's invocations share them. Host threads run
// different workgroups of a dispatch in parallel.
#pragma once

#include "workgroup.h"

struct vec2 {
  float x, y;
  vec2() = default;
  explicit vec2(float a) : x(a), y(a) {}
  vec2(float a, float b) : x(a), y(b) {}
  vec2 operator+(const vec2 &o) const { return vec2(x + o.x, y + o.y); }
  vec2 &operator+=(const vec2 &o) {
    x += o.x;
    y += o.y;
    return *this;
  }
};

extern "C" {
float expf(float);
float powf(float, float);
float cosf(float);
float sinf(float);
float sqrtf(float);
float tanhf(float);
float roundf(float);
}

inline float exp(float x) { return expf(x); }
inline float pow(float x, float y) { return powf(x, y); }
inline float cos(float x) { return cosf(x); }
inline float sin(float x) { return sinf(x); }
inline float inversesqrt(float x) { return 1.0f / sqrtf(x); }
inline float tanh(float x) { return tanhf(x); }
// GLSL leaves the direction of halves to the implementation; roundf takes them away from zero.
inline float round(float x) { return roundf(x); }
inline float max(float a, float b) { return a < b ? b : a; }
inline float min(float a, float b) { return b < a ? b : a; }
inline uint max(uint a, uint b) { return a < b ? b : a; }
inline uint min(uint a, uint b) { return b < a ? b : a; }

inline float uintBitsToFloat(uint u) {
  float f;
  __builtin_memcpy(&f, &u, 4);
  return f;
}
inline uint floatBitsToUint(float f) {
  uint u;
  __builtin_memcpy(&u, &f, 4);
  return u;
}

inline vec2 unpackHalf2x16(uint v) {
  return vec2(vgref::half_to_float(v & 0xFFFFu), vgref::half_to_float(v >> 16));
}
inline uint packHalf2x16(vec2 v) { return vgref::float_to_half(v.x) | (vgref::float_to_half(v.y) << 16); }
inline void barrier() { vgref::barrier(); }

// The shaders declare only local_size_x, so y and z of the global id are the group's.
inline uvec3 vgref_global_id(uint local_size_x) {
  uvec3 g = vgref::group_id();
  g.x = g.x * local_size_x + vgref::local_id().x;
  return g;
}
#define gl_GlobalInvocationID (vgref_global_id(vgref_local_size))
#define gl_LocalInvocationID (::vgref::local_id())
#define gl_WorkGroupID (::vgref::group_id())
#define gl_NumWorkGroups (::vgref::num_groups())
#define shared static thread_local

// Subgroups (GL_KHR_shader_subgroup_basic / _arithmetic) of 32 invocations:
// the _xtx7900 shaders' wave32 reductions (see workgroup.h for the order).
#define gl_SubgroupSize 32u
#define gl_SubgroupInvocationID (::vgref::local_id().x & 31u)
#define gl_SubgroupID (::vgref::local_id().x >> 5)
#define gl_NumSubgroups ((vgref_local_size + 31u) / 32u)
inline float subgroupAdd(float v) { return vgref::subgroup_add(v); }
inline float subgroupMax(float v) { return vgref::subgroup_max(v); }
