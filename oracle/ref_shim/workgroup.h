// workgroup.h — the compute-dispatch emulator behind glsl_shim.h: workgroup
// and invocation ids, barrier(), and dispatch over a grid of workgroups.
// TEST INFRASTRUCTURE ONLY. Includes no math header (see glsl_shim.h).
#pragma once
#include <cstdint>

typedef unsigned int uint;

struct uvec3 {
  uint x, y, z;
};

namespace vgref {
float half_to_float(uint h);
uint float_to_half(float f);
const uvec3 &local_id();
const uvec3 &group_id();
const uvec3 &num_groups();
void barrier();
// Subgroup reductions over the 32 consecutive invocations of the caller's
// subgroup (every invocation of the subgroup calls them together). The sum
// is the balanced pairwise tree over the invocations in order, which is what
// a shuffle-xor butterfly computes: the hardware's own order is not
// specified by GLSL, and this one is an assumption of the emulation.
float subgroup_add(float v);
float subgroup_max(float v);
// Runs fn once for every invocation of a gx*gy*gz grid of workgroups of
// `local` invocations (a 1-D local size). Returns 0, or -1 on a bad argument.
int dispatch(void (*fn)(), uint local, uint gx, uint gy, uint gz);
// Host threads for dispatch (0 = all hardware threads).
void set_threads(int n);
}  // namespace vgref
