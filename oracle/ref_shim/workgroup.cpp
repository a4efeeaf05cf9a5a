// workgroup.cpp — compute-dispatch emulator for shaders compiled as C++.
//
// TEST INFRASTRUCTURE ONLY (the parity pin of the oracle).
//
// Each host thread takes whole workgroups from a shared counter. Inside a
// workgroup every invocation is a fiber with its own stack; a fiber runs until
// it calls barrier() or returns from the shader's main, then control goes
// back to the scheduler, which resumes the next fiber. One sweep over the
// fibers therefore moves every live invocation from one barrier to the next,
// which is exactly the guarantee GLSL's barrier() gives. Invocations that
// returned early drop out of later barriers.
#include "workgroup.h"

#include <atomic>
#include <cstdlib>
#include <cstring>
#include <vector>
#ifdef _OPENMP
#include <omp.h>
#endif

#if !defined(__x86_64__)
#error "the fiber switch below is written for x86-64"
#endif

// Saves the callee-saved registers of the System V x86-64 ABI on the current
// stack, stores the stack pointer in *save_sp, then loads next_sp and restores
// the registers saved there. MXCSR and the x87 control word are never changed
// by the shaders, so they are not switched.
extern "C" void vgref_switch(void **save_sp, void *next_sp);
asm(R"(
  .text
  .p2align 4
  .globl vgref_switch
  .hidden vgref_switch
  .type vgref_switch, @function
vgref_switch:
  pushq %rbp
  pushq %rbx
  pushq %r12
  pushq %r13
  pushq %r14
  pushq %r15
  movq %rsp, (%rdi)
  movq %rsi, %rsp
  popq %r15
  popq %r14
  popq %r13
  popq %r12
  popq %rbx
  popq %rbp
  ret
  .size vgref_switch, .-vgref_switch
)");

namespace vgref {
namespace {

constexpr size_t kStackBytes = 64 * 1024;

struct Fiber {
  void *sp = nullptr;
  uvec3 lid{0, 0, 0};
  bool done = false;
  uint32_t bar = 0;   // workgroup barriers this invocation has reached
  uint32_t sgop = 0;  // subgroup operations this invocation has entered
  std::vector<uint8_t> stack;
};

struct Worker {
  void *sched_sp = nullptr;
  std::vector<Fiber> fibers;
  uint32_t cur = 0;
  uint32_t nlive = 0;          // invocations of the workgroup still running
  uint32_t bar_n[4] = {};      // arrivals at barrier k, in slot k % 4
  uint32_t sg_n[32][4] = {};   // deposits of subgroup s for its operation k, in slot [s][k % 4]
  bool sg_used = false;        // sg_n holds counts of the previous workgroup
  float sg[2][1024];  // subgroup operands, double-buffered by operation parity
  void (*fn)() = nullptr;
  uvec3 wg{0, 0, 0}, nwg{1, 1, 1};
};

thread_local Worker *tw = nullptr;
int g_threads = 0;

// First and every later activation of a fiber: run the shader for the current
// workgroup, mark the invocation done, return to the scheduler; resumed for the
// next workgroup from the same place.
[[noreturn]] void fiber_entry() {
  for (;;) {
    Worker *w = tw;
    Fiber &f = w->fibers[w->cur];
    w->fn();
    f.done = true;
    --w->nlive;
    vgref_switch(&f.sp, w->sched_sp);
  }
}

void init_fiber(Fiber &f) {
  f.stack.assign(kStackBytes, 0);
  uintptr_t top = (reinterpret_cast<uintptr_t>(f.stack.data()) + kStackBytes) & ~uintptr_t(15);
  void **s = reinterpret_cast<void **>(top);
  *--s = nullptr;                                       // fake return address of fiber_entry
  *--s = reinterpret_cast<void *>(&fiber_entry);        // popped by `ret` in vgref_switch
  for (int i = 0; i < 6; ++i) *--s = nullptr;           // rbp rbx r12 r13 r14 r15
  f.sp = s;
}

Worker &worker(uint32_t local) {
  if (!tw) tw = new Worker();  // one per host thread, kept for the thread's life
  Worker &w = *tw;
  if (w.fibers.size() != local) {
    w.fibers.clear();
    w.fibers.resize(local);
    for (auto &f : w.fibers) init_fiber(f);
  }
  return w;
}

void run_group(Worker &w) {
  const uint32_t n = (uint32_t)w.fibers.size();
  for (uint32_t i = 0; i < n; ++i) {
    w.fibers[i].done = false;
    w.fibers[i].lid = uvec3{i, 0, 0};
    w.fibers[i].sgop = 0;
    w.fibers[i].bar = 0;
  }
  w.nlive = n;
  std::memset(w.bar_n, 0, sizeof w.bar_n);
  if (w.sg_used) {
    std::memset(w.sg_n, 0, sizeof w.sg_n);
    w.sg_used = false;
  }
  bool live = true;
  while (live) {
    live = false;
    for (uint32_t i = 0; i < n; ++i) {
      if (w.fibers[i].done) continue;
      w.cur = i;
      vgref_switch(&w.sched_sp, w.fibers[i].sp);
      if (!w.fibers[i].done) live = true;
    }
  }
}

}  // namespace

const uvec3 &local_id() { return tw->fibers[tw->cur].lid; }
const uvec3 &group_id() { return tw->wg; }
const uvec3 &num_groups() { return tw->nwg; }
// An invocation at barrier() runs on only once every live invocation of the
// workgroup has reached it (so subgroup operations inside subgroup-uniform
// branches, which switch fibers a different number of times, cannot skew
// the workgroup's barriers).
// Invocations are at most one barrier apart (none passes barrier k before all
// reached it), so four arrival slots suffice: arriving at k clears slot k + 2,
// whose last use, barrier k - 2, every invocation has passed.
void barrier() {
  Worker *w = tw;
  const uint32_t k = ++w->fibers[w->cur].bar;
  w->bar_n[(k + 2u) & 3u] = 0;
  ++w->bar_n[k & 3u];
  while (w->bar_n[k & 3u] < w->nlive) vgref_switch(&w->fibers[w->cur].sp, w->sched_sp);
}

// Every invocation of the subgroup deposits its operand and switches fibers
// until the other 31 have deposited theirs, then reduces the 32 operands.
// Consecutive operations use the two buffers in turn: an invocation can enter
// operation k + 2 only after all of its subgroup entered k + 1, that is after
// they read operation k's operands.
namespace {
template <bool MAX>
float subgroup_reduce(float v) {
  Worker *w = tw;
  const uint32_t me = w->cur, lane = w->fibers[me].lid.x, base = lane & ~31u, sgi = lane >> 5;
  const uint32_t k = w->fibers[me].sgop++, buf = k & 1u;
  const uint32_t width = w->fibers.size() - base < 32u ? (uint32_t)w->fibers.size() - base : 32u;
  w->sg[buf][lane] = v;
  w->sg_used = true;
  w->sg_n[sgi][(k + 2u) & 3u] = 0;
  ++w->sg_n[sgi][k & 3u];
  while (w->sg_n[sgi][k & 3u] < width) vgref_switch(&w->fibers[me].sp, w->sched_sp);
  float t[32];
  const float *src = w->sg[buf] + base;
  for (int i = 0; i < 32; ++i) t[i] = src[i];
  for (int s = 1; s < 32; s <<= 1)
    for (int i = 0; i < 32; i += 2 * s) t[i] = MAX ? (t[i] < t[i + s] ? t[i + s] : t[i]) : t[i] + t[i + s];
  return t[0];
}
}  // namespace
float subgroup_add(float v) { return subgroup_reduce<false>(v); }
float subgroup_max(float v) { return subgroup_reduce<true>(v); }

void set_threads(int n) { g_threads = n; }

int dispatch(void (*fn)(), uint local, uint gx, uint gy, uint gz) {
  if (!fn || local == 0 || local > 1024) return -1;
  const uint64_t total = (uint64_t)gx * gy * gz;
  if (total == 0) return 0;
  std::atomic<uint64_t> next{0};
#ifdef _OPENMP
  int nt = g_threads > 0 ? g_threads : omp_get_max_threads();
  if ((uint64_t)nt > total) nt = (int)total;
#pragma omp parallel num_threads(nt)
#endif
  {
    Worker &w = worker(local);
    w.fn = fn;
    w.nwg = uvec3{gx, gy, gz};
    for (;;) {
      const uint64_t g = next.fetch_add(1);
      if (g >= total) break;
      w.wg = uvec3{(uint)(g % gx), (uint)((g / gx) % gy), (uint)(g / ((uint64_t)gx * gy))};
      run_group(w);
    }
  }
  return 0;
}

// IEEE binary16 -> binary32, exact.
float half_to_float(uint h) {
  const uint32_t sign = (h & 0x8000u) << 16, e = (h >> 10) & 0x1Fu, m = h & 0x3FFu;
  uint32_t bits;
  if (e == 0x1F) {
    bits = sign | 0x7F800000u | (m << 13);
  } else if (e != 0) {
    bits = sign | ((e - 15u + 127u) << 23) | (m << 13);
  } else if (m == 0) {
    bits = sign;
  } else {
    // subnormal: normalise the mantissa
    int k = 0;
    uint32_t mm = m;
    while (!(mm & 0x400u)) {
      mm <<= 1;
      ++k;
    }
    bits = sign | ((uint32_t)(127 - 15 + 1 - k) << 23) | ((mm & 0x3FFu) << 13);
  }
  float f;
  std::memcpy(&f, &bits, 4);
  return f;
}

// binary32 -> binary16, round to nearest, ties to even; overflow to infinity.
uint float_to_half(float f) {
  uint32_t x;
  std::memcpy(&x, &f, 4);
  const uint32_t sign = (x >> 16) & 0x8000u, e = (x >> 23) & 0xFFu, m = x & 0x7FFFFFu;
  if (e == 0xFF) return sign | 0x7C00u | (m ? 0x200u : 0u);
  const int E = (int)e - 127 + 15;
  if (E >= 31) return sign | 0x7C00u;
  if (E <= 0) {
    if (E < -10) return sign;
    const uint32_t mant = m | 0x800000u;
    const int s = 14 - E;
    uint32_t h = mant >> s;
    const uint32_t rem = mant & ((1u << s) - 1u), halfway = 1u << (s - 1);
    if (rem > halfway || (rem == halfway && (h & 1u))) ++h;
    return sign | h;
  }
  uint32_t h = ((uint32_t)E << 10) | (m >> 13);
  const uint32_t rem = m & 0x1FFFu;
  if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h;
  return sign | h;
}

}  // namespace vgref

extern "C" void vgref_set_threads(int n) { vgref::set_threads(n); }
