// CUDA kernels of the BaseLM decode step (sm_100a): the shared matvec parts
// (producer, activation prologue, tensor-core consumer, epilogues) used by the
// persistent step kernel (step_kernel.cuh) and by the standalone kernels of
// the vg_k_* entry points and the per-kernel step program.
//
// Weight layout in HBM ("segmented 16-row tiles", built by repack_kernel; see
// TileGeom). A tile is 16 output rows, the M of one mma.sync with the weights
// as the A operand. A K-step is 32 Q8_0 quants (one block) or 16 fp16 values
// of the 16 rows, 512 bytes stored as the four 8x16-byte matrices that
// ldmatrix.x4 delivers as the A fragment. A segment is 8 K-steps followed
// (Q8_0) by their fp16 block scales; a tile is its segments back to back and
// tiles follow each other, so a CTA's run of tiles is one contiguous range
// that the TMA engine streams into a shared-memory ring with cp.async.bulk.
//
// Row orders are permuted at load time so that fused epilogues find both
// operands of a pair in one lane: rows l and l + 8 of a tile hold RoPE
// elements (i, i + head_dim/2) of Q and K, and (gate r, up r) of the FFN.
//
// Activations enter the tensor cores exactly. Q8_0: the input vector is
// scaled by one power of two 2^e for the whole vector (max|x| 2^-e in
// [32, 64)) and written as three int8 digits, x = 2^e (d0 + d1 2^-7 + d2
// 2^-14), the B columns of an exact s8 MMA (m16n8k32) whose int32 sums are
// rescaled in fp32 by the fp16 block scale of each K-step. F16: x 2^-e is
// split into fp16 hi + lo, two B columns of an f16 MMA (m16n8k16) with fp32
// accumulation.
#pragma once
#include <type_traits>
#include <cuda_fp16.h>

#include <cstdint>

#include "ptx.cuh"

namespace vg {

// FSQ (step kernel only): bias + round(tanh(y) * scale) / scale, the ResidualLM
// quantiser (fsq_quantize.comp) on linear_bias.comp's output.
enum class Mode { PLAIN, RESID, SWIGLU, QKV, FSQ };
enum class Pro { COPY, RMSNORM };

constexpr int kMvConsumers = 8;                       // consumer warps per matvec CTA
constexpr int kMvThreads = 32 * (kMvConsumers + 1);   // + one producer warp
constexpr uint32_t kTileRows = 16;                     // rows of a tile = M of one MMA
constexpr uint32_t kSegSteps = 8;                      // K-steps per segment
constexpr uint32_t kStepBytes = 512;                   // 16 rows x 32 bytes
constexpr uint32_t kSegQsBytes = kSegSteps * kStepBytes;
constexpr uint32_t kStageSegs = 4;                    // segments per pipeline stage (one bulk copy)
constexpr uint32_t kChunkSteps = kStageSegs * kSegSteps / 8;  // K-steps per consumer warp per stage
static_assert(kChunkSteps == 4 && kSegSteps % kChunkSteps == 0,
              "each consumer warp takes one batch of 4 K-steps of one segment per stage");

// Slots of the per-stream device control block.
constexpr uint32_t kCtrlPos = 0;    // decode position of the step being run
constexpr uint32_t kCtrlToken = 1;  // token id of a token step
constexpr uint32_t kCtrlErr = 2;    // error flag bits (ptx.cuh)
constexpr uint32_t kCtrlWaitNs = 3; // limit of every bounded device wait in ns (0: kWaitLimitNs); read
                                    // through the error word by wait_limit (ptx.cuh), so it follows it
constexpr uint32_t kCtrlBarExtra = 4;  // arrivals added to every grid-barrier target of the next step
                                       // (0 in service; a test sets 1 to make a barrier wait run out)
constexpr uint32_t kCtrlWords = 16;
static_assert(kCtrlWaitNs == kCtrlErr + 1, "wait_limit reads the limit from the word after the error word");

// Segmented 16-row tiles. A K-step is 32 columns of Q8_0 quants or 16 columns
// of fp16 values of the tile's 16 rows: 512 bytes stored as four 8x16-byte
// matrices [rows 0-7, bytes 0-15][rows 8-15, bytes 0-15][rows 0-7, bytes
// 16-31][rows 8-15, bytes 16-31], which is the order ldmatrix.x4 delivers the
// A fragment of mma m16n8k32 (s8) / m16n8k16 (f16) in. A segment is kSegSteps
// K-steps, followed for Q8_0 by their fp16 block scales laid [row % 8]
// [K-step][row / 8] (rows r and r+8 adjacent, a row pair's K-steps contiguous). A tile is its segments back to back and
// the tiles of a matrix follow each other, so a run of tiles is one contiguous
// byte range. Padding rows and columns are zero.
struct TileGeom {
  uint32_t rows, cols, q8;
  __host__ __device__ uint32_t step_cols() const { return q8 ? 32u : 16u; }
  __host__ __device__ uint32_t seg_cols() const { return kSegSteps * step_cols(); }
  __host__ __device__ uint32_t nseg() const { return (cols + seg_cols() - 1) / seg_cols(); }
  __host__ __device__ uint32_t seg_bytes() const { return kSegQsBytes + (q8 ? kSegSteps * kTileRows * 2u : 0u); }
  __host__ __device__ uint32_t tiles() const { return (rows + kTileRows - 1) / kTileRows; }
  __host__ __device__ uint64_t bytes() const { return (uint64_t)tiles() * nseg() * seg_bytes(); }
  __host__ __device__ uint64_t seg_base(uint32_t r, uint32_t seg) const {
    return ((uint64_t)(r / kTileRows) * nseg() + seg) * seg_bytes();
  }
  // byte offset of element (r, k): the int8 quant (Q8_0) or the fp16 value (F16)
  __host__ __device__ uint64_t elem_off(uint32_t r, uint32_t k) const {
    const uint32_t sc = seg_cols(), seg = k / sc, kk = k % sc;
    const uint32_t st = kk / step_cols(), kb = (kk % step_cols()) * (q8 ? 1u : 2u);
    const uint32_t tr = r % kTileRows;
    return seg_base(r, seg) + st * kStepBytes + ((kb >> 4) * 2u + (tr >> 3)) * 128u + (tr & 7u) * 16u + (kb & 15u);
  }
  // byte offset of the fp16 scale of Q8_0 block b of row r
  __host__ __device__ uint64_t scale_off(uint32_t r, uint32_t b) const {
    const uint32_t tr = r % kTileRows;
    return seg_base(r, b / kSegSteps) + kSegQsBytes + (tr & 7u) * 32u + (b % kSegSteps) * 4u + (tr >> 3) * 2u;
  }
};

// KV-cache rows in HBM are stored with their 16-byte chunks (8 fp16 each)
// XOR-permuted by the row's position: chunk c of row r sits at chunk
// c ^ (r & m), m = min(head_dim / 8, 8) - 1. A bulk copy of consecutive rows
// then lands in shared memory so that the 8 rows an ldmatrix reads at one
// chunk column fall in 8 different bank groups (plain rows of 128 or 256
// bytes put all 8 in the same banks). kv_swz gives the stored element index
// of element e of the row at position r.
__host__ __device__ __forceinline__ uint32_t kv_swz(uint32_t r, uint32_t e, uint32_t head_dim) {
  const uint32_t m = (head_dim >= 64u ? 8u : head_dim / 8u) - 1u;
  return ((((e >> 3) ^ (r & m)) << 3) | (e & 7u));
}

struct MvParams {
  const uint8_t *w;       // segmented tiles
  TileGeom g;
  uint32_t stages;        // pipeline stages in the shared-memory ring
  uint32_t rb;            // tiles per CTA (partial-sum buffer rows)
  uint32_t a_bytes;       // shared bytes of the activation operand region (128-aligned)
  uint32_t plane;         // bytes between activation planes
  const float *xsrc;      // input vector (COPY) or hidden state (RMSNORM)
  const float *normw;     // RMSNorm weight
  float eps;
  float *out;             // output vector (q for QKV)
  const float *resid;     // RESID: residual input
  float alpha;            // PLAIN: output scale; RESID: residual branch scale
  // QKV epilogue
  uint32_t q_rows, kv_rows, head_dim, ctx;
  __half *kc, *vc;        // this layer's caches, [kv_head][ctx][head_dim]
  const float *inv_freq;  // [head_dim/2], 1/pow(theta, 2i/d)
  const float *ext;       // [head_dim/2], LongRoPE factors
  float rope_scaling;
  uint32_t *ctrl;
  float *out2;            // step kernel RESID: a second copy of the output (nullptr: none)
};

// Shared-memory plan of one matvec CTA (host and device agree on it).
struct MvSmem {
  uint32_t a, ring, bars, red, scr, total;
  __host__ __device__ MvSmem(const MvParams &p) {
    const uint32_t ns = p.stages;
    a = 0;
    ring = p.a_bytes;
    bars = ring + ns * kStageSegs * p.g.seg_bytes();
    red = bars + ns * 16u;
    scr = red + p.rb * kMvConsumers * kTileRows * 4u;
    total = scr + 64u * 4u;
  }
};

__host__ __device__ inline uint32_t mv_a_plane(uint32_t q8, uint32_t cols_pad) {
  // planes are offset by 32 bytes modulo 128 so the 8-byte B-fragment loads of
  // the 12 (Q8_0) or 8 (F16) lanes that read different planes hit different banks
  const uint32_t b = q8 ? cols_pad : cols_pad * 2u;
  return ((b + 127u) & ~127u) + 32u;
}

// Byte of activation element kk (0..31 of a Q8_0 block, or 0..15 of an F16
// K-step in 2-byte units) inside its 32-byte K-step of a digit / half plane:
// the order of the B fragment, so lane tq finds its b0 and b1 as one 8-byte
// word at tq * 8.
__device__ __forceinline__ uint32_t bfrag_byte_q8(uint32_t kk) {
  return kk < 16u ? (kk >> 2) * 8u + (kk & 3u) : ((kk - 16u) >> 2) * 8u + 4u + (kk & 3u);
}
__device__ __forceinline__ uint32_t bfrag_half_f16(uint32_t kk) {
  return kk < 8u ? (kk >> 1) * 4u + (kk & 1u) : ((kk - 8u) >> 1) * 4u + 2u + (kk & 1u);
}
__host__ __device__ inline uint32_t mv_a_bytes(uint32_t q8, uint32_t cols_pad) {
  const uint32_t pl = mv_a_plane(q8, cols_pad);
  const uint32_t bytes = q8 ? 3u * pl + (cols_pad / 32u) * 4u : 2u * pl + 16u;
  return (bytes + 127u) & ~127u;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
// Largest value over the warp in one redux.sync: fp32 bit patterns mapped to
// u32 keys in the same order (negative values: every bit flipped; others: the
// sign bit set), the largest key taken, and mapped back. Exact, like fmaxf over
// the lanes (NaN inputs excepted).
__device__ __forceinline__ float warp_max(float v) {
  const uint32_t b = __float_as_uint(v);
  const uint32_t k = b ^ ((uint32_t)((int32_t)b >> 31) | 0x80000000u);
  const uint32_t r = __reduce_max_sync(0xffffffffu, k);
  return __uint_as_float(r ^ ((r & 0x80000000u) ? 0x80000000u : 0xFFFFFFFFu));
}

// Sums 8 per-lane values over the warp with 9 shuffles (instead of 8 x 5): on
// return, lane l holds the warp total of value (l >> 2) & 7.
__device__ __forceinline__ float warp_sum8(const float (&v)[8], uint32_t lane) {
  const bool h4 = (lane >> 4) & 1, h2 = (lane >> 3) & 1, h1 = (lane >> 2) & 1;
  float a[4], b[2], c;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float keep = h4 ? v[4 + i] : v[i], send = h4 ? v[i] : v[4 + i];
    a[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
  }
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const float keep = h2 ? a[2 + i] : a[i], send = h2 ? a[i] : a[2 + i];
    b[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
  }
  {
    const float keep = h1 ? b[1] : b[0], send = h1 ? b[0] : b[1];
    c = keep + __shfl_xor_sync(0xffffffffu, send, 4);
  }
  c += __shfl_xor_sync(0xffffffffu, c, 2);
  c += __shfl_xor_sync(0xffffffffu, c, 1);
  return c;
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t (&r)[4], const void *p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}

// The same four 8x8 matrices, each transposed on the way in.
__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t (&r)[4], const void *p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ uint32_t pack_half2(__half lo, __half hi) {
  return (uint32_t)__half_as_ushort(lo) | ((uint32_t)__half_as_ushort(hi) << 16);
}

// D = A(16x32 s8, row) * B(32x8 s8, col) + c (every element), A fragment as
// ldmatrix.x4 delivers it.
__device__ __forceinline__ void mma_s8(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1, int c) {
  asm(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%10, %10, %10, %10};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(c));
}

// C += A(16x16 f16, row) * B(16x8 f16, col) in fp32.
__device__ __forceinline__ void mma_f16(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// RoPE of one (a, b) pair, rope.comp:28-49 with inv_freq precomputed on the host.
__device__ __forceinline__ void rope_pair(float &a, float &b, uint32_t pos, uint32_t i, const float *inv_freq,
                                          const float *ext, float scaling) {
  const float angle = __fdiv_rn(__fmul_rn((float)pos, inv_freq[i]), ext[i]);
  float sn, cs;
  sincosf(angle, &sn, &cs);
  const float c = __fmul_rn(cs, scaling), s = __fmul_rn(sn, scaling);
  const float a2 = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
  const float b2 = __fadd_rn(__fmul_rn(b, c), __fmul_rn(a, s));
  a = a2;
  b = b2;
}

// FSQ quantisation in place (fsq_quantize.comp:8-11): x = round(tanh(x) * scale)
// / scale. GLSL leaves the rounding of halves to the implementation; roundf
// rounds them away from zero.
__global__ void fsq_quantize_kernel(float *x, uint32_t n, float scale) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  x[i] = __fdiv_rn(roundf(__fmul_rn(tanhf(x[i]), scale)), scale);
}

// Power-of-two scale 2^e for a block whose largest magnitude has fp32 bits
// `mbits`, chosen so that max|x| * 2^-e lies in [32, 64). Returns false for a
// block that is zero or below 2^-117 in magnitude (treated as zero).
__device__ __forceinline__ bool block_exponent(uint32_t mbits, int &e) {
  const int ef = (int)((mbits >> 23) & 0xFFu);
  if (ef < 10) return false;
  e = ef - 127 - 5;
  return true;
}
__device__ __forceinline__ float pow2f(int e) { return __uint_as_float((uint32_t)(127 + e) << 23); }

// Epilogue of packed rows R and R + 8 of one tile (R = 16t + l, l < 8). The
// pair modes store the two halves of a pair there: SWIGLU gate row 8t + l and
// up row 8t + l; QKV (Q and K) RoPE elements i and i + d/2 of one head.
template <Mode M>
__device__ __forceinline__ void mv_epilogue(const MvParams &p, uint32_t R, float a, float b, uint32_t pos) {
  const uint32_t R2 = R + 8u;
  if constexpr (M == Mode::PLAIN) {
    if (R < p.g.rows) p.out[R] = __fmul_rn(a, p.alpha);  // matvec.comp:61
    if (R2 < p.g.rows) p.out[R2] = __fmul_rn(b, p.alpha);
  } else if constexpr (M == Mode::RESID) {
    // residual_rmsnorm.comp:27, hidden + branch * scale, with branch = this row's product
    if (R < p.g.rows) p.out[R] = __fadd_rn(p.resid[R], __fmul_rn(a, p.alpha));
    if (R2 < p.g.rows) p.out[R2] = __fadd_rn(p.resid[R2], __fmul_rn(b, p.alpha));
  } else if constexpr (M == Mode::SWIGLU) {
    const uint32_t o = (R / kTileRows) * 8u + (R % kTileRows);
    if (2u * o < p.g.rows) p.out[o] = __fmul_rn(__fdiv_rn(a, __fadd_rn(1.0f, expf(-a))), b);  // matvec_swiglu.comp:67
  } else {
    if (R >= p.g.rows) return;
    const uint32_t hd = p.head_dim, half_d = hd >> 1;
    if (pos >= p.ctx) {
      set_error(p.ctrl + kCtrlErr, kErrPosition);
    } else if (R < p.q_rows + p.kv_rows) {
      // Q or K: tile m of a head holds pair elements i = 8m + l and i + d/2
      const bool isq = R < p.q_rows;
      const uint32_t Rr = isq ? R : R - p.q_rows;
      const uint32_t head = Rr / hd, w = Rr % hd, i = (w / kTileRows) * 8u + (w % kTileRows);
      rope_pair(a, b, pos, i, p.inv_freq, p.ext, p.rope_scaling);
      if (isq) {
        p.out[head * hd + i] = a;
        p.out[head * hd + i + half_d] = b;
      } else {
        __half *dst = p.kc + ((size_t)head * p.ctx + pos) * hd;  // store_kv.comp:21-22, RNE
        dst[kv_swz(pos, i, hd)] = __float2half_rn(a);
        dst[kv_swz(pos, i + half_d, hd)] = __float2half_rn(b);
      }
    } else {
      const uint32_t v = R - p.q_rows - p.kv_rows, kvh = v / hd, j = v % hd;
      __half *dst = p.vc + ((size_t)kvh * p.ctx + pos) * hd;
      dst[kv_swz(pos, j, hd)] = __float2half_rn(a);
      dst[kv_swz(pos, j + 8u, hd)] = __float2half_rn(b);
    }
  }
}

// ---------------------------------------------------------------------------
// Matrix-vector product with fused prologue and epilogue.
//
// A CTA owns a contiguous range of tiles, i.e. a contiguous run of segments in
// HBM. A producer warp streams that run in stages of kStageSegs segments (one
// ~17 KB cp.async.bulk per stage: large copies are what reach full HBM
// bandwidth on this part) into a ring of shared-memory stages. The consumer
// warps build the activation operand (RMSNorm of the hidden state or a copy,
// then the exact int8 digits or the fp16 hi/lo split), run the tensor-core
// K-steps with every warp taking a 4-K-step batch of every stage, keep one
// partial per (tile, warp) in shared memory, and after one barrier reduce each
// tile's 8 partials in warp order (deterministic) and run the epilogue.
//
// The three parts are device functions shared by matvec_kernel (one matrix per
// launch) and the persistent decode-step kernel (all matrices of a step in one
// launch, the ring running across them).
// ---------------------------------------------------------------------------
struct MvRing {
  uint8_t *ring;           // nst slots of `slot` bytes
  uint64_t *full, *empty;  // per slot: bulk copy landed / all consumer warps done
  uint32_t nst, slot;
};

// Position in the ring, advanced without divisions: the slot of the next
// stage, the parity of that slot's current use, and the stage count.
struct RingPos {
  uint32_t slot = 0, phase = 0, n = 0;
  __device__ __forceinline__ void next(uint32_t nst) {
    ++n;
    if (++slot == nst) {
      slot = 0;
      phase ^= 1u;
    }
  }
};

// Producer side of one stage: waits (bounded) until the slot's previous use
// has been released, then announces `bytes` for it. False when the wait gave up.
__device__ __forceinline__ bool ring_claim(const MvRing &R, const RingPos &rp, uint32_t bytes,
                                           const uint32_t *abort_flag, uint32_t *err) {
  if (rp.n >= R.nst && !mbar_wait_backoff(&R.empty[rp.slot], rp.phase ^ 1u, abort_flag)) {
    set_error(err, kErrConsumerWait);
    return false;
  }
  mbar_arrive_expect_tx(&R.full[rp.slot], bytes);
  return true;
}

// Issues the stages of a run of n_items segments of SEGB bytes starting at src
// as the next stages of the ring. False when a wait for a free slot gave up.
__device__ __forceinline__ bool mv_produce(const MvRing &R, const uint8_t *src, uint32_t n_items, uint32_t SEGB,
                                           RingPos &rp, const uint32_t *abort_flag, uint32_t *err) {
  for (uint32_t s = 0; s < n_items; s += kStageSegs) {
    const uint32_t bytes = min(kStageSegs, n_items - s) * SEGB;
    if (!ring_claim(R, rp, bytes, abort_flag, err)) return false;
    bulk_g2s(R.ring + rp.slot * R.slot, src + (uint64_t)s * SEGB, bytes, &R.full[rp.slot]);
    rp.next(R.nst);
  }
  return true;
}

// Waits (bounded) until every bulk copy issued into the ring has landed, so
// that the CTA never exits with copies in flight: the last use of each slot is
// the one just before rp (going back one lap).
__device__ __forceinline__ void mv_drain(const MvRing &R, const RingPos &rp, uint32_t *err) {
  for (uint32_t i = 0; i < R.nst && i < rp.n; ++i) {
    // slot i's last use has parity rp.phase if it lies before rp.slot in this lap, else the previous one
    const uint32_t par = i < rp.slot ? rp.phase : rp.phase ^ 1u;
    if (!mbar_wait_bounded(&R.full[i], par, nullptr)) {
      set_error(err, kErrDrainWait);
      return;
    }
  }
}

// Where a matvec's input vector comes from: an fp32 vector written earlier
// (read through L2), or row `token` of a token table times alpha
// (embedding.comp:28-47).
struct XSrc {
  const float *x;      // fp32 input, or nullptr for a token-table row
  const uint8_t *tab;  // token table (segmented tiles) when x == nullptr
  TileGeom g;
  uint32_t token;
  float alpha;
};
template <bool TAB>
__device__ __forceinline__ float xsrc_elem(const XSrc &s, uint32_t k) {
  if constexpr (!TAB) return __ldcg(s.x + k);
  float v;
  if (s.g.q8) {
    const float d = __half2float(*reinterpret_cast<const __half *>(s.tab + s.g.scale_off(s.token, k / 32u)));
    v = __fmul_rn(d, (float)(int8_t)s.tab[s.g.elem_off(s.token, k)]);
  } else {
    v = __half2float(*reinterpret_cast<const __half *>(s.tab + s.g.elem_off(s.token, k)));
  }
  return __fmul_rn(v, s.alpha);
}

// What the consumer warps wait for before they read the input vector.
struct WaitSpec {
  uint32_t kind;                  // kWaitNone, kWaitPdl (griddepcontrol.wait), kWaitGrid
  const unsigned long long *bar;  // kWaitGrid: arrival counter, and the count to reach
  unsigned long long target;
  uint32_t *err;
};
enum : uint32_t { kWaitNone = 0, kWaitPdl = 1, kWaitGrid = 2 };
__device__ __forceinline__ void consumer_wait(const WaitSpec &w, uint32_t cw, uint32_t lane) {
  if (w.kind == kWaitPdl) {
    pdl_wait();
  } else if (w.kind == kWaitGrid) {
    if (cw == 0 && lane == 0 && !grid_wait(w.bar, w.target, w.err)) set_error(w.err, kErrGridWait);
    named_bar(1, kMvConsumers * 32);
  }
}

// Activation operand of a matvec in shared memory: Q8_0 -> three int8 digit
// planes and the whole-vector power of two *sx; F16 -> fp16 hi and lo planes
// and the whole-vector power of two *xscale. Run by the kMvConsumers consumer
// warps (named barrier 1). The input vector (C elements) comes from src (its
// token table when TAB); with RMS it is RMSNormed with normw, else copied. The wait comes after the RMSNorm
// weights are loaded and before the first input load. With xout set, the
// (normalised) input vector is also written there.
template <bool Q8, bool RMS, bool TAB>
__device__ __forceinline__ void mv_activation(uint32_t C, uint32_t cols_pad, const float *normw, float eps,
                                              uint8_t *areg, uint32_t plane, float *scr, uint32_t cw, uint32_t lane,
                                              const XSrc &src, const WaitSpec &wait, float *xout) {
  constexpr uint32_t NCT = kMvConsumers * 32;
  auto xload = [&](uint32_t k) { return xsrc_elem<TAB>(src, k); };
  float *sx = reinterpret_cast<float *>(areg + 3u * plane);      // Q8: 2^e of the whole vector
  float *xscale = reinterpret_cast<float *>(areg + 2u * plane);  // F16: 2^e of the whole vector
  // Warp cw handles the groups of 4 consecutive 32-element blocks b with
  // (b / 4) % 8 == cw, i.e. 128 consecutive elements per group, 4 per lane:
  // block q of a group is lanes 8q..8q+7, so a block's max takes 3 shuffles
  // and each lane writes its 4 digits of a plane as one 32-bit word. When a
  // tile has a multiple of 4 segments (kStageSegs) these are exactly the Q8_0
  // K-steps that warp cw consumes in mv_consume, so no barrier is needed
  // between the digits and the MMAs. Every activation load is issued up front
  // (one round trip); the RMSNorm weight does not depend on the producer of the
  // input and is loaded before the wait. Register path for up to 4096 (RMSNorm
  // inputs) or 6144 (copied inputs) columns.
  constexpr uint32_t MAXG = RMS ? 4 : 6;
  const uint32_t NGRP = (cols_pad / 32u + 3u) / 4u;                     // groups of 4 blocks
  const uint32_t JG = NGRP > cw ? (NGRP - cw + kMvConsumers - 1) / kMvConsumers : 0u;  // groups of this warp
  auto elem0 = [&](uint32_t g) { return (g * kMvConsumers + cw) * 128u + lane * 4u; };  // first element of lane
  const bool regs = (NGRP + kMvConsumers - 1) / kMvConsumers <= MAXG;
  auto load4 = [&](uint32_t k0, auto fetch) {
    float4 v;
    v.x = k0 < C ? fetch(k0) : 0.f;
    v.y = k0 + 1u < C ? fetch(k0 + 1u) : 0.f;
    v.z = k0 + 2u < C ? fetch(k0 + 2u) : 0.f;
    v.w = k0 + 3u < C ? fetch(k0 + 3u) : 0.f;
    return v;
  };
  float4 xr[MAXG], wr[MAXG];
  if constexpr (RMS) {
#pragma unroll
    for (uint32_t g = 0; g < MAXG; ++g)
      wr[g] = (regs && g < JG) ? load4(elem0(g), [&](uint32_t k) { return normw[k]; }) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  consumer_wait(wait, cw, lane);
#pragma unroll
  for (uint32_t g = 0; g < MAXG; ++g)
    xr[g] = (regs && g < JG) ? load4(elem0(g), xload) : make_float4(0.f, 0.f, 0.f, 0.f);
  // RMSNorm (rmsnorm.comp:21-42, inversesqrt taken as 1/sqrt): x = h * inv_rms * w.
  // Without xout the factor inv_rms is deferred: the operand is h * w and the
  // consumer scales each output row by inv_rms (W (inv_rms h w) = inv_rms W (h w)),
  // so the sum of squares needs no barrier here; this warp's partial goes to
  // scr[8 + cw] for mv_consume. With xout the normalised x itself is formed.
  const bool defer = RMS && xout == nullptr;
  float inv_rms = 1.0f;
  if constexpr (RMS) {
    float ss = 0.f;
    if (regs) {
#pragma unroll
      for (uint32_t g = 0; g < MAXG; ++g) ss += xr[g].x * xr[g].x + xr[g].y * xr[g].y + xr[g].z * xr[g].z + xr[g].w * xr[g].w;
    } else {
      for (uint32_t i = cw * 32u + lane; i < C; i += NCT) {
        const float v = xload(i);
        ss += v * v;
      }
    }
    ss = warp_sum(ss);
    if (defer) {
      if (lane == 0) scr[8 + cw] = ss;
    } else {
      if (lane == 0) scr[cw] = ss;
      named_bar(1, NCT);
      float tot = 0.f;
#pragma unroll
      for (int w = 0; w < kMvConsumers; ++w) tot += scr[w];
      inv_rms = 1.0f / sqrtf(tot / (float)C + eps);
    }
    if (regs) {
#pragma unroll
      for (uint32_t g = 0; g < MAXG; ++g) {
        xr[g].x = __fmul_rn(__fmul_rn(xr[g].x, inv_rms), wr[g].x);
        xr[g].y = __fmul_rn(__fmul_rn(xr[g].y, inv_rms), wr[g].y);
        xr[g].z = __fmul_rn(__fmul_rn(xr[g].z, inv_rms), wr[g].z);
        xr[g].w = __fmul_rn(__fmul_rn(xr[g].w, inv_rms), wr[g].w);
      }
    }
  }
  // element k when the row is too long for the register path
  auto xglobal = [&](uint32_t k) -> float {
    if (k >= C) return 0.f;
    const float v = xload(k);
    if constexpr (RMS) return __fmul_rn(__fmul_rn(v, inv_rms), normw[k]);
    return v;
  };
  // f(g, v) for every group of this warp (register path fully unrolled)
  auto each_group = [&](auto f) {
    if (regs) {
#pragma unroll
      for (uint32_t g = 0; g < MAXG; ++g)
        if (g < JG) f(g, xr[g]);
    } else {
      for (uint32_t g = 0; g < JG; ++g) f(g, load4(elem0(g), xglobal));
    }
  };
  if (xout) {
    each_group([&](uint32_t g, const float4 &v) {
      const uint32_t k0 = elem0(g);
      if (k0 < C) xout[k0] = v.x;
      if (k0 + 1u < C) xout[k0 + 1u] = v.y;
      if (k0 + 2u < C) xout[k0 + 2u] = v.z;
      if (k0 + 3u < C) xout[k0 + 3u] = v.w;
    });
  }
  if constexpr (Q8) {
    // int8 digits and the whole-vector power of two 2^e (max|x| * 2^-e in
    // [32, 64)): v = x * 2^-e (|v| < 64, exact), n = round(v * 2^14) through
    // the 1.5 * 2^23 constant (for |t| < 2^22, t + 1.5 * 2^23 rounds t to an
    // integer and its bit pattern minus 0x4B400000 is that integer), then n =
    // d0 * 2^14 + d1 * 2^7 + d2 with every digit in [-64, 64] by integer shifts.
    float m = 0.f;
    each_group([&](uint32_t, const float4 &v) {
      m = fmaxf(m, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
    });
    m = warp_max(m);
    named_bar(1, NCT);  // scr[] reuse after the RMSNorm reduction
    if (lane == 0) scr[cw] = m;
    named_bar(1, NCT);
    float mx = 0.f;
#pragma unroll
    for (int w = 0; w < kMvConsumers; ++w) mx = fmaxf(mx, scr[w]);
    int e = 0;
    const bool nz = block_exponent(__float_as_uint(mx), e);
    const float inv = nz ? pow2f(-e) : 0.f;
    constexpr float kRnd = 12582912.0f;
    constexpr int kRndBits = 0x4B400000;
    auto split = [&](float x, int &q0, int &q1, int &q2) {
      const int n = __float_as_int(fmaf(x * inv, 16384.0f, kRnd)) - kRndBits;
      q0 = (n + 8192) >> 14;
      const int r = n - (q0 << 14);
      q1 = (r + 64) >> 7;
      q2 = r - (q1 << 7);
    };
    auto digits = [&](uint32_t g, const float4 &v) {
      int q[3][4];
      split(v.x, q[0][0], q[1][0], q[2][0]);
      split(v.y, q[0][1], q[1][1], q[2][1]);
      split(v.z, q[0][2], q[1][2], q[2][2]);
      split(v.w, q[0][3], q[1][3], q[2][3]);
      const uint32_t k0 = elem0(g), b = k0 >> 5;
      if (b * 32u < cols_pad) {
        const uint32_t o = b * 32u + bfrag_byte_q8(k0 & 31u);  // 4 consecutive bytes
#pragma unroll
        for (int d = 0; d < 3; ++d) {
          const uint32_t w = __byte_perm(__byte_perm((uint32_t)q[d][0], (uint32_t)q[d][1], 0x0040u),
                                         __byte_perm((uint32_t)q[d][2], (uint32_t)q[d][3], 0x0040u), 0x5410u);
          *reinterpret_cast<uint32_t *>(areg + d * plane + o) = w;
        }
      }
    };
    each_group(digits);
    if (cw == 0 && lane == 0) *sx = nz ? pow2f(e) : 0.f;
    named_bar(1, NCT);
  } else {
    // whole-vector power-of-two scale, then fp16 hi + lo
    float m = 0.f;
    each_group([&](uint32_t, const float4 &v) {
      m = fmaxf(m, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
    });
    m = warp_max(m);
    named_bar(1, NCT);  // scr[] reuse after the RMSNorm reduction
    if (lane == 0) scr[cw] = m;
    named_bar(1, NCT);
    float mx = 0.f;
#pragma unroll
    for (int w = 0; w < kMvConsumers; ++w) mx = fmaxf(mx, scr[w]);
    const uint32_t ef = (__float_as_uint(mx) >> 23) & 0xFFu;
    const int e = ef < 20 ? 0 : (int)ef - 127 - 13;  // max|x| * 2^-e < 2^14
    const float inv = pow2f(-e);
    __half *hi = reinterpret_cast<__half *>(areg), *lo = reinterpret_cast<__half *>(areg + plane);
    auto halves = [&](uint32_t g, const float4 &v4) {
      const uint32_t k0 = elem0(g);
      const float vv[4] = {v4.x, v4.y, v4.z, v4.w};
#pragma unroll
      for (uint32_t i = 0; i < 4; ++i) {
        const uint32_t k = k0 + i;
        if (k >= cols_pad) continue;
        const uint32_t o = (k & ~15u) + bfrag_half_f16(k & 15u);  // element k of K-step k / 16
        const float v = vv[i] * inv;
        const __half h = __float2half_rn(v);
        hi[o] = h;
        lo[o] = __float2half_rn(v - __half2float(h));
      }
    };
    each_group(halves);
    if (cw == 0 && lane == 0) *xscale = pow2f(e);
    named_bar(1, NCT);
  }
}

// Consumes the n_items segments of this CTA's tile run from ring stages j, j+1,
// ... (tile t0 first), writes per-(tile, warp) partials into red (zeroed by the
// caller for the run's tiles), and after a consumer barrier runs the tile
// reductions and the epilogue. ok turns false when a wait gave up (the
// partials are then incomplete and the error flag is set).
// Consumer side of a matvec over n_items ring segments (tiles t0.. of this
// CTA's run). epilogue(R, a, b, pv) receives the finished rows R and R + 8
// and pv = pre(R); for the first tile of each warp pre runs before the K
// loop, so the loads it makes overlap the loop.
template <bool Q8, class Pre, class Epilogue>
__device__ __forceinline__ void mv_consume(const MvRing &R, RingPos &rp, uint32_t n_items, uint32_t NSEG,
                                           uint32_t SEGB, const uint8_t *areg, uint32_t plane, float *red,
                                           const MvParams &p, uint32_t t0, uint32_t cw, uint32_t lane,
                                           const uint32_t *abort_flag, uint32_t *err, bool &ok,
                                           const float *defer_ss, Pre pre, Epilogue epilogue) {
  constexpr uint32_t NCT = kMvConsumers * 32;
  const float *sx = reinterpret_cast<const float *>(areg + 3u * plane);
  const float *xscale = reinterpret_cast<const float *>(areg + 2u * plane);
  // mma m16n8k32.s8 (Q8_0) / m16n8k16.f16 (F16) with the weights as A (16 rows
  // x one K-step) and the activation as B: column n of B is digit n (Q8_0) or
  // the hi/lo half n (F16); the other columns are zero (their lanes load plane
  // 0 and mask it). Lane (gq, tq) receives D rows gq and gq + 8, columns 2tq
  // and 2tq + 1.
  const uint32_t gq = lane >> 2, tq = lane & 3u;
  // Q8: columns 3-7 of B may hold anything (their sums are dropped: column 3
  // by c7 = 0 in lane tq = 1, columns 4-7 by lane_scale = 0), so every lane
  // loads a digit plane unmasked; F16: columns 2-7 are zero (masked), since
  // fp16 products of arbitrary bytes need not be finite
  const bool brow = Q8 ? (gq < 3) : (gq < 2);
  const uint8_t *bplane = areg + (Q8 ? gq % 3u : (brow ? gq : 0u)) * plane;
  const uint32_t bmask = (Q8 || brow) ? 0xFFFFFFFFu : 0u;
  const float c7 = tq == 0 ? 0.0078125f : 0.f;
  // Q8_0: the int32 accumulator of the MMA starts at the bit pattern of
  // 1.5 * 2^23, so the result read as a float is 1.5 * 2^23 + S exactly
  // (|S| <= 32 * 127 * 64 < 2^22) and one exact subtraction gives S. Lane tq=0
  // combines digits 0 and 1 as S0 + S1 * 2^-7, lane tq=1 has S2 (column 3 is
  // zero), so a row's partial is acc (tq=0) + acc * 2^-14 (tq=1).
  // F16: lane tq=0 holds hi (column 0) and lo (column 1).
  constexpr int kMagicBits = 0x4B400000;
  constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23
  const float lane_scale = Q8 ? (tq == 0 ? 1.f : tq == 1 ? 6.103515625e-05f : 0.f) : (tq == 0 ? 1.f : 0.f);
  const float xsc = Q8 ? *sx : *xscale;  // the activation's power of two
  float acc0 = 0.f, acc1 = 0.f;
  float acc0b = 0.f, acc1b = 0.f;  // Q8_0: second chain when two stages are processed together
  float cf[2][4] = {};  // F16: two accumulator chains

  // This warp's partial of one tile: after the tq reduction, lane (gq, 0)
  // holds rows gq and gq + 8; they go to red[tile][warp][row].
  auto flush = [&](uint32_t rel) {
    float v0, v1;
    if constexpr (Q8) {
      v0 = (acc0 + acc0b) * (lane_scale * xsc);
      v1 = (acc1 + acc1b) * (lane_scale * xsc);
    } else {
      v0 = (cf[0][0] + cf[0][1] + cf[1][0] + cf[1][1]) * lane_scale;
      v1 = (cf[0][2] + cf[0][3] + cf[1][2] + cf[1][3]) * lane_scale;
    }
    v0 += __shfl_xor_sync(0xffffffffu, v0, 1);
    v1 += __shfl_xor_sync(0xffffffffu, v1, 1);
    v0 += __shfl_xor_sync(0xffffffffu, v0, 2);
    v1 += __shfl_xor_sync(0xffffffffu, v1, 2);
    if (tq == 0) {
      if constexpr (!Q8) {
        v0 *= xsc;
        v1 *= xsc;
      }
      red[(rel * kMvConsumers + cw) * kTileRows + gq] = v0;
      red[(rel * kMvConsumers + cw) * kTileRows + gq + 8u] = v1;
    }
    acc0 = acc1 = acc0b = acc1b = 0.f;
#pragma unroll
    for (int a = 0; a < 2; ++a)
#pragma unroll
      for (int b = 0; b < 4; ++b) cf[a][b] = 0.f;
  };

  // Every warp reads every stage: a stage holds 4 consecutive segments and
  // warp cw takes K-steps 4*(cw%2) .. 4*(cw%2)+3 of segment cw/2 of it, so all
  // 8 warps work on the stage at once. A segment never spans two tiles. Every
  // warp waits for every stage and releases it (the empty barrier counts 8
  // arrivals), so no warp can run more than one ring phase ahead.
  const uint32_t sq = (cw & 1u) * kChunkSteps;  // first K-step of this warp within its segment
  // this warp's segment of the current stage: index i in the run = tile rel, segment seg of the tile
  uint32_t i = cw >> 1, rel = 0, seg = i;
  while (seg >= NSEG) {
    seg -= NSEG;
    ++rel;
  }
  uint32_t cur = 0xFFFFFFFFu;  // tile (relative) of the accumulated partial
  const uint32_t ntiles = (n_items + NSEG - 1) / NSEG;
  float2 pv0 = make_float2(0.f, 0.f);
  if (lane < 8 && cw < ntiles) pv0 = pre((t0 + cw) * kTileRows + lane);
  // K-steps of NB stages (segment bases sgs, first K-steps kss): all
  // shared-memory loads first, then the NB * 4 independent MMAs, then the rescale
  auto run = [&](auto nbc, const uint8_t *const (&sgs)[2], const uint32_t (&kss)[2]) {
    constexpr int NB = decltype(nbc)::value;
    uint32_t a[NB][4][4], b0[NB][4], b1[NB][4];
#pragma unroll
    for (int nb = 0; nb < NB; ++nb)
#pragma unroll
      for (uint32_t q = 0; q < 4; ++q) {
        ldmatrix_x4(a[nb][q], sgs[nb] + (sq + q) * kStepBytes + lane * 16u);
        // B fragment: one 8-byte word per lane per K-step (planes in B-fragment order)
        const uint2 bw = *reinterpret_cast<const uint2 *>(bplane + (kss[nb] + q) * 32u + tq * 8u);
        b0[nb][q] = bw.x & bmask;
        b1[nb][q] = bw.y & bmask;
      }
    if constexpr (Q8) {
      // the scales of rows gq and gq + 8 for the 4 K-steps
      uint4 wsv[NB];
#pragma unroll
      for (int nb = 0; nb < NB; ++nb) wsv[nb] = *reinterpret_cast<const uint4 *>(sgs[nb] + kSegQsBytes + gq * 32u + sq * 4u);
      int r[NB][4][4];
#pragma unroll
      for (int nb = 0; nb < NB; ++nb)
#pragma unroll
        for (uint32_t q = 0; q < 4; ++q) mma_s8(r[nb][q], a[nb][q], b0[nb][q], b1[nb][q], kMagicBits);
#pragma unroll
      for (int nb = 0; nb < NB; ++nb) {
        const uint32_t wsw[4] = {wsv[nb].x, wsv[nb].y, wsv[nb].z, wsv[nb].w};
        float &A0 = nb == 0 ? acc0 : acc0b, &A1 = nb == 0 ? acc1 : acc1b;
#pragma unroll
        for (uint32_t q = 0; q < 4; ++q) {
          const float2 w = __half22float2(*reinterpret_cast<const __half2 *>(&wsw[q]));
          const float v0 = fmaf(__int_as_float(r[nb][q][1]) - kMagic, c7, __int_as_float(r[nb][q][0]) - kMagic);
          const float v1 = fmaf(__int_as_float(r[nb][q][3]) - kMagic, c7, __int_as_float(r[nb][q][2]) - kMagic);
          A0 = fmaf(v0, w.x, A0);
          A1 = fmaf(v1, w.y, A1);
        }
      }
    } else {
#pragma unroll
      for (int nb = 0; nb < NB; ++nb)
#pragma unroll
        for (uint32_t q = 0; q < 4; ++q) mma_f16(cf[q & 1], a[nb][q], b0[nb][q], b1[nb][q]);
    }
  };
  auto advance = [&] {
    rp.next(R.nst);
    i += kStageSegs;
    seg += kStageSegs;
    while (seg >= NSEG) {
      seg -= NSEG;
      ++rel;
    }
  };
  if (NSEG % (2u * kStageSegs) == 0) {
    // Tiles of an even number of stages: every iteration takes two stages of
    // one tile (this warp's segment cw / 2 of each), every tile ends on a pair.
    const uint32_t ntl = n_items / NSEG, spt = NSEG / kStageSegs;
    for (uint32_t t = 0; t < ntl && ok; ++t) {
      for (uint32_t j = 0; j < spt; j += 2) {
        RingPos nx = rp;
        nx.next(R.nst);
        if (!mbar_wait_bounded(&R.full[rp.slot], rp.phase, abort_flag) ||
            !mbar_wait_bounded(&R.full[nx.slot], nx.phase, abort_flag)) {
          set_error(err, kErrConsumerWait);
          ok = false;
          break;
        }
        const uint32_t ks0 = (j * kStageSegs + (cw >> 1)) * kSegSteps + sq;
        const uint8_t *const sgs[2] = {R.ring + rp.slot * R.slot + (cw >> 1) * SEGB,
                                       R.ring + nx.slot * R.slot + (cw >> 1) * SEGB};
        const uint32_t kss[2] = {ks0, ks0 + kStageSegs * kSegSteps};
        run(std::integral_constant<int, 2>{}, sgs, kss);
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&R.empty[rp.slot]);
          mbar_arrive(&R.empty[nx.slot]);
        }
        rp = nx;
        rp.next(R.nst);
      }
      if (ok) flush(t);
    }
    cur = 0xFFFFFFFFu;  // flushed
  } else
  for (uint32_t s = 0; s < n_items && ok; s += kStageSegs) {
    const uint32_t slot0 = rp.slot;
    if (!mbar_wait_bounded(&R.full[slot0], rp.phase, abort_flag)) {
      set_error(err, kErrConsumerWait);
      ok = false;
      break;
    }
    // Two stages at once when this warp's segment of the next stage continues
    // the same tile: twice the work per wait, and the two batches overlap.
    const bool pair = i < n_items && i + kStageSegs < n_items && seg + kStageSegs < NSEG;
    if (i < n_items) {
      if (rel != cur) {
        if (cur != 0xFFFFFFFFu) flush(cur);
        cur = rel;
      }
      const uint32_t ks0 = seg * kSegSteps + sq;  // K-step index in the row
      const uint8_t *sg0 = R.ring + slot0 * R.slot + (cw >> 1) * SEGB;
      if (pair) {
        RingPos nx = rp;
        nx.next(R.nst);
        if (!mbar_wait_bounded(&R.full[nx.slot], nx.phase, abort_flag)) {
          set_error(err, kErrConsumerWait);
          ok = false;
          break;
        }
        const uint8_t *const sgs[2] = {sg0, R.ring + nx.slot * R.slot + (cw >> 1) * SEGB};
        const uint32_t kss[2] = {ks0, ks0 + kStageSegs * kSegSteps};
        run(std::integral_constant<int, 2>{}, sgs, kss);
      } else {
        const uint8_t *const sgs[2] = {sg0, sg0};
        const uint32_t kss[2] = {ks0, ks0};
        run(std::integral_constant<int, 1>{}, sgs, kss);
      }
    }
    // release the stage (or both)
    __syncwarp();
    if (lane == 0) mbar_arrive(&R.empty[slot0]);
    advance();
    if (pair) {
      if (lane == 0) mbar_arrive(&R.empty[rp.slot]);
      advance();
      s += kStageSegs;
    }
  }
  if (ok && cur != 0xFFFFFFFFu) flush(cur);
  named_bar(1, NCT);  // every partial written

  // Deferred RMSNorm (mv_activation without xout): the rows are scaled by
  // 1/sqrt(sum of squares / C + eps), the warps' partial sums of squares being
  // in defer_ss[0..7].
  float row_scale = 1.0f;
  if (defer_ss) {
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < kMvConsumers; ++w) tot += defer_ss[w];
    row_scale = 1.0f / sqrtf(tot / (float)p.g.cols + p.eps);
  }
  // Tile reduction and epilogue: tile rel goes to warp rel % 8, lanes 0-7
  // take rows (l, l + 8), summing the 8 warps' partials in order.
  for (uint32_t t = cw; t < ntiles; t += kMvConsumers) {
    if (lane < 8) {
      float a = 0.f, b = 0.f;
#pragma unroll
      for (int w = 0; w < kMvConsumers; ++w) {
        a += red[(t * kMvConsumers + w) * kTileRows + lane];
        b += red[(t * kMvConsumers + w) * kTileRows + lane + 8u];
      }
      const uint32_t R0 = (t0 + t) * kTileRows + lane;
      epilogue(R0, a * row_scale, b * row_scale, t == cw ? pv0 : pre(R0));
    }
  }
}

template <bool Q8, Mode M, Pro P>
__global__ void __launch_bounds__(kMvThreads, 1) matvec_kernel(const __grid_constant__ MvParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const MvSmem L(p);
  const TileGeom g = p.g;
  const uint32_t NSEG = g.nseg(), SEGB = g.seg_bytes();
  MvRing R;
  R.ring = smem + L.ring;
  R.full = reinterpret_cast<uint64_t *>(smem + L.bars);
  R.empty = R.full + p.stages;
  R.nst = p.stages;
  R.slot = kStageSegs * SEGB;
  float *red = reinterpret_cast<float *>(smem + L.red);  // [tile][warp][row] partial sums
  float *scr = reinterpret_cast<float *>(smem + L.scr);

  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
  const uint32_t T = g.tiles();
  const uint32_t t0 = (uint32_t)((uint64_t)blockIdx.x * T / gridDim.x);
  const uint32_t t1 = (uint32_t)((uint64_t)(blockIdx.x + 1) * T / gridDim.x);
  const uint32_t n_items = (t1 - t0) * NSEG;  // segments of this CTA
  uint32_t *err = p.ctrl + kCtrlErr;

  if (threadIdx.x == 0) {
    for (uint32_t i = 0; i < R.nst; ++i) {
      mbar_init(&R.full[i], 1);
      mbar_init(&R.empty[i], kMvConsumers);  // every consumer warp releases every stage
    }
    fence_mbar_init();
  }
  for (uint32_t i = threadIdx.x; i < (t1 - t0) * kMvConsumers * kTileRows; i += blockDim.x) red[i] = 0.f;
  __syncthreads();
  pdl_launch_dependents();

  if (warp == kMvConsumers) {
    // producer: starts before griddepcontrol.wait, so the weights stream in
    // while the previous kernel of the step is still running
    if (lane == 0) {
      RingPos rp;
      if (mv_produce(R, p.w + (uint64_t)t0 * NSEG * SEGB, n_items, SEGB, rp, nullptr, err)) mv_drain(R, rp, err);
    }
    return;
  }
  const uint32_t cw = warp;
  XSrc src{};
  src.x = p.xsrc;
  WaitSpec wait{};
  wait.kind = kWaitPdl;
  mv_activation<Q8, P == Pro::RMSNORM, false>(g.cols, NSEG * g.seg_cols(), p.normw, p.eps, smem + L.a, p.plane, scr,
                                              cw, lane, src, wait, nullptr);
  const uint32_t pos = (M == Mode::QKV) ? p.ctrl[kCtrlPos] : 0u;
  bool ok = true;
  RingPos rp;
  mv_consume<Q8>(R, rp, n_items, NSEG, SEGB, smem + L.a, p.plane, red, p, t0, cw, lane, nullptr, err, ok,
                 P == Pro::RMSNORM ? scr + 8 : nullptr,
                 [](uint32_t) { return make_float2(0.f, 0.f); },
                 [&](uint32_t R0, float a, float b, float2) { mv_epilogue<M>(p, R0, a, b, pos); });
}

// ---------------------------------------------------------------------------
// Split-K flash-decoding GQA attention over one layer.
// grid = (nsplit, kv_heads), clusters of 8 CTAs along the split axis. Each CTA
// takes a chunk of at most chunk_cap positions of one KV head and all of that
// head's query heads: the K/V rows of the chunk are staged into shared memory
// by two cp.async.bulk copies issued before griddepcontrol.wait (the row of
// the current position, written by this step's QKV kernel, is loaded after
// it). It computes the scores (attn_scores.comp), a chunk-local softmax
// (softmax.comp) and the value sum (attn_values.comp). The 8 CTAs of a cluster
// merge their (m, l, o) partials through distributed shared memory (CTA r
// merges query heads r, r+8, ...); the last cluster of a KV head to finish
// (atomic ticket, no waiting) merges the cluster partials into the output.
// ---------------------------------------------------------------------------
constexpr uint32_t kAttnCluster = 8;
constexpr uint32_t kAttnThreads = 256;

struct AttnParams {
  const float *q;
  const __half *kc, *vc;   // this layer: [kv_head][ctx][head_dim]
  float *out;              // [heads * head_dim]
  float *part;             // [kv_heads][nsplit / 8][G][head_dim + 2]
  uint32_t *tickets;       // [kv_heads * G], zero between launches
  uint32_t heads, kv_heads, ctx, nsplit, chunk_cap;
  float scale;             // 1 / sqrt(head_dim)
  uint32_t fixed_pos;      // position to use, or 0xFFFFFFFF to read ctrl
  uint32_t *ctrl;
  uint32_t swz;            // 1: rows stored chunk-permuted (kv_swz, a stream's cache); 0: plain rows
};

__host__ __device__ inline uint32_t attention_smem_bytes(uint32_t G, uint32_t head_dim, uint32_t chunk_cap) {
  const uint32_t kv = 2u * chunk_cap * head_dim * 2u;          // K and V rows (fp16)
  const uint32_t f = G * chunk_cap + 2u * G * head_dim + 2u * G;  // scores, o, m, l, q (fp32)
  return ((kv + 15u) & ~15u) + f * 4u + 16u;
}

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ float ld_dsmem(const float *p, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_u32(p)), "r"(rank));
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(remote) : "memory");
  return v;
}

template <int DPL>
__global__ void __launch_bounds__(kAttnThreads) attention_kernel(const __grid_constant__ AttnParams p) {
  constexpr uint32_t D = 32u * DPL;
  extern __shared__ __align__(128) uint8_t sa[];
  const uint32_t split = blockIdx.x, kvh = blockIdx.y;
  const uint32_t G = p.heads / p.kv_heads;
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u, nwarps = kAttnThreads / 32;
  __half *sK = reinterpret_cast<__half *>(sa);
  __half *sV = sK + p.chunk_cap * D;
  float *sS = reinterpret_cast<float *>(sa + ((2u * p.chunk_cap * D * 2u + 15u) & ~15u));  // [G][chunk_cap]
  float *sO = sS + G * p.chunk_cap;  // [G][D]
  float *sM = sO + G * D;            // [G]
  float *sL = sM + G;                // [G]
  float *sQ = sL + G;                // [G][D]
  __shared__ __align__(8) uint64_t bar;
  __shared__ uint32_t is_last;

  uint32_t pos = p.fixed_pos != 0xFFFFFFFFu ? p.fixed_pos : p.ctrl[kCtrlPos];
  if (pos >= p.ctx) {
    if (threadIdx.x == 0 && p.ctrl) set_error(p.ctrl + kCtrlErr, kErrPosition);
    pos = p.ctx - 1;
  }
  const uint32_t n = pos + 1;
  const uint32_t chunk = (n + p.nsplit - 1) / p.nsplit;
  const uint32_t t0 = min(split * chunk, n), t1 = min(t0 + chunk, n), len = t1 - t0;
  const uint32_t tp = min(t1, pos);  // rows [t0, tp) were written by earlier steps
  const __half *kb = p.kc + (size_t)kvh * p.ctx * D;
  const __half *vb = p.vc + (size_t)kvh * p.ctx * D;
  const bool staged = tp > t0;

  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0 && staged) {
    const uint32_t bytes = (tp - t0) * D * 2u;
    mbar_arrive_expect_tx(&bar, 2u * bytes);
    bulk_g2s(sK, kb + (size_t)t0 * D, bytes, &bar);
    bulk_g2s(sV, vb + (size_t)t0 * D, bytes, &bar);
  }
  pdl_launch_dependents();
  pdl_wait();
  if (pos >= t0 && pos < t1) {
    const uint32_t r = pos - t0;
    for (uint32_t i = threadIdx.x; i < D / 2u; i += blockDim.x) {
      reinterpret_cast<__half2 *>(sK + r * D)[i] = reinterpret_cast<const __half2 *>(kb + (size_t)pos * D)[i];
      reinterpret_cast<__half2 *>(sV + r * D)[i] = reinterpret_cast<const __half2 *>(vb + (size_t)pos * D)[i];
    }
  }
  for (uint32_t i = threadIdx.x; i < G * D; i += blockDim.x) sQ[i] = p.q[(size_t)kvh * G * D + i];
  if (threadIdx.x == 0 && staged && !mbar_wait_bounded(&bar, 0) && p.ctrl)
    set_error(p.ctrl + kCtrlErr, kErrConsumerWait);
  __syncthreads();

  // scores: warp per position; lane holds DPL dims of K; query heads in groups of 8
  for (uint32_t t = warp; t < len; t += nwarps) {
    float kf[DPL];
    const __half *kr = sK + t * D + (p.swz ? kv_swz(t0 + t, lane * DPL, D) : lane * DPL);
#pragma unroll
    for (int j = 0; j < DPL; ++j) kf[j] = __half2float(kr[j]);
    for (uint32_t gb = 0; gb < G; gb += 8) {
      float part[8];
#pragma unroll
      for (uint32_t i = 0; i < 8; ++i) {
        float acc = 0.f;
        if (gb + i < G) {
          const float *qg = sQ + (gb + i) * D + lane * DPL;
#pragma unroll
          for (int j = 0; j < DPL; ++j) acc = fmaf(qg[j], kf[j], acc);
        }
        part[i] = acc;
      }
      const float tot = warp_sum8(part, lane);
      const uint32_t gi = gb + ((lane >> 2) & 7u);
      if ((lane & 3u) == 0 && gi < G) sS[gi * p.chunk_cap + t] = __fmul_rn(tot, p.scale);
    }
  }
  __syncthreads();

  // chunk-local softmax and value sum: warp per query head
  for (uint32_t g0 = warp; g0 < G; g0 += nwarps) {
    float *sg = sS + g0 * p.chunk_cap;
    float m = -INFINITY;
    for (uint32_t t = lane; t < len; t += 32) m = fmaxf(m, sg[t]);
    m = warp_max(m);
    float l = 0.f;
    for (uint32_t t = lane; t < len; t += 32) {
      const float e = expf(sg[t] - m);
      sg[t] = e;
      l += e;
    }
    l = warp_sum(l);
    __syncwarp();
    float o[DPL];
#pragma unroll
    for (int j = 0; j < DPL; ++j) o[j] = 0.f;
    for (uint32_t t = 0; t < len; ++t) {
      const float pw = sg[t];
      const __half *vr = sV + t * D + (p.swz ? kv_swz(t0 + t, lane * DPL, D) : lane * DPL);
#pragma unroll
      for (int j = 0; j < DPL; ++j) o[j] = fmaf(pw, __half2float(vr[j]), o[j]);
    }
#pragma unroll
    for (int j = 0; j < DPL; ++j) sO[g0 * D + lane * DPL + j] = o[j];
    if (lane == 0) {
      sM[g0] = len ? m : -INFINITY;
      sL[g0] = l;
    }
  }

  // merge the 8 chunks of this cluster through distributed shared memory
  cluster_sync();
  const uint32_t rank = cluster_rank();
  const uint32_t ncl = p.nsplit / kAttnCluster, cl = split / kAttnCluster;
  __shared__ float wts[32];
  __shared__ float stat[2];
  for (uint32_t g0 = rank; g0 < G; g0 += kAttnCluster) {
    if (warp == 0) {
      // lanes 0-7 read one peer each
      const float mj = lane < kAttnCluster ? ld_dsmem(&sM[g0], lane) : -INFINITY;
      const float lj = lane < kAttnCluster ? ld_dsmem(&sL[g0], lane) : 0.f;
      const float M = warp_max(mj);
      const float w = mj == -INFINITY ? 0.f : expf(mj - M);
      const float Lsum = warp_sum(w * lj);
      if (lane < kAttnCluster) wts[lane] = w;
      if (lane == 0) {
        stat[0] = M;
        stat[1] = Lsum;
      }
    }
    __syncthreads();
    float *dst = p.part + (((size_t)kvh * ncl + cl) * G + g0) * (D + 2);
    for (uint32_t d = threadIdx.x; d < D; d += blockDim.x) {
      float o[kAttnCluster];
#pragma unroll
      for (uint32_t j = 0; j < kAttnCluster; ++j) o[j] = ld_dsmem(&sO[g0 * D + d], j);
      float acc = 0.f;
#pragma unroll
      for (uint32_t j = 0; j < kAttnCluster; ++j) acc = fmaf(wts[j], o[j], acc);
      dst[d] = acc;
    }
    if (threadIdx.x == 0) {
      dst[D] = stat[0];
      dst[D + 1] = stat[1];
    }
    __syncthreads();
  }
  cluster_sync();  // peers' shared memory stays alive until every merge has read it

  // merge the clusters of this KV head: the last one to arrive does it
  for (uint32_t g0 = rank; g0 < G; g0 += kAttnCluster) {
    if (threadIdx.x == 0) {
      __threadfence();
      is_last = atomicAdd(&p.tickets[kvh * G + g0], 1u) == ncl - 1;
    }
    __syncthreads();
    if (is_last) {
      __threadfence();
      const float *pb = p.part + ((size_t)kvh * ncl * G + g0) * (D + 2);
      const size_t stride = (size_t)G * (D + 2);
      for (uint32_t c0 = 0; c0 < ncl; c0 += 32) {
        // weights of up to 32 clusters per pass (ncl is small: nsplit / 8)
        if (warp == 0) {
          float M = stat[0];
          if (c0 == 0) {
            M = -INFINITY;
            for (uint32_t c = lane; c < ncl; c += 32) M = fmaxf(M, __ldcg(pb + c * stride + D));
            M = warp_max(M);
          }
          float Lpart = 0.f;
          const uint32_t c = c0 + lane;
          if (c < ncl) {
            const float mc = __ldcg(pb + c * stride + D);
            const float w = mc == -INFINITY ? 0.f : expf(mc - M);
            wts[lane] = w;
            Lpart = w * __ldcg(pb + c * stride + D + 1);
          } else {
            wts[lane] = 0.f;
          }
          Lpart = warp_sum(Lpart);
          if (lane == 0) {
            stat[0] = M;
            stat[1] = c0 == 0 ? Lpart : stat[1] + Lpart;
          }
        }
        __syncthreads();
        const uint32_t nc = min(32u, ncl - c0);
        for (uint32_t d = threadIdx.x; d < D; d += blockDim.x) {
          float acc = c0 == 0 ? 0.f : p.out[((size_t)kvh * G + g0) * D + d];
          for (uint32_t c = 0; c < nc; ++c) acc = fmaf(wts[c], __ldcg(pb + (c0 + c) * stride + d), acc);
          p.out[((size_t)kvh * G + g0) * D + d] = acc;
        }
        __syncthreads();
      }
      const float invL = 1.0f / stat[1];
      for (uint32_t d = threadIdx.x; d < D; d += blockDim.x) p.out[((size_t)kvh * G + g0) * D + d] *= invL;
      if (threadIdx.x == 0) p.tickets[kvh * G + g0] = 0;
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// Token embedding: hidden[i] = dequant(W[token][i]) * alpha (embedding.comp).
// ---------------------------------------------------------------------------
__global__ void embedding_kernel(const uint8_t *w, TileGeom g, const uint32_t *token_ptr, uint32_t token_fixed,
                                 float alpha, float *out, uint32_t *err) {
  uint32_t tok = token_ptr ? *token_ptr : token_fixed;
  if (tok >= g.rows) {
    if (blockIdx.x == 0 && threadIdx.x == 0) set_error(err, kErrBadToken);
    tok = 0;
  }
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < g.cols; i += gridDim.x * blockDim.x) {
    float v;
    if (g.q8) {
      const float d = __half2float(*reinterpret_cast<const __half *>(w + g.scale_off(tok, i / 32u)));
      v = __fmul_rn(d, (float)(int8_t)w[g.elem_off(tok, i)]);
    } else {
      v = __half2float(*reinterpret_cast<const __half *>(w + g.elem_off(tok, i)));
    }
    out[i] = __fmul_rn(v, alpha);
  }
  pdl_launch_dependents();
}

// ---------------------------------------------------------------------------
// (Residual) RMSNorm in one CTA: residual_rmsnorm.comp / rmsnorm.comp. With
// branch == nullptr, hidden is only read. Optionally advances the position.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(1024) residual_rmsnorm_kernel(float *hidden, const float *branch, const float *w,
                                                                uint32_t n, float eps, float scale, float *y,
                                                                uint32_t *ctrl, int advance_pos) {
  __shared__ float red[32];
  __shared__ float inv_rms_s;
  pdl_launch_dependents();
  pdl_wait();
  float ss = 0.f;
  for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
    float v = hidden[i];
    if (branch) {
      v = __fadd_rn(v, __fmul_rn(branch[i], scale));
      hidden[i] = v;
    }
    ss += v * v;
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31u) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (uint32_t i = 0; i < blockDim.x / 32; ++i) t += red[i];
    inv_rms_s = 1.0f / sqrtf(t / (float)n + eps);
  }
  __syncthreads();
  const float inv_rms = inv_rms_s;
  for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) y[i] = __fmul_rn(__fmul_rn(hidden[i], inv_rms), w[i]);
  if (advance_pos && threadIdx.x == 0) ctrl[kCtrlPos] += 1u;
}

// ---------------------------------------------------------------------------
// GGUF matrix -> segmented tiles. One CTA per source row; the destination is
// zero-filled beforehand (padding rows and columns stay zero). The packed row
// of source row r is
//   kPermIdentity: r
//   kPermRope:     within each group of `group` rows (one head of d rows),
//                  element i < d/2 and its RoPE partner i + d/2 go to rows l
//                  and l + 8 of tile i / 8 of the head (l = i % 8)
//   kPermHalves:   tile r / 8, row r % 8 + 8 * half (gate rows half 0, up
//                  rows half 1 of an interleaved gate/up matrix)
// ---------------------------------------------------------------------------
enum : uint32_t { kPermIdentity = 0, kPermRope = 1, kPermHalves = 2 };

__host__ __device__ inline uint32_t packed_row(uint32_t r, uint32_t perm, uint32_t group, uint32_t half) {
  if (perm == kPermRope) {
    const uint32_t w = r % group, h = group / 2, i = w < h ? w : w - h;
    return (r / group) * group + (i / 8u) * kTileRows + (i % 8u) + (w < h ? 0u : 8u);
  }
  if (perm == kPermHalves) return (r / 8u) * kTileRows + (r % 8u) + 8u * half;
  return r;
}

__global__ void repack_kernel(const uint8_t *src, uint32_t src_rows, TileGeom g, uint8_t *dst, uint32_t perm,
                              uint32_t group, uint32_t half) {
  const uint32_t cols = g.cols;
  for (uint32_t r = blockIdx.x; r < src_rows; r += gridDim.x) {
    const uint32_t R = packed_row(r, perm, group, half);
    if (g.q8) {
      const uint32_t nb = cols / 32;
      const uint8_t *in = src + (size_t)r * nb * 34;
      for (uint32_t i = threadIdx.x; i < cols; i += blockDim.x) dst[g.elem_off(R, i)] = in[(i >> 5) * 34 + 2 + (i & 31)];
      for (uint32_t b = threadIdx.x; b < nb; b += blockDim.x) {
        const uint64_t o = g.scale_off(R, b);
        dst[o] = in[b * 34];
        dst[o + 1] = in[b * 34 + 1];
      }
    } else {
      const uint8_t *in = src + (size_t)r * cols * 2;
      for (uint32_t i = threadIdx.x; i < cols; i += blockDim.x) {
        const uint64_t o = g.elem_off(R, i);
        dst[o] = in[2 * i];
        dst[o + 1] = in[2 * i + 1];
      }
    }
  }
}

}  // namespace vg
