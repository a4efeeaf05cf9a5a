// CUDA kernels of the BaseLM decode step (sm_100a).
//
// Weight layout in HBM ("segmented 8-row tiles", built by repack_kernel).
// Every matrix is cut into tiles of 8 rows, and each tile into K-segments of
// 16 K-steps; a K-step is 32 int8 quants (Q8_0: exactly one block) or 16 fp16
// values, i.e. 8 rows x 32 bytes. A K-step is stored as two 128-byte 8x16-byte
// matrices (bytes 0-15 and 16-31 of the 8 rows), which is the order ldmatrix
// reads, so the tensor-core B operand loads are bank-conflict free. A Q8_0
// segment ends with the 16 x 8 fp16 block scales. One segment (4352 B Q8_0,
// 4096 B F16) is the unit the TMA engine streams into a shared-memory ring
// slot with one cp.async.bulk.
//
// Row orders are permuted at load time so that fused epilogues find both
// operands in one lane: rows 2j and 2j+1 of a tile are (i, i + head_dim/2) for
// the Q and K projections (RoPE pairs) and (gate r, up r) for the FFN.
//
// Activations enter the tensor cores exactly: for Q8_0, x is split per
// 32-element block into three int8 digits with a power-of-two block scale,
//   x = 2^e (d0 + d1 2^-7 + d2 2^-14),  |d_i| <= 64,
// so each K-step is an exact int32 mma (m16n8k32, digits as the A rows, the 8
// weight rows as B) that is then scaled by the fp16 block scale and 2^e in
// fp32. For F16 weights x is scaled by a power of two and split into fp16
// hi + lo, accumulated in fp32 by m16n8k16.
#pragma once
#include <cuda_fp16.h>

#include <cstdint>

#include "ptx.cuh"

namespace vg {

enum class Mode { PLAIN, RESID, SWIGLU, QKV };
enum class Pro { COPY, RMSNORM };

constexpr int kMvConsumers = 8;                       // consumer warps per matvec CTA
constexpr int kMvThreads = 32 * (1 + kMvConsumers);   // + one producer warp
constexpr uint32_t kTileRows = 8;
constexpr uint32_t kSegSteps = 16;                    // K-steps per segment
constexpr uint32_t kStepBytes = 256;                  // 8 rows x 32 bytes
constexpr uint32_t kSegQsBytes = kSegSteps * kStepBytes;

// Slots of the per-stream device control block.
constexpr uint32_t kCtrlPos = 0;    // decode position of the step being run
constexpr uint32_t kCtrlToken = 1;  // token id of a token step
constexpr uint32_t kCtrlErr = 2;    // error flag bits (ptx.cuh)
constexpr uint32_t kCtrlWords = 16;

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
    return seg_base(r, seg) + st * kStepBytes + (kb >> 4) * 128u + (r % kTileRows) * 16u + (kb & 15u);
  }
  // byte offset of the fp16 scale of Q8_0 block b of row r
  __host__ __device__ uint64_t scale_off(uint32_t r, uint32_t b) const {
    return seg_base(r, b / kSegSteps) + kSegQsBytes + ((b % kSegSteps) * kTileRows + (r % kTileRows)) * 2u;
  }
};

struct MvParams {
  const uint8_t *w;       // segmented tiles
  TileGeom g;
  uint32_t spw;           // ring slots per consumer warp
  uint32_t rb;            // tile reduction buffers (power of two)
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
};

// Shared-memory plan of one matvec CTA (host and device agree on it).
struct MvSmem {
  uint32_t a, ring, bars, red, cnt, gen, scr, total;
  __host__ __device__ MvSmem(const MvParams &p) {
    const uint32_t ns = kMvConsumers * p.spw;
    a = 0;
    ring = p.a_bytes;
    bars = ring + ns * p.g.seg_bytes();
    red = bars + ns * 16u;
    cnt = red + p.rb * kMvConsumers * kTileRows * 4u;
    gen = cnt + p.rb * 4u;
    scr = gen + p.rb * 4u;
    total = scr + 64u * 4u;
  }
};

__host__ __device__ inline uint32_t mv_a_plane(uint32_t q8, uint32_t cols_pad) {
  // planes are offset by 16 bytes modulo 128 so the 12 (Q8_0) or 8 (F16) lanes
  // that load A fragments from different planes hit different banks
  const uint32_t b = q8 ? cols_pad : cols_pad * 2u;
  return ((b + 127u) & ~127u) + 16u;
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
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t (&r)[4], const void *p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}

// D = A(16x32 s8, row) * B(32x8 s8, col); rows 8-15 of A are zero.
__device__ __forceinline__ void mma_s8(int (&d)[4], uint32_t a0, uint32_t a2, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%10, %11, %12, %13};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1), "r"(0), "r"(0), "r"(0), "r"(0));
}

// C += A(16x16 f16, row) * B(16x8 f16, col) in fp32; rows 8-15 of A are zero.
__device__ __forceinline__ void mma_f16(float (&c)[4], uint32_t a0, uint32_t a2, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1));
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

// Epilogue of one pair of adjacent packed rows (R even for pair modes).
template <Mode M>
__device__ __forceinline__ void mv_epilogue(const MvParams &p, uint32_t R, float a, float b, uint32_t pos) {
  if constexpr (M == Mode::PLAIN) {
    if (R < p.g.rows) p.out[R] = __fmul_rn(a, p.alpha);  // matvec.comp:61
    if (R + 1 < p.g.rows) p.out[R + 1] = __fmul_rn(b, p.alpha);
  } else if constexpr (M == Mode::RESID) {
    // residual_rmsnorm.comp:27, hidden + branch * scale, with branch = this row's product
    if (R < p.g.rows) p.out[R] = __fadd_rn(p.resid[R], __fmul_rn(a, p.alpha));
    if (R + 1 < p.g.rows) p.out[R + 1] = __fadd_rn(p.resid[R + 1], __fmul_rn(b, p.alpha));
  } else if constexpr (M == Mode::SWIGLU) {
    if (R < p.g.rows) p.out[R >> 1] = __fmul_rn(__fdiv_rn(a, __fadd_rn(1.0f, expf(-a))), b);  // matvec_swiglu.comp:67
  } else {
    if (R >= p.g.rows) return;
    const uint32_t hd = p.head_dim, half_d = hd >> 1;
    if (pos >= p.ctx) {
      set_error(p.ctrl + kCtrlErr, kErrPosition);
    } else if (R < p.q_rows) {
      const uint32_t pi = R >> 1, head = pi / half_d, i = pi % half_d;
      rope_pair(a, b, pos, i, p.inv_freq, p.ext, p.rope_scaling);
      p.out[head * hd + i] = a;
      p.out[head * hd + i + half_d] = b;
    } else if (R < p.q_rows + p.kv_rows) {
      const uint32_t pi = (R - p.q_rows) >> 1, kvh = pi / half_d, i = pi % half_d;
      rope_pair(a, b, pos, i, p.inv_freq, p.ext, p.rope_scaling);
      __half *dst = p.kc + ((size_t)kvh * p.ctx + pos) * hd;  // store_kv.comp:21-22, RNE
      dst[i] = __float2half_rn(a);
      dst[i + half_d] = __float2half_rn(b);
    } else {
      const uint32_t R2 = R - p.q_rows - p.kv_rows, kvh = R2 / hd, j = R2 % hd;
      __half *dst = p.vc + ((size_t)kvh * p.ctx + pos) * hd;
      dst[j] = __float2half_rn(a);
      dst[j + 1] = __float2half_rn(b);
    }
  }
}

// ---------------------------------------------------------------------------
// Matrix-vector product with fused prologue and epilogue.
//
// CTA c owns a contiguous range of tiles; its segments ("items", tile-major)
// are dealt round-robin to the 8 consumer warps. Warp 0 (lane 0) streams the
// items into the ring with cp.async.bulk; each consumer warp owns `spw` slots
// and consumes its items in order, so every mbarrier parity wait is at most
// one phase ahead. Streaming starts before griddepcontrol.wait: the weights
// arrive while the previous kernel of the step is still running.
// After the dependency resolves the consumers build the activation operand
// (RMSNorm of the hidden state or a copy, then the exact int8 digits or fp16
// hi/lo split), run the tensor-core K-steps of their items, and reduce each
// tile's 8 rows across warps through shared memory; the last warp to finish a
// tile (arrival counter) sums the warps' partials in warp order (so results
// are deterministic) and runs the epilogue.
// ---------------------------------------------------------------------------
template <bool Q8, Mode M, Pro P>
__global__ void __launch_bounds__(kMvThreads, 1) matvec_kernel(const __grid_constant__ MvParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const MvSmem L(p);
  const TileGeom g = p.g;
  const uint32_t NSEG = g.nseg(), SEGB = g.seg_bytes(), SPW = p.spw, NS = kMvConsumers * SPW;
  uint8_t *ring = smem + L.ring;
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + L.bars);
  uint64_t *empty = full + NS;
  float *red = reinterpret_cast<float *>(smem + L.red);
  uint32_t *cnt = reinterpret_cast<uint32_t *>(smem + L.cnt);
  uint32_t *gen = reinterpret_cast<uint32_t *>(smem + L.gen);
  float *scr = reinterpret_cast<float *>(smem + L.scr);

  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
  const uint32_t T = g.tiles();
  const uint32_t t0 = (uint32_t)((uint64_t)blockIdx.x * T / gridDim.x);
  const uint32_t t1 = (uint32_t)((uint64_t)(blockIdx.x + 1) * T / gridDim.x);
  const uint32_t n_items = (t1 - t0) * NSEG;
  uint32_t *err = p.ctrl + kCtrlErr;

  if (threadIdx.x == 0) {
    for (uint32_t i = 0; i < NS; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    fence_mbar_init();
  }
  for (uint32_t i = threadIdx.x; i < p.rb; i += blockDim.x) {
    cnt[i] = 0;
    gen[i] = 0;
  }
  __syncthreads();
  pdl_launch_dependents();

  if (warp == 0) {
    if (lane == 0) {
      uint32_t kw[kMvConsumers] = {};
      bool ok = true;
      for (uint32_t i = 0; i < n_items && ok; ++i) {
        const uint32_t w = i % kMvConsumers, k = kw[w];
        const uint32_t slot = w * SPW + k % SPW;
        if (k >= SPW && !mbar_wait_bounded(&empty[slot], ((k / SPW) - 1u) & 1u)) {
          set_error(err, kErrProducerWait);
          ok = false;
          break;
        }
        kw[w] = k + 1;
        const uint8_t *src = p.w + ((uint64_t)(t0 + i / NSEG) * NSEG + i % NSEG) * SEGB;
        mbar_arrive_expect_tx(&full[slot], SEGB);
        bulk_g2s(ring + slot * SEGB, src, SEGB, &full[slot]);
      }
      // Never leave with copies in flight: wait (bounded) for the last phase
      // armed on every slot.
      for (uint32_t w = 0; w < kMvConsumers && ok; ++w)
        for (uint32_t j = 0; j < SPW && j < kw[w]; ++j) {
          const uint32_t last = j + ((kw[w] - 1u - j) / SPW) * SPW;
          if (!mbar_wait_bounded(&full[w * SPW + j], (last / SPW) & 1u)) {
            set_error(err, kErrDrainWait);
            ok = false;
            break;
          }
        }
    }
    return;
  }

  // ---------------- consumers ----------------
  constexpr uint32_t NCT = kMvConsumers * 32;
  const uint32_t cw = warp - 1;
  const uint32_t C = g.cols;
  const uint32_t cols_pad = NSEG * g.seg_cols();
  uint8_t *areg = smem + L.a;
  float *sx = reinterpret_cast<float *>(areg + 3u * p.plane);  // Q8: per-block 2^e
  float *xscale = reinterpret_cast<float *>(areg + 2u * p.plane);  // F16: 2^e of the whole vector

  pdl_wait();
  float inv_rms = 1.0f;
  if constexpr (P == Pro::RMSNORM) {
    // rmsnorm.comp:21-42 (inversesqrt taken as 1/sqrt); x = h * inv_rms * w.
    float ss = 0.f;
    for (uint32_t i = threadIdx.x - 32; i < C; i += NCT) {
      const float v = p.xsrc[i];
      ss += v * v;
    }
    ss = warp_sum(ss);
    if (lane == 0) scr[cw] = ss;
    named_bar(1, NCT);
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < kMvConsumers; ++w) tot += scr[w];
    inv_rms = 1.0f / sqrtf(tot / (float)C + p.eps);
  }
  auto xval = [&](uint32_t k) -> float {
    if (k >= C) return 0.f;
    const float v = p.xsrc[k];
    if constexpr (P == Pro::RMSNORM) return __fmul_rn(__fmul_rn(v, inv_rms), p.normw[k]);
    return v;
  };
  if constexpr (Q8) {
    // one warp per 32-element block: digits and the block exponent
    int8_t *d0p = reinterpret_cast<int8_t *>(areg), *d1p = d0p + p.plane, *d2p = d1p + p.plane;
    for (uint32_t b = cw; b < cols_pad / 32u; b += kMvConsumers) {
      const uint32_t k = b * 32u + lane;
      const float x = xval(k);
      const uint32_t mb = __reduce_max_sync(0xffffffffu, __float_as_uint(fabsf(x)));
      int e = 0;
      int q0 = 0, q1 = 0, q2 = 0;
      const bool nz = block_exponent(mb, e);
      if (nz) {
        const float v = x * pow2f(-e);  // exact, |v| < 64
        const float f0 = rintf(v), r0 = (v - f0) * 128.0f;
        const float f1 = rintf(r0), r1 = (r0 - f1) * 128.0f;
        q0 = (int)f0;
        q1 = (int)f1;
        q2 = (int)rintf(r1);
      }
      d0p[k] = (int8_t)q0;
      d1p[k] = (int8_t)q1;
      d2p[k] = (int8_t)q2;
      if (lane == 0) sx[b] = nz ? pow2f(e) : 0.f;
    }
  } else {
    // whole-vector power-of-two scale, then fp16 hi + lo
    float m = 0.f;
    for (uint32_t k = threadIdx.x - 32; k < C; k += NCT) m = fmaxf(m, fabsf(xval(k)));
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
    __half *hi = reinterpret_cast<__half *>(areg), *lo = reinterpret_cast<__half *>(areg + p.plane);
    for (uint32_t k = threadIdx.x - 32; k < cols_pad; k += NCT) {
      const float v = xval(k) * inv;
      const __half h = __float2half_rn(v);
      hi[k] = h;
      lo[k] = __float2half_rn(v - __half2float(h));
    }
    if (threadIdx.x == 32) *xscale = pow2f(e);
  }
  named_bar(1, NCT);

  const uint32_t pos = (M == Mode::QKV) ? p.ctrl[kCtrlPos] : 0u;
  const uint32_t gq = lane >> 2, tq = lane & 3u;
  // digit / half plane this lane feeds into the A fragment (rows 0-2 or 0-1)
  const bool arow = Q8 ? (gq < 3) : (gq < 2);
  const uint8_t *aplane = areg + (arow ? gq : 0u) * p.plane;
  const float dscale = gq == 0 ? 1.0f : gq == 1 ? 0.0078125f : 6.103515625e-05f;  // 2^(-7 gq)
  uint32_t k = 0;  // items consumed by this warp
  bool ok = true;
  for (uint32_t t = t0; t < t1; ++t) {
    float acc0 = 0.f, acc1 = 0.f;
    float cf[4] = {0.f, 0.f, 0.f, 0.f};
    const uint32_t i0 = (t - t0) * NSEG;
    for (uint32_t s = (cw + kMvConsumers - i0 % kMvConsumers) % kMvConsumers; ok && s < NSEG;
         s += kMvConsumers) {
      const uint32_t slot = cw * SPW + k % SPW;
      if (!mbar_wait_bounded(&full[slot], (k / SPW) & 1u)) {
        set_error(err, kErrConsumerWait);
        ok = false;
        break;
      }
      const uint8_t *seg = ring + slot * SEGB;
      const uint32_t ks0 = s * kSegSteps;
#pragma unroll 2
      for (uint32_t ks = 0; ks < kSegSteps; ks += 2) {
        uint32_t b[4];
        ldmatrix_x4(b, seg + ks * kStepBytes + lane * 16u);
#pragma unroll
        for (uint32_t j = 0; j < 2; ++j) {
          const uint32_t kg = ks0 + ks + j;
          if constexpr (Q8) {
            uint32_t a0 = 0, a2 = 0;
            if (arow) {
              a0 = *reinterpret_cast<const uint32_t *>(aplane + kg * 32u + tq * 4u);
              a2 = *reinterpret_cast<const uint32_t *>(aplane + kg * 32u + 16u + tq * 4u);
            }
            int c[4];
            mma_s8(c, a0, a2, b[2 * j], b[2 * j + 1]);
            if (arow) {
              const __half2 dp =
                  *reinterpret_cast<const __half2 *>(seg + kSegQsBytes + ((ks + j) * kTileRows + 2u * tq) * 2u);
              const float sc = sx[kg] * dscale;
              acc0 = fmaf((float)c[0], __low2float(dp) * sc, acc0);
              acc1 = fmaf((float)c[1], __high2float(dp) * sc, acc1);
            }
          } else {
            uint32_t a0 = 0, a2 = 0;
            if (arow) {
              a0 = *reinterpret_cast<const uint32_t *>(aplane + (kg * 16u + tq * 2u) * 2u);
              a2 = *reinterpret_cast<const uint32_t *>(aplane + (kg * 16u + 8u + tq * 2u) * 2u);
            }
            mma_f16(cf, a0, a2, b[2 * j], b[2 * j + 1]);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
      ++k;
    }
    // this warp's partial for the 8 rows of tile t: lanes 0-3 hold rows 2tq, 2tq+1
    float v0, v1;
    if constexpr (Q8) {
      v0 = acc0 + __shfl_down_sync(0xffffffffu, acc0, 4) + __shfl_down_sync(0xffffffffu, acc0, 8);
      v1 = acc1 + __shfl_down_sync(0xffffffffu, acc1, 4) + __shfl_down_sync(0xffffffffu, acc1, 8);
    } else {
      v0 = (cf[0] + __shfl_down_sync(0xffffffffu, cf[0], 4)) * *xscale;
      v1 = (cf[1] + __shfl_down_sync(0xffffffffu, cf[1], 4)) * *xscale;
    }
    const uint32_t rel = t - t0, buf = rel & (p.rb - 1u), want_gen = rel / p.rb;
    // the previous use of this buffer must have been reduced (bounded wait)
    if (lane == 0 && rel >= p.rb) {
      const uint64_t ts = globaltimer();
      uint32_t it = 0;
      while (*reinterpret_cast<volatile uint32_t *>(&gen[buf]) != want_gen) {
        if (++it > kWaitMaxIters || ((it & 255u) == 0 && globaltimer() - ts > kWaitLimitNs)) {
          set_error(err, kErrConsumerWait);
          break;
        }
      }
    }
    __syncwarp();
    if (lane < 4) {
      red[(buf * kMvConsumers + cw) * kTileRows + 2 * lane] = v0;
      red[(buf * kMvConsumers + cw) * kTileRows + 2 * lane + 1] = v1;
    }
    __syncwarp();
    uint32_t last = 0;
    if (lane == 0) {
      __threadfence_block();
      last = atomicAdd(&cnt[buf], 1u) == kMvConsumers - 1;
    }
    last = __shfl_sync(0xffffffffu, last, 0);
    if (last) {
      __threadfence_block();
      if (lane < 4) {
        float a = 0.f, bsum = 0.f;
#pragma unroll
        for (int w = 0; w < kMvConsumers; ++w) {
          a += *reinterpret_cast<volatile float *>(&red[(buf * kMvConsumers + w) * kTileRows + 2 * lane]);
          bsum += *reinterpret_cast<volatile float *>(&red[(buf * kMvConsumers + w) * kTileRows + 2 * lane + 1]);
        }
        mv_epilogue<M>(p, t * kTileRows + 2 * lane, a, bsum, pos);
      }
      __syncwarp();
      if (lane == 0) {
        cnt[buf] = 0;
        __threadfence_block();
        *reinterpret_cast<volatile uint32_t *>(&gen[buf]) = want_gen + 1;
      }
    }
    if (!ok) break;
  }
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

  // scores: warp per position; lane holds DPL dims of K
  for (uint32_t t = warp; t < len; t += nwarps) {
    float kf[DPL];
    const __half *kr = sK + t * D + lane * DPL;
#pragma unroll
    for (int j = 0; j < DPL; ++j) kf[j] = __half2float(kr[j]);
    for (uint32_t g0 = 0; g0 < G; ++g0) {
      const float *qg = sQ + g0 * D + lane * DPL;
      float s = 0.f;
#pragma unroll
      for (int j = 0; j < DPL; ++j) s = fmaf(qg[j], kf[j], s);
      s = warp_sum(s);
      if (lane == 0) sS[g0 * p.chunk_cap + t] = __fmul_rn(s, p.scale);
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
      const __half *vr = sV + t * D + lane * DPL;
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
  __shared__ float wts[kAttnCluster];
  __shared__ float stat[2];
  for (uint32_t g0 = rank; g0 < G; g0 += kAttnCluster) {
    if (threadIdx.x == 0) {
      float mj[kAttnCluster], M = -INFINITY;
      for (uint32_t j = 0; j < kAttnCluster; ++j) {
        mj[j] = ld_dsmem(&sM[g0], j);
        M = fmaxf(M, mj[j]);
      }
      float Lsum = 0.f;
      for (uint32_t j = 0; j < kAttnCluster; ++j) {
        const float w = mj[j] == -INFINITY ? 0.f : expf(mj[j] - M);
        wts[j] = w;
        Lsum += w * ld_dsmem(&sL[g0], j);
      }
      stat[0] = M;
      stat[1] = Lsum;
    }
    __syncthreads();
    float *dst = p.part + (((size_t)kvh * ncl + cl) * G + g0) * (D + 2);
    for (uint32_t d = threadIdx.x; d < D; d += blockDim.x) {
      float acc = 0.f;
      for (uint32_t j = 0; j < kAttnCluster; ++j) acc = fmaf(wts[j], ld_dsmem(&sO[g0 * D + d], j), acc);
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
      if (threadIdx.x < 32) {
        float M = -INFINITY;
        for (uint32_t c = lane; c < ncl; c += 32) M = fmaxf(M, __ldcg(pb + c * stride + D));
        M = warp_max(M);
        float Lsum = 0.f;
        for (uint32_t c = lane; c < ncl; c += 32) {
          const float mc = __ldcg(pb + c * stride + D);
          Lsum += (mc == -INFINITY ? 0.f : expf(mc - M)) * __ldcg(pb + c * stride + D + 1);
        }
        Lsum = warp_sum(Lsum);
        if (lane == 0) {
          stat[0] = M;
          stat[1] = 1.0f / Lsum;
        }
      }
      __syncthreads();
      for (uint32_t d = threadIdx.x; d < D; d += blockDim.x) {
        float acc = 0.f;
        for (uint32_t c = 0; c < ncl; ++c) {
          const float mc = __ldcg(pb + c * stride + D);
          const float w = mc == -INFINITY ? 0.f : expf(mc - stat[0]);
          acc = fmaf(w, __ldcg(pb + c * stride + d), acc);
        }
        p.out[((size_t)kvh * G + g0) * D + d] = acc * stat[1];
      }
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
// is perm(row) * dst_stride + dst_offset, where perm interleaves the two
// halves of each group of `pair_group` rows (0 = identity).
// ---------------------------------------------------------------------------
__global__ void repack_kernel(const uint8_t *src, uint32_t src_rows, TileGeom g, uint8_t *dst, uint32_t dst_stride,
                              uint32_t dst_offset, uint32_t pair_group) {
  const uint32_t cols = g.cols;
  for (uint32_t r = blockIdx.x; r < src_rows; r += gridDim.x) {
    uint32_t pr = r;
    if (pair_group) {
      const uint32_t grp = r / pair_group, w = r % pair_group, h = pair_group / 2;
      pr = grp * pair_group + (w < h ? 2 * w : 2 * (w - h) + 1);
    }
    const uint32_t R = pr * dst_stride + dst_offset;
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
