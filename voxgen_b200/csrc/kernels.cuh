// CUDA kernels of the BaseLM decode step (sm_100a).
//
// Weights live in HBM as "row records" (see repack_kernel): one record per
// matrix row, 16-byte aligned, so a contiguous range of rows is one contiguous
// byte range that the TMA engine can stream into shared memory with a single
// cp.async.bulk per ring slot. Row orders are permuted at load time so that
// every fused epilogue finds its operands in one warp:
//   * QKV: Q and K rows of each head are interleaved as (i, i + head_dim/2)
//     pairs, so a warp holds both halves of a RoPE rotation;
//   * gate/up: gate row r and up row r are adjacent, so a warp holds both
//     inputs of SwiGLU.
#pragma once
#include <cuda_fp16.h>

#include <cstdint>

#include "ptx.cuh"

namespace vg {

enum class WFmt { Q8, F16 };
enum class Mode { PLAIN, RESID, SWIGLU, QKV };
enum class Pro { COPY, RMSNORM };

constexpr int kConsumerWarps = 8;
constexpr int kMatvecThreads = 32 * (1 + kConsumerWarps);

// Slots of the per-stream device control block.
constexpr uint32_t kCtrlPos = 0;    // decode position of the step being run
constexpr uint32_t kCtrlToken = 1;  // token id of a token step
constexpr uint32_t kCtrlErr = 2;    // error flag bits (ptx.cuh)
constexpr uint32_t kCtrlWords = 16;

// ---- packed layouts -------------------------------------------------------
// Q8_0 row record: int8 quants [cols] | fp16 scales [cols/32] | pad to 16 B.
// F16 row record : fp16 [cols] | pad to 16 B.
__host__ __device__ constexpr uint32_t round16(uint32_t x) { return (x + 15u) & ~15u; }
__host__ __device__ constexpr uint32_t q8_row_bytes(uint32_t cols) { return round16(cols + cols / 16u); }
__host__ __device__ constexpr uint32_t f16_row_bytes(uint32_t cols) { return round16(cols * 2u); }

template <WFmt F> struct Fmt;
// A lane reads 16 bytes of a row per step: 16 int8 (Q8) or 8 fp16 (F16).
// x is kept in shared memory with 4 floats of padding every 16 (Q8) or 32
// (F16) elements so that the warp's 128-bit x loads are bank-conflict free.
template <> struct Fmt<WFmt::Q8> {
  static constexpr uint32_t EPL = 16, CHUNK = 512;
  __host__ __device__ static constexpr uint32_t xpad(uint32_t i) { return i + (i >> 4) * 4u; }
  __host__ __device__ static constexpr uint32_t row_bytes(uint32_t cols) { return q8_row_bytes(cols); }
};
template <> struct Fmt<WFmt::F16> {
  static constexpr uint32_t EPL = 8, CHUNK = 256;
  __host__ __device__ static constexpr uint32_t xpad(uint32_t i) { return i + (i >> 5) * 4u; }
  __host__ __device__ static constexpr uint32_t row_bytes(uint32_t cols) { return f16_row_bytes(cols); }
};

struct MvParams {
  const uint8_t *w;        // row records
  uint32_t rows, cols, row_bytes;
  uint32_t units;          // ceil(rows / RW)
  uint32_t slots;          // ring slots in shared memory
  uint32_t x_bytes;        // shared bytes reserved for x (128-aligned)
  const float *xsrc;       // input vector (COPY) or hidden state (RMSNORM)
  const float *normw;      // RMSNorm weight
  float eps;
  float *out;              // output vector (q for QKV)
  const float *resid;      // RESID: residual input
  float alpha;             // PLAIN: output scale; RESID: residual branch scale
  // QKV epilogue
  uint32_t q_rows, kv_rows, head_dim, ctx;
  __half *kc, *vc;         // this layer's caches, [kv_head][ctx][head_dim]
  const float *inv_freq;   // [head_dim/2], 1/pow(theta, 2i/d)
  const float *ext;        // [head_dim/2], LongRoPE factors
  float rope_scaling;
  uint32_t *ctrl;
};

__host__ __device__ inline uint32_t matvec_smem_bytes(uint32_t x_bytes, uint32_t slots, uint32_t slot_bytes) {
  return x_bytes + slots * slot_bytes + slots * 16u + 64u * 4u;
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

// sum_k q_k * x_k over 16 int8 quants. Each signed byte b becomes the float
// 2^23 + (b + 128) by placing (b ^ 0x80) in the low mantissa byte; subtracting
// 2^23 + 128 gives b exactly, with one byte permute and one add per value.
__device__ __forceinline__ float dot16_q8(uint4 q, const float *x) {
  const float2 bias = make_float2(-8388736.0f, -8388736.0f);
  float2 s0 = make_float2(0.f, 0.f), s1 = make_float2(0.f, 0.f);
  const uint32_t w[4] = {q.x ^ 0x80808080u, q.y ^ 0x80808080u, q.z ^ 0x80808080u, q.w ^ 0x80808080u};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float2 f01 = make_float2(__uint_as_float(__byte_perm(w[j], 0x4B000000u, 0x7650)),
                             __uint_as_float(__byte_perm(w[j], 0x4B000000u, 0x7651)));
    float2 f23 = make_float2(__uint_as_float(__byte_perm(w[j], 0x4B000000u, 0x7652)),
                             __uint_as_float(__byte_perm(w[j], 0x4B000000u, 0x7653)));
    f01 = __fadd2_rn(f01, bias);
    f23 = __fadd2_rn(f23, bias);
    s0 = __ffma2_rn(f01, make_float2(x[4 * j], x[4 * j + 1]), s0);
    s1 = __ffma2_rn(f23, make_float2(x[4 * j + 2], x[4 * j + 3]), s1);
  }
  return (s0.x + s0.y) + (s1.x + s1.y);
}

__device__ __forceinline__ float dot8_f16(uint4 h, const float *x) {
  const __half2 *h2 = reinterpret_cast<const __half2 *>(&h);
  float2 s = make_float2(0.f, 0.f);
#pragma unroll
  for (int j = 0; j < 4; ++j) s = __ffma2_rn(__half22float2(h2[j]), make_float2(x[2 * j], x[2 * j + 1]), s);
  return s.x + s.y;
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

// ---------------------------------------------------------------------------
// Matrix-vector product with fused prologue / epilogue.
//
// Warp 0 is the producer: lane 0 streams this CTA's contiguous slice of row
// records into a ring of shared-memory slots with cp.async.bulk, one mbarrier
// per slot. It starts before griddepcontrol.wait, so the weights of this
// kernel stream in while the previous kernel of the step is still running.
// Warps 1..8 are consumers: after the dependency resolves they build x in
// shared memory (copy, or RMSNorm of the hidden state), then each takes every
// 8th unit of RW rows, computes RW dot products from the slot (x held in
// registers per 512-column chunk, reused across the RW rows), releases the
// slot and runs the epilogue.
// ---------------------------------------------------------------------------
template <WFmt F, Mode M, Pro P, int RW>
__global__ void __launch_bounds__(kMatvecThreads, 1) matvec_kernel(const __grid_constant__ MvParams p) {
  using T = Fmt<F>;
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t C = p.cols;
  const uint32_t slot_bytes = RW * p.row_bytes;
  const uint32_t NS = p.slots;
  float *xs = reinterpret_cast<float *>(smem);
  uint8_t *ring = smem + p.x_bytes;
  uint64_t *full = reinterpret_cast<uint64_t *>(ring + NS * slot_bytes);
  uint64_t *empty = full + NS;
  float *red = reinterpret_cast<float *>(empty + NS);

  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
  const uint32_t u0 = (uint32_t)((uint64_t)blockIdx.x * p.units / gridDim.x);
  const uint32_t u1 = (uint32_t)((uint64_t)(blockIdx.x + 1) * p.units / gridDim.x);
  const uint32_t n = u1 - u0;
  uint32_t *err = p.ctrl + kCtrlErr;

  if (threadIdx.x == 0) {
    for (uint32_t i = 0; i < NS; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    fence_mbar_init();
  }
  __syncthreads();
  pdl_launch_dependents();

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t total = (uint64_t)p.rows * p.row_bytes;
      uint32_t s = 0;
      for (; s < n; ++s) {
        const uint32_t slot = s % NS;
        if (s >= NS && !mbar_wait_bounded(&empty[slot], ((s / NS) - 1u) & 1u)) {
          set_error(err, kErrProducerWait);
          break;
        }
        const uint64_t off = (uint64_t)(u0 + s) * slot_bytes;
        const uint64_t left = total - off;
        const uint32_t bytes = left < slot_bytes ? (uint32_t)left : slot_bytes;
        mbar_arrive_expect_tx(&full[slot], bytes);
        bulk_g2s(ring + slot * slot_bytes, p.w + off, bytes, &full[slot]);
      }
      // Never leave with copies in flight: wait (bounded) for the last phase
      // armed on each slot.
      const uint32_t armed = s < NS ? s : NS;
      for (uint32_t i = 0; i < armed; ++i) {
        const uint32_t last = i + ((s - 1u - i) / NS) * NS;
        if (!mbar_wait_bounded(&full[i], (last / NS) & 1u)) {
          set_error(err, kErrDrainWait);
          break;
        }
      }
    }
    return;
  }

  // ---- consumers ----
  constexpr uint32_t NCT = kConsumerWarps * 32;
  const uint32_t cw = warp - 1, ctid = threadIdx.x - 32;
  pdl_wait();
  if constexpr (P == Pro::RMSNORM) {
    // rmsnorm.comp:21-42 (inversesqrt taken as 1/sqrt); y = x * inv_rms * w.
    float ss = 0.f;
    for (uint32_t i = ctid * 4; i < C; i += NCT * 4) {
      const float4 v = *reinterpret_cast<const float4 *>(p.xsrc + i);
      ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
    }
    ss = warp_sum(ss);
    if (lane == 0) red[cw] = ss;
    named_bar(1, NCT);
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) tot += red[w];
    const float inv_rms = 1.0f / sqrtf(tot / (float)C + p.eps);
    for (uint32_t i = ctid * 4; i < C; i += NCT * 4) {
      float4 v = *reinterpret_cast<const float4 *>(p.xsrc + i);
      const float4 g = *reinterpret_cast<const float4 *>(p.normw + i);
      v.x = __fmul_rn(__fmul_rn(v.x, inv_rms), g.x);
      v.y = __fmul_rn(__fmul_rn(v.y, inv_rms), g.y);
      v.z = __fmul_rn(__fmul_rn(v.z, inv_rms), g.z);
      v.w = __fmul_rn(__fmul_rn(v.w, inv_rms), g.w);
      *reinterpret_cast<float4 *>(xs + T::xpad(i)) = v;
    }
  } else {
    for (uint32_t i = ctid * 4; i < C; i += NCT * 4)
      *reinterpret_cast<float4 *>(xs + T::xpad(i)) = *reinterpret_cast<const float4 *>(p.xsrc + i);
  }
  named_bar(1, NCT);

  const uint32_t pos = (M == Mode::QKV) ? p.ctrl[kCtrlPos] : 0u;
  for (uint32_t s = cw; s < n; s += kConsumerWarps) {
    const uint32_t slot = s % NS;
    if (!mbar_wait_bounded(&full[slot], (s / NS) & 1u)) {
      set_error(err, kErrConsumerWait);
      break;
    }
    const uint8_t *base = ring + slot * slot_bytes;
    float acc[RW];
#pragma unroll
    for (int r = 0; r < RW; ++r) acc[r] = 0.f;
    for (uint32_t col0 = lane * T::EPL; col0 < C; col0 += T::CHUNK) {
      float xv[T::EPL];
#pragma unroll
      for (uint32_t k = 0; k < T::EPL / 4; ++k) {
        const float4 v = *reinterpret_cast<const float4 *>(xs + T::xpad(col0) + 4 * k);
        xv[4 * k] = v.x;
        xv[4 * k + 1] = v.y;
        xv[4 * k + 2] = v.z;
        xv[4 * k + 3] = v.w;
      }
#pragma unroll
      for (int r = 0; r < RW; ++r) {
        const uint8_t *row = base + r * p.row_bytes;
        if constexpr (F == WFmt::Q8) {
          const uint4 q = *reinterpret_cast<const uint4 *>(row + col0);
          const float d = __half2float(*reinterpret_cast<const __half *>(row + C + (col0 >> 5) * 2u));
          acc[r] = fmaf(d, dot16_q8(q, xv), acc[r]);
        } else {
          const uint4 h = *reinterpret_cast<const uint4 *>(row + col0 * 2u);
          acc[r] += dot8_f16(h, xv);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);
#pragma unroll
    for (int r = 0; r < RW; ++r) acc[r] = warp_sum(acc[r]);

    const uint32_t rbase = (u0 + s) * RW;
    if constexpr (M == Mode::PLAIN || M == Mode::RESID) {
#pragma unroll
      for (int r = 0; r < RW; ++r) {
        const uint32_t R = rbase + r;
        if (lane == (uint32_t)r && R < p.rows) {
          if constexpr (M == Mode::PLAIN)
            p.out[R] = __fmul_rn(acc[r], p.alpha);  // matvec.comp:61
          else  // residual_rmsnorm.comp:27 with branch = this row's product
            p.out[R] = __fadd_rn(p.resid[R], __fmul_rn(acc[r], p.alpha));
        }
      }
    } else {
#pragma unroll
      for (int pr = 0; pr < RW / 2; ++pr) {
        const uint32_t R = rbase + 2 * pr;
        if (lane != (uint32_t)pr || R >= p.rows) continue;
        float a = acc[2 * pr], b = acc[2 * pr + 1];
        if constexpr (M == Mode::SWIGLU) {
          // matvec_swiglu.comp:65-68
          p.out[R >> 1] = __fmul_rn(__fdiv_rn(a, __fadd_rn(1.0f, expf(-a))), b);
        } else {
          const uint32_t hd = p.head_dim, half_d = hd >> 1;
          if (pos >= p.ctx) {
            set_error(err, kErrPosition);
          } else if (R < p.q_rows) {
            const uint32_t pi = R >> 1, head = pi / half_d, i = pi % half_d;
            rope_pair(a, b, pos, i, p.inv_freq, p.ext, p.rope_scaling);
            p.out[head * hd + i] = a;
            p.out[head * hd + i + half_d] = b;
          } else if (R < p.q_rows + p.kv_rows) {
            const uint32_t pi = (R - p.q_rows) >> 1, kvh = pi / half_d, i = pi % half_d;
            rope_pair(a, b, pos, i, p.inv_freq, p.ext, p.rope_scaling);
            // store_kv.comp:21-22: fp16 round-to-nearest-even
            __half *dst = p.kc + ((size_t)kvh * p.ctx + pos) * hd;
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
    }
  }
}

// ---------------------------------------------------------------------------
// Split-K flash-decoding GQA attention over one layer.
// grid = (nsplit, kv_heads); each CTA takes a contiguous chunk of positions of
// one KV head and all of that head's query heads (the K/V rows are read from
// HBM once for the whole group): scores (attn_scores.comp), a chunk-local
// softmax (softmax.comp) and the value sum (attn_values.comp), written as a
// partial (m, l, o). The last CTA of each KV head (atomic ticket, no waiting)
// merges the partials into the output.
// ---------------------------------------------------------------------------
struct AttnParams {
  const float *q;
  const __half *kc, *vc;   // this layer: [kv_head][ctx][head_dim]
  float *out;              // [heads * head_dim]
  float *part;             // [kv_heads][nsplit][G][head_dim + 2]
  uint32_t *tickets;       // [kv_heads], zero between launches
  uint32_t heads, kv_heads, ctx, nsplit, chunk_cap;
  float scale;             // 1 / sqrt(head_dim)
  uint32_t fixed_pos;      // position to use, or 0xFFFFFFFF to read ctrl
  uint32_t *ctrl;
};

__host__ __device__ inline uint32_t attention_smem_bytes(uint32_t G, uint32_t head_dim, uint32_t chunk_cap,
                                                         uint32_t nsplit) {
  const uint32_t a = G * head_dim + G * chunk_cap + 4 * G;
  const uint32_t b = 2 * G * nsplit + 2 * G;  // combine: weights and per-head stats
  return (a + b) * 4u + 16u;
}

template <int DPL>
__global__ void __launch_bounds__(256) attention_kernel(const __grid_constant__ AttnParams p) {
  constexpr uint32_t D = 32u * DPL;
  extern __shared__ __align__(16) float sa[];
  const uint32_t split = blockIdx.x, kvh = blockIdx.y;
  const uint32_t G = p.heads / p.kv_heads;
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u, nwarps = blockDim.x >> 5;
  float *qs = sa;                       // [G][D]
  float *sc = qs + G * D;               // [G][chunk_cap]
  float *mrow = sc + G * p.chunk_cap;   // [G]
  float *lrow = mrow + G;               // [G]
  float *wts = lrow + 2 * G;            // combine: [nsplit][G]
  float *stat = wts + G * p.nsplit;     // combine: [G] max, [G] 1/L
  __shared__ uint32_t is_last;

  pdl_launch_dependents();
  uint32_t pos = p.fixed_pos != 0xFFFFFFFFu ? p.fixed_pos : p.ctrl[kCtrlPos];
  if (pos >= p.ctx) {
    if (threadIdx.x == 0) set_error(p.ctrl ? p.ctrl + kCtrlErr : nullptr, kErrPosition);
    pos = p.ctx - 1;
  }
  const uint32_t n = pos + 1;
  const uint32_t chunk = (n + p.nsplit - 1) / p.nsplit;
  const uint32_t t0 = min(split * chunk, n), t1 = min(t0 + chunk, n);
  const __half *kb = p.kc + (size_t)kvh * p.ctx * D;
  const __half *vb = p.vc + (size_t)kvh * p.ctx * D;

  // Rows before `pos` were written by earlier steps: pull them toward L2 while
  // the QKV kernel of this step finishes.
  {
    const uint32_t tp = min(t1, pos);
    const uint32_t lines_per_row = (D * 2u + 127u) / 128u;
    const uint32_t nl = (tp > t0 ? tp - t0 : 0u) * lines_per_row;
    for (uint32_t i = threadIdx.x; i < 2 * nl; i += blockDim.x) {
      const uint32_t li = i < nl ? i : i - nl;
      const __half *base = i < nl ? kb : vb;
      prefetch_l2(reinterpret_cast<const uint8_t *>(base + (size_t)(t0 + li / lines_per_row) * D) +
                  (li % lines_per_row) * 128u);
    }
  }
  pdl_wait();

  for (uint32_t i = threadIdx.x; i < G * D; i += blockDim.x) qs[i] = p.q[(size_t)kvh * G * D + i];
  __syncthreads();

  // scores: warp per position, lane holds DPL dims
  for (uint32_t t = t0 + warp; t < t1; t += nwarps) {
    float kf[DPL];
    const __half *kr = kb + (size_t)t * D + lane * DPL;
    if constexpr (DPL == 1) {
      kf[0] = __half2float(*kr);
    } else if constexpr (DPL == 2) {
      kf[0] = __low2float(*reinterpret_cast<const __half2 *>(kr));
      kf[1] = __high2float(*reinterpret_cast<const __half2 *>(kr));
    } else {
#pragma unroll
      for (int k = 0; k < DPL; k += 4) {
        const uint2 raw = *reinterpret_cast<const uint2 *>(kr + k);
        const float2 f0 = __half22float2(*reinterpret_cast<const __half2 *>(&raw.x));
        const float2 f1 = __half22float2(*reinterpret_cast<const __half2 *>(&raw.y));
        kf[k] = f0.x;
        kf[k + 1] = f0.y;
        kf[k + 2] = f1.x;
        kf[k + 3] = f1.y;
      }
    }
    for (uint32_t g = 0; g < G; ++g) {
      const float *qg = qs + g * D + lane * DPL;
      float s = 0.f;
#pragma unroll
      for (int k = 0; k < DPL; ++k) s = fmaf(qg[k], kf[k], s);
      s = warp_sum(s);
      if (lane == 0) sc[g * p.chunk_cap + (t - t0)] = __fmul_rn(s, p.scale);
    }
  }
  __syncthreads();

  // chunk-local softmax and value sum: warp per query head
  const uint32_t len = t1 - t0;
  for (uint32_t g = warp; g < G; g += nwarps) {
    float *sg = sc + g * p.chunk_cap;
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
    for (int k = 0; k < DPL; ++k) o[k] = 0.f;
    for (uint32_t t = 0; t < len; ++t) {
      const float pw = sg[t];
      const __half *vr = vb + (size_t)(t0 + t) * D + lane * DPL;
#pragma unroll
      for (int k = 0; k < DPL; ++k) o[k] = fmaf(pw, __half2float(vr[k]), o[k]);
    }
    float *dst = p.part + (((size_t)kvh * p.nsplit + split) * G + g) * (D + 2);
#pragma unroll
    for (int k = 0; k < DPL; ++k) dst[lane * DPL + k] = o[k];
    if (lane == 0) {
      dst[D] = len ? m : -INFINITY;
      dst[D + 1] = l;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const uint32_t ticket = atomicAdd(&p.tickets[kvh], 1u);
    is_last = ticket == p.nsplit - 1;
  }
  __syncthreads();
  if (!is_last) return;
  __threadfence();

  // merge: M = max m_s, w_s = exp(m_s - M), out = sum w_s o_s / sum w_s l_s
  const float *pb = p.part + (size_t)kvh * p.nsplit * G * (D + 2);
  for (uint32_t g = warp; g < G; g += nwarps) {
    float M = -INFINITY;
    for (uint32_t s = lane; s < p.nsplit; s += 32) M = fmaxf(M, __ldcg(pb + ((size_t)s * G + g) * (D + 2) + D));
    M = warp_max(M);
    float L = 0.f;
    for (uint32_t s = lane; s < p.nsplit; s += 32) {
      const float *e = pb + ((size_t)s * G + g) * (D + 2);
      const float ms = __ldcg(e + D);
      const float w = ms == -INFINITY ? 0.f : expf(ms - M);
      wts[s * G + g] = w;
      L += w * __ldcg(e + D + 1);
    }
    L = warp_sum(L);
    if (lane == 0) stat[g] = 1.0f / L;
  }
  __syncthreads();
  for (uint32_t i = threadIdx.x; i < G * D; i += blockDim.x) {
    const uint32_t g = i / D, d = i % D;
    float acc = 0.f;
    for (uint32_t s = 0; s < p.nsplit; ++s) acc = fmaf(wts[s * G + g], __ldcg(pb + ((size_t)s * G + g) * (D + 2) + d), acc);
    p.out[((size_t)kvh * G + g) * D + d] = acc * stat[g];
  }
  if (threadIdx.x == 0) p.tickets[kvh] = 0;
}

// ---------------------------------------------------------------------------
// Token embedding: hidden[i] = dequant(W[token][i]) * alpha (embedding.comp).
// ---------------------------------------------------------------------------
__global__ void embedding_kernel(const uint8_t *w, int q8, uint32_t rows, uint32_t cols, uint32_t row_bytes,
                                 const uint32_t *token_ptr, uint32_t token_fixed, float alpha, float *out,
                                 uint32_t *err) {
  uint32_t tok = token_ptr ? *token_ptr : token_fixed;
  if (tok >= rows) {
    if (blockIdx.x == 0 && threadIdx.x == 0) set_error(err, kErrBadToken);
    tok = 0;
  }
  const uint8_t *row = w + (size_t)tok * row_bytes;
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < cols; i += gridDim.x * blockDim.x) {
    float v;
    if (q8) {
      const float d = __half2float(*reinterpret_cast<const __half *>(row + cols + (i >> 5) * 2u));
      v = __fmul_rn(d, (float)(int8_t)row[i]);
    } else {
      v = __half2float(reinterpret_cast<const __half *>(row)[i]);
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
// GGUF matrix -> row records. One CTA per source row. The destination row is
// perm(row) * dst_stride + dst_offset, where perm interleaves the two halves of
// each group of `pair_group` rows (0 = identity).
// ---------------------------------------------------------------------------
__global__ void repack_kernel(const uint8_t *src, int q8, uint32_t rows, uint32_t cols, uint8_t *dst,
                              uint32_t row_bytes, uint32_t dst_stride, uint32_t dst_offset, uint32_t pair_group) {
  for (uint32_t r = blockIdx.x; r < rows; r += gridDim.x) {
    uint32_t pr = r;
    if (pair_group) {
      const uint32_t g = r / pair_group, w = r % pair_group, h = pair_group / 2;
      pr = g * pair_group + (w < h ? 2 * w : 2 * (w - h) + 1);
    }
    uint8_t *out = dst + (size_t)(pr * dst_stride + dst_offset) * row_bytes;
    if (q8) {
      const uint32_t nb = cols / 32;
      const uint8_t *in = src + (size_t)r * nb * 34;
      for (uint32_t i = threadIdx.x; i < cols; i += blockDim.x) out[i] = in[(i >> 5) * 34 + 2 + (i & 31)];
      for (uint32_t b = threadIdx.x; b < nb; b += blockDim.x) {
        out[cols + 2 * b] = in[b * 34];
        out[cols + 2 * b + 1] = in[b * 34 + 1];
      }
      for (uint32_t i = cols + 2 * nb + threadIdx.x; i < row_bytes; i += blockDim.x) out[i] = 0;
    } else {
      const uint8_t *in = src + (size_t)r * cols * 2;
      for (uint32_t i = threadIdx.x; i < cols * 2; i += blockDim.x) out[i] = in[i];
      for (uint32_t i = cols * 2 + threadIdx.x; i < row_bytes; i += blockDim.x) out[i] = 0;
    }
  }
}

}  // namespace vg
